"""The expert cache of the streaming path, over the C-ABI (``trc_cache_*``, ``trc_rejouer``,
``trc_trace_lire``): the host-side mirror of trc-cache's ``Cache``, ``Trace``, ``rejouer``
(moteur/crates/trc-cache/src/lib.rs:105-301, trace.rs:1-171), same names and meaning.

Differences: a request that finds no free or evictable slot, and ``pret`` on a slot not in
flight, raise ``ErreurUsage`` (the reference panics); policies are chosen by name ("lru",
"belady"), with ``casser=True`` for the reference's broken-policy witness (hits not told)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import ErreurUsage, lib, verifier


class _Decision(C.Structure):
    _fields_ = [("sorte", C.c_uint32), ("emplacement", C.c_uint32), ("tiede", C.c_int32), ("reserve", C.c_uint32)]


class _Compteurs(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("succes_vram", "succes_ram", "defauts_disque", "octets_disque",
                                            "octets_copies", "evictions", "evictions_ram")]


class _TraceDims(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("experts", "couches", "k", "jetons", "erreur", "erreur_ligne",
                                            "erreur_expert", "reserve")]


_u16p, _u32, _u64, _vp, _sz, _i32, _i64 = (C.POINTER(C.c_uint16), C.c_uint32, C.c_uint64, C.c_void_p, C.c_size_t,
                                           C.c_int, C.c_int64)
for _n, (_r, _a) in {
    "trc_cache_nouveau": (_vp, [_u32, _u32, _u32, _vp, _u32, C.c_uint16, C.c_uint16, _u32]),
    "trc_cache_detruire": (None, [_vp]),
    "trc_cache_fixer_tailles": (_i32, [_vp, _vp, C.c_uint16, C.c_uint16]),
    "trc_cache_demander": (_i32, [_vp, C.c_uint16, _vp, _u32, _u64, _vp]),
    "trc_cache_pret": (_i32, [_vp, _u32]),
    "trc_cache_liberer": (_i32, [_vp, C.c_uint16]),
    "trc_cache_compteurs": (None, [_vp, _vp]),
    "trc_cache_etat": (_i32, [_vp, _u32, _vp, _vp]),
    "trc_cache_occupant": (_i64, [_vp, _u32]),
    "trc_cache_emplacement_de": (_i64, [_vp, C.c_uint16, C.c_uint16]),
    "trc_cache_tiede_de": (_i64, [_vp, C.c_uint16, C.c_uint16]),
    "trc_cache_epingles": (_u32, [_vp, _vp, _u32]),
    "trc_rejouer": (_i32, [_vp, _u32, C.c_uint16, C.c_uint16, _u32, _u32, _u32, _u32, _vp]),
    "trc_trace_lire": (_i32, [C.c_char_p, _sz, _vp, _vp, _sz]),
}.items():
    getattr(lib, _n).restype = _r
    getattr(lib, _n).argtypes = _a

POLITIQUES = {"lru": 0, "belady": 1}
SORTES = {0: "succes", 1: "defaut_ram", 2: "defaut_disque"}
ETATS = {0: "libre", 1: "en_vol", 2: "present"}


@dataclass(frozen=True)
class Decision:
    """Succes{emplacement}, DefautRam{emplacement, tiede}, DefautDisque{emplacement, tiede|None}."""
    sorte: str
    emplacement: int
    tiede: int | None = None


@dataclass
class Compteurs:
    succes_vram: int = 0
    succes_ram: int = 0
    defauts_disque: int = 0
    octets_disque: int = 0
    octets_copies: int = 0
    evictions: int = 0
    evictions_ram: int = 0

    def acces(self) -> int:
        return self.succes_vram + self.succes_ram + self.defauts_disque


def _compteurs(c: _Compteurs) -> Compteurs:
    return Compteurs(**{n: int(getattr(c, n)) for n, _ in _Compteurs._fields_})


class ErreurTrace(ValueError):
    """A trace that is refused (trace.rs:150-171): ``sorte`` "ligne" (``numero``), "hors_bornes"
    (``expert``, ``experts``), "vide" or "lecture"."""

    def __init__(self, message, sorte, numero=0, expert=0, experts=0):
        super().__init__(message)
        self.sorte, self.numero, self.expert, self.experts = sorte, numero, expert, experts


@dataclass
class Trace:
    """A routing trace: choix[T][L][k], the k experts each layer chose at each token."""
    experts: int
    couches: int
    k: int
    jetons: int
    choix: np.ndarray
    commentaires: list = field(default_factory=list)

    def groupe(self, jeton: int, couche: int) -> np.ndarray:
        return self.choix[jeton, couche]

    def acces(self) -> int:
        return int(self.choix.size)

    @classmethod
    def depuis_texte(cls, texte: str) -> "Trace":
        b = texte.encode()
        d = _TraceDims()
        st = lib.trc_trace_lire(b, len(b), C.byref(d), None, 0)
        if st != 0:
            msg = lib.trc_derniere_erreur().decode()
            sorte = {1: "ligne", 2: "hors_bornes", 3: "vide"}.get(d.erreur, "ligne")
            raise ErreurTrace(msg, sorte, d.erreur_ligne, d.erreur_expert, d.experts)
        choix = np.zeros((d.jetons, d.couches, d.k), np.uint16)
        verifier(lib.trc_trace_lire(b, len(b), C.byref(d), choix.ctypes.data, choix.size))
        comm = [l.strip()[1:].strip() for l in texte.splitlines() if l.strip().startswith("#")]
        return cls(int(d.experts), int(d.couches), int(d.k), int(d.jetons), choix, comm)

    @classmethod
    def depuis_choix(cls, choix, experts: int) -> "Trace":
        ch = np.ascontiguousarray(choix, np.uint16)
        return cls(experts, ch.shape[1], ch.shape[2], ch.shape[0], ch)


def lire_trace(chemin: str) -> Trace:
    try:
        with open(chemin, encoding="utf-8") as f:
            texte = f.read()
    except OSError as e:
        raise ErreurTrace(f"unreadable trace ({chemin}): {e}", "lecture") from e
    return Trace.depuis_texte(texte)


class Cache:
    """The two-tier expert cache (Cache::nouveau): `emplacements` device slots, `tiedes` host
    entries; `politique` "lru" or "belady" (Belady reads the future from `trace`)."""

    def __init__(self, emplacements: int, tiedes: int = 0, politique: str = "lru", trace: Trace | None = None,
                 casser: bool = False):
        ch = None if trace is None else np.ascontiguousarray(trace.choix, np.uint16)
        self._choix = ch
        p = lib.trc_cache_nouveau(emplacements, tiedes, POLITIQUES[politique],
                                  None if ch is None else ch.ctypes.data, 0 if ch is None else ch.shape[0],
                                  0 if ch is None else ch.shape[1], 0 if ch is None else ch.shape[2], int(casser))
        if not p:
            raise ErreurUsage(lib.trc_derniere_erreur().decode())
        self._p = C.c_void_p(p)
        self.emplacements = emplacements
        self._d = (_Decision * 64)()

    def __del__(self):
        p = getattr(self, "_p", None)
        if p:
            lib.trc_cache_detruire(p)
            self._p = None

    def fixer_tailles(self, tailles) -> None:
        """tailles[couche][expert]: the bytes of each expert's part."""
        t = np.ascontiguousarray(tailles, np.uint64)
        self._tailles = t
        verifier(lib.trc_cache_fixer_tailles(self._p, t.ctypes.data, t.shape[0], t.shape[1]))

    def demander(self, couche: int, experts, t: int) -> list:
        ex = np.ascontiguousarray(experts, np.uint16)
        if ex.size > len(self._d):
            self._d = (_Decision * ex.size)()
        verifier(lib.trc_cache_demander(self._p, couche, ex.ctypes.data, ex.size, t, self._d))
        return [Decision(SORTES[d.sorte], int(d.emplacement), None if d.tiede < 0 else int(d.tiede))
                for d in self._d[:ex.size]]

    def pret(self, emplacement: int) -> None:
        verifier(lib.trc_cache_pret(self._p, emplacement))

    def liberer(self, couche: int) -> None:
        verifier(lib.trc_cache_liberer(self._p, couche))

    def compteurs(self) -> Compteurs:
        c = _Compteurs()
        lib.trc_cache_compteurs(self._p, C.byref(c))
        return _compteurs(c)

    def evictions_ram(self) -> int:
        return self.compteurs().evictions_ram

    def etat(self, emplacement: int):
        """("libre" | "en_vol" | "present", niveau): niveau 1 (exact) unless free."""
        e, n = C.c_uint32(), C.c_uint32()
        verifier(lib.trc_cache_etat(self._p, emplacement, C.byref(e), C.byref(n)))
        return ETATS[e.value], n.value

    def occupant(self, emplacement: int):
        v = lib.trc_cache_occupant(self._p, emplacement)
        return None if v < 0 else (v >> 16, v & 0xFFFF)

    def emplacement_de(self, id_) -> int | None:
        v = lib.trc_cache_emplacement_de(self._p, id_[0], id_[1])
        return None if v < 0 else int(v)

    def tiede_de(self, id_) -> int | None:
        v = lib.trc_cache_tiede_de(self._p, id_[0], id_[1])
        return None if v < 0 else int(v)

    def epingles(self) -> list:
        n = lib.trc_cache_epingles(self._p, None, 0)
        a = (C.c_uint32 * max(n, 1))()
        lib.trc_cache_epingles(self._p, a, n)
        return [(v >> 16, v & 0xFFFF) for v in a[:n]]


def rejouer(trace: Trace, emplacements: int, tiedes: int = 0, politique: str = "lru", casser: bool = False) -> Compteurs:
    """The simulator (lib.rs:272-301): the trace through a new cache, counted in accesses."""
    ch = np.ascontiguousarray(trace.choix, np.uint16)
    c = _Compteurs()
    verifier(lib.trc_rejouer(ch.ctypes.data, ch.shape[0], ch.shape[1], ch.shape[2], emplacements, tiedes,
                             POLITIQUES[politique], int(casser), C.byref(c)))
    return _compteurs(c)

