"""The streaming layer executor over the C-ABI (``trc_flux_*``): MoE layers whose experts' parts
live in pinned host memory and come to the GPU on demand, through the expert cache (trc-ordo's
on-demand step, moteur/crates/trc-ordo/src/lib.rs:1054-1367)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import DimsExpert, lib, verifier
from .cache import Compteurs, _Compteurs, _compteurs


class FluxConfig(C.Structure):
    """trc_flux_config: 128 bytes."""
    _fields_ = [("couches", C.c_uint32), ("experts", C.c_uint32), ("k", C.c_uint32), ("jetons_max", C.c_uint32),
                ("dims", DimsExpert), ("emplacements", C.c_uint32), ("n_delta", C.c_uint32),
                ("n_codes", C.c_uint32), ("reserve", C.c_uint32), ("taille_emplacement", C.c_uint64),
                ("emplacements_carte", C.c_uint64), ("parties_hote", C.c_uint64), ("tailles_parties", C.c_uint64),
                ("luts", C.c_uint64), ("routeurs", C.c_uint64), ("biais_routeurs", C.c_uint64),
                ("espace", C.c_uint64), ("flux", C.c_uint64)]


class FluxStats(C.Structure):
    """trc_flux_stats: 32 bytes."""
    _fields_ = [("uniques", C.c_uint32), ("succes", C.c_uint32), ("defauts", C.c_uint32), ("reserve", C.c_uint32),
                ("octets_copies", C.c_uint64), ("attente_routeur_s", C.c_double)]


_vp, _u32 = C.c_void_p, C.c_uint32
for _n, (_r, _a) in {
    "trc_flux_espace_octets": (C.c_uint64, [_vp]),
    "trc_flux_nouveau": (_vp, [_vp]),
    "trc_flux_detruire": (None, [_vp]),
    "trc_flux_couche": (C.c_int, [_vp, _u32, _vp, _u32, _vp, _u32, _vp, _vp, _vp]),
    "trc_flux_compteurs": (C.c_int, [_vp, _vp]),
    "trc_flux_controle": (C.c_int, [_vp, _vp, _u32]),
}.items():
    getattr(lib, _n).restype = _r
    getattr(lib, _n).argtypes = _a


def tiers_hote(parties: list, alignement: int = 4096):
    """The host tier: every part (bytes) in one pinned buffer, each at an `alignement`-aligned
    offset. Returns (buffer, addresses u64[n], sizes u64[n])."""
    import torch

    decal, p = [], 0
    for b in parties:
        decal.append(p)
        p += (len(b) + alignement - 1) // alignement * alignement
    tampon = torch.empty(max(p, alignement), dtype=torch.uint8).pin_memory()
    vue = tampon.numpy()
    for d, b in zip(decal, parties):
        vue[d:d + len(b)] = np.frombuffer(b, np.uint8)
    base = tampon.data_ptr()
    return tampon, np.array([base + d for d in decal], np.uint64), np.array([len(b) for b in parties], np.uint64)


class Flux:
    """An executor for `couches` layers of `experts` experts: parts_hote / tailles u64[couches][experts]
    (addresses in pinned host memory and sizes), luts u32[couches][3][4][4096] on the device,
    routeurs f32[couches][experts][d] and biais f32[couches][experts] (or None: imposed routing
    only), `emplacements` device slots of `taille_emplacement` bytes."""

    def __init__(self, dims: DimsExpert, couches: int, experts: int, k: int, emplacements: int, parties_hote,
                 tailles, luts, routeurs=None, biais=None, jetons_max: int = 1, taille_emplacement: int | None = None,
                 n_delta: int = 0, n_codes: int = 0, flux=None):
        import torch

        self.dims = dims
        self.parties_hote = np.ascontiguousarray(parties_hote, np.uint64).reshape(couches, experts)
        self.tailles = np.ascontiguousarray(tailles, np.uint64).reshape(couches, experts)
        te = taille_emplacement or int((int(self.tailles.max()) + 4095) // 4096 * 4096)
        self.emplacements_carte = torch.empty(emplacements * te + 256, dtype=torch.uint8, device="cuda")
        self.luts, self.routeurs, self.biais = luts, routeurs, biais
        self.flux = flux if flux is not None else torch.cuda.current_stream()
        c = FluxConfig()
        c.couches, c.experts, c.k, c.jetons_max = couches, experts, k, jetons_max
        c.dims = dims
        c.emplacements, c.n_delta, c.n_codes = emplacements, n_delta, n_codes
        c.taille_emplacement = te
        c.emplacements_carte = self.emplacements_carte.data_ptr() + (-self.emplacements_carte.data_ptr()) % 256
        c.parties_hote = self.parties_hote.ctypes.data
        c.tailles_parties = self.tailles.ctypes.data
        c.luts = luts.data_ptr()
        c.routeurs = 0 if routeurs is None else routeurs.data_ptr()
        c.biais_routeurs = 0 if biais is None else biais.data_ptr()
        c.flux = self.flux.cuda_stream
        n = int(lib.trc_flux_espace_octets(C.byref(c)))
        self.espace = torch.empty(n + 256, dtype=torch.uint8, device="cuda")
        c.espace = self.espace.data_ptr() + (-self.espace.data_ptr()) % 256
        self.config = c
        p = lib.trc_flux_nouveau(C.byref(c))
        if not p:
            verifier(1)
        self._p = C.c_void_p(p)
        self.k = k
        self._stats = FluxStats()

    def __del__(self):
        p = getattr(self, "_p", None)
        if p:
            lib.trc_flux_detruire(p)
            self._p = None

    def couche(self, couche: int, x, residu, experts=None, poids=None) -> FluxStats:
        """Layer `couche` on x [jetons][d] (CUDA bf16 or f32) and residu (CUDA f32, in place);
        experts / poids (numpy [jetons][k]) impose the routing, else the layer's router runs."""
        import torch

        jetons = x.shape[0] if x.dim() == 2 else 1
        ie = pe = None
        if experts is not None:
            ie = np.ascontiguousarray(experts, np.uint32)
            pe = np.ascontiguousarray(poids, np.float32)
        verifier(lib.trc_flux_couche(self._p, couche, x.data_ptr(), int(x.dtype == torch.bfloat16), residu.data_ptr(),
                                     jetons, None if ie is None else ie.ctypes.data,
                                     None if pe is None else pe.ctypes.data, C.byref(self._stats)))
        s = FluxStats()
        C.memmove(C.byref(s), C.byref(self._stats), C.sizeof(FluxStats))
        return s

    def compteurs(self) -> Compteurs:
        c = _Compteurs()
        verifier(lib.trc_flux_compteurs(self._p, C.byref(c)))
        return _compteurs(c)

    def controle(self) -> np.ndarray:
        n = 4 * self.k * self.config.jetons_max
        out = np.zeros(n, np.uint32)
        verifier(lib.trc_flux_controle(self._p, out.ctypes.data, n))
        return out
