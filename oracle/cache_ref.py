"""Test infrastructure only (a checker, never on the product path): a plain-Python restatement of
the reference's expert cache, to check troncons_b200's C++ cache (troncons_b200/csrc/cache.cpp)
on any trace. It follows moteur/crates/trc-cache/src/lib.rs:105-301 (Cache, rejouer) and
politiques.rs:47-260 (Lru, Belady) step by step; pinned by the same golden counts as the C++
(the reference's own rejouer outputs on its committed routing traces)."""
from __future__ import annotations

from collections import OrderedDict


class Lru:
    """politiques.rs:47-160: an order from oldest to newest; a hit moves to the newest end."""

    def __init__(self):
        self.ordre = OrderedDict()

    def acceder(self, id_, t):
        self.ordre.move_to_end(id_)

    def inserer(self, id_, t):
        assert id_ not in self.ordre
        self.ordre[id_] = None

    def retirer(self, id_):
        del self.ordre[id_]

    def victime(self, epingle):
        for id_ in self.ordre:
            if not epingle(id_):
                return id_
        return None


class Belady:
    """politiques.rs:162-260: the present unprotected id used furthest in the future (never: +inf);
    ties to the smallest (layer, expert). Instants t = token * L + layer."""

    def __init__(self, trace):
        self.usages = {}
        T, L, k = trace.shape
        for t in range(T):
            for c in range(L):
                instant = t * L + c
                for e in trace[t, c]:
                    v = self.usages.setdefault((c, int(e)), [])
                    if not v or v[-1] != instant:
                        v.append(instant)
        self.prochain = {}

    def _apres(self, id_, t):
        import bisect
        v = self.usages.get(id_, [])
        i = bisect.bisect_right(v, t)
        return v[i] if i < len(v) else float("inf")

    def acceder(self, id_, t):
        self.prochain[id_] = self._apres(id_, t)

    def inserer(self, id_, t):
        assert id_ not in self.prochain
        self.prochain[id_] = self._apres(id_, t)

    def retirer(self, id_):
        del self.prochain[id_]

    def victime(self, epingle):
        meilleur = None
        for id_, p in self.prochain.items():
            if epingle(id_):
                continue
            if meilleur is None or p > meilleur[0] or (p == meilleur[0] and id_ < meilleur[1]):
                meilleur = (p, id_)
        return None if meilleur is None else meilleur[1]


class Cache:
    """lib.rs:105-257. Decisions: ("succes", slot, None), ("defaut_ram", slot, entry),
    ("defaut_disque", slot, entry or None)."""

    def __init__(self, emplacements, tiedes, vram, ram, casser=False):
        self.vram, self.ram, self.casser = vram, ram, casser
        self.etats = ["libre"] * emplacements
        self.occupant = [None] * emplacements
        self.ou_vram = {}
        self.libres_vram = list(range(emplacements))[::-1]
        self.occupant_tiede = [None] * tiedes
        self.ou_ram = {}
        self.libres_ram = list(range(tiedes))[::-1]
        self.epingles = []
        self.taille = None
        self.c = dict(succes_vram=0, succes_ram=0, defauts_disque=0, octets_disque=0, octets_copies=0, evictions=0,
                      evictions_ram=0)

    def _acceder(self, p, id_, t):
        if not self.casser:
            p.acceder(id_, t)

    def demander(self, couche, experts, t):
        for e in experts:
            if (couche, e) not in self.epingles:
                self.epingles.append((couche, e))
        sortie = []
        for e in experts:
            id_ = (couche, e)
            if id_ in self.ou_vram:
                self._acceder(self.vram, id_, t)
                if id_ in self.ou_ram:
                    self._acceder(self.ram, id_, t)
                self.c["succes_vram"] += 1
                sortie.append(("succes", self.ou_vram[id_], None))
                continue
            s = self._emplacement_pour_defaut()
            self.vram.inserer(id_, t)
            self.etats[s] = "en_vol"
            self.occupant[s] = id_
            self.ou_vram[id_] = s
            octets = self.taille(id_) if self.taille else 0
            self.c["octets_copies"] += octets
            if id_ in self.ou_ram:
                self._acceder(self.ram, id_, t)
                self.c["succes_ram"] += 1
                sortie.append(("defaut_ram", s, self.ou_ram[id_]))
            else:
                self.c["defauts_disque"] += 1
                self.c["octets_disque"] += octets
                sortie.append(("defaut_disque", s, self._entree_tiede_pour(id_, t)))
        return sortie

    def _emplacement_pour_defaut(self):
        if self.libres_vram:
            return self.libres_vram.pop()

        def epingle(id_):
            return id_ in self.epingles or (id_ in self.ou_vram and self.etats[self.ou_vram[id_]] == "en_vol")

        v = self.vram.victime(epingle)
        if v is None:
            raise RuntimeError("no free or evictable device slot")
        self.vram.retirer(v)
        s = self.ou_vram.pop(v)
        self.occupant[s] = None
        self.etats[s] = "libre"
        self.c["evictions"] += 1
        return s

    def _entree_tiede_pour(self, id_, t):
        if not self.occupant_tiede:
            return None
        if self.libres_ram:
            r = self.libres_ram.pop()
        else:
            v = self.ram.victime(lambda x: x in self.epingles)
            if v is None:
                return None
            self.ram.retirer(v)
            r = self.ou_ram.pop(v)
            self.occupant_tiede[r] = None
            self.c["evictions_ram"] += 1
        self.ram.inserer(id_, t)
        self.occupant_tiede[r] = id_
        self.ou_ram[id_] = r
        return r

    def pret(self, s):
        if self.etats[s] != "en_vol":
            raise RuntimeError(f"pret({s}) on a {self.etats[s]} slot")
        self.etats[s] = "present"

    def liberer(self, couche):
        self.epingles = [i for i in self.epingles if i[0] != couche]


def rejouer(trace, emplacements, tiedes=0, politique="lru", casser=False) -> dict:
    """lib.rs:272-301 on trace[T][L][k] (numpy or nested lists)."""
    import numpy as np

    tr = np.asarray(trace)
    mk = (lambda: Lru()) if politique == "lru" else (lambda: Belady(tr))
    c = Cache(emplacements, tiedes, mk(), mk(), casser)
    T, L, _ = tr.shape
    for t in range(T):
        for l in range(L):
            for sorte, s, _ in c.demander(l, [int(e) for e in tr[t, l]], t * L + l):
                if sorte != "succes":
                    c.pret(s)
            c.liberer(l)
    return c.c
