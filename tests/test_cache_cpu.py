"""CPU: the expert cache (troncons_b200/csrc/cache.cpp through troncons_b200.cache) on the
reference's own cache tests (moteur/crates/trc-cache/src/tests.rs), its golden counts, and the
oracle's restatement.

- golden: the reference's engine counters and its simulator's replays on two routing traces of
  its engine (gpt-oss-120b and -20b, 708 tokens; tests/golden/traces_boucle.*), and, when the
  reference is mounted, on its two 5,120-token traces with the broken-policy witness too;
- tests.rs, each with its known answer: frozen routing (exact hit counts), pinning keeps a
  layer's k experts together (hits = |S_t & S_t-1|), a slot in flight is never evicted, a
  present unpinned slot is, two tiers equal two stack caches, Belady never below LRU, the broken
  policy gives another count, LRU order and victim, the trace format and its refusals, bytes
  counted per tier, Belady's hand-computed case, the global LRU cliff;
- the C++ cache against oracle/cache_ref.py (a step-by-step restatement) on random sticky
  traces, both policies, with and without the host tier."""
import json
import os

import numpy as np
import pytest

from troncons_b200 import ErreurUsage
from troncons_b200.cache import Cache, ErreurTrace, Trace, lire_trace, rejouer

ICI = os.path.dirname(os.path.abspath(__file__))
REF_O3 = os.path.join(os.environ.get("TRONCONS_REF", "/root/reference"), "mesures/moteur/O/journaux/o3")
M64 = (1 << 64) - 1


class Alea:
    """splitmix64 (tests.rs:6-21)."""

    def __init__(self, graine):
        self.x = graine & M64

    def suivant(self):
        self.x = (self.x + 0x9E3779B97F4A7C15) & M64
        z = self.x
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
        return z ^ (z >> 31)

    def sous(self, n):
        return self.suivant() % n

    def reel(self):
        return (self.suivant() >> 11) / float(1 << 53)


def trace_collante(t, l, e, k, rho, graine) -> Trace:
    """tests.rs:25-53: each place keeps its expert with probability rho, else draws one not in the set."""
    a = Alea(graine)
    etat = []
    for _ in range(l):
        s = []
        while len(s) < k:
            x = a.sous(e)
            if x not in s:
                s.append(x)
        etat.append(s)
    choix = np.zeros((t, l, k), np.uint16)
    for j in range(t):
        for c, s in enumerate(etat):
            for i in range(k):
                if a.reel() >= rho:
                    while True:
                        x = a.sous(e)
                        if x not in s:
                            s[i] = x
                            break
            choix[j, c] = s
    return Trace.depuis_choix(choix, e)


def trace_figee(t, l, k) -> Trace:
    choix = np.array([[list(range(c, c + k)) for c in range(l)] for _ in range(t)], np.uint16)
    return Trace.depuis_choix(choix, 32)


# ---------------------------------------------------------------- golden counts


with open(os.path.join(ICI, "golden", "traces_boucle.json")) as f:
    GOLD = json.load(f)
NPZ = np.load(os.path.join(ICI, "golden", "traces_boucle.npz"))


@pytest.mark.parametrize("nom", ["t120-boucle", "t20-boucle"])
def test_comptes_du_moteur_et_du_simulateur_de_reference(nom):
    tr = Trace.depuis_choix(NPZ[nom.replace("-", "_")], GOLD[nom]["experts"])
    for r in GOLD[nom]["resultats"]:
        c = rejouer(tr, r["emplacements"], r["tiedes"], "lru", r.get("casser", False))
        obtenu = {k: getattr(c, k) for k in ("succes_vram", "succes_ram", "defauts_disque", "evictions")}
        assert obtenu == {k: r[k] for k in obtenu}, r["source"]
        assert c.acces() == r["acces"]


@pytest.mark.parametrize("nom", ["o3-120b-2026-10-15-s1", "o3-2026-10-15-s1"])
def test_rejouer_de_reference_sur_ses_traces_longues(nom):
    chemin = os.path.join(REF_O3, nom + "-code.trace")
    if not os.path.exists(chemin):
        pytest.skip("the reference's 5,120-token traces are read where the reference is mounted")
    tr = lire_trace(chemin)
    with open(os.path.join(REF_O3, nom + "-rejouer.json")) as f:
        d = json.load(f)
    assert (tr.jetons, tr.couches, tr.experts, tr.k) == (d["temoin"]["T"], d["temoin"]["L"], d["temoin"]["E"],
                                                         d["temoin"]["k"])
    for cle in ("temoin", "casse"):
        for r in d[cle]["resultats"]:
            c = rejouer(tr, r["emplacements"], r["tiedes"], d[cle]["politique"], d[cle]["casser"])
            assert (c.acces(), c.succes_vram, c.succes_ram, c.defauts_disque, c.evictions) == (
                r["acces"], r["succes_vram"], r["succes_ram"], r["defauts_disque"], r["evictions"]), cle


# ---------------------------------------------------------------- tests.rs


def test_routage_fige_reponses_exactes():
    t, l, k = 4000, 4, 4
    tr = trace_figee(t, l, k)
    lk = l * k
    c0 = rejouer(tr, lk - k)
    assert c0.succes_vram == 0
    c1 = rejouer(tr, lk - 1)
    assert c1.succes_vram == (k - 1) * l * (t - 1)
    c2 = rejouer(tr, lk)
    assert c2.succes_vram == lk * (t - 1)
    assert c2.evictions == 0
    for c in (c0, c1, c2):
        assert c.acces() == tr.acces()


def test_epinglage_tient_les_k_experts_ensemble():
    tr = trace_collante(2000, 1, 12, 4, 0.5, 7)
    cache = Cache(4, 0)
    precedent = []
    for t in range(tr.jetons):
        for c in range(tr.couches):
            g = [int(x) for x in tr.groupe(t, c)]
            d = cache.demander(c, g, 0)
            assert sum(x.sorte == "succes" for x in d) == sum(e in precedent for e in g), f"token {t}"
            precedent = g
            for i, e in enumerate(g):
                s = cache.emplacement_de((c, e))
                assert s is not None, "a pinned expert was evicted"
                assert s == d[i].emplacement and cache.occupant(s) == (c, e)
            for x in d:
                if x.sorte == "defaut_disque":
                    assert x.tiede is None
                    cache.pret(x.emplacement)
            cache.liberer(c)


def test_en_vol_jamais_evince():
    cache = Cache(1, 0)
    cache.demander(0, [3], 0)
    cache.liberer(0)  # unpinned, but not ready
    with pytest.raises(ErreurUsage, match="no free or evictable device slot"):
        cache.demander(1, [5], 1)


def test_present_desepingle_est_evincable():
    cache = Cache(1, 0)
    d = cache.demander(0, [3], 0)
    assert [(x.sorte, x.emplacement, x.tiede) for x in d] == [("defaut_disque", 0, None)]
    cache.pret(0)
    cache.liberer(0)
    d = cache.demander(1, [5], 1)
    assert [(x.sorte, x.emplacement, x.tiede) for x in d] == [("defaut_disque", 0, None)]
    assert cache.compteurs().evictions == 1
    assert cache.etat(0) == ("en_vol", 1)


def test_pret_sur_un_emplacement_qui_n_est_pas_en_vol():
    cache = Cache(2, 0)
    with pytest.raises(ErreurUsage):
        cache.pret(0)


def test_deux_etages_egalent_deux_caches_a_pile():
    for graine in range(4):
        tr = trace_collante(800, 5, 32, 4, 0.55, 100 + graine)
        for v, r in [(8, 8), (8, 20), (16, 40), (30, 90), (12, 160)]:
            for pol in ("lru", "belady"):
                deux = rejouer(tr, v, r, pol)
                seul_v = rejouer(tr, v, 0, pol)
                seul_r = rejouer(tr, r, 0, pol)
                assert deux.succes_vram == seul_v.succes_vram, (pol, v, r)
                assert deux.succes_vram + deux.succes_ram == seul_r.succes_vram, (pol, v, r)
                assert deux.acces() == tr.acces()


def test_belady_jamais_sous_lru():
    for graine in range(6):
        tr = trace_collante(600, 4, 64, 4, 0.3 + 0.1 * graine, graine)
        for n in (4, 8, 16, 33, 64, 128):
            assert rejouer(tr, n, 0, "belady").succes_vram >= rejouer(tr, n).succes_vram, (graine, n)


def test_politique_faussee_donne_un_autre_compte():
    tr = trace_collante(1000, 4, 64, 4, 0.6, 3)
    assert rejouer(tr, 32).succes_vram != rejouer(tr, 32, casser=True).succes_vram


def test_lru_ordre_et_victime():
    """tests.rs:172-186 through the cache: 4 slots holding (0,0..3) in that order, (0,1) hit;
    then each new expert evicts the oldest unpinned: (0,0), then (0,2), then (0,3), then (0,1)."""
    cache = Cache(4, 0)
    for e in range(4):
        for d in cache.demander(0, [e], e):
            cache.pret(d.emplacement)
        cache.liberer(0)
    assert cache.demander(0, [1], 4)[0].sorte == "succes"
    cache.liberer(0)
    attendues = [(0, 0), (0, 2), (0, 3), (0, 1)]
    for i, e in enumerate((10, 11, 12, 13)):
        avant = {cache.occupant(s) for s in range(4)}
        d = cache.demander(1, [e], 5 + i)[0]
        cache.pret(d.emplacement)
        cache.liberer(1)
        apres = {cache.occupant(s) for s in range(4)}
        assert avant - apres == {attendues[i]}


def test_trace_lue_comme_l_outil_python():
    tr = Trace.depuis_texte("# source\nE=32\n3 17 | 5 9\n\n3 31 | 5 2\n")
    assert (tr.experts, tr.couches, tr.k, tr.jetons) == (32, 2, 2, 2)
    assert list(tr.groupe(1, 0)) == [3, 31] and list(tr.groupe(1, 1)) == [5, 2]
    assert tr.commentaires == ["source"]
    assert Trace.depuis_texte("3 17 | 5 9").experts == 18


def test_trace_mal_formee_refusee():
    for texte, sorte, numero in [("1 2 | 3 4\n1 2\n", "ligne", 2), ("1 2 | 3 4\n1 2 | 3\n", "ligne", 2),
                                 ("# rien\n", "vide", 0), ("1 x\n", "ligne", 1)]:
        with pytest.raises(ErreurTrace) as e:
            Trace.depuis_texte(texte)
        assert e.value.sorte == sorte and e.value.numero == numero, texte
    with pytest.raises(ErreurTrace) as e:
        Trace.depuis_texte("E=4\n1 7\n")
    assert (e.value.sorte, e.value.expert, e.value.experts) == ("hors_bornes", 7, 4)


def test_octets_comptes_par_etage():
    cache = Cache(1, 2)
    cache.fixer_tailles(np.array([[1000 + e for e in range(8)]], np.uint64))
    for c, e in [(0, 1), (0, 2), (0, 1)]:
        for d in cache.demander(c, [e], 0):
            if d.sorte != "succes":
                cache.pret(d.emplacement)
        cache.liberer(c)
    k = cache.compteurs()
    assert (k.succes_vram, k.succes_ram, k.defauts_disque) == (0, 1, 2)
    assert k.octets_disque == 1001 + 1002
    assert k.octets_copies == 1001 + 1002 + 1001
    assert k.evictions == 2


def test_belady_cas_calcule_a_la_main():
    tr = Trace.depuis_texte("E=3\n0\n1\n2\n0\n")
    assert rejouer(tr, 2, 0, "belady").succes_vram == 1
    assert rejouer(tr, 2).succes_vram == 0


def test_falaise_du_lru_global():
    for graine in range(4):
        l, k = 6, 4
        tr = trace_collante(700, l, 16, k, 0.7, 40 + graine)
        seuil = (l - 1) * k
        for n in (k, 7, 13, seuil):
            assert rejouer(tr, n).succes_vram == 0, n
        assert rejouer(tr, seuil + 1).succes_vram > 0
        assert rejouer(tr, seuil, 0, "belady").succes_vram > 0


# ---------------------------------------------------------------- against the oracle


@pytest.mark.parametrize("graine", range(6))
def test_cache_contre_l_oracle(graine):
    import oracle.cache_ref as R

    tr = trace_collante(120, 3, 24, 4, 0.4 + 0.08 * graine, 900 + graine)
    for pol in ("lru", "belady"):
        for v, r in [(4, 0), (7, 0), (9, 5), (6, 30), (40, 12)]:
            for casser in (False, True):
                a = rejouer(tr, v, r, pol, casser)
                b = R.rejouer(tr.choix, v, r, pol, casser)
                assert {k: getattr(a, k) for k in b} == b, (pol, v, r, casser)
