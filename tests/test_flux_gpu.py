"""GPU: the streaming executor (trc_flux_*): parts in pinned host memory, a pool of device slots
managed by the expert cache, copies on their own stream, the fused layer on the compute stream.

- its results are those of the layer with every part resident (bit for bit), with the router
  choosing the experts and with imposed routing, while slots are evicted and refilled;
- on a routing trace of the reference's engine (gpt-oss-20b, 708 tokens x 24 layers, 32
  experts, 362 slots: tests/golden/traces_boucle.*), its cache counts are the reference
  engine's own counters for that run (trc-ordo's "engine count = simulator count" witness),
  the bytes copied are its misses' part sizes, and no integrity counter is set."""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ICI = os.path.dirname(os.path.abspath(__file__))


def _couches(c, couches):
    """`couches` layers sharing one layer's parts, LUTs and router (each (layer, expert) is its own
    cache entry and its own copy)."""
    import troncons_b200.flux as F

    tampon, adr, tailles = F.tiers_hote(c.parties)
    adr = np.tile(adr, couches)
    tailles = np.tile(tailles, couches)
    luts = torch.from_numpy(np.tile(c.luts.view(np.int32), couches)).cuda()
    wr = torch.from_numpy(np.tile(c.wr.reshape(1, -1), (couches, 1))).cuda()
    br = torch.from_numpy(np.tile(c.br.reshape(1, -1), (couches, 1))).cuda()
    return tampon, adr, tailles, luts, wr, br


def test_flux_egale_la_couche_residente():
    import troncons_b200 as T
    import troncons_b200.flux as F
    import troncons_b200.synth as S
    from troncons_b200.carte import CoucheCarte

    dims = T.DimsExpert.de([256, 256, 512], [512, 512, 256])
    c = S.couche(11, dims, 8, brut=False)
    L = 3
    tampon, adr, tailles, luts, wr, br = _couches(c, L)
    fl = F.Flux(dims, L, 8, 4, 6, adr, tailles, luts, wr, br)  # 6 slots for 3 x 8 experts: evictions
    cc = CoucheCarte(c, k=4, brut=False)
    rng = np.random.default_rng(5)
    defauts = 0
    for pas in range(12):
        r0 = torch.from_numpy(rng.standard_normal(512).astype(np.float32)).cuda()
        rf, rr = r0.clone(), r0.clone()
        for l in range(L):
            x = torch.from_numpy(rng.standard_normal(512).astype(np.float32)).to(torch.bfloat16).cuda()
            if pas % 2 == 0:
                defauts += fl.couche(l, x.view(1, -1), rf).defauts
                cc.couche(x, rr)
            else:  # imposed routing
                e = rng.choice(8, 4, replace=False).astype(np.uint32)
                w = rng.random(4).astype(np.float32)
                defauts += fl.couche(l, x.view(1, -1), rf, e.reshape(1, 4), w.reshape(1, 4)).defauts
                cc.idx.copy_(torch.from_numpy(e.astype(np.int32)))
                cc.poids.copy_(torch.from_numpy(w))
                cc.couche(x, rr, routeur=False)
        torch.cuda.synchronize()
        assert torch.equal(rf.view(torch.int32), rr.view(torch.int32)), f"step {pas}"
    k = fl.compteurs()
    assert k.defauts_disque == defauts and k.evictions > 0
    assert (fl.controle() == 0).all() and (cc.controle.cpu().numpy() == 0).all()


def test_compte_du_moteur_de_reference_sur_sa_trace():
    import troncons_b200 as T
    import troncons_b200.flux as F
    import troncons_b200.synth as S

    with open(os.path.join(ICI, "golden", "traces_boucle.json")) as f:
        gold = json.load(f)["t20-boucle"]
    choix = np.load(os.path.join(ICI, "golden", "traces_boucle.npz"))["t20_boucle"]  # [708][24][4]
    moteur = gold["resultats"][0]
    T_, L, k = choix.shape
    dims = T.DimsExpert.de([256, 256, 256], [256, 256, 256])
    c = S.couche(13, dims, gold["experts"], brut=False)
    tampon, adr, tailles, luts, wr, br = _couches(c, L)
    fl = F.Flux(dims, L, gold["experts"], k, moteur["emplacements"], adr, tailles, luts)
    x = torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda")
    r = torch.zeros(1, 256, dtype=torch.float32, device="cuda")
    w = np.full((1, k), 0.25, np.float32)
    octets = 0
    for t in range(T_):
        for l in range(L):
            s = fl.couche(l, x, r, choix[t, l].reshape(1, k), w)
            octets += s.octets_copies
    torch.cuda.synchronize()
    cpt = fl.compteurs()
    assert (cpt.acces(), cpt.succes_vram, cpt.defauts_disque, cpt.evictions) == (
        moteur["acces"], moteur["succes_vram"], moteur["defauts_disque"], moteur["evictions"])
    # the bytes copied: the parts of the misses, as the cache counts them given the sizes
    from troncons_b200.cache import Cache

    ref = Cache(moteur["emplacements"], 0)
    ref.fixer_tailles(tailles.reshape(L, gold["experts"]))
    for t in range(T_):
        for l in range(L):
            for d in ref.demander(l, choix[t, l], t * L + l):
                if d.sorte != "succes":
                    ref.pret(d.emplacement)
            ref.liberer(l)
    assert octets == ref.compteurs().octets_copies
    assert (fl.controle() == 0).all()
