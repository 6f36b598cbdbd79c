"""GPU: the layer "par flux" (trc_moe_couche_par_flux, the reference's prefill by stream): each
distinct routed expert decoded once for the batch, then applied to every position routed to it.

Its residuals equal the fused layer's bit for bit (the token-by-token arithmetic: the
reference's proposition 5, layer-by-layer order = token-by-token order) on the same routing,
for batches of 1 to 128 positions, k = 4 and 8, the small and gpt-oss shapes; a routed expert
whose part is absent is counted as a format error of every activation routed to it."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _deux(cc, x, r0):
    rf, rp = r0.clone(), r0.clone()
    cc.controle.zero_()
    cc.couche(x, rf)
    ctl_f = cc.controle.clone()
    cc.controle.zero_()
    cc.couche_par_flux(x, rp, routeur=False)
    torch.cuda.synchronize()
    return rf, rp, ctl_f, cc.controle.clone()


@pytest.mark.parametrize("nom,k,jetons", [("couche_petite", 4, 1), ("couche_petite", 4, 7), ("couche_petite", 4, 128),
                                          ("couche_petite", 8, 33), ("couche_gpt_oss", 4, 16),
                                          ("couche_gpt_oss", 8, 5)])
def test_par_flux_egale_la_couche_fusionnee(nom, k, jetons, request):
    from troncons_b200.carte import CoucheCarte

    c = request.getfixturevalue(nom)
    cc = CoucheCarte(c, k=k, brut=False, jetons=jetons)
    rng = np.random.default_rng(17 + jetons + k)
    d = c.dims.colonnes[0]
    for pas in range(3):
        x = torch.from_numpy(rng.standard_normal((jetons, d)).astype(np.float32)).to(torch.bfloat16).cuda()
        r0 = torch.from_numpy(rng.standard_normal((jetons, c.dims.lignes[2])).astype(np.float32)).cuda()
        rf, rp, ctl_f, ctl_p = _deux(cc, x, r0)
        assert (ctl_f == 0).all() and (ctl_p == 0).all()
        assert torch.equal(rf.view(torch.int32), rp.view(torch.int32)), f"step {pas}"


def test_par_flux_expert_absent_compte(couche_petite):
    """Expert 3's part is absent: the activations routed to it are counted as format errors and
    left out of their positions' sums; the others are unaffected."""
    from troncons_b200.carte import CoucheCarte

    cc = CoucheCarte(couche_petite, k=4, brut=False, jetons=4)
    cc.adresses[3] = 0
    idx = np.array([[0, 1, 2, 4], [3, 5, 6, 7], [1, 3, 0, 2], [4, 5, 6, 7]], np.int32)
    cc.idx.copy_(torch.from_numpy(idx.reshape(-1)))
    cc.poids.copy_(torch.full((16,), 0.25))
    x = torch.ones(4, 512, dtype=torch.bfloat16, device="cuda")
    r = torch.zeros(4, couche_petite.dims.lignes[2], dtype=torch.float32, device="cuda")
    cc.controle.zero_()
    cc.couche_par_flux(x, r, routeur=False)
    torch.cuda.synchronize()
    ctl = cc.controle.cpu().numpy().reshape(16, 4)
    touche = (idx.reshape(-1) == 3)
    assert (ctl[touche, 1] >= 1).all() and (ctl[~touche, 1] == 0).all()
    assert torch.isfinite(r).all()


@pytest.mark.parametrize("jetons,tenus", [(16, (2, 6)), (40, (0, 3)), (9, (5, 8))])
def test_par_flux_sur_une_part_partielle(couche_petite, jetons, tenus):
    """An expert share with the partial combine (the expert-parallel layer's form): par flux
    writes the fused layer's bits, each position's share of the sum alone, with no counter set
    for the activations of experts held elsewhere."""
    from troncons_b200.carte import CoucheCarte

    cc = CoucheCarte(couche_petite, k=4, brut=False, jetons=jetons, tenus=tenus)
    rng = np.random.default_rng(jetons)
    d = couche_petite.dims.colonnes[0]
    for pas in range(2):
        x = torch.from_numpy(rng.standard_normal((jetons, d)).astype(np.float32)).to(torch.bfloat16).cuda()
        r0 = torch.from_numpy(rng.standard_normal((jetons, couche_petite.dims.lignes[2])).astype(np.float32)).cuda()
        rf, rp = r0.clone(), r0.clone()
        cc.controle.zero_()
        cc.couche(x, rf, partiel=True)
        ctl_f = cc.controle.clone()
        cc.controle.zero_()
        cc.couche_par_flux(x, rp, routeur=False, partiel=True)
        torch.cuda.synchronize()
        assert (ctl_f == 0).all() and (cc.controle == 0).all()
        assert torch.equal(rf.view(torch.int32), rp.view(torch.int32)), f"step {pas}"
        idx = cc.idx.cpu().numpy().reshape(jetons, 4)
        sans = ~((idx >= tenus[0]) & (idx < tenus[1])).any(1)
        assert (rp[torch.from_numpy(sans).cuda()] == 0).all()


@pytest.mark.parametrize("nom,k,jetons", [("couche_petite", 4, 12), ("couche_petite", 8, 5), ("couche_gpt_oss", 4, 6)])
def test_par_flux_contre_l_oracle(nom, k, jetons, request):
    """A batch of positions par flux against the oracle's CPU port of the layer, position by
    position (oracle/couche_cpu.c: router, the reference CPU decoder, the GEMVs, SwiGLU and the
    combine): the same routed experts, and every position's residual within 1e-4 of its max|r|
    (the port sums the GEMV in another f32 order). Independent of the fused CUDA layer."""
    import oracle as O
    from troncons_b200.carte import CoucheCarte

    c = request.getfixturevalue(nom)
    cc = CoucheCarte(c, k=k, brut=False, jetons=jetons)
    rng = np.random.default_rng(41 + jetons + k)
    d, R2 = c.dims.colonnes[0], c.dims.lignes[2]
    xf = rng.standard_normal((jetons, d)).astype(np.float32)
    x = torch.from_numpy(xf).to(torch.bfloat16)
    r0 = rng.standard_normal((jetons, R2)).astype(np.float32)
    r = torch.from_numpy(r0.copy()).cuda()
    cc.controle.zero_()
    cc.couche_par_flux(x.cuda(), r)
    torch.cuda.synchronize()
    assert (cc.controle == 0).all()
    rg = r.cpu().numpy()
    idx_gpu = cc.idx.cpu().numpy().reshape(jetons, k).astype(np.uint32)
    xb = x.float().numpy()
    for j in range(jetons):
        res, idx, _ = O.couche_moe_cpu(c.parties, c.luts, c.dims.lignes, c.dims.colonnes, c.wr, c.br, xb[j], k, r0[j])
        assert (idx_gpu[j] == idx).all(), f"position {j}: other experts routed"
        assert np.abs(rg[j] - res).max() <= 1e-4 * max(1.0, np.abs(res).max()), f"position {j}"


@pytest.mark.parametrize("jetons,seuil", [(32, 16), (64, 1), (48, 28)])
def test_par_flux_mma_dans_la_tolerance(couche_gpt_oss, jetons, seuil):
    """The layer par flux with the experts of at least `seuil` activations on the tensor cores
    (trc_moe_couche_par_flux_mma: x and h quantized to MXFP8, the GEMMs' rows gathered and
    scattered through the experts' activation lists), against the exact layer par flux on the
    same routing: within the quantization's tolerance. Two quantized inputs in a row (x for
    gate/up, then h for down) compound the single GEMM's ~3 % RMS: measured ~4 % RMS of the
    layer's added term, so the bounds are 10 % of its largest value at the worst element and 6 %
    in RMS. seuil 1: every expert on the tensor cores; 28: a mix of both paths."""
    from troncons_b200.carte import CoucheCarte

    c = couche_gpt_oss
    cc = CoucheCarte(c, k=4, brut=False, jetons=jetons)
    rng = np.random.default_rng(jetons + seuil)
    d = c.dims.colonnes[0]
    for pas in range(2):
        x = torch.from_numpy(rng.standard_normal((jetons, d)).astype(np.float32)).to(torch.bfloat16).cuda()
        r0 = torch.from_numpy(rng.standard_normal((jetons, c.dims.lignes[2])).astype(np.float32)).cuda()
        ra, rb = r0.clone(), r0.clone()
        cc.controle.zero_()
        cc.couche_par_flux(x, ra)
        cc.couche_par_flux(x, rb, routeur=False, mma_seuil=seuil)
        torch.cuda.synchronize()
        assert (cc.controle == 0).all() and int(cc.erreur_pf.item()) == 0
        da, db = (ra - r0).cpu().numpy(), (rb - r0).cpu().numpy()
        m = np.abs(da).max()
        assert m > 0
        assert np.abs(db - da).max() <= 1e-1 * m, (pas, np.abs(db - da).max() / m)
        assert np.sqrt(np.mean((db - da) ** 2)) <= 6e-2 * np.sqrt(np.mean(da ** 2))
        n_par_expert = np.bincount(cc.idx.cpu().numpy(), minlength=c.experts)
        if seuil == 28:
            assert (n_par_expert >= 28).any() and ((n_par_expert > 0) & (n_par_expert < 28)).any(), n_par_expert


@pytest.mark.parametrize("nom,jetons,seuil", [("couche_petite", 9, 0), ("couche_gpt_oss", 16, 0), ("couche_gpt_oss", 48, 16)])
def test_par_flux_brut_egal_compresse(nom, jetons, seuil, request):
    """The layer par flux on raw parts (each distinct expert's streams copied into its slot)
    gives the compressed parts' residual bits, on the exact path and on the tensor cores."""
    from troncons_b200.carte import CoucheCarte

    c = request.getfixturevalue(nom)
    cc = CoucheCarte(c, k=4, brut=True, jetons=jetons)
    rng = np.random.default_rng(jetons + 3)
    d = c.dims.colonnes[0]
    x = torch.from_numpy(rng.standard_normal((jetons, d)).astype(np.float32)).to(torch.bfloat16).cuda()
    r0 = torch.from_numpy(rng.standard_normal((jetons, c.dims.lignes[2])).astype(np.float32)).cuda()
    rc, rb = r0.clone(), r0.clone()
    cc.controle.zero_()
    cc.couche_par_flux(x, rc, mma_seuil=seuil)
    cc.couche_par_flux(x, rb, routeur=False, mma_seuil=seuil, brute=True)
    torch.cuda.synchronize()
    assert (cc.controle == 0).all()
    assert torch.equal(rc.view(torch.int32), rb.view(torch.int32))
