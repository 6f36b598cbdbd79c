"""GPU: the MoE layer around the decoder.

- router logits bit for bit against the CPU replica of troncons_b200's order, top-k indices
  exact and weights within 1e-6 of the f64 softmax (ARCHITECTURE.md 5.6), the reference's
  tie-break known answer and mailbox protocol (trc-noyaux/tests/passe.rs:303-321);
- SwiGLU within 1e-6 of f64, combine bit for bit against the same sum on the host (no FMA);
- the exactness invariant: the fused compressed layer (both schedules: down decoded alongside
  gate/up, or after SwiGLU), the fused raw layer and the decode-then-multiply sequence give the
  same bits, step after step;
- the layer against the CPU port of the path within a stated tolerance."""
import ctypes as C

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def adresse_carte(hote: int) -> int:
    """Device address of page-locked host memory (cudaHostGetDevicePointer)."""
    try:
        from cuda.bindings import runtime as rt
    except ImportError:  # older cuda-python
        from cuda import cudart as rt
    err, d = rt.cudaHostGetDevicePointer(hote, 0)
    if int(err) != 0:
        pytest.skip(f"pinned memory not mapped for the device ({err})")
    return int(d)


def test_topk_egalites_et_boite(noyaux):
    l = np.array([1.0, 3.0, 3.0, 0.0, 2.0, -1.0], np.float32)
    iv = torch.zeros(4, dtype=torch.int32, device="cuda")
    pv = torch.zeros(4, dtype=torch.float32, device="cuda")
    boite = torch.zeros(64, dtype=torch.int32).pin_memory()
    adresse = adresse_carte(boite.data_ptr())
    noyaux.routeur_topk(t(l), 6, 4, iv, pv, adresse, 77)
    torch.cuda.synchronize()
    idx = iv.cpu().numpy()
    assert list(idx) == [1, 2, 4, 0]
    e = np.exp(np.array([3.0, 3.0, 2.0, 1.0]) - 3.0)
    att = (e / e.sum()).astype(np.float32)
    pw = pv.cpu().numpy()
    assert (pw == att).all()
    mots = boite.numpy()
    assert mots[0] == 77 and list(mots[1:5]) == [1, 2, 4, 0]
    assert (mots[5:9].view(np.float32) == pw).all()


def test_routeur_ordre_au_bit(noyaux):
    rng = np.random.default_rng(2)
    E, Cc = 128, 2880
    w = (rng.standard_normal((E, Cc)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(E) * 0.01).astype(np.float32)
    x = rng.standard_normal(Cc).astype(np.float32)
    lv = torch.zeros(E, dtype=torch.float32, device="cuda")
    noyaux.gemv_f32(t(w), t(x), t(b), lv, E, Cc)
    torch.cuda.synchronize()
    y = lv.cpu().numpy()
    assert (y.view(np.uint32) == O.ordre_gemv_f32(w, x, b, E, Cc).view(np.uint32)).all()
    iv = torch.zeros(4, dtype=torch.int32, device="cuda")
    pv = torch.zeros(4, dtype=torch.float32, device="cuda")
    noyaux.routeur_topk(lv, E, 4, iv, pv)
    torch.cuda.synchronize()
    i_ref, w_ref = O.routeur_topk(y, 4)
    assert (iv.cpu().numpy().astype(np.uint32) == i_ref).all()
    assert np.abs(pv.cpu().numpy() - w_ref).max() <= 1e-6


def test_swiglu_et_combiner(noyaux):
    g = np.array([100.0, 7.0, -3.0, 0.0, 1.5], np.float32)
    u = np.array([100.0, 7.0, -100.0, 5.0, -0.25], np.float32)
    yv = torch.zeros(5, dtype=torch.float32, device="cuda")
    noyaux.swiglu_oai(t(g), t(u), yv, 5)
    torch.cuda.synchronize()
    y = yv.cpu().numpy()
    assert y[0] == y[1]
    ref = O.swiglu(g, u)
    assert np.all(np.abs(y - ref) <= 1e-6 * np.maximum(np.abs(ref), 1e-30))
    rng = np.random.default_rng(3)
    d = 2880
    x = ((rng.random(d) - 0.5) * 1e3).astype(np.float32)
    s = ((rng.random(4 * d) - 0.5) * 7.0).astype(np.float32)
    w = np.array([0.4123, 0.3001, 0.2, 0.0876], np.float32)
    xv = t(x)
    noyaux.combiner(xv, t(s), d, t(w), 4, d)
    torch.cuda.synchronize()
    att = O.combiner(x, s, d, w, 4, d)
    assert (xv.cpu().numpy().view(np.uint32) == att.view(np.uint32)).all()


def _trois_chemins(cc, x, residu0):
    r_f = t(residu0)
    cc.controle.zero_()
    cc.couche(x, r_f, brute=False)
    ctl_f = cc.controle.clone()
    r_b = t(residu0)
    cc.controle.zero_()
    cc.couche(x, r_b, brute=True)
    ctl_b = cc.controle.clone()
    r_d = t(residu0)
    cc.decodee(x, r_d)
    torch.cuda.synchronize()
    assert (ctl_f == 0).all() and (ctl_b == 0).all() and (cc.ctl_d == 0).all()
    return r_f.cpu().numpy(), r_b.cpu().numpy(), r_d.cpu().numpy()


@pytest.mark.parametrize("recouvrement", [True, False])
@pytest.mark.parametrize("nom,k", [("couche_petite", 4), ("couche_impaire", 4), ("couche_gpt_oss", 4),
                                   ("couche_gpt_oss", 8)])
def test_compresse_brut_decode_au_bit(nom, k, recouvrement, request):
    """k = 8 on the gpt-oss shapes has more CODES_CTX tiles (8 x 2 x 127) than the producer /
    consumer form holds at once: the launch takes the one-warp-per-tile form. Both schedules:
    the down projection decoded alongside gate/up (its GEMV later, from the decoded words), and
    the sequential one (its decode fused into its GEMV after SwiGLU)."""
    from troncons_b200.carte import CoucheCarte

    c = request.getfixturevalue(nom)
    cc = CoucheCarte(c, k=k, recouvrement=recouvrement)
    cc.preparer_decodee()
    rng = np.random.default_rng(4)
    n_pas = 16 if nom == "couche_gpt_oss" else 32
    for pas in range(n_pas if k == 4 else 4):
        x = torch.from_numpy(rng.standard_normal(c.dims.colonnes[0]).astype(np.float32)).to(torch.bfloat16).cuda()
        residu0 = rng.standard_normal(c.dims.lignes[2]).astype(np.float32)
        f, b, d = _trois_chemins(cc, x, residu0)
        assert (f.view(np.uint32) == b.view(np.uint32)).all(), f"step {pas}: compressed != raw"
        assert (f.view(np.uint32) == d.view(np.uint32)).all(), f"step {pas}: fused != decode-then-GEMV"


def test_couche_contre_le_port_cpu(couche_gpt_oss):
    """The fused layer against the oracle's CPU port of the path (f32 GEMV in a different order,
    f64 SwiGLU and softmax): same experts, outputs within a stated tolerance."""
    from troncons_b200.carte import CoucheCarte

    c = couche_gpt_oss
    cc = CoucheCarte(c, k=4, brut=False)
    rng = np.random.default_rng(8)
    for _ in range(4):
        xf = rng.standard_normal(c.dims.colonnes[0]).astype(np.float32)
        x = torch.from_numpy(xf).to(torch.bfloat16).cuda()
        xb = x.float().cpu().numpy()
        residu0 = rng.standard_normal(c.dims.lignes[2]).astype(np.float32)
        r = t(residu0)
        cc.controle.zero_()
        cc.couche(x, r)
        torch.cuda.synchronize()
        res_cpu, idx, w = O.couche_moe_cpu(c.parties, c.luts, c.dims.lignes, c.dims.colonnes, c.wr, c.br, xb, 4, residu0)
        assert (cc.idx.cpu().numpy().astype(np.uint32) == idx).all()
        g = r.cpu().numpy()
        # Tolerance: f32 sums of 2,880 terms in two orders (a few ulps of the row magnitudes).
        assert np.abs(g - res_cpu).max() <= 1e-4 * max(1.0, np.abs(res_cpu).max())


@pytest.mark.parametrize("jetons,n_codes", [(1, 32), (3, 64), (8, 256)])
def test_ordonnancements_au_bit(couche_gpt_oss, jetons, n_codes):
    """The same layer through both schedules (the workspace's size picks one): the sequential
    (down decoded into its GEMV after SwiGLU) and the overlapped (down decoded alongside gate/up,
    its GEMV later on the decoded words) give the same residual bits, for 4 to 32 activations and
    tiles of 32, 64 and 256 macro-steps (parts re-encoded with that tile length)."""
    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.carte import CoucheCarte

    c = S.couche(20261201, T.DimsExpert.gpt_oss(), 8, brut=False, n_delta=n_codes, n_codes=n_codes) \
        if n_codes != 256 else couche_gpt_oss
    d = c.dims
    na = 4 * jetons
    seq = T.espace_octets(d, na)
    rec = T.espace_recouvrant_octets(d, na)
    assert rec > seq
    cs = CoucheCarte(c, k=4, brut=False, jetons=jetons, n_delta=n_codes, n_codes=n_codes, espace=seq)
    cr = CoucheCarte(c, k=4, brut=False, jetons=jetons, n_delta=n_codes, n_codes=n_codes, espace=rec)
    rng = np.random.default_rng(jetons + n_codes)
    for _ in range(3):
        x = torch.from_numpy(rng.standard_normal((jetons, d.colonnes[0])).astype(np.float32)).to(torch.bfloat16).cuda()
        r0 = torch.from_numpy(rng.standard_normal((jetons, d.lignes[2])).astype(np.float32)).cuda()
        a, b = r0.clone(), r0.clone()
        cs.couche(x, a)
        cr.couche(x, b)
        torch.cuda.synchronize()
        assert (cs.controle == 0).all() and (cr.controle == 0).all()
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))


@pytest.mark.parametrize("nom,k,jetons,recouvrement,tenus", [
    ("couche_petite", 4, 1, True, None), ("couche_gpt_oss", 4, 1, True, None), ("couche_gpt_oss", 4, 1, False, None),
    ("couche_gpt_oss", 8, 3, True, None), ("couche_gpt_oss", 4, 2, True, (2, 6))])
def test_deltas_predecodes_au_bit(nom, k, jetons, recouvrement, tenus, request):
    """Every expert's DELTA decoded once (trc_moe_predecoder_deltas): the bytes are the oracle's
    deltas (scale - median + 128 per block, trc-codec/src/lib.rs:348-373) and the layer that reads
    them instead of decoding DELTA gives the same residual bits as the one that decodes it, in
    both schedules, for token batches and an expert-parallel share (partial combine)."""
    import troncons_b200 as T
    from troncons_b200.carte import CoucheCarte

    c = request.getfixturevalue(nom)
    d = c.dims
    a = CoucheCarte(c, k=k, brut=False, jetons=jetons, recouvrement=recouvrement, tenus=tenus)
    p = CoucheCarte(c, k=k, brut=False, jetons=jetons, recouvrement=recouvrement, tenus=tenus, deltas_predecodes=True)
    torch.cuda.synchronize()
    assert (p.controle_deltas == 0).all()
    # The predecoded bytes: matrix j of expert e at ek[j] + e * nb_j, ek 256-aligned per matrix.
    dl = p.deltas.cpu().numpy()
    off = 0
    for j in range(3):
        nb = d.lignes[j] * (d.colonnes[j] // 32)
        for e in (0, c.experts - 1):
            _, delta, _ = O.preparer_matrice(c.blocs[j][e], d.lignes[j], d.colonnes[j] // 32, True)
            assert (dl[off + e * nb:off + (e + 1) * nb] == delta[:nb]).all(), f"matrix {j} expert {e}"
        off = (off + nb * c.experts + 255) // 256 * 256
    assert int(T.lib.trc_moe_deltas_octets(C.byref(d), c.experts)) == off
    rng = np.random.default_rng(9 + k + jetons)
    for _ in range(3):
        x = torch.from_numpy(rng.standard_normal((jetons, d.colonnes[0])).astype(np.float32)).to(torch.bfloat16).cuda()
        r0 = torch.from_numpy(rng.standard_normal((jetons, d.lignes[2])).astype(np.float32)).cuda()
        ra, rp = r0.clone(), r0.clone()
        a.controle.zero_()
        p.controle.zero_()
        a.couche(x, ra, partiel=tenus is not None)
        p.couche(x, rp, partiel=tenus is not None)
        torch.cuda.synchronize()
        assert (a.controle == 0).all() and (p.controle == 0).all()
        assert torch.equal(a.idx, p.idx)
        assert torch.equal(ra.view(torch.int32), rp.view(torch.int32))
