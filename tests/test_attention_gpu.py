"""GPU: the attention side of a layer (Q8_0 GEMV, RMSNorm, YaRN, KV write, attention with sinks
and the sliding window) through the C-ABI.

- against the reference's own kernels on the same GPU (oracle/_ref, passe.cuh compiled for
  sm_100a): bit for bit for the Q8_0 GEMV, RMSNorm, rotation and KV write (the same arithmetic
  order and the same CUDA math); within 1e-5 of max|out| for the attention, which is split over
  positions and merged in a cluster (another order of the same f32 sums);
- against the CPU restatement (oracle/attention_cpu.c): bit for bit for the Q8_0 GEMV, RMSNorm
  and the KV write; the YaRN rotation and the attention call the host's libm (pow, log, sin,
  cos, expf), so within 2e-7 relative for the rotation and 1e-5 of max|out| for attention (the
  reference's own attention threshold, ARCHITECTURE.md 6.5);
- shapes of gpt-oss-120b: q 4096 x 2880, k / v 512 x 2880, o 2880 x 4096 (Q8_0), 64 query heads
  over 8 kv heads of 64; a sliding layer (ring of 128 cases, positions past the ring) and a full
  layer (up to 3,000 positions)."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def q8_0(rng, R, C):
    """A seeded Q8_0 matrix (ggml layout): per block of 32, d = f16(max|w| / 127), q = round(w / d)."""
    w = (rng.standard_normal((R, C // 32, 32)) * 0.02).astype(np.float32)
    d = (np.abs(w).max(axis=2) / 127.0).astype(np.float16)
    dq = np.where(d == 0, 1, d).astype(np.float32)
    q = np.clip(np.rint(w / dq[:, :, None]), -127, 127).astype(np.int8)
    blocs = np.zeros((R, C // 32, 34), np.uint8)
    blocs[:, :, 0:2] = d.view(np.uint8).reshape(R, C // 32, 2)
    blocs[:, :, 2:] = q.view(np.uint8)
    return blocs.reshape(-1)


@pytest.mark.parametrize("R,C", [(4096, 2880), (512, 2880), (2880, 4096), (37, 96), (1, 32)])
def test_gemv_q8_0(noyaux, R, C):
    rng = np.random.default_rng(R + C)
    W = q8_0(rng, R, C)
    x = rng.standard_normal(C).astype(np.float32)
    b = (rng.standard_normal(R) * 0.01).astype(np.float32)
    y = torch.zeros(R, dtype=torch.float32, device="cuda")
    Wd, xd, bd = t(W), t(x), t(b)
    noyaux.gemv_q8_0(Wd, xd, bd, y, R, C)
    torch.cuda.synchronize()
    nous = y.cpu().numpy()
    assert (nous.view(np.uint32) == O.gemv_q8_0(W, x, b, R, C).view(np.uint32)).all()
    ref = O.ref()
    if ref is not None:
        yr = torch.zeros(R, dtype=torch.float32, device="cuda")
        assert ref.ref_gemv_q8_0(Wd.data_ptr(), xd.data_ptr(), bd.data_ptr(), yr.data_ptr(), R, C,
                                 torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert (yr.cpu().numpy().view(np.uint32) == nous.view(np.uint32)).all()


def test_gemv_q8_0_sans_biais_et_refus(noyaux):
    import troncons_b200 as T

    rng = np.random.default_rng(1)
    W = q8_0(rng, 64, 256)
    x = rng.standard_normal(256).astype(np.float32)
    y = torch.zeros(64, dtype=torch.float32, device="cuda")
    noyaux.gemv_q8_0(t(W), t(x), None, y, 64, 256)
    torch.cuda.synchronize()
    assert (y.cpu().numpy().view(np.uint32) == O.gemv_q8_0(W, x, None, 64, 256).view(np.uint32)).all()
    Wd = t(np.concatenate([np.zeros(2, np.uint8), W]))
    with pytest.raises(T.ErreurUsage):  # a matrix not 16-aligned
        noyaux.gemv_q8_0(T.VueCarte(Wd.data_ptr() + 2, W.size), t(x), None, y, 64, 256)


@pytest.mark.parametrize("n,lignes", [(2880, 1), (2880, 3), (100, 2)])
def test_rmsnorm(noyaux, n, lignes):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n * lignes).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    y = torch.zeros(n * lignes, dtype=torch.float32, device="cuda")
    xd, wd = t(x), t(w)
    noyaux.rmsnorm(xd, wd, y, n, lignes, 1e-5)
    torch.cuda.synchronize()
    nous = y.cpu().numpy()
    assert (nous.view(np.uint32) == O.rmsnorm(x, w, n, lignes, 1e-5).view(np.uint32)).all()
    ref = O.ref()
    if ref is not None:
        yr = torch.zeros_like(y)
        assert ref.ref_rmsnorm(xd.data_ptr(), wd.data_ptr(), yr.data_ptr(), n, lignes, 1e-5,
                               torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert (yr.cpu().numpy().view(np.uint32) == nous.view(np.uint32)).all()
    # in place
    noyaux.rmsnorm(xd, wd, xd, n, lignes, 1e-5)
    torch.cuda.synchronize()
    assert (xd.cpu().numpy().view(np.uint32) == nous.view(np.uint32)).all()


@pytest.mark.parametrize("position", [0, 1, 127, 4095, 131071])
@pytest.mark.parametrize("variante", [0, 1])
def test_rope_yarn(noyaux, position, variante):
    import troncons_b200 as T

    rng = np.random.default_rng(position + 7 * variante)
    p = T.ParamsRope.gpt_oss()
    p.variante = variante
    q = rng.standard_normal(64 * 64).astype(np.float32)
    k = rng.standard_normal(8 * 64).astype(np.float32)
    qd, kd = t(q), t(k)
    noyaux.rope_yarn(qd, kd, 64, 8, position, p)
    torch.cuda.synchronize()
    qo, ko = O.rope_yarn(q, k, 64, 8, position, p)
    for a, b in ((qd.cpu().numpy(), qo), (kd.cpu().numpy(), ko)):
        assert np.abs(a - b).max() <= 2e-7 * max(1.0, np.abs(b).max())
    ref = O.ref()
    if ref is not None:
        import ctypes as C

        qr, kr = t(q), t(k)
        assert ref.ref_rope_yarn(qr.data_ptr(), kr.data_ptr(), 64, 8, position, C.addressof(p),
                                 torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(qr.view(torch.int32), qd.view(torch.int32))
        assert torch.equal(kr.view(torch.int32), kd.view(torch.int32))


def _cache(rng, cases, dkv):
    k = rng.standard_normal((cases, dkv)).astype(np.float32)
    v = rng.standard_normal((cases, dkv)).astype(np.float32)
    return O.f16(k).reshape(cases, dkv), O.f16(v).reshape(cases, dkv)


def test_ecrire_kv(noyaux):
    rng = np.random.default_rng(3)
    dkv, cases = 512, 130
    k = (rng.standard_normal(dkv) * 100).astype(np.float32)
    v = (rng.standard_normal(dkv) * 1e-5).astype(np.float32)  # subnormal f16 values included
    ck = torch.zeros(cases * dkv, dtype=torch.int16, device="cuda")
    cv = torch.zeros_like(ck)
    noyaux.ecrire_kv(t(k), t(v), ck, cv, dkv, 129)
    torch.cuda.synchronize()
    hk = np.zeros(cases * dkv, np.uint16)
    hv = np.zeros_like(hk)
    O.ecrire_kv(k, v, hk, hv, dkv, 129)
    assert (ck.cpu().numpy().view(np.uint16) == hk).all() and (cv.cpu().numpy().view(np.uint16) == hv).all()
    assert (hk[129 * dkv:] == np.float16(k).view(np.uint16)).all()


@pytest.mark.parametrize("position,fenetre,tetes,tetes_kv", [
    (0, 128, 64, 8), (200, 128, 64, 8), (1000, 128, 64, 8), (5, 0, 64, 8), (2999, 0, 64, 8),
    (31, 0, 64, 8), (32, 0, 64, 8), (511, 0, 64, 8), (4095, 0, 64, 8), (8191, 0, 64, 8),
    (700, 0, 8, 8), (700, 0, 64, 1), (130, 128, 16, 4)])
def test_attention(noyaux, position, fenetre, tetes, tetes_kv):
    """Split over positions in slices (1 to 16 per key/value head, each staged 128 positions at a
    time with the online rescale) and merged in a cluster: within 1e-5 of max|out| of the oracle
    (the reference's single-pass order restated) and of the reference's own kernel, for 1 to
    8,192 positions, the ring of a sliding layer, and 1, 4, 8 and 64 query heads per key/value
    head."""
    import ctypes as C

    import troncons_b200 as T

    rng = np.random.default_rng(position + fenetre + tetes)
    p = T.ParamsAttention.gpt_oss(position, fenetre)
    p.tetes, p.tetes_kv = tetes, tetes_kv
    dkv = 64 * tetes_kv
    cases = fenetre if fenetre else position + 1
    ck, cv = _cache(rng, cases, dkv)
    q = rng.standard_normal(tetes * 64).astype(np.float32)
    puits = rng.standard_normal(tetes).astype(np.float32)
    sortie = torch.zeros(tetes * 64, dtype=torch.float32, device="cuda")
    qd, ckd, cvd, pd = t(q), t(ck.view(np.int16)), t(cv.view(np.int16)), t(puits)
    noyaux.attention(qd, ckd, cvd, pd, sortie, p)
    torch.cuda.synchronize()
    nous = sortie.cpu().numpy()
    att = O.attention(q, ck.reshape(-1), cv.reshape(-1), puits, p)
    assert np.abs(nous - att).max() <= 1e-5 * max(1.0, np.abs(att).max())
    ref = O.ref()
    if ref is not None and tetes == 64 and tetes_kv == 8:
        sr = torch.zeros_like(sortie)
        assert ref.ref_attention(qd.data_ptr(), ckd.data_ptr(), cvd.data_ptr(), pd.data_ptr(), sr.data_ptr(),
                                 C.addressof(p), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        r = sr.cpu().numpy()
        assert np.abs(nous - r).max() <= 1e-5 * max(1.0, np.abs(r).max())
