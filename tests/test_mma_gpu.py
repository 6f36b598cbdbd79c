"""GPU: the MXFP4 expert GEMM on the tensor cores (trc_gemm_mxfp4: tcgen05.mma
kind::mxf8f6f4.block_scale, the weights' own E2M1 codes and E8M0 block scales, the activations
quantized to MXFP8 on the GPU), for experts that receive 16 to 256 tokens at once.

Tolerances, stated:
- against an f64 GEMM of the same operands (the weights dequantized exactly, x quantized by the
  oracle's restatement of the OCP MX rule): within 1e-5 of max|y| (the products are exact, the
  tensor core sums them in f32);
- against the f64 GEMM of the unquantized x (the model's arithmetic): within 8e-2 of max|y| at
  the worst element and 5e-2 in RMS (E4M3 keeps 3 mantissa bits of each activation: half an ulp
  is 6.25 % of the element; measured 3.1 % of max|y| at the worst element of a 2,880-term sum,
  3 % in RMS)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _matrice(graine, R, Cc):
    import troncons_b200.synth as S

    bl, bi = S.matrices(graine, R, Cc, 1)
    b = bl[0].reshape(R * (Cc // 32), 17)
    return b[:, 1:].reshape(-1).copy(), b[:, 0].copy(), bi[0]


def _gemm(codes, ech, biais, x, R, Cc, bf16=False):
    import troncons_b200 as T

    n = x.shape[0]
    cd, ed, bd = (torch.from_numpy(a).cuda() for a in (codes, ech, biais))
    xt = torch.from_numpy(x).cuda()
    if bf16:
        xt = xt.to(torch.bfloat16)
    y = torch.full((n, R), float("nan"), dtype=torch.float32, device="cuda")
    octets = int(T.lib.trc_gemm_mxfp4_espace_octets(Cc, n))
    esp = torch.empty(octets + 256, dtype=torch.uint8, device="cuda")
    e0 = esp.data_ptr() + (-esp.data_ptr()) % 256
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    r = T.lib.trc_gemm_mxfp4(cd.data_ptr(), ed.data_ptr(), bd.data_ptr(), R, Cc, xt.data_ptr(), int(bf16), n,
                             y.data_ptr(), e0, octets, err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert r == T.TRC_OK, T.lib.trc_derniere_erreur()
    torch.cuda.synchronize()
    assert int(err.item()) == 0, "a bounded wait gave up"
    return y.cpu().numpy(), (xt.float().cpu().numpy() if bf16 else x)


@pytest.mark.parametrize("R,Cc,n", [(128, 128, 16), (256, 2880, 16), (2880, 2880, 64), (200, 96, 24),
                                    (2880, 2880, 256), (384, 512, 100)])
def test_gemm_contre_f64(R, Cc, n):
    codes, ech, biais = _matrice(R + Cc + n, R, Cc)
    rng = np.random.default_rng(n)
    x = rng.standard_normal((n, Cc)).astype(np.float32)
    x[:, :32] *= 1e-3  # a block of small activations: their own scale
    y, xs = _gemm(codes, ech, biais, x, R, Cc)
    xq, _ = O.mxfp8(xs)
    ref_q = O.gemm_mxfp4_f64(codes, ech, biais, xq, R, Cc)
    m = max(1.0, np.abs(ref_q).max())
    assert np.abs(y - ref_q).max() <= 1e-5 * m, np.abs(y - ref_q).max() / m
    ref = O.gemm_mxfp4_f64(codes, ech, biais, xs, R, Cc)
    assert np.abs(y - ref).max() <= 8e-2 * max(1.0, np.abs(ref).max())
    assert np.sqrt(np.mean((y - ref) ** 2)) <= 5e-2 * np.sqrt(np.mean(ref ** 2))


def test_tuiles_par_copies_egales_tma():
    """Codes 16 bytes off a 32-byte boundary: the weight tiles come by 8-byte copies instead of
    TMA (the 4-bit unpacking tensor map needs 32-aligned codes); the same bits either way."""
    import troncons_b200 as T

    R, Cc, n = 384, 2880, 48
    codes, ech, biais = _matrice(5, R, Cc)
    x = np.random.default_rng(6).standard_normal((n, Cc)).astype(np.float32)
    y_tma, _ = _gemm(codes, ech, biais, x, R, Cc)
    brut = torch.zeros(codes.size + 48, dtype=torch.uint8, device="cuda")
    debut = (-brut.data_ptr()) % 32 + 16  # 16 mod 32
    brut[debut:debut + codes.size] = torch.from_numpy(codes).cuda()
    ed, bd, xt = (torch.from_numpy(a).cuda() for a in (ech, biais, x))
    y = torch.full((n, R), float("nan"), dtype=torch.float32, device="cuda")
    octets = int(T.lib.trc_gemm_mxfp4_espace_octets(Cc, n))
    esp = torch.empty(octets + 256, dtype=torch.uint8, device="cuda")
    e0 = esp.data_ptr() + (-esp.data_ptr()) % 256
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert (brut.data_ptr() + debut) % 32 == 16
    assert T.lib.trc_gemm_mxfp4(brut.data_ptr() + debut, ed.data_ptr(), bd.data_ptr(), R, Cc, xt.data_ptr(), 0, n,
                                y.data_ptr(), e0, octets, err.data_ptr(),
                                torch.cuda.current_stream().cuda_stream) == T.TRC_OK, T.lib.trc_derniere_erreur()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(y.cpu().numpy().view(np.uint32), y_tma.view(np.uint32))


def test_gemm_bf16_et_refus():
    import troncons_b200 as T

    codes, ech, biais = _matrice(3, 256, 512)
    x = np.random.default_rng(1).standard_normal((32, 512)).astype(np.float32)
    y, xs = _gemm(codes, ech, biais, x, 256, 512, bf16=True)
    xq, _ = O.mxfp8(xs)
    ref_q = O.gemm_mxfp4_f64(codes, ech, biais, xq, 256, 512)
    assert np.abs(y - ref_q).max() <= 1e-5 * max(1.0, np.abs(ref_q).max())
    v = C.c_void_p(256)
    assert T.lib.trc_gemm_mxfp4(v, v, None, 256, 100, v, 0, 16, v, v, 1 << 20, v, None) == T.TRC_ERR_USAGE
    assert T.lib.trc_gemm_mxfp4(v, v, None, 256, 512, v, 0, 257, v, v, 1 << 20, v, None) == T.TRC_ERR_USAGE


def test_lot_egal_seul():
    """A batch of GEMMs of different shapes (trc_gemm_mxfp4_lot: one quantization launch, one MMA
    launch with the matrix as grid y) gives each matrix's single-call bits."""
    import troncons_b200 as T

    formes = [(2880, 2880, 16), (256, 512, 64), (384, 2880, 33)]
    rng = np.random.default_rng(77)
    garde, descs, attendus = [], [], []
    for j, (R, Cc, n) in enumerate(formes):
        codes, ech, biais = _matrice(90 + j, R, Cc)
        x = rng.standard_normal((n, Cc)).astype(np.float32)
        y1, _ = _gemm(codes, ech, biais, x, R, Cc)
        attendus.append(y1)
        t = [torch.from_numpy(a).cuda() for a in (codes, ech, biais, x)]
        y = torch.full((n, R), float("nan"), dtype=torch.float32, device="cuda")
        garde += t + [y]
        descs.append(T.DescGemm(t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), t[3].data_ptr(), y.data_ptr(),
                                R, Cc, n, 0))
    nb = len(formes)
    hote = (T.DescGemm * nb)(*descs)  # host descriptors: copied into the launches' parameters
    octets = int(T.lib.trc_gemm_mxfp4_lot_espace_octets(2880, 64, nb))
    esp = torch.empty(octets + 256, dtype=torch.uint8, device="cuda")
    e0 = esp.data_ptr() + (-esp.data_ptr()) % 256
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert T.lib.trc_gemm_mxfp4_lot(C.addressof(hote), nb, 2880, 2880, 64, e0, octets, err.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream) == T.TRC_OK, T.lib.trc_derniere_erreur()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for j in range(nb):
        y = garde[5 * j + 4].cpu().numpy()
        assert np.array_equal(y.view(np.uint32), attendus[j].view(np.uint32)), formes[j]
