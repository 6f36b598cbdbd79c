"""GPU: the MXFP4 GEMV on a slot (trc_gemv / trc_gemv_lot).

- integer-exact case of the reference (trc-noyaux/tests/carte.rs:330-407): scales in [117, 123]
  and x in {-2..2} make every partial sum exact in f32, so the GPU must equal the exact result
  bit for bit, whatever its order;
- bit for bit against the CPU replica of troncons_b200's own reduction order;
- within the reference's GEMV tolerance (1e-5 relative, ARCHITECTURE.md 5.6) of an f64 host
  evaluation, and of the reference's own gemv_mxfp4 when oracle/_ref is built;
- code 8 (-0) reads as code 0, bit for bit (carte.rs:481-554);
- a batch gives the bits of single launches."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def t(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def matrice_slot(codes, ech, biais, R, C):
    """An SoA matrix (codes, scales at al256, biases at al256)."""
    nb = R * (C // 32)
    eo = (nb * 16 + 255) & ~255
    bo = (eo + nb + 255) & ~255
    pas = (bo + 4 * R + 255) & ~255
    m = np.zeros(pas, np.uint8)
    m[:nb * 16] = codes
    m[eo:eo + nb] = ech
    m[bo:bo + 4 * R] = np.asarray(biais, np.float32).view(np.uint8)
    return m


def gemv(noyaux, m, x, R, C):
    y = torch.zeros(R, dtype=torch.float32, device="cuda")
    noyaux.gemv(t(m), t(np.asarray(x, np.float32)), y, R, C)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def synth(graine, R, C):
    import troncons_b200.synth as S

    bl, bi = S.matrices(graine, R, C, 1)
    nb = R * (C // 32)
    b = bl[0].reshape(nb, 17)
    return b[:, 1:].reshape(-1).copy(), b[:, 0].copy(), bi[0]


def test_gemv_exacte_sur_entiers(noyaux):
    rng = np.random.default_rng(11)
    for R, C in [(2880, 2880), (37, 96), (64, 8192)]:
        codes, _, _ = synth(3, R, C)
        ech = rng.integers(117, 124, R * (C // 32)).astype(np.uint8)
        biais = (rng.integers(-1000, 1001, R) / 2048.0).astype(np.float32)
        x = rng.integers(-2, 3, C).astype(np.float32)
        y = gemv(noyaux, matrice_slot(codes, ech, biais, R, C), x, R, C)
        exact = O.gemv_f64(codes, ech, biais, x, R, C)
        assert (y.view(np.uint32) == exact.astype(np.float32).view(np.uint32)).all(), (R, C)


def test_gemv_ordre_au_bit_et_tolerance(noyaux):
    rng = np.random.default_rng(5)
    for R, C in [(2880, 2880), (100, 9024), (8, 256)]:
        codes, ech, biais = synth(4, R, C)
        x = rng.standard_normal(C).astype(np.float32)
        y = gemv(noyaux, matrice_slot(codes, ech, biais, R, C), x, R, C)
        ordre = O.ordre_gemv(codes, ech, biais, x, R, C)
        assert (y.view(np.uint32) == ordre.view(np.uint32)).all(), (R, C)
        f64 = O.gemv_f64(codes, ech, biais, x, R, C)
        assert np.abs(y - f64).max() <= 1e-5 * np.abs(f64).max()


def test_code_8_lu_comme_0(noyaux):
    codes, ech, biais = synth(9, 2880, 2880)
    lo, hi = codes & 15, codes >> 4
    n8 = int((lo == 8).sum() + (hi == 8).sum())
    assert n8 > 100_000
    canon = (np.where(lo == 8, 0, lo) | (np.where(hi == 8, 0, hi) << 4)).astype(np.uint8)
    rng = np.random.default_rng(17)
    x = rng.standard_normal(2880).astype(np.float32)
    x[::97] = 0.0
    x[1::97] = -0.0
    y0 = gemv(noyaux, matrice_slot(codes, ech, biais, 2880, 2880), x, 2880, 2880)
    y1 = gemv(noyaux, matrice_slot(canon, ech, biais, 2880, 2880), x, 2880, 2880)
    assert (y0.view(np.uint32) == y1.view(np.uint32)).all()
    # the check bites: a code 0 facing a non-zero x changed to 1 changes row 0
    casse = canon.copy()
    i = next(i for i in range(16) if (casse[i] & 15) == 0 and x[i] != 0.0)
    casse[i] |= 1
    y2 = gemv(noyaux, matrice_slot(casse, ech, biais, 2880, 2880), x, 2880, 2880)
    assert y2[0] != y1[0]


def test_lot_egal_seul(noyaux):
    import troncons_b200 as T

    R, C = 2880, 2880
    mats, xs, ys = [], [], []
    rng = np.random.default_rng(3)
    for j in range(3):
        codes, ech, biais = synth(20 + j, R, C)
        mats.append(t(matrice_slot(codes, ech, biais, R, C)))
        xs.append(t(rng.standard_normal(C).astype(np.float32)))
    seul = []
    for j in range(3):
        y = torch.zeros(R, dtype=torch.float32, device="cuda")
        noyaux.gemv(mats[j], xs[j], y, R, C)
        seul.append(y)
        ys.append(torch.zeros(R, dtype=torch.float32, device="cuda"))
    descs = (T.DescGemv * 3)(*[T.DescGemv(mats[j].data_ptr(), xs[j].data_ptr(), ys[j].data_ptr(), R, C) for j in range(3)])
    dd = torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).cuda()
    noyaux.gemv_lot(dd, 3, R)
    torch.cuda.synchronize()
    for j in range(3):
        assert torch.equal(seul[j].view(torch.int32), ys[j].view(torch.int32))


def test_gemv_de_reference_dans_la_tolerance(noyaux):
    ref = O.ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    R, C = 2880, 2880
    codes, ech, biais = synth(31, R, C)
    x = np.random.default_rng(1).standard_normal(C).astype(np.float32)
    m = t(matrice_slot(codes, ech, biais, R, C))
    xv = t(x)
    yr = torch.zeros(R, dtype=torch.float32, device="cuda")
    assert ref.ref_gemv(m.data_ptr(), xv.data_ptr(), yr.data_ptr(), R, C, torch.cuda.current_stream().cuda_stream) == 0
    y = gemv(noyaux, matrice_slot(codes, ech, biais, R, C), x, R, C)
    yr = yr.cpu().numpy()
    assert np.abs(y - yr).max() <= 1e-5 * np.abs(yr).max()


def test_refus_des_tailles_fausses(noyaux):
    import troncons_b200 as T

    petit = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(T.ErreurUsage):
        noyaux.decoder_expert(petit, petit, petit, T.DimsExpert.gpt_oss(), petit)
    with pytest.raises(T.ErreurUsage):
        noyaux.gemv(petit, petit, petit, 2880, 2880)


@pytest.mark.parametrize("formes", [
    [(2880, 2880)] * 12,                      # decode-then-multiply's gate/up batch of six experts
    [(16, 64), (32, 8192), (48, 96), (100, 512), (2880, 2880)],  # B = 2 / 256 / odd / R % 16 / gpt-oss
    [(512, 256), (256, 512), (64, 7936)],
])
def test_lot_en_groupes_egal_l_ordre(noyaux, formes):
    """trc_gemv_lot (rows in groups of 16 per warp, codes and scales staged by bulk copies, the
    quads' chains in f32x2 FMAs; shapes the groups cannot take fall back to the row walk) against
    the CPU replica of the library's reduction order, bit for bit, in one launch of mixed shapes:
    B = 2 to 256 blocks per row, odd B, rows not a multiple of 16, one and two segments per row."""
    import troncons_b200 as T

    rng = np.random.default_rng(len(formes))
    mats, xs, ys, attendus = [], [], [], []
    for j, (R, C) in enumerate(formes):
        codes, ech, biais = synth(40 + j, R, C)
        x = rng.standard_normal(C).astype(np.float32)
        mats.append(t(matrice_slot(codes, ech, biais, R, C)))
        xs.append(t(x))
        ys.append(torch.full((R,), float("nan"), dtype=torch.float32, device="cuda"))
        attendus.append(O.ordre_gemv(codes, ech, biais, x, R, C))
    descs = (T.DescGemv * len(formes))(*[T.DescGemv(mats[j].data_ptr(), xs[j].data_ptr(), ys[j].data_ptr(), R, C)
                                         for j, (R, C) in enumerate(formes)])
    dd = torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).cuda()
    noyaux.gemv_lot(dd, len(formes), max(R for R, _ in formes))
    torch.cuda.synchronize()
    for j, (R, C) in enumerate(formes):
        y = ys[j].cpu().numpy()
        assert (y.view(np.uint32) == attendus[j].view(np.uint32)).all(), (R, C)
