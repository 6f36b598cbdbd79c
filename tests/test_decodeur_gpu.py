"""GPU: the sm_100a decoder (trc_decoder_expert / trc_decoder_lot / trc_copier_brut) against the
CPU oracle, byte for byte, with the reference's fault injections
(trc-noyaux/tests/carte.rs:247-328): a corrupted LUT slot, a flipped stream bit, a bad magic,
a batch mixing a corrupted expert. Where oracle/_ref is built, also against the reference's own
kernels compiled for sm_100a on the same bytes."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def carte(b) -> "torch.Tensor":
    a = np.frombuffer(bytes(b), np.uint8) if not isinstance(b, np.ndarray) else b.view(np.uint8).reshape(-1)
    return torch.from_numpy(a.copy()).cuda()


def decoder(noyaux, partie: bytes, luts: np.ndarray, dims, brut=False):
    import troncons_b200 as T

    te = T.taille_emplacement(dims)
    p = carte(partie)
    l = carte(luts)
    e = torch.zeros(te, dtype=torch.uint8, device="cuda")
    ctl = torch.zeros(4, dtype=torch.int32, device="cuda")
    if brut:
        noyaux.copier_brut(p, e, dims, ctl)
    else:
        noyaux.decoder_expert(p, e, l, dims, ctl)
    torch.cuda.synchronize()
    return e.cpu().numpy(), ctl.cpu().numpy().astype(np.uint32)


def test_decodage_exact_petite(noyaux, couche_petite):
    import troncons_b200.synth as S

    c = couche_petite
    for x in range(c.experts):
        slot, ctl = decoder(noyaux, c.parties[x], c.luts, c.dims)
        assert (ctl == 0).all(), ctl
        assert (slot == S.slot_attendu(c, x)).all()


def test_decodage_exact_gpt_oss(noyaux, couche_gpt_oss):
    import troncons_b200.synth as S

    c = couche_gpt_oss
    for x in range(c.experts):
        slot, ctl = decoder(noyaux, c.parties[x], c.luts, c.dims)
        assert (ctl == 0).all(), (x, ctl)
        att = S.slot_attendu(c, x)
        assert (slot == att).all(), f"expert {x}: {(slot != att).sum()} bytes differ"


def test_decodage_egal_oracle_sur_flux_casse(noyaux, couche_petite):
    """A flipped bit in CODES_CTX of matrix 1: the GPU's bytes and counters equal the CPU
    decoder's (words past a tile's end read 0 on both sides, rans.rs:427-436)."""
    c = couche_petite
    p = bytearray(c.parties[1])
    e = 64 + 16 * 7
    dec = int.from_bytes(p[e + 4:e + 8], "little")
    lon = int.from_bytes(p[e + 8:e + 12], "little")
    p[dec + lon // 2] ^= 0x10
    slot, ctl = decoder(noyaux, bytes(p), c.luts, c.dims)
    ref, ctl_ref = O.decoder_expert(bytes(p), c.luts, list(c.dims.lignes), list(c.dims.colonnes), slot.size)
    assert ctl[0] > 0, "a flipped stream bit must leave lanes off L"
    assert ctl[0] == ctl_ref[0] and ctl[2] == ctl_ref[2], (ctl, ctl_ref)
    assert (slot == ref).all()


def test_cassures(noyaux, couche_gpt_oss):
    import troncons_b200.synth as S

    c = couche_gpt_oss
    att = S.slot_attendu(c, 0)
    # 1. a CODES_CTX LUT slot (class 1, matrix 0) corrupted
    luts = c.luts.copy()
    luts[4096 + 4096 // 2] ^= 1
    slot, _ = decoder(noyaux, c.parties[0], luts, c.dims)
    assert (slot != att).any(), "the corrupted LUT changed nothing"
    # 2. a stream bit flipped in CODES_CTX of matrix 1 (stream 7)
    p = bytearray(c.parties[0])
    e = 64 + 16 * 7
    dec = int.from_bytes(p[e + 4:e + 8], "little")
    lon = int.from_bytes(p[e + 8:e + 12], "little")
    p[dec + lon // 2] ^= 0x10
    slot, ctl = decoder(noyaux, bytes(p), c.luts, c.dims)
    assert ctl[0] > 0 and (slot != att).any()
    # 3. no magic: a format error, nothing decoded
    p = bytearray(c.parties[0])
    p[0] ^= 0xFF
    _, ctl = decoder(noyaux, bytes(p), c.luts, c.dims)
    assert ctl[1] > 0


def test_lot_egal_seul(noyaux, couche_gpt_oss):
    import troncons_b200 as T
    import troncons_b200.synth as S

    c = couche_gpt_oss
    dims = c.dims
    te = T.taille_emplacement(dims)
    parties = [bytearray(c.parties[i]) for i in range(3)]
    e7 = 64 + 16 * 7
    dec = int.from_bytes(parties[1][e7 + 4:e7 + 8], "little")
    lon = int.from_bytes(parties[1][e7 + 8:e7 + 12], "little")
    parties[1][dec + lon // 2] ^= 0x10
    p = [carte(bytes(x)) for x in parties]
    l = carte(c.luts)
    empl = torch.zeros(3 * te, dtype=torch.uint8, device="cuda")
    ctl = torch.zeros(12, dtype=torch.int32, device="cuda")
    descs = (T.DescDecodage * 3)(*[T.DescDecodage(p[i].data_ptr(), empl.data_ptr() + i * te, l.data_ptr(),
                                                  ctl.data_ptr() + 16 * i) for i in range(3)])
    dd = torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).cuda()
    noyaux.decoder_lot(dd, 3, dims)
    torch.cuda.synchronize()
    tout = empl.cpu().numpy()
    c_lot = ctl.cpu().numpy().astype(np.uint32).reshape(3, 4)
    for i in (0, 2):
        assert (c_lot[i] == 0).all()
        assert (tout[i * te:(i + 1) * te] == S.slot_attendu(c, i)).all()
    assert c_lot[1][0] > 0
    seul, c1 = decoder(noyaux, bytes(parties[1]), c.luts, dims)
    assert (seul == tout[te:2 * te]).all() and (c1 == c_lot[1]).all()


def test_tuiles_de_taille_quelconque(noyaux):
    """DELTA with N = 32 and CODES_CTX with N = 64 (the format carries N per stream)."""
    import troncons_b200 as T
    import troncons_b200.synth as S

    dims = T.DimsExpert.de([320, 320, 640], [640, 640, 320])
    c = S.couche(11, dims, 2, n_delta=32, n_codes=64)
    for x in range(2):
        slot, ctl = decoder(noyaux, c.parties[x], c.luts, dims)
        assert (ctl == 0).all()
        assert (slot == S.slot_attendu(c, x)).all()


def test_copier_brut(noyaux, couche_gpt_oss):
    import troncons_b200.synth as S

    c = couche_gpt_oss
    slot, ctl = decoder(noyaux, c.parties_brutes[0], c.luts, c.dims, brut=True)
    assert ctl[1] == 0
    assert (slot == S.slot_attendu(c, 0, canonique=False)).all()
    p = bytearray(c.parties_brutes[0])
    p[0] ^= 0xFF
    _, ctl = decoder(noyaux, bytes(p), c.luts, c.dims, brut=True)
    assert ctl[1] > 0


def test_noyaux_de_reference_memes_octets(noyaux, couche_gpt_oss):
    """The reference's own decoder (noyaux.cu, compiled unchanged for sm_100a) on the same parts
    gives the same slot bytes and lane counters."""
    ref = O.ref()
    if ref is None:
        pytest.skip("oracle/_ref not built (the reference checkout was absent at build time)")
    import troncons_b200 as T

    c = couche_gpt_oss
    te = T.taille_emplacement(c.dims)
    dims6 = np.array(list(c.dims.lignes) + list(c.dims.colonnes), np.uint32)
    for x in range(3):
        p = carte(c.parties[x])
        l = carte(c.luts)
        e = torch.zeros(te, dtype=torch.uint8, device="cuda")
        ctl = torch.zeros(4, dtype=torch.int32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        assert ref.ref_decoder_expert(p.data_ptr(), e.data_ptr(), l.data_ptr(), O.p(dims6, O.P32), ctl.data_ptr(), s) == 0
        torch.cuda.synchronize()
        nous, c_nous = decoder(noyaux, c.parties[x], c.luts, c.dims)
        assert (e.cpu().numpy() == nous).all()
        assert (ctl.cpu().numpy() == 0).all() and (c_nous == 0).all()
