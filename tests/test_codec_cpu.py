"""CPU: the oracle's codec on the reference codec's own test cases (trc-codec/tests/rans.rs).

- round trip with a per-lane context (the scale class of each 16-byte block), at 8, 1,000 and
  16,200 blocks, tiles of 256 and 32 macro-steps (rans.rs:115-138);
- faults (rans.rs:184-249): a table with two frequencies swapped, a flipped word, a flipped
  state give a wrong output AND a record that says so; a surplus word leaves the output right
  and is seen only by the words-consumed check; a tampered or truncated header is refused;
- a v1.0 matrix rebuilt bit for bit from its part; a tampered median is seen (rans.rs:283-316);
- v1.2: signed zeros folded, the canonical expert rebuilt bit for bit, no nibble 8 left, and
  fewer CODES_CTX bytes than v1.0 by at least half a bit per folded -0 (rans.rs:318-363)."""
import numpy as np
import pytest

import oracle as O
import trc_aides as A


def _source_et_tables(rng, n_blocs):
    src = A.octets_geometriques(rng, 16 * n_blocs)
    kappa = rng.choice(np.array([0, 1, 1, 2], np.uint8), n_blocs)
    # Blocks of class 2 are pulled towards 0, as in MXFP4.
    src = np.where(np.repeat(kappa, 16) == 2, src & 0x33, src).astype(np.uint8)
    f = np.stack([O.table_depuis_comptes(np.bincount(src.reshape(-1, 16)[kappa == k].reshape(-1),
                                                     minlength=256).astype(np.uint64)) for k in range(3)])
    return src, kappa, f


def _bourrer(a):
    return np.concatenate([a, np.zeros((-a.size) % 128, np.uint8)])


@pytest.mark.parametrize("N", [256, 32])
@pytest.mark.parametrize("n_blocs", [8, 1000, 8 * 2025])
def test_aller_retour_par_voie(n_blocs, N):
    rng = np.random.default_rng(3 + n_blocs + N)
    src, kappa, f = _source_et_tables(rng, n_blocs)
    src_p = _bourrer(src)
    # Padding symbols (beyond the blocks) use table 0; make sure it holds symbol 0.
    if n_blocs * 16 != src_p.size and f[0][0] == 0:
        pytest.skip("padding symbol absent from table 0")
    flux = O.coder_g1(src_p, f, kappa, N)
    assert O.flux_valide(flux) == 0
    luts = np.stack([O.lut(x) for x in f])
    d, b = O.decoder(flux, luts, kappa)
    assert b.intact()
    assert (d[:src.size] == src).all()
    banc = O.banc()
    if banc is not None:
        assert banc.coder_g1(src_p, f, kappa, N) == flux


def test_cassures_tombent():
    rng = np.random.default_rng(5)
    n_blocs = 4000
    src, kappa, f = _source_et_tables(rng, n_blocs)
    luts = np.stack([O.lut(x) for x in f])
    flux = O.coder_g1(src, f, kappa)
    d, b = O.decoder(flux, luts, kappa)
    assert b.intact() and (d == src).all(), "the original must pass"

    # 1. Table of class 1 with its two most frequent symbols' frequencies swapped.
    f1 = f[1].copy()
    i, j = np.argsort(-f1.astype(np.int64), kind="stable")[:2]
    f1[i], f1[j] = f1[j], f1[i]
    luts_f = np.stack([luts[0], O.lut(f1), luts[2]])
    d, b = O.decoder(flux, luts_f, kappa)
    assert (d != src).any(), "swapped table: same output"
    assert b.voies_hors_l > 0, "swapped table: no lane off L"

    # 2. A flipped word, then a flipped state.
    fl = A.Flux.lire(flux)
    g = A.Flux.lire(flux)
    g.mots[g.mots.size // 2] ^= 0x0100
    d, b = O.decoder(g.ecrire(), luts, kappa)
    assert (d != src).any() and not b.intact()
    g = A.Flux.lire(flux)
    g.etats[5] ^= 1
    d, b = O.decoder(g.ecrire(), luts, kappa)
    assert (d != src).any() and b.voies_hors_l > 0
    # A surplus word at the end of the last tile: output and lanes stay right; only the
    # words-consumed check sees it.
    g = A.Flux.lire(flux)
    g.mots = np.append(g.mots, np.uint16(0xABCD))
    d, b = O.decoder(g.ecrire(), luts, kappa)
    assert (d == src).all() and b.voies_hors_l == 0 and b.tuiles_mots_faux == 1

    # 3. Tampered header fields are refused: P, reserved byte, T, geometry.
    s = fl.ecrire()
    assert s == flux
    for pos in (0, 7, 8, 6):
        q = bytearray(s)
        q[pos] ^= 0x41
        assert O.flux_valide(bytes(q)) != 0, f"tampered byte {pos} accepted"
    # Truncated stream: refused.
    assert O.flux_valide(s[:-64]) != 0


def _matrice(rng, R, B, experts, canonique, zeros_signes=False):
    blocs = [A.blocs_mxfp4(rng, R, B, zeros_signes) for _ in range(experts)]
    preps = [O.preparer_matrice(b, R, B, canonique) for b in blocs]
    return blocs, preps, A.tables_matrice(preps)


def _partie(prep, biais, f4, R, nb, expert):
    return O.assembler_partie(0, expert, 0, 1, A.flux_matrice(prep, biais, f4, 0, R, nb))[0]


def _origine(blocs, R, B):
    b = blocs.reshape(R * B, 17)
    return b[:, 1:].reshape(-1), b[:, 0]


@pytest.mark.parametrize("R,B", [(64, 2), (90, 3), (2880 // 8, 90)])
def test_matrice_v10_se_reconstruit(R, B):
    rng = np.random.default_rng(6 + R)
    nb = R * B
    blocs, preps, f4 = _matrice(rng, R, B, 3, canonique=False)
    luts4 = np.stack([O.lut(x) for x in f4])
    for x, prep in enumerate(preps):
        biais = bytes((i * 7 + x) & 255 for i in range(4 * R))
        partie = _partie(prep, biais, f4, R, nb, x)
        codes, ech, bi, bd, bc = O.decoder_matrice_v10(partie, 0, R, B, luts4)
        assert bd.intact() and bc.intact()
        q0, e0 = _origine(blocs[x], R, B)
        assert (codes == q0).all() and (ech == e0).all(), f"matrix ({R}, {B}) expert {x}"
        assert bi.tobytes() == biais
        # A tampered median gives wrong scales.
        _, dm, _, _ = O.trouver_flux(partie, A.SORTE_MEDIANES, 0)
        q = bytearray(partie)
        q[dm] ^= 1
        _, ech_q, _, _, _ = O.decoder_matrice_v10(bytes(q), 0, R, B, luts4)
        assert (ech_q != e0).any(), "tampered median not seen"


def _porte_un_8(o):
    o = np.asarray(o)
    return ((o & 15) == 8) | ((o >> 4) == 8)


def _canonique(q):
    lo, hi = q & 15, q >> 4
    return (np.where(lo == 8, 0, lo) | (np.where(hi == 8, 0, hi) << 4)).astype(np.uint8)


def test_matrice_canonique_se_reconstruit_et_gagne():
    R, B = 2880 // 8, 90
    nb = R * B
    rng = np.random.default_rng(20261017)
    blocs = [A.blocs_mxfp4(rng, R, B, zeros_signes=True) for _ in range(3)]
    n8 = sum(int(((_origine(b, R, B)[0] & 15) == 8).sum() + ((_origine(b, R, B)[0] >> 4) == 8).sum()) for b in blocs)
    assert n8 > 0, "the test set must carry -0 codes"
    octets = [0, 0]
    for i, canonique in enumerate([False, True]):
        preps = [O.preparer_matrice(b, R, B, canonique) for b in blocs]
        f4 = A.tables_matrice(preps)
        if canonique:
            sym8 = _porte_un_8(np.arange(256))
            for k in range(1, 4):
                assert (f4[k][sym8] == 0).all(), f"canonical table k = {k - 1} gives a slot to a nibble 8"
        luts4 = np.stack([O.lut(x) for x in f4])
        for x, prep in enumerate(preps):
            biais = bytes((i * 3 + x) & 255 for i in range(4 * R))
            fl = A.flux_matrice(prep, biais, f4, 0, R, nb)
            octets[i] += len(fl[3][4])
            partie = O.assembler_partie(0, x, 0, 1, fl)[0]
            codes, ech, _, bd, bc = O.decoder_matrice_v10(partie, 0, R, B, luts4)
            assert bd.intact() and bc.intact()
            q0, e0 = _origine(blocs[x], R, B)
            attendu = _canonique(q0) if canonique else q0
            assert (codes == attendu).all() and (ech == e0).all(), f"canonical = {canonique}, expert {x}"
            if canonique:
                assert not _porte_un_8(codes).any()
                assert (codes != q0).any()
    # Each folded -0 removes about one bit (a coin toss): at least half of n8 bits.
    gain_bits = (octets[0] - octets[1]) * 8.0
    assert gain_bits > 0.5 * n8, f"gain {gain_bits} bits for {n8} folded -0 ({octets[1]} vs {octets[0]} bytes)"
