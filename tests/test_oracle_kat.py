"""CPU: the oracle against the reference's known answers, and the product's host helpers
against the oracle.

Known answers (reference test, file:line):
- empreinte64("abc") = first 8 bytes of SHA-256("abc"), little-endian
  (trc-format/tests/aller_retour.rs:411-416), plus the FIPS 180-4 SHA-256 vectors;
- LUT entries of a known table, and a full-frequency single symbol (trc-noyaux/src/abi.rs:384-406);
- frequency tables refused / accepted, all-zero counts (trc-codec/tests/rans.rs:251-262);
- slot layout of gpt-oss: 4,147,200 / 4,406,528 / 4,418,048 per matrix, 13,254,144 per expert
  (abi.rs:340-349);
- tile counts of gpt-oss streams: DELTA 259,200 B -> 2,025 macro-steps -> T = 8 at N = 256
  (64 at N = 32), CODES_CTX 4,147,200 B -> 32,400 macro-steps -> T = 127 (abi.rs:351-383)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import troncons_b200 as T


def test_empreinte64_connue():
    assert O.empreinte64(b"abc") == int.from_bytes(bytes([0xBA, 0x78, 0x16, 0xBF, 0x8F, 0x01, 0xCF, 0xEA]), "little")


@pytest.mark.parametrize("message,condensat", [
    (b"abc", "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"),
    (b"", "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"),
    (b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq",
     "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1"),
])
def test_sha256_fips180(message, condensat):
    assert O.sha256(message).hex() == condensat


def test_sha256_million_a():
    assert O.sha256(b"a" * 1_000_000).hex() == "cdc76e5c9914fb9281a1c7e284d73e67f1809a48a497200e046d39ccc7112cd0"


def _lut_produit(f):
    out = np.zeros(4096, np.uint32)
    fa = np.ascontiguousarray(f, np.uint16)
    s = T.lib.trc_lut_geometrie1(fa.ctypes.data, out.ctypes.data)
    return s, out


def test_lut_d_une_table_connue():
    f = np.zeros(256, np.uint16)
    f[3], f[200] = 4000, 96
    for l in (O.lut(f), _lut_produit(f)[1]):
        assert l[0] == 3 | (3999 << 8)
        assert l[3999] == 3 | (3999 << 8) | (3999 << 20)
        assert l[4000] == 200 | (95 << 8)
        assert l[4095] == 200 | (95 << 8) | (95 << 20)
    f[3] = 3999  # a wrong sum is refused
    with pytest.raises(ValueError):
        O.lut(f)
    assert _lut_produit(f)[0] == T.TRC_ERR_USAGE


def test_symbole_unique_a_frequence_pleine():
    f = np.zeros(256, np.uint16)
    f[7] = 4096
    assert O.lut(f)[4095] == 7 | (4095 << 8) | (4095 << 20)
    assert _lut_produit(f)[1][4095] == 7 | (4095 << 8) | (4095 << 20)


def test_tables_refusees_et_comptes_nuls():
    f = np.zeros(16, np.uint16)
    f[0] = 4095
    with pytest.raises(ValueError):
        O.lut(f, geometrie=2)
    f[1] = 1
    O.lut(f, geometrie=2)
    assert O.table_depuis_comptes(np.zeros(256, np.uint64))[0] == 4096


@pytest.mark.parametrize("geometrie", [1, 2])
def test_tables_somme_et_presence(geometrie):
    """Every counted symbol keeps a non-zero frequency; frequencies sum to 4096; the product's
    normalisation (geometry 1) gives the oracle's frequencies."""
    rng = np.random.default_rng(11 + geometrie)
    n = 256 if geometrie == 1 else 16
    for _ in range(200):
        c = np.zeros(n, np.uint64)
        k = int(rng.integers(1, n + 1))
        sym = rng.choice(n, k, replace=False)
        c[sym] = rng.integers(1, 10 ** int(rng.integers(1, 9)), k).astype(np.uint64)
        f = O.table_depuis_comptes(c, geometrie)
        assert int(f.sum()) == 4096
        assert ((c > 0) <= (f > 0)).all()
        if geometrie == 1:
            fp = np.zeros(256, np.uint16)
            assert T.lib.trc_table_depuis_comptes(c.ctypes.data, 1, fp.ctypes.data) == T.TRC_OK
            assert (fp == f).all()


def test_disposition_gpt_oss():
    assert O.disposition(2880, 2880) == (4_147_200, 4_406_528, 4_418_048)
    d = T.DimsExpert.gpt_oss()
    assert T.taille_emplacement(d) == 13_254_144
    assert int(T.lib.trc_taille_emplacement(C.byref(d))) == 13_254_144


@pytest.mark.parametrize("n_delta,t_delta", [(256, 8), (32, 64)])
def test_tuiles_gpt_oss(n_delta, t_delta):
    """The product's encoder on one gpt-oss-shaped matrix: stream sizes P and tile counts T."""
    import trc_aides as A

    rng = np.random.default_rng(3)
    R, B = 2880, 90
    blocs = A.blocs_mxfp4(rng, R, B)
    prep = O.preparer_matrice(blocs, R, B, True)
    f4 = A.tables_matrice([prep])
    fl = A.flux_matrice(prep, b"\0" * 4 * R, f4, 0, R, R * B, n_delta=n_delta)
    fd, fc = A.Flux.lire(fl[2][4]), A.Flux.lire(fl[3][4])
    assert (fd.P, fd.debuts.size) == (259_200, t_delta)
    assert (fc.P, fc.debuts.size) == (4_147_200, 127)
