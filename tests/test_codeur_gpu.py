"""GPU: the `.trc` encoder on the GPU against the CPU encoders.

Streams (trc_coder_flux_gpu) against the oracle's coder:
The oracle's coder is pinned byte for byte to the reference bench's coder_g1 (banc_k.cu:277-321)
and to trc-codec's stream layout (rans.rs:186-228, 296-334); the GPU's stream must be the same
bytes, for:
- random sources with a per-block context (the scale class of each 16-byte block), tiles of 256
  and 32 macro-steps, one partial last tile, one tile only;
- the DELTA and CODES_CTX streams of MXFP4 matrices with gpt-oss's shapes (2880 x 5760 gate/up,
  the v1.2 canonical preparation), the streams a `.trc` part holds;
- a symbol absent from its table, and a context with no table, which are refused.
The decoded stream gives the source back (oracle decoder).

Whole level-0 parts (trc_coder_parties_gpu) and the layer's symbol counts (trc_comptes_gpu)
against this library's CPU encoder (trc_coder_partie, trc_comptes_matrice, whose parts are
pinned to the reference bench's assembler): byte for byte, for v1.2 (canonical) and v1.0 codes,
tiles of 256, 32 and odd sizes, shapes whose deltas and codes need padding (3, 1 and 100 blocks
per row), and gpt-oss's expert shape; a table missing a symbol the expert holds is refused."""
import numpy as np
import pytest

import oracle as O
import trc_aides as A

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def T():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import troncons_b200

    return troncons_b200


def _sur_gpu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _source_et_tables(rng, n_blocs):
    src = A.octets_geometriques(rng, 16 * n_blocs)
    kappa = rng.choice(np.array([0, 1, 1, 2], np.uint8), n_blocs)
    src = np.where(np.repeat(kappa, 16) == 2, src & 0x33, src).astype(np.uint8)
    f = np.stack([O.table_depuis_comptes(np.bincount(src.reshape(-1, 16)[kappa == k].reshape(-1),
                                                     minlength=256).astype(np.uint64)) for k in range(3)])
    return src, kappa, f


@pytest.mark.parametrize("N", [256, 32, 1])
@pytest.mark.parametrize("n_blocs", [8, 1000, 8 * 2025, 200_000])
def test_flux_gpu_egale_oracle(T, n_blocs, N):
    rng = np.random.default_rng(11 + n_blocs + N)
    src, kappa, f = _source_et_tables(rng, n_blocs)
    src = np.concatenate([src, np.zeros((-src.size) % 128, np.uint8)])
    if f[0][0] == 0 and src.size != 16 * n_blocs:
        f[0][0], f[0][int(np.argmax(f[0]))] = 1, f[0][int(np.argmax(f[0]))] - 1
    attendu = O.coder_g1(src, f, kappa, N)
    obtenu = T.coder_flux_gpu(_sur_gpu(src), _sur_gpu(f), _sur_gpu(kappa), N)
    assert obtenu == attendu
    if n_blocs <= 8 * 2025:
        d, b = O.decoder(obtenu, np.stack([O.lut(x) for x in f]), kappa)
        assert b.intact() and (d[:src.size] == src).all()


def test_flux_gpu_sans_contexte(T):
    rng = np.random.default_rng(4)
    src = A.octets_geometriques(rng, 128 * 777)
    f = O.table_depuis_comptes(np.bincount(src, minlength=256).astype(np.uint64))[None]
    for N in (256, 7):
        assert T.coder_flux_gpu(_sur_gpu(src), _sur_gpu(f), None, N) == O.coder_g1(src, f, None, N)


@pytest.mark.parametrize("n_delta,n_codes", [(256, 256), (32, 32)])
def test_flux_gpu_matrice_gpt_oss(T, n_delta, n_codes):
    """The DELTA and CODES_CTX streams of a 2880 x 5760 MXFP4 matrix (v1.2 canonical)."""
    rng = np.random.default_rng(29)
    R, B = 5760, 2880 // 32
    prep = O.preparer_matrice(A.blocs_mxfp4(rng, R, B, zeros_signes=True), R, B, True)
    f4 = A.tables_matrice([prep])
    _, delta, qs = prep
    kappa = A.classe(delta[:R * B])
    fd = T.coder_flux_gpu(_sur_gpu(delta), _sur_gpu(f4[0:1]), None, n_delta)
    assert fd == O.coder_g1(delta, f4[0:1], None, n_delta)
    fc = T.coder_flux_gpu(_sur_gpu(qs), _sur_gpu(f4[1:4]), _sur_gpu(kappa), n_codes)
    assert fc == O.coder_g1(qs, f4[1:4], kappa, n_codes)


def test_flux_gpu_refuse_symbole_absent(T):
    rng = np.random.default_rng(8)
    src = A.octets_geometriques(rng, 128 * 40)
    f = O.table_depuis_comptes(np.bincount(src, minlength=256).astype(np.uint64))[None]
    src[1000] = int(np.flatnonzero(f[0] == 0)[0])  # a byte the table has no slot for
    with pytest.raises(ValueError):
        T.coder_flux_gpu(_sur_gpu(src), _sur_gpu(f), None, 256)
    # a context with no table
    src2 = A.octets_geometriques(rng, 128 * 40)
    f2 = np.stack([O.table_depuis_comptes(np.bincount(src2, minlength=256).astype(np.uint64))] * 2)
    kappa = np.zeros(src2.size // 16, np.uint8)
    kappa[17] = 2
    with pytest.raises(ValueError):
        T.coder_flux_gpu(_sur_gpu(src2), _sur_gpu(f2), _sur_gpu(kappa), 256)


def test_flux_gpu_usage(T):
    src = torch.zeros(100, dtype=torch.uint8, device="cuda")
    f = torch.zeros(256, dtype=torch.int16, device="cuda")
    with pytest.raises(T.ErreurUsage):
        T.coder_flux_gpu(src, f, None, 256)


# ---------------------------------------------------------------- whole parts


def _lot(graine, dims, n):
    """n experts' blocks and biases (synthetic MXFP4), on the host and on the GPU."""
    import troncons_b200.synth as S

    hote = [S.matrices(graine + j, dims.lignes[j], dims.colonnes[j], n) for j in range(3)]
    blocs = [[torch.from_numpy(hote[j][0][e]).cuda() for j in range(3)] for e in range(n)]
    biais = [[torch.from_numpy(hote[j][1][e]).cuda() for j in range(3)] for e in range(n)]
    return hote, blocs, biais


FORMES = {
    "petite": ([256, 256, 512], [512, 512, 256]),
    "impaire": ([37, 5, 130], [96, 32, 3200]),  # B = 3, 1, 100; padded deltas and codes
}


@pytest.mark.parametrize("forme", list(FORMES))
@pytest.mark.parametrize("canonique", [True, False])
def test_comptes_et_parties_gpu_egalent_le_codeur_cpu(T, forme, canonique):
    import troncons_b200.synth as S

    dims = T.DimsExpert.de(*FORMES[forme])
    n = 6
    hote, blocs, biais = _lot(5, dims, n)
    c_cpu = S.comptes([hote[j][0] for j in range(3)], dims, canonique)
    c_gpu = S.comptes_gpu(blocs, dims, canonique).cpu().numpy().astype(np.uint64).reshape(3, 4, 256)
    assert (c_gpu == c_cpu).all()
    freqs = S.tables_de_comptes(c_cpu)
    for nd, nc in ((256, 256), (32, 32), (7, 33)):
        parts = S.coder_parties_gpu(blocs, biais, dims, freqs, canonique, couche=3, experts=[10 + e for e in range(n)],
                                    n_delta=nd, n_codes=nc)
        for e in range(n):
            attendu = S.coder_partie([hote[j][0][e] for j in range(3)], [hote[j][1][e] for j in range(3)], dims, freqs,
                                     canonique, couche=3, expert=10 + e, n_delta=nd, n_codes=nc)
            assert parts[e] == attendu, f"expert {e}, tiles {nd}/{nc}"


def test_parties_gpu_gpt_oss(T):
    """Two gpt-oss experts (3 x 2880 x 2880): counts and parts as the CPU encoder's."""
    import troncons_b200.synth as S

    dims = T.DimsExpert.gpt_oss()
    hote, blocs, biais = _lot(41, dims, 2)
    c_cpu = S.comptes([hote[j][0] for j in range(3)], dims)
    c_gpu = S.comptes_gpu(blocs, dims).cpu().numpy().astype(np.uint64).reshape(3, 4, 256)
    assert (c_gpu == c_cpu).all()
    freqs = S.tables_de_comptes(c_cpu)
    parts = S.coder_parties_gpu(blocs, biais, dims, freqs)
    for e in range(2):
        attendu = S.coder_partie([hote[j][0][e] for j in range(3)], [hote[j][1][e] for j in range(3)], dims, freqs,
                                 expert=e)
        assert parts[e] == attendu


def test_parties_gpu_refusent_un_symbole_absent(T):
    """A table with no slot for a symbol the expert holds: the CPU encoder refuses, the GPU
    reports length 0 and writes nothing."""
    import troncons_b200.synth as S

    dims = T.DimsExpert.de(*FORMES["petite"])
    hote, blocs, biais = _lot(9, dims, 2)
    freqs = S.tables_de_comptes(S.comptes([hote[j][0] for j in range(3)], dims))
    # delta 128 (a scale equal to its row's median) is in every row: give its mass to another symbol
    f = freqs[1, 0].astype(np.int64)
    autre = int(np.argmax(np.where(np.arange(256) == 128, -1, f)))
    f[autre] += f[128]
    f[128] = 0
    freqs[1, 0] = f.astype(np.uint16)
    with pytest.raises(ValueError):
        S.coder_partie([hote[j][0][0] for j in range(3)], [hote[j][1][0] for j in range(3)], dims, freqs)
    with pytest.raises(ValueError):
        S.coder_parties_gpu(blocs, biais, dims, freqs)
