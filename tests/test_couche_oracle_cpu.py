"""CPU: the layer the CPU baseline builds with the oracle alone (oracle.CoucheOracle) is the
product's synthetic layer (troncons_b200.synth.couche) byte for byte: the same weights from the
same seeds, the same tables, LUTs and v1.2 parts, and the same router. So the bench's reference
arm times the same workload as the GPU arm without loading the product library."""
import numpy as np
import pytest

import oracle as O
import troncons_b200 as T
import troncons_b200.synth as S


@pytest.mark.parametrize("graine,lignes,colonnes,premier,n", [
    (5, 64, 64, 0, 3), (11, 2880, 2880, 7, 2), (20261201 * 7 + 2, 2880, 2880, 126, 2)])
def test_poids_egaux(graine, lignes, colonnes, premier, n):
    b0, i0 = S.matrices(graine, lignes, colonnes, n, premier=premier)
    b1, i1 = O.synth_matrices(graine, lignes, colonnes, n, premier=premier)
    assert np.array_equal(b0, b1)
    assert np.array_equal(i0.view(np.uint32), i1.view(np.uint32))


@pytest.mark.parametrize("lignes,colonnes,experts,n_delta,n_codes", [
    ([256, 256, 512], [512, 512, 256], 8, 256, 256),
    ([96, 96, 64], [64, 64, 96], 5, 32, 64),
    ([2880, 2880, 2880], [2880, 2880, 2880], 3, 256, 256),
])
def test_couche_egale(lignes, colonnes, experts, n_delta, n_codes):
    c = S.couche(2026, T.DimsExpert.de(lignes, colonnes), experts, brut=False, n_delta=n_delta, n_codes=n_codes)
    o = O.CoucheOracle(2026, lignes, colonnes, experts, n_delta, n_codes)
    assert np.array_equal(c.freqs, o.freqs)
    assert np.array_equal(c.luts, o.luts)
    assert all(a == b for a, b in zip(c.parties, o.parties))
    assert np.array_equal(c.wr, o.wr) and np.array_equal(c.br, o.br)


def test_bf16():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(3).standard_normal(100000).astype(np.float32)
    x[:4] = [0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8]  # ties to even, both ways
    attendu = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16(x).view(np.uint32), attendu.view(np.uint32))
