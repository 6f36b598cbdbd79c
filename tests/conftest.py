"""Shared fixtures. Tests marked `gpu` need a CUDA device (a B200); the others run on CPU.

The oracle (oracle/, CPU restatement of the reference) is the checker; the product under test
is troncons_b200 (the C-ABI library and its CUDA kernels)."""
import os
import sys

import pytest

RACINE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if RACINE not in sys.path:
    sys.path.insert(0, RACINE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        gpu = False
    if gpu:
        return
    saut = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(saut)


@pytest.fixture(scope="session")
def noyaux():
    import troncons_b200 as T

    return T.Noyaux()


@pytest.fixture(scope="session")
def couche_gpt_oss():
    """A synthetic gpt-oss-shaped layer of 8 experts (2880 x 2880 matrices), v1.2 + raw parts."""
    import troncons_b200 as T
    import troncons_b200.synth as S

    return S.couche(20261201, T.DimsExpert.gpt_oss(), 8)


@pytest.fixture(scope="session")
def couche_impaire():
    """A small layer whose down matrix has an odd number of blocks per row (9: 256 x 288), so
    that its GEMVs take the row walks (k_moe_bas, k_moe_brut) instead of the row groups."""
    import troncons_b200 as T
    import troncons_b200.synth as S

    return S.couche(11, T.DimsExpert.de([288, 288, 256], [256, 256, 288]), 8)


@pytest.fixture(scope="session")
def couche_petite():
    """A small layer (8 experts: gate and up 256 x 512, down 512 x 256) for quick checks."""
    import troncons_b200 as T
    import troncons_b200.synth as S

    return S.couche(7, T.DimsExpert.de([256, 256, 512], [512, 512, 256]), 8)
