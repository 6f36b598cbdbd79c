"""CPU: the encoders pinned to the reference's own encoder.

The reference bench (trc-noyaux/banc/banc_k.cu) carries a second .trc encoder written from the
format specification alone. tests/golden/codeur_banc.json holds the SHA-256 of parts it wrote
(tests/golden/generer_codeur_banc.py, from seeded synthetic experts and the oracle's frequency
tables). Here:
- the oracle's encoder (oracle/trc_oracle.c) writes those exact parts;
- the product's encoder (troncons_b200/csrc/codeur.cpp, trc_coder_partie) writes them too, from
  its own counts and normalisation (trc_comptes_matrice, trc_table_depuis_comptes);
- when oracle/_ref is built, the bench encoder itself still writes them."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

import oracle as O
import troncons_b200 as T
import troncons_b200.synth as S

ICI = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ICI, "golden"))

from generer_codeur_banc import parties_banc  # noqa: E402

with open(os.path.join(ICI, "golden", "codeur_banc.json")) as f:
    GOLDEN = json.load(f)["cas"]


def _sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def _cas(c):
    return (c["graine"], c["lignes"], c["colonnes"], c["experts"], c["canonique"], c["n_delta"], c["n_codes"])


@pytest.mark.parametrize("c", GOLDEN, ids=lambda c: f"g{c['graine']}")
def test_oracle_ecrit_les_parties_du_banc(c):
    _, _, _, freqs, parties = parties_banc(*_cas(c), codeur=O,
                                           assembleur=lambda co, x, fl: O.assembler_partie(co, x, 0, 3, fl)[0])
    assert _sha(freqs.astype("<u2").tobytes()) == c["tables_sha256"]
    assert [(len(p), _sha(p)) for p in parties] == [(q["octets"], q["sha256"]) for q in c["parties"]]


@pytest.mark.parametrize("c", GOLDEN, ids=lambda c: f"g{c['graine']}")
def test_produit_ecrit_les_parties_du_banc(c):
    graine, lignes, colonnes, experts, canonique, n_delta, n_codes = _cas(c)
    dims = T.DimsExpert.de(lignes, colonnes)
    blocs, biais = [], []
    for j in range(3):
        b, bi = S.matrices(graine * 7 + j, lignes[j], colonnes[j], experts)
        blocs.append(b)
        biais.append(bi)
    freqs = S.tables(blocs, dims, canonique)
    assert _sha(freqs.astype("<u2").tobytes()) == c["tables_sha256"]
    for x, q in enumerate(c["parties"]):
        p = S.coder_partie([blocs[j][x] for j in range(3)], [biais[j][x] for j in range(3)], dims, freqs, canonique,
                           0, x, n_delta, n_codes)
        assert (len(p), _sha(p)) == (q["octets"], q["sha256"]), f"expert {x}"


@pytest.mark.parametrize("c", GOLDEN[:2], ids=lambda c: f"g{c['graine']}")
def test_banc_toujours_egal(c):
    banc = O.banc()
    if banc is None:
        pytest.skip("oracle/_ref/libtrc_banc.so not built (make -C oracle ref)")
    _, _, _, _, parties = parties_banc(*_cas(c), codeur=banc, assembleur=banc.assembler_partie)
    assert [_sha(p) for p in parties] == [q["sha256"] for q in c["parties"]]


def test_luts_couche_produit_egale_oracle_et_banc():
    rng = np.random.default_rng(9)
    freqs = np.zeros((3, 4, 256), np.uint16)
    for j in range(3):
        for t in range(4):
            cpt = rng.integers(0, 1000, 256).astype(np.uint64) * (rng.random(256) < 0.6)
            cpt[0] += 1
            freqs[j, t] = O.table_depuis_comptes(cpt)
    luts = S.luts(freqs).reshape(3, 4, 4096)
    banc = O.banc()
    for j in range(3):
        for t in range(4):
            assert (luts[j, t] == O.lut(freqs[j, t])).all()
            if banc is not None:
                assert (luts[j, t] == banc.lut(freqs[j, t])).all()


def test_symbole_absent_refuse():
    """A code byte with no slot in its table cannot be encoded: the product refuses."""
    dims = T.DimsExpert.de([64, 64, 64], [64, 64, 64])
    blocs, biais = [], []
    for j in range(3):
        b, bi = S.matrices(5 + j, 64, 64, 1)
        blocs.append(b)
        biais.append(bi)
    freqs = S.tables(blocs, dims, True)
    freqs[0, 1] = 0
    freqs[0, 1, 0] = 4096  # class-0 table knows only byte 0
    with pytest.raises(ValueError):
        S.coder_partie([b[0] for b in blocs], [b[0] for b in biais], dims, freqs, True)
