"""CPU: the oracle against outputs of the reference's own CUDA kernels.

tests/golden/noyaux_ref.json was written on a B200 by tests/golden/generer_noyaux_ref.py, with
the reference's kernels (trc-noyaux/noyaux/noyaux.cu compiled unchanged for sm_100a). Here, with
no GPU, the same seeded inputs are rebuilt (their SHA-256 is checked first) and:
- the oracle's normative decoder gives the reference decoder's slot bytes, bit for bit, with
  clean integrity counters (decodeur.cuh against rans.rs:388-451, lib.rs:190-260);
- the f64 GEMV agrees with gemv_mxfp4 within the reference's own tolerance, max|y - y64| <=
  1e-5 max|y64| (ARCHITECTURE.md 6.5, K2);
- top-k indices are equal and weights equal bit for bit (passe.cuh:455-514 against
  ops.rs:123-131); SwiGLU bit for bit, or within 1 ulp where the f64 exp of the device and of
  the host libm round differently (counted, at most 1 in 1,000); the combine bit for bit; the
  router GEMV within 1e-5 relative of f64."""
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

from generer_noyaux_ref import entrees_gemv_f32  # noqa: E402

with open(os.path.join(ICI, "golden", "noyaux_ref.json")) as f:
    G = json.load(f)


def _sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def _f32(bits) -> np.ndarray:
    return np.array(bits, np.uint32).view(np.float32)


_couches = {}


def _couche(cg):
    if cg["graine"] not in _couches:
        _couches[cg["graine"]] = S.couche(cg["graine"], T.DimsExpert.de(cg["lignes"], cg["colonnes"]), cg["experts"],
                                          brut=False)
    return _couches[cg["graine"]]


def _slot(cg, x):
    c = _couche(cg)
    slot, ctl = O.decoder_expert(c.parties[x], c.luts, cg["lignes"], cg["colonnes"], T.taille_emplacement(c.dims))
    return slot, ctl


@pytest.mark.parametrize("cg", G["couches"], ids=lambda c: f"g{c['graine']}")
def test_decodeur_du_oracle_egale_le_noyau_de_reference(cg):
    c = _couche(cg)
    assert _sha(c.luts.astype("<u4").tobytes()) == cg["luts_sha256"], "LUTs differ from the fixture's"
    for x, e in enumerate(cg["experts_decodes"]):
        assert _sha(c.parties[x]) == e["partie_sha256"], f"expert {x}: part differs from the fixture's"
        assert e["controle"] == [0, 0, 0, 0]
        slot, ctl = _slot(cg, x)
        assert (ctl == 0).all()
        assert _sha(slot.tobytes()) == e["emplacement_sha256"], f"expert {x}: slot differs from the reference kernel's"


@pytest.mark.parametrize("i", range(len(G["gemv"])))
def test_gemv_f64_contre_gemv_mxfp4(i):
    g = G["gemv"][i]
    cg = next(c for c in G["couches"] if c["graine"] == g["graine"])
    slot, _ = _slot(cg, g["expert"])
    j = g["matrice"]
    R, C = cg["lignes"][j], cg["colonnes"][j]
    base = sum(O.disposition(cg["lignes"][a], cg["colonnes"][a])[2] for a in range(j))
    e_off, b_off, _ = O.disposition(R, C)
    nb = R * (C // 32)
    m = slot[base:]
    codes, ech = m[:16 * nb], m[e_off:e_off + nb]
    biais = m[b_off:b_off + 4 * R].view(np.float32)
    x = _f32(g["x_bits"])
    y64 = O.gemv_f64(codes, ech, biais, x, R, C)
    y = _f32(g["y_bits"]).astype(np.float64)
    assert np.abs(y - y64).max() <= 1e-5 * np.abs(y64).max()


@pytest.mark.parametrize("i", range(len(G["topk"])))
def test_topk_contre_routeur_topk(i):
    t = G["topk"][i]
    idx, w = O.routeur_topk(_f32(t["logits_bits"]), t["k"])
    assert [int(v) for v in idx] == t["indices"]
    assert [int(v) for v in w.view(np.uint32)] == t["poids_bits"]


def test_swiglu_contre_swiglu_oai():
    s = G["swiglu"]
    y = O.swiglu(_f32(s["g_bits"]), _f32(s["u_bits"])).view(np.int32).astype(np.int64)
    yr = np.array(s["y_bits"], np.uint32).view(np.int32).astype(np.int64)
    ulp = np.abs(y - yr)
    assert ulp.max() <= 1
    assert (ulp > 0).sum() <= len(ulp) // 1000


def test_combiner_contre_combiner():
    c = G["combiner"]
    d = len(c["residu_bits"])
    so = _f32(c["sorties_bits"])
    w = _f32(c["poids_bits"])
    r = O.combiner(_f32(c["residu_bits"]), so, d, w, len(w), d)
    assert [int(v) for v in r.view(np.uint32)] == c["sortie_bits"]


def test_gemv_f32_routeur():
    g = G["gemv_f32"]
    E, C = len(g["b_bits"]), len(g["x_bits"])
    W, x, b = entrees_gemv_f32(E, C)
    assert _sha(W.tobytes()) == g["W_sha256"]
    assert [int(v) for v in x.view(np.uint32)] == g["x_bits"]
    y64 = W.astype(np.float64) @ x.astype(np.float64) + b
    y = _f32(g["y_bits"]).astype(np.float64)
    assert np.abs(y - y64).max() <= 1e-5 * np.abs(y64).max()
