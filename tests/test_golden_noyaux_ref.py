"""CPU: the oracle against outputs of the reference's own CUDA kernels.

tests/golden/noyaux_ref.json was written on a B200 by tests/golden/generer_noyaux_ref.py, with
the reference's kernels (trc-noyaux/noyaux/noyaux.cu compiled unchanged for sm_100a). Here, with
no GPU, the same seeded inputs are rebuilt (their SHA-256 is checked first) and:
- the oracle's normative decoder gives the reference decoder's slot bytes, bit for bit, with
  clean integrity counters (decodeur.cuh against rans.rs:388-451, lib.rs:190-260);
- the attention side: the Q8_0 GEMV, RMSNorm and the f16 KV write bit for bit; the YaRN
  rotation within 2e-7 relative and the attention within 1e-5 of max|out| (host libm against
  the device's math functions);
- the f64 GEMV agrees with gemv_mxfp4 within the reference's own tolerance, max|y - y64| <=
  1e-5 max|y64| (ARCHITECTURE.md 6.5, K2);
- top-k indices are equal and weights equal bit for bit (passe.cuh:455-514 against
  ops.rs:123-131); SwiGLU bit for bit, or within 1 ulp where the f64 exp of the device and of
  the host libm round differently (counted, at most 1 in 1,000); the combine bit for bit; the
  router GEMV within 1e-5 relative of f64."""
import base64
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


def _u32(b64) -> np.ndarray:
    return np.frombuffer(base64.b64decode(b64), "<u4").astype(np.uint32)


def _f32(b64) -> np.ndarray:
    return _u32(b64).view(np.float32)


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
    assert (w.view(np.uint32) == _u32(t["poids_bits"])).all()


def test_swiglu_contre_swiglu_oai():
    s = G["swiglu"]
    y = O.swiglu(_f32(s["g_bits"]), _f32(s["u_bits"])).view(np.int32).astype(np.int64)
    yr = _u32(s["y_bits"]).view(np.int32).astype(np.int64)
    ulp = np.abs(y - yr)
    assert ulp.max() <= 1
    assert (ulp > 0).sum() <= len(ulp) // 1000


def test_combiner_contre_combiner():
    c = G["combiner"]
    d = len(_u32(c["residu_bits"]))
    so = _f32(c["sorties_bits"])
    w = _f32(c["poids_bits"])
    r = O.combiner(_f32(c["residu_bits"]), so, d, w, len(w), d)
    assert (r.view(np.uint32) == _u32(c["sortie_bits"])).all()


def test_gemv_f32_routeur():
    g = G["gemv_f32"]
    E, C = len(_u32(g["b_bits"])), len(_u32(g["x_bits"]))
    W, x, b = entrees_gemv_f32(E, C)
    assert _sha(W.tobytes()) == g["W_sha256"]
    assert (x.view(np.uint32) == _u32(g["x_bits"])).all()
    y64 = W.astype(np.float64) @ x.astype(np.float64) + b
    y = _f32(g["y_bits"]).astype(np.float64)
    assert np.abs(y - y64).max() <= 1e-5 * np.abs(y64).max()


# ---------------------------------------------------------------- the attention side

from generer_noyaux_ref import entrees_attention  # noqa: E402

A = G["attention"]
_E = {}


def _e():
    if not _E:
        _E.update(entrees_attention())
        for n, v in _E.items():
            assert _sha(np.ascontiguousarray(v).tobytes()) == A["entrees_sha256"][n], f"input {n} differs"
    return _E


def test_gemv_q8_0_et_rmsnorm_au_bit():
    e = _e()
    y = O.gemv_q8_0(e["W"], e["x"], e["b"], 512, 2880)
    assert (y.view(np.uint32) == _u32(A["gemv_q8_0_bits"])).all()
    yn = O.rmsnorm(e["xn"], e["wn"], 2880, 2, 1e-5)
    assert (yn.view(np.uint32) == _u32(A["rmsnorm_bits"])).all()


@pytest.mark.parametrize("i", range(4))
def test_rope_yarn(i):
    import troncons_b200 as T2

    e = _e()
    r = A["rope"][i]
    p = T2.ParamsRope.gpt_oss()
    p.variante = r["variante"]
    q, k = O.rope_yarn(e["q"], e["k"], 64, 8, r["position"], p)
    for a, b in ((q, _f32(r["q_bits"])), (k, _f32(r["k_bits"]))):
        assert np.abs(a - b).max() <= 2e-7 * max(1.0, np.abs(b).max())


def test_ecrire_kv_au_bit():
    e = _e()
    ck = np.zeros(3 * 512, np.uint16)
    cv = np.zeros_like(ck)
    O.ecrire_kv(e["kv_k"], e["kv_v"], ck, cv, 512, 2)
    k = np.frombuffer(base64.b64decode(A["ecrire_kv"]["k"]), "<u2")
    v = np.frombuffer(base64.b64decode(A["ecrire_kv"]["v"]), "<u2")
    assert (ck[1024:] == k).all() and (cv[1024:] == v).all()


@pytest.mark.parametrize("i", range(2))
def test_attention(i):
    import troncons_b200 as T2

    e = _e()
    a = A["attention"][i]
    p = T2.ParamsAttention.gpt_oss(a["position"], a["fenetre"])
    cases = a["fenetre"] if a["fenetre"] else a["position"] + 1
    out = O.attention(e["q"], e["cache_k"][:cases].reshape(-1), e["cache_v"][:cases].reshape(-1), e["puits"], p)
    ref = _f32(a["sortie_bits"])
    assert np.abs(out - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
