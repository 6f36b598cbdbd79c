"""GPU: the whole decode step (trc_modele_pas) on a small synthetic gpt-oss-shaped model.

- the embedding row and the argmax (trc_ligne_q8_0, trc_argmax) against numpy, bit for bit:
  ties to the smallest index, NaN never chosen, all NaN -> 0xFFFFFFFF (passe.cuh:623-669);
- the project's exactness invariant on the whole model: greedy decode from the .trc v1.2 parts
  and from the raw MXFP4 parts of the same weights gives the same logits bit for bit and the same
  tokens, step after step;
- the logits against a CPU port of the step composed from the oracle (attention side and MoE
  layer on host cores, different reduction orders): max|dz| <= 1e-3 max|z| and the same greedy
  token at every step;
- the logits against an fp64 host evaluation of the same weights (storage formats kept: Q8_0
  rows, the MXFP4 experts decoded by the oracle, the f16 KV cache; every product and sum in
  f64): max|dz| <= 1e-4 max|z| and the same greedy token at every step."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def petit():
    import troncons_b200.modele as M

    return M.Modele(couches=2, d=256, tetes=8, tetes_kv=2, experts=8, k=4, vocab=512, contexte=64, ffn=256,
                    fenetre=16, graine=7, compresse=True, brut=True)


def test_ligne_q8_0_et_argmax():
    import ctypes as C

    import troncons_b200 as T
    import troncons_b200.modele as M

    w = M.synth_q8_0(40, 256, 3, 11)
    y = torch.zeros(256, dtype=torch.float32, device="cuda")
    T.verifier(T.lib.trc_ligne_q8_0(w.data_ptr(), w.numel(), 17, 256, y.data_ptr(), 1024, M._flux()))
    b = w.cpu().numpy().reshape(40, 8, 34)[17]
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    assert np.array_equal(y.cpu().numpy(), (d * q).reshape(-1))

    def am(v):
        t = torch.from_numpy(np.asarray(v, np.float32)).cuda()
        o = torch.zeros(1, dtype=torch.int32, device="cuda")
        T.verifier(T.lib.trc_argmax(t.data_ptr(), t.numel() * 4, t.numel(), o.data_ptr(), 4, M._flux()))
        return int(o.cpu().numpy().view(np.uint32)[0])

    v = np.random.default_rng(2).standard_normal(5000).astype(np.float32)
    assert am(v) == int(np.argmax(v))
    v[[100, 4000]] = 9.0
    assert am(v) == 100
    v[50] = np.nan
    assert am(v) == 100
    assert am([np.nan] * 7) == 0xFFFFFFFF
    assert am([-np.inf, -np.inf]) == 0
    del C


def _glouton(m, n, jeton0=1):
    lg, jt, ct = m.vues()
    ct.zero_()
    logits, jetons, j = [], [], jeton0
    for pos in range(n):
        m.pas(j, pos)
        torch.cuda.synchronize()
        logits.append(lg.cpu().numpy().copy())
        j = int(jt.cpu().numpy()[0])
        jetons.append(j)
    assert (ct.cpu().numpy() == 0).all()
    return logits, jetons


def test_compresse_et_brut_au_bit(petit):
    petit.choisir("compresse")
    lc, jc = _glouton(petit, 40)
    petit.choisir("brut")
    lb, jb = _glouton(petit, 40)
    assert jc == jb
    for s, (a, b) in enumerate(zip(lc, lb)):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"step {s}"


def test_deltas_predecodes_au_bit(petit):
    """The same model with every layer's DELTA decoded once at load (deltas_predecodes): 40
    greedy steps give the logits of the model that decodes DELTA at every step, bit for bit, and
    so those of its raw parts (the exactness invariant holds with the predecoded scales too)."""
    import troncons_b200.modele as M

    p = M.Modele(couches=2, d=256, tetes=8, tetes_kv=2, experts=8, k=4, vocab=512, contexte=64, ffn=256,
                 fenetre=16, graine=7, compresse=True, brut=True, deltas_predecodes=True)
    assert len(p.deltas) == 2
    petit.choisir("compresse")
    la, ja = _glouton(petit, 40)
    lp, jp = _glouton(p, 40)
    p.choisir("brut")
    lb, jb = _glouton(p, 40)
    assert ja == jp == jb
    for s, (a, b, c) in enumerate(zip(la, lp, lb)):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"step {s}"
        assert np.array_equal(a.view(np.uint32), c.view(np.uint32)), f"step {s}"


def test_contre_le_port_cpu(petit):
    import oracle as O
    import troncons_b200 as T

    m = petit
    m.choisir("compresse")
    L, d, dq, dkv = m.couches, m.d, m.tetes * 64, m.tetes_kv * 64
    h = [{n: (v.cpu().numpy() if torch.is_tensor(v) else v) for n, v in t.items()} for t in m.tenseurs]
    parts = []
    for l in range(L):
        tampon, adr, tailles = m.parties["compresse"][l]
        base = tampon.data_ptr()
        brut = tampon.cpu().numpy()
        parts.append([brut[int(a) - base:int(a) - base + int(s)].tobytes() for a, s in zip(adr, tailles)])
    luts = [x.cpu().numpy().view(np.uint32) for x in m.luts]
    emb = m.enchassement.cpu().numpy().reshape(m.vocab, d // 32, 34)
    wout = m.sortie_w.cpu().numpy()
    nsortie = m.norme_sortie.cpu().numpy()
    caches = [[np.zeros(t["cache_k"].size, np.uint16), np.zeros(t["cache_v"].size, np.uint16)] for t in h]
    lg, jt, _ = m.vues()
    j = 1
    for pos in range(20):  # past the sliding layers' ring of 16 cases
        m.pas(j, pos)
        torch.cuda.synchronize()
        z_gpu = lg.cpu().numpy().copy()
        # the CPU port of the same step
        b = emb[j]
        x = (b[:, :2].copy().view(np.float16).astype(np.float32) * b[:, 2:].view(np.int8).astype(np.float32)).reshape(-1)
        for l in range(L):
            t = h[l]
            hh = O.rmsnorm(x, t["attn_norm"], d, 1, m.eps)
            q = O.gemv_q8_0(t["wq"], hh, t["bq"], dq, d)
            k = O.gemv_q8_0(t["wk"], hh, t["bk"], dkv, d)
            v = O.gemv_q8_0(t["wv"], hh, t["bv"], dkv, d)
            q, k = O.rope_yarn(q, k, m.tetes, m.tetes_kv, pos, m.rope)
            an = t["anneau"]
            O.ecrire_kv(k, v, caches[l][0], caches[l][1], dkv, pos % an if an else pos)
            fin = pos + 1
            pa = T.ParamsAttention(m.tetes, m.tetes_kv, 64, max(0, fin - an) if an else 0, fin, an, 0.125, 0)
            a = O.attention(q, caches[l][0], caches[l][1], t["puits"], pa)
            o = O.gemv_q8_0(t["wo"], a, t["bo"], d, dq)
            x = O.combiner(x, o, d, None, 1, d)
            h2 = O.rmsnorm(x, t["post_norm"], d, 1, m.eps)
            x, _, _ = O.couche_moe_cpu(parts[l], luts[l], list(m.dims.lignes), list(m.dims.colonnes),
                                       t["wr"], t["br"], h2, m.k, x)
        hn = O.rmsnorm(x, nsortie, d, 1, m.eps)
        z = O.gemv_q8_0(wout, hn, None, m.vocab, d)
        assert np.abs(z_gpu - z).max() <= 1e-3 * np.abs(z).max(), f"step {pos}"
        assert int(np.argmax(z)) == int(jt.cpu().numpy()[0]), f"step {pos}"
        j = int(jt.cpu().numpy()[0])


# ---------------------------------------------------------------- against an fp64 evaluation

def test_contre_une_evaluation_f64(petit):
    """The model's logits against the same model evaluated in f64 on the host (oracle/modele_f64:
    the storage formats kept: Q8_0, MXFP4, the f16 KV cache): max|dz| <= 1e-4 max|z| and the same
    greedy token at every step."""
    from oracle.modele_f64 import ModeleF64

    m = petit
    m.choisir("compresse")
    ref = ModeleF64(m, kv16=True)
    lg, jt, _ = m.vues()
    j = 3
    for pos in range(24):  # past the sliding layers' ring of 16 cases
        m.pas(j, pos)
        torch.cuda.synchronize()
        z_gpu = lg.cpu().numpy().astype(np.float64)
        z = ref.pas(j, pos)
        assert np.abs(z_gpu - z).max() <= 1e-4 * np.abs(z).max(), f"step {pos}: {np.abs(z_gpu - z).max()}"
        assert int(np.argmax(z)) == int(jt.cpu().numpy()[0]), f"step {pos}"
        j = int(jt.cpu().numpy()[0])
