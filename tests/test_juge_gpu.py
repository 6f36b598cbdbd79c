"""GPU: the quality judge (csrc/juge.cu over the C-ABI, troncons_b200.juge) against the oracle
(oracle/juge_ref.py, the reference's trc-juge restated).

- entry coding (trc_juge_coder, kld::coder_entree): codes and step bit for bit, log_p_min within
  one f32 ulp (the log-sum-exp is summed in another order), f32 and f64 logits, odd and even
  vocabularies up to gpt-oss's 201,088, flat rows (step 0), rows spread past max - 16;
- judged positions (trc_juge_positions): KL within 1e-9 relative (f64 sums in another order),
  NLLs and dp within 1e-12, first choices exact (ties to the first index), for Q coded (not
  renormalised) and raw f32 / f64 logits (renormalised); a coded entry against itself gives a KL
  of exactly 0 (stats.rs:203-221);
- files and judgements: entries written through the GPU read back equal to the oracle's; `kl` of
  a file against itself is 0 with every first choice kept; `comparer` with A = B gives zero
  paired differences and all four verdicts, a perturbed B fails them;
- the whole model judged: the engine's logits from the .trc parts and from the raw parts against
  the f64 truth of the same weights (oracle/modele_f64, KV stored in f16 as the engine does),
  through `.kld` files: compressed and raw give identical entries (KL exactly 0 between them);
  against the truth, the KL of the coded entries is the 16-bit coding's resolution and every
  first choice is kept; the engine's raw logits against the truth's entries differ from the
  truth's own raw logits by less than 1e-9 in KL at every position, over windows that wrap the
  sliding layers' KV ring."""
import numpy as np
import pytest

import oracle.juge_ref as R

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _lignes(rng, m, n, f64):
    x = rng.standard_normal((m, n)) * 4
    if m > 1:
        x[1] = 0.75  # flat: step 0, every code 0
    if m > 2:
        x[2, ::3] -= 40.0  # a third of the row below max - 16
    return x if f64 else x.astype(np.float32)


@pytest.mark.parametrize("n", [1, 7, 1000, 4097, 201088])
@pytest.mark.parametrize("f64", [False, True])
def test_coder_contre_l_oracle(n, f64):
    import troncons_b200.juge as J

    rng = np.random.default_rng(n + f64)
    m = 2 if n == 201088 else 4
    x = _lignes(rng, m, n, f64)
    e = J.coder(torch.from_numpy(x).cuda()).cpu().numpy().view(np.uint16)
    assert e.shape == (m, R.mots_par_entree(n))
    for i in range(m):
        o = R.coder_entree(x[i].astype(np.float64))
        assert np.array_equal(e[i, 4:], o[4:]), i
        assert e[i, 0] == o[0] and e[i, 1] == o[1], i
        lpm_g = int(e[i, 2]) | (int(e[i, 3]) << 16)
        lpm_o = int(o[2]) | (int(o[3]) << 16)
        assert abs(lpm_g - lpm_o) <= 1, i


def _comparer(r, o):
    assert r["premier_p"] == o["premier_p"] and r["premier_q"] == o["premier_q"]
    assert bool(r["meme_premier"]) == o["meme_premier"]
    assert r["kl"] == pytest.approx(o["kl"], rel=1e-9, abs=1e-15)
    for k in ("nll_q", "nll_p", "dp"):
        assert r[k] == pytest.approx(o[k], rel=1e-12, abs=1e-15), k


@pytest.mark.parametrize("n", [7, 1001, 201088])
@pytest.mark.parametrize("mode", ["code", "f32", "f64"])
def test_positions_contre_l_oracle(n, mode):
    import troncons_b200.juge as J

    rng = np.random.default_rng(3 * n + len(mode))
    m = 2 if n == 201088 else 3
    a = rng.standard_normal((m, n)) * 3
    b = a + rng.standard_normal((m, n)) * 0.3
    a[0, [1, 4]] = a[0].max() + 1.0  # a tie for the first choice of P: the first index wins
    b[-1, [2, 5]] = b[-1].max() + 1.0
    ep = J.coder(torch.from_numpy(a).cuda())
    if mode == "code":
        q = J.coder(torch.from_numpy(b).cuda())
    else:
        q = torch.from_numpy(b.astype(np.float32) if mode == "f32" else b).cuda()
    s = rng.integers(0, n, m)
    r = J.positions(ep, q, s, n)
    ep_h = ep.cpu().numpy().view(np.uint16)
    for i in range(m):
        p = R.Entree(ep_h[i], n)
        if mode == "code":
            o = R.position_decodee(p, R.Entree(q.cpu().numpy().view(np.uint16)[i], n), n, int(s[i]))
        else:
            o = R.position(p, q.cpu().numpy()[i].astype(np.float64), n, int(s[i]))
        _comparer(r[i], o)
    assert r[0]["premier_p"] == 1


def test_entree_contre_elle_meme():
    import troncons_b200.juge as J

    n = 20_000
    a = np.array([30.0 if i == 7 else 12.0 - (i % 23) for i in range(n)])
    e = J.coder(torch.from_numpy(a).cuda())
    r = J.positions(e, e, [7], n)
    assert r[0]["kl"] == 0.0 and r[0]["meme_premier"] == 1
    renorm = J.positions(e, torch.from_numpy(R.Entree(e.cpu().numpy().view(np.uint16)[0], n).tous()).cuda(), [7], n)
    assert renorm[0]["kl"] > 1e-4


def test_suivant_hors_vocabulaire():
    import troncons_b200.juge as J

    e = J.coder(torch.zeros(2, 10, dtype=torch.float32, device="cuda"))
    with pytest.raises(ValueError, match="n_vocab"):
        J.positions(e, e, [3, 10], 10)
    with pytest.raises(ValueError):
        J.positions(e, e, [3], 10)


def _ecrire(chemin, n_ctx, jetons, lignes):
    import troncons_b200.juge as J

    w = J.EcrivainKld(chemin, n_ctx, lignes.shape[-1], jetons)
    for c in range(lignes.shape[0]):
        w.ecrire(torch.from_numpy(lignes[c]).cuda())
    w.finir()


def test_fichiers_et_jugements(tmp_path):
    import troncons_b200.juge as J

    rng = np.random.default_rng(11)
    n_ctx, n, fen = 16, 3001, 3
    notees = len(J.positions_notees(n_ctx))
    jetons = rng.integers(0, n, n_ctx * fen)
    v = rng.standard_normal((fen, notees, n)) * 3
    a = v + rng.standard_normal(v.shape) * 0.05
    b = v + rng.standard_normal(v.shape) * 0.8
    for nom, x in (("v", v), ("a", a), ("b", b)):
        _ecrire(str(tmp_path / f"{nom}.kld"), n_ctx, jetons, x)
    f = J.FichierKld(str(tmp_path / "v.kld"))
    assert f.n_chunk == fen and np.array_equal(f.jetons, jetons)
    for c in range(fen):
        e = f.fenetre(c)
        for k in range(notees):
            o = R.coder_entree(v[c, k])
            assert np.array_equal(e[k, 4:], o[4:]) and np.array_equal(e[k, :2], o[:2])
    soi = J.kl(str(tmp_path / "v.kld"), str(tmp_path / "v.kld"), csv=str(tmp_path / "p.csv"))
    assert soi["resume"]["kl_max"] == 0.0 and soi["resume"]["meme_premier"] == 1.0
    assert soi["resume"]["n"] == fen * notees
    lignes = open(tmp_path / "p.csv").read().splitlines()
    assert len(lignes) == 1 + fen * notees and lignes[1].split(",")[2] == "0.000000000e0"
    pareil = J.comparer(str(tmp_path / "v.kld"), str(tmp_path / "a.kld"), str(tmp_path / "a.kld"))
    assert pareil["apparie"]["kl_difference_b_moins_a"] == 0.0 and all(pareil["verdicts"].values())
    pire = J.comparer(str(tmp_path / "v.kld"), str(tmp_path / "a.kld"), str(tmp_path / "b.kld"))
    assert pire["apparie"]["kl_difference_b_moins_a"] > 0
    assert not pire["verdicts"]["litteral_kl"] and not pire["verdicts"]["statistique_kl"]
    # the summary against the oracle's, positions recomputed by the oracle
    ps = []
    for c in range(fen):
        ev, ea = f.fenetre(c), J.FichierKld(str(tmp_path / "a.kld")).fenetre(c)
        for k in range(notees):
            ps.append(R.position_decodee(R.Entree(ev[k], n), R.Entree(ea[k], n), n,
                                         int(jetons[c * n_ctx + n_ctx // 2 + k + 1])))
    o = R.resumer(ps)
    assert pareil["a_contre_verite"]["kl_moyenne"] == pytest.approx(o["kl_moyenne"], rel=1e-9)
    assert pareil["a_contre_verite"]["meme_premier"] == o["meme_premier"]


@pytest.fixture(scope="module")
def petit():
    import troncons_b200.modele as M

    return M.Modele(couches=2, d=256, tetes=8, tetes_kv=2, experts=8, k=4, vocab=512, contexte=64, ffn=256,
                    fenetre=16, graine=5, compresse=True, brut=True)


def test_modele_juge(petit, tmp_path):
    import troncons_b200.juge as J
    from oracle.modele_f64 import ModeleF64

    m = petit
    n_ctx, fen = 24, 2
    notees = J.positions_notees(n_ctx)
    jetons = np.random.default_rng(9).integers(0, m.vocab, n_ctx * fen)
    # the truth keeps the engine's f16 KV storage: with f64 keys and values, the f16 rounding alone
    # swaps two near-tied routed experts at one of these positions (top-k routing is discontinuous)
    verite = ModeleF64(m, kv16=True)
    lignes = {"verite": [], "compresse": [], "brut": []}
    for c in range(fen):
        verite.reinitialiser()
        w = jetons[c * n_ctx:(c + 1) * n_ctx]
        for t in range(n_ctx - 1):
            z = verite.pas(int(w[t]), t)
            if t in notees:
                lignes["verite"].append(z)
    for actifs in ("compresse", "brut"):
        m.choisir(actifs)
        lg, _, _ = m.vues()
        for c in range(fen):
            m.choisir(actifs)  # clears the KV caches
            lg, _, _ = m.vues()
            w = jetons[c * n_ctx:(c + 1) * n_ctx]
            for t in range(n_ctx - 1):
                m.pas(int(w[t]), t)
                if t in notees:
                    lignes[actifs].append(lg.clone())
    for nom, l in lignes.items():
        x = np.stack(l) if nom == "verite" else torch.stack(l).cpu().numpy()
        _ecrire(str(tmp_path / f"{nom}.kld"), n_ctx, jetons, x.reshape(fen, len(notees), m.vocab))
    entre = J.kl(str(tmp_path / "compresse.kld"), str(tmp_path / "brut.kld"))
    assert entre["resume"]["kl_max"] == 0.0 and entre["resume"]["meme_premier"] == 1.0
    # both sides coded on 16 bits (log p to within pas / 2, pas <= 16 / 65535)
    contre = J.kl(str(tmp_path / "verite.kld"), str(tmp_path / "compresse.kld"))
    assert contre["resume"]["n"] == fen * len(notees)
    assert contre["resume"]["kl_moyenne"] < 1e-6 and contre["resume"]["meme_premier"] == 1.0
    c = J.comparer(str(tmp_path / "verite.kld"), str(tmp_path / "compresse.kld"), str(tmp_path / "brut.kld"))
    assert c["apparie"]["kl_difference_b_moins_a"] == 0.0 and all(c["verdicts"].values())
    # the engine's own error: its raw logits (renormalised) against the truth's entries, beside the
    # truth's raw logits against its own entries (the coding floor)
    ev = J.FichierKld(str(tmp_path / "verite.kld"))
    s = np.concatenate([ev.jetons_fenetre(w)[notees.start + 1:notees.stop + 1] for w in range(fen)])
    pv = np.concatenate([ev.fenetre(w) for w in range(fen)])
    plancher = J.positions(pv, np.stack(lignes["verite"]), s, m.vocab)
    moteur = J.positions(pv, torch.stack(lignes["compresse"]), s, m.vocab)
    ecart = np.abs(moteur["kl"] - plancher["kl"])
    print("model vs f64 truth: coded", {k: contre["resume"][k] for k in ("kl_moyenne", "kl_max", "meme_premier")},
          "raw engine KL", float(moteur["kl"].mean()), "coding floor", float(plancher["kl"].mean()),
          "max |engine - floor|", float(ecart.max()))
    assert (moteur["meme_premier"] == 1).all()
    assert ecart.max() < 1e-9
