"""CPU: the quality judge without a GPU.

- the oracle (oracle/juge_ref.py) pinned by the reference's own known-answer tests: an entry's
  round trip within half a step (kld.rs:192-217), KL of a distribution against itself below the
  step and positive against another (stats.rs:183-201), a decoded entry against itself exactly 0
  and its renormalisation positive (stats.rs:203-221), Wilson's interval of 95 / 100
  (stats.rs:223-229), the ABBA rule's three cases (abba.rs:46-52);
- the host mirror (troncons_b200/juge.py): summary, quantiles, Wilson, ABBA against the oracle;
  `.kld` files written by the oracle read back (header, tokens, entries), truncated and foreign
  files refused; Rust's number formats in the CSV."""
import math
import struct

import numpy as np
import pytest

import oracle.juge_ref as R
import troncons_b200.juge as J


def test_aller_retour_d_une_entree():
    n = 1001
    logits = [((i * 37) % 101) * 0.2 - 10.0 for i in range(n)]
    e = R.Entree(R.coder_entree(logits), n)
    mx = max(logits)
    lse = math.log(sum(math.exp(l - mx) for l in logits))
    for i in range(n):
        if logits[i] > mx - 16.0:
            assert abs(float(e.log_p(i)) - (logits[i] - mx - lse)) < 1.3e-4, i


def test_kl_nulle_contre_soi_meme_et_positive_sinon():
    n = 500
    a = [((i * 13) % 37) * 0.3 for i in range(n)]
    e = R.Entree(R.coder_entree(a), n)
    soi = R.position(e, a, n, 3)
    assert abs(soi["kl"]) < float(e.pas) and soi["meme_premier"]
    b = [a[i] + ((i * 7) % 5) * 0.4 for i in range(n)]
    assert R.position(e, b, n, 3)["kl"] > 1e-3


def test_entree_decodee_contre_elle_meme():
    n = 20_000
    a = [30.0 if i == 7 else 12.0 - (i % 23) for i in range(n)]
    e = R.Entree(R.coder_entree(a), n)
    assert R.position_decodee(e, e, n, 7)["kl"] == 0.0
    assert R.position(e, e.tous().astype(np.float64), n, 7)["kl"] > 1e-4


def test_wilson_connu():
    for f in (R.wilson95, J.wilson95):
        a, b = f(95, 100)
        assert abs(a - 0.8882) < 1e-3 and abs(b - 0.9785) < 1e-3


def test_abba():
    cas = [([(10.0, 11.0, 11.0, 10.2), (10.1, 11.1, 10.9, 10.0)], True), ([(10.0, 10.25, 10.25, 10.0)], False),
           ([(10.0, 10.8, 10.8, 10.5)], False)]
    for series, reel in cas:
        o, p = R.decider(series), J.decider(series)
        assert o["reel"] is reel and p.reel is reel
        assert (p.moyenne_a, p.moyenne_b, p.ecart_relatif, p.plus_grand_bruit, p.seuil) == (
            o["moyenne_a"], o["moyenne_b"], o["ecart_relatif"], o["plus_grand_bruit"], o["seuil"])
    with pytest.raises(ValueError):
        J.decider([])


def _positions_oracle(rng, m, n):
    ps = []
    for _ in range(m):
        a = rng.standard_normal(n) * 3
        b = a + rng.standard_normal(n) * 0.05
        ps.append(R.position(R.Entree(R.coder_entree(a), n), b, n, int(rng.integers(n))))
    return ps


@pytest.mark.parametrize("m", [1, 2, 9, 10, 37])
def test_resume_contre_l_oracle(m):
    rng = np.random.default_rng(m)
    ps = _positions_oracle(rng, m, 300)
    o = R.resumer(ps)
    r = J.resumer([J.Position(p["kl"], p["meme_premier"], p["nll_q"], p["nll_p"], p["dp"], p["premier_p"],
                              p["premier_q"]) for p in ps])
    for k, v in o.items():
        w = getattr(r, k)
        if isinstance(v, tuple):
            assert np.allclose(w, v, rtol=1e-9, atol=0), k
        elif isinstance(v, float) and math.isnan(v):
            assert math.isnan(w), k
        else:
            # numpy's pairwise sums against the reference's serial ones; the uncertainties are
            # differences of such sums (sum x^2 / n - mean^2)
            assert w == pytest.approx(v, rel=1e-9, abs=1e-15), k


def test_quantiles():
    t = sorted(np.random.default_rng(1).random(101))
    for f in (-1.0, 0.0, 0.1, 0.5, 0.9, 0.99, 0.999, 1.0, 2.0):
        assert J.quantile(np.array(t), f) == R.quantile(t, f)


def _fichier(tmp_path, n_ctx=12, n_vocab=37, fenetres=3, graine=0):
    rng = np.random.default_rng(graine)
    jetons = rng.integers(0, n_vocab, n_ctx * fenetres)
    lignes = [rng.standard_normal(n_vocab) * 4 for _ in range(fenetres * len(R.positions_notees(n_ctx)))]
    chemin = str(tmp_path / f"f{graine}.kld")
    R.ecrire_kld(chemin, n_ctx, n_vocab, jetons, lignes)
    return chemin, jetons, lignes


@pytest.mark.parametrize("n_vocab", [37, 40])
def test_lecture_d_un_fichier(tmp_path, n_vocab):
    chemin, jetons, lignes = _fichier(tmp_path, n_vocab=n_vocab)
    f = J.FichierKld(chemin)
    assert (f.n_ctx, f.n_vocab, f.n_chunk) == (12, n_vocab, 3)
    assert f.entrees_par_fenetre() == 5 and np.array_equal(f.jetons, jetons)
    for c in range(3):
        assert np.array_equal(f.jetons_fenetre(c), jetons[12 * c:12 * c + 12])
        e = f.fenetre(c)
        assert e.shape == (5, J.mots_par_entree(n_vocab))
        for k in range(5):
            assert np.array_equal(e[k], R.coder_entree(lignes[5 * c + k]))
    with pytest.raises(IndexError):
        f.fenetre(3)


def test_fichiers_refuses(tmp_path):
    chemin, _, _ = _fichier(tmp_path)
    b = open(chemin, "rb").read()
    (tmp_path / "court.kld").write_bytes(b[:-2])
    with pytest.raises(J.ErreurKld, match="bytes instead of"):
        J.FichierKld(str(tmp_path / "court.kld"))
    (tmp_path / "autre.kld").write_bytes(b"_logitz_" + b[8:])
    with pytest.raises(J.ErreurKld, match="not a llama-perplexity"):
        J.FichierKld(str(tmp_path / "autre.kld"))
    (tmp_path / "tete.kld").write_bytes(b[:8] + struct.pack("<Iii", 1, 37, 0))
    with pytest.raises(J.ErreurKld):
        J.FichierKld(str(tmp_path / "tete.kld"))
    with pytest.raises(J.ErreurKld, match="not a multiple"):
        J.EcrivainKld(str(tmp_path / "x.kld"), 12, 37, np.zeros(13))


def test_fenetres_incompatibles(tmp_path):
    a, _, _ = _fichier(tmp_path, graine=0)
    b, _, _ = _fichier(tmp_path, graine=1)
    with pytest.raises(J.ErreurKld, match="tokens differ"):
        J._fenetres([J.FichierKld(a), J.FichierKld(b)], None)
    c, _, _ = _fichier(tmp_path, n_vocab=40, graine=2)
    with pytest.raises(J.ErreurKld, match="incompatible"):
        J._fenetres([J.FichierKld(a), J.FichierKld(c)], None)


def test_formats_rust():
    assert J._exp_rust(1.2345e-5, 9) == "1.234500000e-5"
    assert J._exp_rust(0.0, 9) == "0.000000000e0"
    assert J._exp_rust(-3.5e12, 6) == "-3.500000e12"
    assert J._exp_rust(float("nan"), 6) == "NaN" and J._exp_rust(float("inf"), 6) == "inf"
    assert J._fix_rust(2.5, 6) == "2.500000"


def test_ligne_de_commande_usage(capsys):
    """The command line names its two sub-commands and refuses anything else (exit status 2)."""
    assert J.main([]) == 2
    assert J.main(["reference"]) == 2
    assert "kl|comparer" in capsys.readouterr().err
    assert J._args(["--base", "p.kld", "--test", "q.kld", "--fenetres", "3", "--drapeau"]) == {
        "base": "p.kld", "test": "q.kld", "fenetres": "3"}
