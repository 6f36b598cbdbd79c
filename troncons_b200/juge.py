"""The quality judge, the reference's trc-juge (moteur/crates/trc-juge): llama-perplexity's `.kld`
logit files read and written (kld.rs), every per-position figure (KL, first choice, NLL) and
the entry coding computed on the GPU over the C-ABI (`trc_juge_positions`, `trc_juge_coder`),
the summary statistics and the ABBA decision rule on the host (stats.rs, abba.rs).

Command line, the reference's `juge kl` and `juge comparer` (bin/juge.rs:239-296, 298-400):

    python -m troncons_b200.juge kl --base P.kld --test Q.kld [--fenetres N] [--csv c.csv] [--json j.json]
    python -m troncons_b200.juge comparer --verite V.kld --a A.kld --b B.kld [--fenetres N] [--json j.json]
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os
import struct
import sys
from dataclasses import asdict, dataclass

import numpy as np

from . import lib, verifier

MAGIE = b"_logits_"
_u32, _u64, _vp, _sz, _i32 = C.c_uint32, C.c_uint64, C.c_void_p, C.c_size_t, C.c_int

for _n, (_r, _a) in {
    "trc_juge_mots_par_entree": (_u64, [_u32]),
    "trc_juge_coder": (_i32, [_vp, _u32, _sz, _u32, _u32, _vp, _sz, _vp]),
    "trc_juge_positions": (_i32, [_vp, _sz, _vp, _sz, _u32, _vp, _sz, _u32, _u32, _vp, _sz, _vp]),
}.items():
    getattr(lib, _n).restype = _r
    getattr(lib, _n).argtypes = _a


class ErreurKld(ValueError):
    """A `.kld` file that is not one, truncated, or inconsistent with another."""


def mots_par_entree(n_vocab: int) -> int:
    """u16 words per entry (kld.rs:27-29), from the library."""
    return int(lib.trc_juge_mots_par_entree(n_vocab))


def positions_notees(n_ctx: int) -> range:
    """The scored positions of a window of n_ctx tokens: [n_ctx / 2, n_ctx - 1) (kld.rs:32-34)."""
    return range(n_ctx // 2, n_ctx - 1)


# ---------------------------------------------------------------- files (kld.rs:36-121, 188-235)

class FichierKld:
    """A `.kld` file opened for reading (kld.rs:36-121): header, tokens, then per window the
    entries of its scored positions."""

    def __init__(self, chemin: str):
        self.chemin = chemin
        taille = os.path.getsize(chemin)
        with open(chemin, "rb") as f:
            tete = f.read(20)
        if len(tete) < 20 or tete[:8] != MAGIE:
            raise ErreurKld(f"{chemin}: not a llama-perplexity logits file")
        self.n_ctx, self.n_vocab, self.n_chunk = struct.unpack("<Iii", tete[8:20])
        if self.n_ctx < 2 or self.n_vocab <= 0 or self.n_chunk < 0:
            raise ErreurKld(f"{chemin}: header n_ctx {self.n_ctx}, n_vocab {self.n_vocab}, n_chunk {self.n_chunk}")
        self.debut = 20 + 4 * self.n_ctx * self.n_chunk
        nv = mots_par_entree(self.n_vocab)
        attendu = self.debut + self.n_chunk * self.entrees_par_fenetre() * nv * 2
        if taille != attendu:
            raise ErreurKld(f"{chemin}: {taille} bytes instead of {attendu} (truncated file or another format)")
        self.jetons = np.fromfile(chemin, "<i4", self.n_ctx * self.n_chunk, offset=20).astype(np.uint32)

    ouvrir = classmethod(lambda cls, chemin: cls(chemin))

    def entrees_par_fenetre(self) -> int:
        return len(positions_notees(self.n_ctx))

    def fenetre(self, c: int) -> np.ndarray:
        """The entries of window c: u16[scored positions][nv]."""
        if not 0 <= c < self.n_chunk:
            raise IndexError(f"window {c} of {self.n_chunk}")
        nv = mots_par_entree(self.n_vocab)
        n = self.entrees_par_fenetre() * nv
        e = np.fromfile(self.chemin, "<u2", n, offset=self.debut + 2 * c * n)
        return e.reshape(self.entrees_par_fenetre(), nv)

    def jetons_fenetre(self, c: int) -> np.ndarray:
        return self.jetons[c * self.n_ctx:(c + 1) * self.n_ctx]


class EcrivainKld:
    """A `.kld` file being written (kld.rs:188-235); each row of logits is coded on the GPU."""

    def __init__(self, chemin: str, n_ctx: int, n_vocab: int, jetons):
        jetons = np.asarray(jetons, np.int64)
        if jetons.size % n_ctx != 0:
            raise ErreurKld(f"{jetons.size} tokens: not a multiple of n_ctx = {n_ctx}")
        self.n_vocab = n_vocab
        self.entrees_ecrites = 0
        self._f = open(chemin, "wb")
        self._f.write(MAGIE)
        self._f.write(struct.pack("<Iii", n_ctx, n_vocab, jetons.size // n_ctx))
        self._f.write(jetons.astype("<i4").tobytes())

    creer = classmethod(lambda cls, chemin, n_ctx, n_vocab, jetons: cls(chemin, n_ctx, n_vocab, jetons))

    def ecrire(self, logits, flux=None) -> None:
        """Rows of logits (a CUDA tensor or a host array, f32 or f64, [n_vocab] or [m][n_vocab]),
        coded on the GPU (coder) and appended."""
        e = coder(logits, flux=flux)
        self._f.write(e.cpu().numpy().view("<u2").tobytes())
        self.entrees_ecrites += e.shape[0]

    def finir(self) -> None:
        self._f.close()


def _sur_gpu(x, dtypes):
    import torch

    t = x if torch.is_tensor(x) else torch.from_numpy(np.ascontiguousarray(x))
    if t.dtype not in dtypes:
        raise TypeError(f"dtype {t.dtype}: expected one of {dtypes}")
    return t.cuda().contiguous()


def _flux(flux) -> int:
    import torch

    return int((flux or torch.cuda.current_stream()).cuda_stream)


def coder(logits, flux=None):
    """Entries of rows of logits (f32 or f64, [n_vocab] or [m][n_vocab]) coded on the GPU by the
    rule of kld::coder_entree: int16 CUDA tensor [m][nv] (the u16 words' bits)."""
    import torch

    t = _sur_gpu(logits, (torch.float32, torch.float64))
    if t.dim() == 1:
        t = t.unsqueeze(0)
    m, n = t.shape
    nv = mots_par_entree(n)
    sortie = torch.empty((m, nv), dtype=torch.int16, device=t.device)
    verifier(lib.trc_juge_coder(t.data_ptr(), int(t.dtype == torch.float64), t.numel() * t.element_size(), m, n,
                                sortie.data_ptr(), sortie.numel() * 2, _flux(flux)))
    return sortie


@dataclass
class Position:
    """One judged position (stats.rs:24-33)."""

    kl: float
    meme_premier: bool
    nll_q: float
    nll_p: float
    dp: float
    premier_p: int
    premier_q: int


class JugePosition(C.Structure):
    """trc_juge_position: 48 bytes."""

    _fields_ = [("kl", C.c_double), ("nll_q", C.c_double), ("nll_p", C.c_double), ("dp", C.c_double),
                ("premier_p", C.c_uint32), ("premier_q", C.c_uint32), ("meme_premier", C.c_uint32),
                ("suivant_valide", C.c_uint32)]


_POSITION = np.dtype([(n, "<f8" if t is C.c_double else "<u4") for n, t in JugePosition._fields_])
assert _POSITION.itemsize == C.sizeof(JugePosition) == 48


def positions(p, q, suivants, n_vocab: int, flux=None) -> np.ndarray:
    """Per-position figures of P (coded entries [m][nv]) against Q: coded entries [m][nv] (taken
    as log-probabilities, stats::position_decodee) or raw logits [m][n_vocab] f32 / f64
    (renormalised, stats::position); suivants[m] the next tokens. A structured array of m
    records (kl, nll_q, nll_p, dp, premier_p, premier_q, meme_premier, suivant_valide)."""
    import torch

    tp = _sur_gpu(np.asarray(p).view(np.int16) if not torch.is_tensor(p) else p.view(torch.int16), (torch.int16,))
    if torch.is_tensor(q):
        tq = q.view(torch.int16) if q.dtype in (torch.int16, torch.uint16) else q
        tq = _sur_gpu(tq, (torch.int16, torch.float32, torch.float64))
    else:
        qa = np.asarray(q)
        tq = _sur_gpu(qa.view(np.int16) if qa.dtype == np.uint16 else qa, (torch.int16, torch.float32, torch.float64))
    mode = {torch.int16: 0, torch.float32: 1, torch.float64: 2}[tq.dtype]
    tp = tp.unsqueeze(0) if tp.dim() == 1 else tp
    m = tp.shape[0]
    s = np.asarray(suivants, np.int64).reshape(-1)
    if s.size != m or (s < 0).any():
        raise ValueError(f"{s.size} next tokens for {m} positions, or a negative token")
    ts = torch.from_numpy(np.minimum(s, 0xFFFFFFFF).astype(np.uint32).view(np.int32)).cuda()
    sortie = torch.empty(m * _POSITION.itemsize, dtype=torch.uint8, device=tp.device)
    verifier(lib.trc_juge_positions(tp.data_ptr(), tp.numel() * 2, tq.data_ptr(), tq.numel() * tq.element_size(), mode,
                                    ts.data_ptr(), ts.numel() * 4, m, n_vocab, sortie.data_ptr(), sortie.numel(),
                                    _flux(flux)))
    r = sortie.cpu().numpy().view(_POSITION)
    if not r["suivant_valide"].all():
        raise ValueError(f"a next token is >= n_vocab = {n_vocab}")
    return r


def en_positions(r: np.ndarray) -> list:
    return [Position(float(x["kl"]), bool(x["meme_premier"]), float(x["nll_q"]), float(x["nll_p"]), float(x["dp"]),
                     int(x["premier_p"]), int(x["premier_q"])) for x in r]


# ---------------------------------------------------------------- statistics (stats.rs:87-177)

@dataclass
class Resume:
    n: int
    kl_moyenne: float
    kl_incertitude: float
    kl_mediane: float
    kl_p90: float
    kl_p99: float
    kl_p999: float
    kl_max: float
    kl_min: float
    meme_premier: float
    meme_premier_incertitude: float
    meme_premier_wilson95: tuple
    ppl_q: float
    ppl_p: float
    ln_rapport_ppl: float
    ln_rapport_ppl_incertitude: float
    dp_rms: float


def _moyenne_incertitude(v: np.ndarray) -> tuple:
    n = float(v.size)
    m = float(v.sum()) / n
    var = float((v * v).sum()) / n - m * m
    return m, (math.sqrt(var / (n - 1.0)) if var > 0.0 and n > 10.0 else 0.0)


def quantile(tries, f: float) -> float:
    """Linear interpolation between the sorted values of indices floor(f (n - 1)) and the next."""
    if f <= 0.0:
        return float(tries[0])
    if f >= 1.0:
        return float(tries[-1])
    p = f * (len(tries) - 1)
    i = int(p)
    r = p - i
    return float((1.0 - r) * tries[i] + r * tries[min(i + 1, len(tries) - 1)])


def wilson95(k: int, n: int) -> tuple:
    """Wilson's 95 % score interval (z = 1.959964) of k successes out of n."""
    z = 1.959963984540054
    p = k / n
    d = 1.0 + z * z / n
    c = (p + z * z / (2.0 * n)) / d
    h = z * math.sqrt(p * (1.0 - p) / n + z * z / (4.0 * n * n)) / d
    return (c - h, c + h)


def resumer(r) -> Resume:
    """The summary of judged positions (a `positions` array or a list of Position)."""
    if isinstance(r, np.ndarray):
        kl, mp, nq, np_, dp = (r["kl"].astype(np.float64), r["meme_premier"].astype(bool), r["nll_q"], r["nll_p"],
                               r["dp"])
    else:
        kl = np.array([x.kl for x in r])
        mp = np.array([x.meme_premier for x in r])
        nq, np_, dp = (np.array([x.nll_q for x in r]), np.array([x.nll_p for x in r]), np.array([x.dp for x in r]))
    n = kl.size
    if n == 0:
        raise ValueError("no position to summarise")
    kl_m, kl_i = _moyenne_incertitude(kl)
    tries = np.sort(kl)
    med = 0.5 * (tries[n // 2] + tries[n // 2 - 1]) if n % 2 == 0 else tries[n // 2]
    k = int(mp.sum())
    top = k / n
    lq, lq_i = _moyenne_incertitude(nq)
    lp, lp_i = _moyenne_incertitude(np_)
    cov = (float((nq * np_).sum()) / n - lq * lp) / (n - 1.0) if n >= 10 else 0.0
    with np.errstate(divide="ignore", invalid="ignore"):
        inc_top = float(np.sqrt(np.float64(top * (1.0 - top)) / np.float64(n - 1.0)))
    return Resume(n, kl_m, kl_i, float(med), quantile(tries, 0.90), quantile(tries, 0.99), quantile(tries, 0.999),
                  float(tries[-1]), float(tries[0]), top, inc_top, wilson95(k, n), math.exp(lq), math.exp(lp), lq - lp,
                  math.sqrt(max(lq_i * lq_i + lp_i * lp_i - 2.0 * cov, 0.0)), math.sqrt(float((dp * dp).sum()) / n))


# ---------------------------------------------------------------- ABBA series (abba.rs:1-40)

@dataclass
class Verdict:
    moyenne_a: float
    moyenne_b: float
    ecart_relatif: float
    plus_grand_bruit: float
    seuil: float
    reel: bool


def decider(series) -> Verdict:
    """Series A1 B1 B2 A2: the noise of a configuration is |X1 - X2| / mean; a difference between A
    and B is real only when |mean(B) - mean(A)| / mean(A) exceeds both twice the largest noise and
    3 %."""
    if not series:
        raise ValueError("no series")
    bruit, sa, sb = 0.0, 0.0, 0.0
    for a1, b1, b2, a2 in series:
        bruit = max(bruit, abs(a1 - a2) / ((a1 + a2) / 2.0), abs(b1 - b2) / ((b1 + b2) / 2.0))
        sa += a1 + a2
        sb += b1 + b2
    n = 2.0 * len(series)
    ma, mb = sa / n, sb / n
    ecart = (mb - ma) / ma
    seuil = max(2.0 * bruit, 0.03)
    return Verdict(ma, mb, ecart, bruit, seuil, abs(ecart) > seuil)


# ---------------------------------------------------------------- the two judgements

def _exp_rust(x: float, prec: int) -> str:
    """`{:.Ne}` of Rust: mantissa, 'e', exponent without padding or '+'."""
    if math.isnan(x):
        return "NaN"
    if math.isinf(x):
        return "inf" if x > 0 else "-inf"
    m, e = f"{x:.{prec}e}".split("e")
    return f"{m}e{int(e)}"


def _fix_rust(x: float, prec: int) -> str:
    return "NaN" if math.isnan(x) else (("inf" if x > 0 else "-inf") if math.isinf(x) else f"{x:.{prec}f}")


def _fenetres(fichiers, fenetres):
    n = min(f.n_chunk for f in fichiers)
    n = n if fenetres is None else min(fenetres, n)
    for f in fichiers[1:]:
        if f.n_vocab != fichiers[0].n_vocab or f.n_ctx != fichiers[0].n_ctx:
            raise ErreurKld(f"incompatible files: n_vocab {f.n_vocab}/{fichiers[0].n_vocab}, "
                            f"n_ctx {f.n_ctx}/{fichiers[0].n_ctx}")
    for c in range(n):
        for f in fichiers[1:]:
            if not np.array_equal(f.jetons_fenetre(c), fichiers[0].jetons_fenetre(c)):
                raise ErreurKld(f"window {c}: the tokens differ between the files")
    return n


def kl(base: str, test: str, fenetres: int | None = None, csv: str | None = None, json_chemin: str | None = None,
       flux=None) -> dict:
    """`juge kl` (bin/juge.rs:239-296): KL(P || Q) position by position, Q decoded from its own
    16-bit coding and taken as is."""
    p, q = FichierKld(base), FichierKld(test)
    n_fen = _fenetres([p, q], fenetres)
    notees = positions_notees(p.n_ctx)
    toutes = []
    lignes = ["fenetre,position,kl,meme_premier,nll_test,nll_base,dp,premier_base,premier_test"]
    for c in range(n_fen):
        jet = p.jetons_fenetre(c)
        r = positions(p.fenetre(c), q.fenetre(c), jet[notees.start + 1:notees.stop + 1], p.n_vocab, flux=flux)
        for k, x in enumerate(r):
            lignes.append(f"{c},{notees.start + k},{_exp_rust(float(x['kl']), 9)},{int(x['meme_premier'])},"
                          f"{_fix_rust(float(x['nll_q']), 6)},{_fix_rust(float(x['nll_p']), 6)},"
                          f"{_exp_rust(float(x['dp']), 6)},{int(x['premier_p'])},{int(x['premier_q'])}")
        toutes.append(r)
    res = {"outil": "juge kl", "fenetres": n_fen, "resume": asdict(resumer(np.concatenate(toutes)))}
    if json_chemin:
        with open(json_chemin, "w") as f:
            json.dump(res, f, indent=2)
    if csv:
        with open(csv, "w") as f:
            f.write("\n".join(lignes) + "\n")
    return res


def comparer(verite: str, a: str, b: str, fenetres: int | None = None, json_chemin: str | None = None,
             flux=None) -> dict:
    """`juge comparer` (bin/juge.rs:298-400): engines A and B against the same truth V on the same
    positions; paired differences d = kl_B - kl_A and e = t_B - t_A; literal verdicts (mean KL_B <=
    mean KL_A, first-choice rate B >= A) and statistical ones (d <= 2 sigma(d), e >= -2 sigma(e))."""
    v, fa, fb = FichierKld(verite), FichierKld(a), FichierKld(b)
    n_fen = _fenetres([v, fa, fb], fenetres)
    notees = positions_notees(v.n_ctx)
    pa, pb, ia, ib = [], [], [], []
    for c in range(n_fen):
        ev, ea, eb = v.fenetre(c), fa.fenetre(c), fb.fenetre(c)
        s = v.jetons_fenetre(c)[notees.start + 1:notees.stop + 1]
        pa.append(positions(ev, ea, s, v.n_vocab, flux=flux))
        pb.append(positions(ev, eb, s, v.n_vocab, flux=flux))
        ia.append(positions(ea, ev, s, v.n_vocab, flux=flux)["kl"])
        ib.append(positions(eb, ev, s, v.n_vocab, flux=flux)["kl"])
    pa, pb, ia, ib = np.concatenate(pa), np.concatenate(pb), np.concatenate(ia), np.concatenate(ib)
    m = float(pa.size)

    def apparie(x):
        moy = float(x.sum()) / m
        var = max(float((x * x).sum()) / m - moy * moy, 0.0)
        return moy, math.sqrt(var / (m - 1.0))

    d_kl, sd_kl = apparie(pb["kl"] - pa["kl"])
    d_inv, sd_inv = apparie(ib - ia)
    d_top, sd_top = apparie(pb["meme_premier"].astype(np.float64) - pa["meme_premier"].astype(np.float64))
    ra, rb = resumer(pa), resumer(pb)
    res = {
        "outil": "juge comparer", "fenetres": n_fen, "positions": int(pa.size),
        "a_contre_verite": asdict(ra), "b_contre_verite": asdict(rb),
        "kl_inverse": {"a": float(ia.mean()), "b": float(ib.mean()), "difference": d_inv, "ecart_type": sd_inv},
        "apparie": {"kl_difference_b_moins_a": d_kl, "kl_ecart_type": sd_kl,
                    "premier_difference_b_moins_a": d_top, "premier_ecart_type": sd_top},
        "verdicts": {"litteral_kl": rb.kl_moyenne <= ra.kl_moyenne, "litteral_premier": rb.meme_premier >= ra.meme_premier,
                     "statistique_kl": d_kl <= 2.0 * sd_kl, "statistique_premier": d_top >= -2.0 * sd_top},
    }
    if json_chemin:
        with open(json_chemin, "w") as f:
            json.dump(res, f, indent=2)
    return res


def _args(brut):
    mots, i = {}, 0
    while i < len(brut):
        if brut[i].startswith("--") and i + 1 < len(brut) and not brut[i + 1].startswith("--"):
            mots[brut[i][2:]] = brut[i + 1]
            i += 2
        else:
            i += 1
    return mots


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv or argv[0] not in ("kl", "comparer"):
        print("usage: python -m troncons_b200.juge <kl|comparer> ...", file=sys.stderr)
        return 2
    a = _args(argv[1:])
    fen = int(a["fenetres"]) if "fenetres" in a else None
    if argv[0] == "kl":
        r = kl(a["base"], a["test"], fen, a.get("csv"), a.get("json"))
    else:
        r = comparer(a["verite"], a["a"], a["b"], fen, a.get("json"))
    print(json.dumps(r, indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
