"""Test infrastructure only (a checker, never on the product path): a plain-Python restatement of
the reference's quality judge, trc-juge, to check troncons_b200's judge (csrc/juge.cu and
troncons_b200/juge.py):

- the `.kld` logit entry of llama-perplexity and its coding, moteur/crates/trc-juge/src/kld.rs:
  1-16 (format), 27-34 (sizes), 126-143 (decoding), 148-186 (coding);
- one judged position, stats.rs:36-85 (`position`, `position_decodee`, `position_avec`);
- the summary, stats.rs:87-177 (`Resume`, `moyenne_incertitude`, `quantile`, `wilson95`,
  `resumer`);
- the ABBA decision rule, abba.rs:17-40.

Every loop is the reference's, in its order, with Python floats (IEEE f64) and numpy.float32 for
the f32 steps. Pinned by the reference's own known-answer tests (kld.rs:192-217, stats.rs:
179-233, abba.rs:42-52), restated in tests/test_juge_cpu.py."""
from __future__ import annotations

import math
import struct

import numpy as np

MAGIE = b"_logits_"


def mots_par_entree(n_vocab: int) -> int:
    """kld.rs:27-29."""
    return 2 * ((n_vocab + 1) // 2) + 4


def positions_notees(n_ctx: int) -> range:
    """kld.rs:32-34: the scored positions of a window."""
    return range(n_ctx // 2, n_ctx - 1)


def _f32(x: float) -> np.float32:
    return np.float32(x)


def _ln(x: float) -> float:
    """f64::ln: -inf at 0, NaN below 0 or at NaN."""
    if math.isnan(x) or x < 0:
        return math.nan
    return -math.inf if x == 0 else math.log(x)


def coder_entree(logits) -> np.ndarray:
    """kld.rs:148-186: one row of f64 logits -> nv u16 words."""
    n = len(logits)
    mx, mn = -math.inf, math.inf
    for l in logits:
        l = float(l)
        if not math.isnan(l):  # f64::max / f64::min ignore a NaN
            mx, mn = max(mx, l), min(mn, l)
    mn = max(mn, mx - 16.0)
    somme = 0.0
    for l in logits:
        somme += math.exp(float(l) - mx)
    lse = _ln(somme)
    log_p_min = _f32(mn - mx - lse)
    pas = _f32((mx - mn) / 65535.0)
    sortie = np.zeros(mots_par_entree(n), np.uint16)
    pb = int(np.array(pas, np.float32).view(np.uint32))
    mb = int(np.array(log_p_min, np.float32).view(np.uint32))
    sortie[0], sortie[1], sortie[2], sortie[3] = pb & 0xFFFF, pb >> 16, mb & 0xFFFF, mb >> 16
    if pas > 0:
        inv = 1.0 / float(pas)
        for i in range(n):
            l = float(logits[i])
            if l > mn:
                v = (l - mn) * inv
                r = math.floor(v + 0.5) if v >= 0 else -math.floor(-v + 0.5)  # f64::round: half away from 0
                sortie[4 + i] = int(min(max(r, 0.0), 65535.0))
    return sortie


class Entree:
    """kld.rs:126-143: log p_i = pas * code_i + log_p_min, in f32 (product and sum rounded apart)."""

    def __init__(self, mots, n_vocab: int):
        m = np.asarray(mots, np.uint16)
        self.pas = np.array(int(m[0]) | (int(m[1]) << 16), np.uint32).view(np.float32)[()]
        self.log_p_min = np.array(int(m[2]) | (int(m[3]) << 16), np.uint32).view(np.float32)[()]
        self.codes = m[4:4 + n_vocab]

    def log_p(self, i: int) -> np.float32:
        return np.float32(np.float32(self.pas * np.float32(int(self.codes[i]))) + self.log_p_min)

    def tous(self) -> np.ndarray:
        """Every log p_i (vectorised, the same f32 operations)."""
        return ((self.pas * self.codes.astype(np.float32)).astype(np.float32) + self.log_p_min).astype(np.float32)


def position_avec(p: Entree, q, n: int, suivant: int, normaliser: bool) -> dict:
    """stats.rs:41-85. `q`: f64 values (raw logits, or a decoded entry's log-probabilities)."""
    lp_tous = p.tous().astype(np.float64)
    qv = [float(v) for v in q]
    max_q, imax_q = -math.inf, 0
    for i in range(n):
        if qv[i] > max_q:
            max_q, imax_q = qv[i], i
    if normaliser:
        s = 0.0
        for i in range(n):
            s += math.exp(qv[i] - max_q)
        lse_q = max_q + _ln(s)
    else:
        lse_q = 0.0
    kl, imax_p, lp_max = 0.0, 0, -math.inf
    for i in range(n):
        lp = float(lp_tous[i])
        if lp > lp_max:
            lp_max, imax_p = lp, i
        if lp > -16.0:
            kl += math.exp(lp) * (lp - (qv[i] - lse_q))
    nll_q = lse_q - qv[suivant]
    nll_p = -float(lp_tous[suivant])
    dp = math.exp(-nll_q) - math.exp(-nll_p)
    return {"kl": kl, "meme_premier": imax_p == imax_q, "nll_q": nll_q, "nll_p": nll_p, "dp": dp,
            "premier_p": imax_p, "premier_q": imax_q}


def position(p: Entree, q, n: int, suivant: int) -> dict:
    """stats.rs:36-38: Q raw logits, renormalised."""
    return position_avec(p, q, n, suivant, True)


def position_decodee(p: Entree, q: Entree, n: int, suivant: int) -> dict:
    """stats.rs:33-39: Q a decoded entry, not renormalised."""
    return position_avec(p, q.tous().astype(np.float64), n, suivant, False)


def moyenne_incertitude(v) -> tuple:
    """stats.rs:110-117."""
    v = list(v)
    n = float(len(v))
    s = 0.0
    for x in v:
        s += x
    s2 = 0.0
    for x in v:
        s2 += x * x
    m = s / n
    var = s2 / n - m * m
    return m, (math.sqrt(var / (n - 1.0)) if var > 0.0 and n > 10.0 else 0.0)


def quantile(tries, f: float) -> float:
    """stats.rs:119-130."""
    if f <= 0.0:
        return tries[0]
    if f >= 1.0:
        return tries[-1]
    p = f * (len(tries) - 1)
    i = int(p)
    r = p - i
    return (1.0 - r) * tries[i] + r * tries[min(i + 1, len(tries) - 1)]


def wilson95(k: int, n: int) -> tuple:
    """stats.rs:132-142."""
    z = 1.959963984540054
    k, n = float(k), float(n)
    p = k / n
    d = 1.0 + z * z / n
    c = (p + z * z / (2.0 * n)) / d
    h = z * math.sqrt(p * (1.0 - p) / n + z * z / (4.0 * n * n)) / d
    return (c - h, c + h)


def _div(a: float, b: float) -> float:
    """f64 division with IEEE results for a zero divisor (as Rust's f64)."""
    with np.errstate(divide="ignore", invalid="ignore"):
        return float(np.float64(a) / np.float64(b))


def resumer(ps: list) -> dict:
    """stats.rs:144-177."""
    n = len(ps)
    kl_m, kl_i = moyenne_incertitude(p["kl"] for p in ps)
    tries = sorted(p["kl"] for p in ps)
    med = 0.5 * (tries[n // 2] + tries[n // 2 - 1]) if n % 2 == 0 else tries[n // 2]
    k = sum(1 for p in ps if p["meme_premier"])
    top = k / n
    lq, lq_i = moyenne_incertitude(p["nll_q"] for p in ps)
    lp, lp_i = moyenne_incertitude(p["nll_p"] for p in ps)
    if n >= 10:
        sab = 0.0
        for p in ps:
            sab += p["nll_q"] * p["nll_p"]
        cov = (sab / n - lq * lp) / (n - 1.0)
    else:
        cov = 0.0
    dp2 = 0.0
    for p in ps:
        dp2 += p["dp"] * p["dp"]
    dp2 /= n
    return {
        "n": n, "kl_moyenne": kl_m, "kl_incertitude": kl_i, "kl_mediane": med,
        "kl_p90": quantile(tries, 0.90), "kl_p99": quantile(tries, 0.99), "kl_p999": quantile(tries, 0.999),
        "kl_max": tries[-1], "kl_min": tries[0], "meme_premier": top,
        "meme_premier_incertitude": math.sqrt(_div(top * (1.0 - top), n - 1.0)),
        "meme_premier_wilson95": wilson95(k, n), "ppl_q": math.exp(lq), "ppl_p": math.exp(lp),
        "ln_rapport_ppl": lq - lp,
        "ln_rapport_ppl_incertitude": math.sqrt(max(lq_i * lq_i + lp_i * lp_i - 2.0 * cov, 0.0)),
        "dp_rms": math.sqrt(dp2),
    }


def decider(series) -> dict:
    """abba.rs:17-40: series of (a1, b1, b2, a2)."""
    assert series
    bruit, sa, sb = 0.0, 0.0, 0.0
    for a1, b1, b2, a2 in series:
        bruit = max(bruit, abs(a1 - a2) / ((a1 + a2) / 2.0))
        bruit = max(bruit, abs(b1 - b2) / ((b1 + b2) / 2.0))
        sa += a1 + a2
        sb += b1 + b2
    n = 2.0 * len(series)
    ma, mb = sa / n, sb / n
    ecart = (mb - ma) / ma
    seuil = max(2.0 * bruit, 0.03)
    return {"moyenne_a": ma, "moyenne_b": mb, "ecart_relatif": ecart, "plus_grand_bruit": bruit, "seuil": seuil,
            "reel": abs(ecart) > seuil}


def ecrire_kld(chemin: str, n_ctx: int, n_vocab: int, jetons, lignes) -> None:
    """A `.kld` file (kld.rs:188-235), every entry coded by coder_entree: `lignes` = f64 logit rows
    in file order (each window's scored positions, window after window)."""
    with open(chemin, "wb") as f:
        f.write(MAGIE)
        f.write(struct.pack("<Iii", n_ctx, n_vocab, len(jetons) // n_ctx))
        f.write(np.asarray(jetons, np.int32).astype("<i4").tobytes())
        for l in lignes:
            f.write(coder_entree(l).astype("<u2").tobytes())


def lire_kld(chemin: str):
    """(n_ctx, n_vocab, n_chunk, tokens i32[], entries u16[n_chunk][scored][nv]) (kld.rs:48-75)."""
    b = open(chemin, "rb").read()
    assert b[:8] == MAGIE
    n_ctx, n_vocab, n_chunk = struct.unpack("<Iii", b[8:20])
    jetons = np.frombuffer(b, "<i4", n_ctx * n_chunk, 20)
    nv = mots_par_entree(n_vocab)
    e = np.frombuffer(b, "<u2", offset=20 + 4 * n_ctx * n_chunk)
    return n_ctx, n_vocab, n_chunk, jetons, e.reshape(n_chunk, len(positions_notees(n_ctx)), nv)
