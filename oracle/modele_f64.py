"""Test infrastructure only (a checker, never on the product path): the f64 evaluation of a
gpt-oss model on the host, the reference's trc-reference (moteur/crates/trc-reference), to judge
troncons_b200's whole decode step (troncons_b200.modele.Modele) against the truth:

- `pas` = Reference::pas (trc-reference/src/modele.rs:527-550): embedding row, per layer
  RMSNorm (ops.rs:8-19), q / k / v + biases, YaRN (ops.rs:46-88; the OpenAI ramp, real bounds),
  KV append, attention with sinks over the window (ops.rs:90-121, modele.rs:552-573), output +
  residual, RMSNorm, router top-k and softmax (ops.rs:123-132, ties to the smaller index),
  clamped SwiGLU (ops.rs:134-141), the weighted experts' sum, then RMSNorm and the unembedding
  (modele.rs:508-515);
- every product and sum in f64; the weights are the model's own (Q8_0 rows and MXFP4 experts,
  the experts decoded from their `.trc` parts by the CPU codec, dequantised exactly to f64);
- `kv16=True` rounds the cached keys and values to f16 as the engine stores them (the
  reference's `--imiter kv16`, bin/juge.rs:150-160); the default keeps them in f64, the truth.

The GPU model's tensors are read back once at construction (torch); nothing here launches a kernel."""
from __future__ import annotations

import numpy as np

import oracle as O

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def q8_0_f64(w, R: int, C_: int) -> np.ndarray:
    """A Q8_0 matrix (34-byte blocks: f16 d, 32 x i8) as f64 [R][C], exact."""
    b = np.asarray(w, np.uint8).reshape(R, C_ // 32, 34)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float64)
    return (d * b[:, :, 2:].view(np.int8).astype(np.float64)).reshape(R, C_)


def experts_f64(part: bytes, luts, dims, taille_emplacement: int) -> list:
    """[(W f64 [R][C], bias f64 [R]) for gate, up, down] of one expert, from its level-0 part
    decoded by the CPU codec: E2M1(code) * 2^(e - 127), element i of a block in the low nibble
    of byte i and element 16 + i in its high nibble."""
    slot, ctl = O.decoder_expert(part, luts, list(dims.lignes), list(dims.colonnes), taille_emplacement)
    if (ctl != 0).any():
        raise ValueError(f"the part does not decode cleanly: {ctl}")
    out, base = [], 0
    for j in range(3):
        R, C_ = dims.lignes[j], dims.colonnes[j]
        e_off, b_off, pas = O.disposition(R, C_)
        nb = R * (C_ // 32)
        m = slot[base:base + pas]
        codes = m[:16 * nb].reshape(nb, 16)
        ech = m[e_off:e_off + nb].astype(np.int64)
        biais = m[b_off:b_off + 4 * R].view(np.float32).astype(np.float64)
        nib = np.concatenate([codes & 15, codes >> 4], axis=1).astype(np.int64)
        val = E2M1[nib & 7] * np.where(nib & 8, -1.0, 1.0) * np.ldexp(1.0, ech - 127)[:, None]
        out.append((val.reshape(R, C_), biais))
        base += pas
    return out


def inv_freq(p) -> tuple:
    """(inv_freq[d/2], concentration) of YaRN (ops.rs:46-72) for a trc_params_rope."""
    d, demi = p.dim_tete, p.dim_tete // 2
    i = np.arange(demi, dtype=np.float64)
    freq = p.base ** (2 * i / d)
    if p.facteur <= 1.0:
        return 1.0 / freq, 1.0
    conc = 0.1 * np.log(p.facteur) + 1.0
    bas = demi * np.log(p.ctx_origine / (p.beta_rapide * 2 * np.pi)) / np.log(p.base)
    haut = demi * np.log(p.ctx_origine / (p.beta_lent * 2 * np.pi)) / np.log(p.base)
    if p.variante == 1:
        bas, haut = max(np.floor(bas), 0.0), min(np.ceil(haut), d - 1.0)
    rampe = np.clip((i - bas) / (haut - bas), 0.0, 1.0)
    return (1.0 / (p.facteur * freq)) * rampe + (1.0 / freq) * (1.0 - rampe), conc


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    return x * (1.0 / np.sqrt(np.mean(x * x) + eps)) * w


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.minimum(g, 7.0)
    u = np.clip(u, -7.0, 7.0)
    return g / (1.0 + np.exp(-1.702 * g)) * (u + 1.0)


class ModeleF64:
    """The f64 evaluation of a troncons_b200.modele.Modele's weights (its compressed parts)."""

    def __init__(self, m, kv16: bool = False):
        import torch

        import troncons_b200 as T

        self.L, self.d, self.H, self.Hk, self.k = m.couches, m.d, m.tetes, m.tetes_kv, m.k
        self.experts, self.vocab, self.kv16 = m.experts, m.vocab, kv16
        self.eps = float(np.float32(m.eps))
        self.inv, self.conc = inv_freq(m.rope)
        dq, dkv = m.tetes * 64, m.tetes_kv * 64
        hote = lambda t: t.cpu().numpy() if torch.is_tensor(t) else t  # noqa: E731
        te = T.taille_emplacement(m.dims)
        self.couches = []
        for l in range(m.couches):
            t = {n: hote(v) for n, v in m.tenseurs[l].items() if not n.startswith("cache")}
            tampon, adr, tailles = m.parties["compresse"][l]
            base, brut = tampon.data_ptr(), tampon.cpu().numpy()
            lut = m.luts[l].cpu().numpy().view(np.uint32)
            ex = [experts_f64(brut[int(a) - base:int(a) - base + int(s)].tobytes(), lut, m.dims, te)
                  for a, s in zip(adr, tailles)]
            f = lambda n: t[n].astype(np.float64)  # noqa: E731
            self.couches.append({
                "an": f("attn_norm"), "pn": f("post_norm"), "puits": f("puits"), "anneau": int(t["anneau"]),
                "q": (q8_0_f64(t["wq"], dq, m.d), f("bq")), "k": (q8_0_f64(t["wk"], dkv, m.d), f("bk")),
                "v": (q8_0_f64(t["wv"], dkv, m.d), f("bv")), "o": (q8_0_f64(t["wo"], m.d, dq), f("bo")),
                "r": (f("wr").reshape(m.experts, m.d), f("br")), "ex": ex})
        self.emb = q8_0_f64(hote(m.enchassement), m.vocab, m.d)
        self.sortie = q8_0_f64(hote(m.sortie_w), m.vocab, m.d)
        self.norme = hote(m.norme_sortie).astype(np.float64)
        self.reinitialiser()

    def reinitialiser(self) -> None:
        self.cache = [([], []) for _ in range(self.L)]

    def _tourner(self, v: np.ndarray, tetes: int, pos: int) -> np.ndarray:
        v = v.reshape(tetes, 64)
        c, s = np.cos(pos * self.inv) * self.conc, np.sin(pos * self.inv) * self.conc
        a, b = v[:, :32], v[:, 32:]
        return np.concatenate([a * c - b * s, b * c + a * s], axis=1).reshape(-1)

    def pas(self, jeton: int, position: int) -> np.ndarray:
        """Logits f64[vocab] of `jeton` at `position` (the next position after the cached ones)."""
        if position != len(self.cache[0][0]):
            raise ValueError(f"position {position}: the next one is {len(self.cache[0][0])}")
        x = self.emb[jeton].copy()
        for l, c in enumerate(self.couches):
            h = rmsnorm(x, c["an"], self.eps)
            q = c["q"][0] @ h + c["q"][1]
            k = c["k"][0] @ h + c["k"][1]
            v = c["v"][0] @ h + c["v"][1]
            q, k = self._tourner(q, self.H, position), self._tourner(k, self.Hk, position)
            if self.kv16:
                k, v = k.astype(np.float16).astype(np.float64), v.astype(np.float16).astype(np.float64)
            self.cache[l][0].append(k)
            self.cache[l][1].append(v)
            n = position + 1
            debut = max(0, n - c["anneau"]) if c["anneau"] else 0
            K, V = np.array(self.cache[l][0][debut:n]), np.array(self.cache[l][1][debut:n])
            a = np.zeros(self.H * 64)
            for t in range(self.H):
                tk = t // (self.H // self.Hk)
                sc = K[:, tk * 64:(tk + 1) * 64] @ q[t * 64:(t + 1) * 64] * 0.125
                m = max(sc.max(), c["puits"][t])
                e = np.exp(sc - m)
                a[t * 64:(t + 1) * 64] = (e / (e.sum() + np.exp(c["puits"][t] - m))) @ V[:, tk * 64:(tk + 1) * 64]
            x = x + c["o"][0] @ a + c["o"][1]
            h2 = rmsnorm(x, c["pn"], self.eps)
            lr = c["r"][0] @ h2 + c["r"][1]
            top = sorted(range(self.experts), key=lambda e_: (-lr[e_], e_))[:self.k]
            w = np.exp(lr[top] - lr[top[0]])
            w /= w.sum()
            for wi, e_ in zip(w, top):
                (Wg, bg), (Wu, bu), (Wd, bd) = c["ex"][e_]
                x = x + wi * (Wd @ swiglu(Wg @ h2 + bg, Wu @ h2 + bu) + bd)
        return self.sortie @ rmsnorm(x, self.norme, self.eps)
