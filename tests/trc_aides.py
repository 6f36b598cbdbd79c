"""Helpers for the CPU tests: a geometry-1 rANS stream as fields (parse / write back), the
scale class of a delta, seeded synthetic MXFP4 blocks, and a level-0 part built from the
oracle's primitives alone (the way trc-codec's coder_matrice_v10 composes one,
trc-codec/src/lib.rs:399-428)."""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

import oracle as O

SORTE_MEDIANES, SORTE_BIAIS, SORTE_DELTA, SORTE_CODES_CTX = 0x01, 0x02, 0x03, 0x04


@dataclass
class Flux:
    """Fields of a serialised stream (header of 16 bytes, rans.rs:186-228)."""

    P: int
    N: int
    geo: int
    res: int
    debuts: np.ndarray
    etats: np.ndarray
    mots: np.ndarray

    @staticmethod
    def lire(b: bytes) -> "Flux":
        P, N, geo, res, T, W = struct.unpack_from("<IHBBII", b, 0)
        d = np.frombuffer(b, np.uint32, T, 16).copy()
        e = np.frombuffer(b, np.uint32, 32 * T, 16 + 4 * T).copy()
        m = np.frombuffer(b, np.uint16, W, 16 + 132 * T).copy()
        return Flux(P, N, geo, res, d, e, m)

    def ecrire(self) -> bytes:
        T, W = self.debuts.size, self.mots.size
        o = struct.pack("<IHBBII", self.P, self.N, self.geo, self.res, T, W)
        o += self.debuts.astype("<u4").tobytes() + self.etats.astype("<u4").tobytes() + self.mots.astype("<u2").tobytes()
        return o + b"\0" * ((-len(o)) % 16)


def classe(delta: np.ndarray) -> np.ndarray:
    """Scale class of a block from its delta: 0 below 128, 1 at 128, 2 above (lib.rs:48-55)."""
    d = np.asarray(delta)
    return np.where(d < 128, 0, np.where(d == 128, 1, 2)).astype(np.uint8)


def octets_geometriques(rng: np.random.Generator, n: int, p_lo: float = 0.3, p_hi: float = 0.25) -> np.ndarray:
    """n bytes whose two nibbles follow truncated geometric laws (peaked like MXFP4 codes)."""
    lo = np.minimum(rng.geometric(p_lo, n) - 1, 15)
    hi = np.minimum(rng.geometric(p_hi, n) - 1, 15)
    return (lo | (hi << 4)).astype(np.uint8)


def blocs_mxfp4(rng: np.random.Generator, R: int, B: int, zeros_signes: bool = False) -> np.ndarray:
    """R*B MXFP4 blocks of 17 bytes (E8M0 scale, 16 code bytes): per-row median scale near
    2^-8..-10, block scales spread around it, peaked codes; with `zeros_signes`, half of the
    zero nibbles carry the sign bit (code 8, -0), as in gpt-oss's weights."""
    med = 118 + rng.integers(0, 4, R)
    e = np.clip(med[:, None] + np.minimum(rng.geometric(0.5, (R, B)) - 1, 4) - 2, 0, 255).astype(np.uint8)
    q = octets_geometriques(rng, R * B * 16, 0.3, 0.3).reshape(R * B, 16)
    if zeros_signes:
        lo, hi = q & 15, q >> 4
        lo = np.where((lo == 0) & (rng.integers(0, 2, lo.shape) == 1), 8, lo)
        hi = np.where((hi == 0) & (rng.integers(0, 2, hi.shape) == 1), 8, hi)
        q = (lo | (hi << 4)).astype(np.uint8)
    return np.concatenate([e.reshape(-1, 1), q], axis=1).reshape(-1)


def tables_matrice(preps) -> np.ndarray:
    """Frequencies u16[4][256] (DELTA, CODES k = 0, 1, 2) from the counts of prepared matrices."""
    c = np.zeros(4 * 256, np.uint64)
    for _, d, q in preps:
        O.ajouter_comptes(d, q, c)
    return np.stack([O.table_depuis_comptes(c[256 * t:256 * (t + 1)]) for t in range(4)])


def flux_matrice(prep, biais: bytes, f4: np.ndarray, j: int, R: int, nb: int, n_delta: int = 256,
                 n_codes: int = 256, codeur=None):
    """The four streams of matrix j (MEDIANES, BIAIS, DELTA, CODES_CTX) as assembler_partie
    takes them; `codeur` = an object with coder_g1 (the oracle module by default)."""
    codeur = codeur or O
    med, delta, qs = prep
    fd = codeur.coder_g1(delta, f4[0:1], None, n_delta)
    fc = codeur.coder_g1(qs, f4[1:4], classe(delta[:nb]), n_codes)
    return [(SORTE_MEDIANES, j, 0xFF, R, med.tobytes()), (SORTE_BIAIS, j, 0xFF, len(biais), biais),
            (SORTE_DELTA, j, 0, delta.size, fd), (SORTE_CODES_CTX, j, 0xFF, qs.size, fc)]
