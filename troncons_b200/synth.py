"""Seeded synthetic gpt-oss-shaped MoE layers, encoded as `.trc` v1.2 parts.

There are no real weights here, so every input is synthetic: per row
sigma = 0.02 * LogNormal(0, 0.3), weights N(0, sigma), per 32-block E8M0 = floor(log2 max|w|) - 2,
E2M1 round-to-nearest-even with the sign kept (so -0 codes exist, as in gpt-oss's GGUF), biases
N(0, 0.01) rounded to bf16 and stored as f32. The layer's tables are built from the counts of
all its experts, as trc-codeur does (bins/trc-codeur/src/coder.rs:207-240), then each expert is
encoded into a v1.2 part (canonical codes) and, for the raw path, into a raw part.
"""
from __future__ import annotations

import ctypes as C
import concurrent.futures as cf
import os
from dataclasses import dataclass, field

import numpy as np

from . import DimsExpert, lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def matrices(graine: int, lignes: int, colonnes: int, n: int, fils: int = 0, premier: int = 0):
    """Synthetic MXFP4 matrices premier .. premier + n - 1: (blocs uint8[n, R*B*17], biais
    float32[n, R]); matrix x is the same whichever others are drawn with it."""
    B = colonnes // 32
    blocs = np.empty((n, lignes * B * 17), np.uint8)
    biais = np.empty((n, lignes), np.float32)
    r = lib.trc_synth_matrices(graine, lignes, colonnes, premier, n, _p(blocs), _p(biais), fils)
    if r != 0:
        raise ValueError("synthetic generation refused its arguments")
    return blocs, biais


def comptes(blocs_j: list, dims: DimsExpert, canonique: bool = True) -> np.ndarray:
    """The symbol counts u64[3][4][256] (DELTA, CODES k = 0, 1, 2 per matrix) of the experts in
    blocs_j (bins/trc-codeur/src/coder.rs:207-240 counts all experts of a layer)."""
    c = np.zeros((3, 4, 256), np.uint64)
    for j in range(3):
        R, B = dims.lignes[j], dims.colonnes[j] // 32
        cj = np.zeros((4, 256), np.uint64)
        for x in range(blocs_j[j].shape[0]):
            lib.trc_comptes_matrice(_p(blocs_j[j][x]), R, B, int(canonique), _p(cj))
        c[j] = cj
    return c


def tables_de_comptes(c: np.ndarray) -> np.ndarray:
    """Frequencies u16[3][4][256] from counts u64[3][4][256]."""
    freqs = np.zeros((3, 4, 256), np.uint16)
    for j in range(3):
        for t in range(4):
            f = np.zeros(256, np.uint16)
            lib.trc_table_depuis_comptes(_p(np.ascontiguousarray(c[j, t])), 1, _p(f))
            freqs[j, t] = f
    return freqs


def tables(blocs_j: list, dims: DimsExpert, canonique: bool = True) -> np.ndarray:
    """The layer's frequency tables u16[3][4][256] from all experts' counts."""
    return tables_de_comptes(comptes(blocs_j, dims, canonique))


def luts(freqs: np.ndarray) -> np.ndarray:
    """u32[3][4][4096] in the kernels' layout (abi.rs:207-221)."""
    out = np.zeros(3 * 4 * 4096, np.uint32)
    f = np.ascontiguousarray(freqs, np.uint16)
    if lib.trc_luts_couche(_p(f), None, _p(out)) != 0:
        raise ValueError("a table does not sum to 4096")
    return out


def coder_partie(blocs3, biais3, dims: DimsExpert, freqs: np.ndarray, canonique: bool = True, couche: int = 0,
                 expert: int = 0, n_delta: int = 256, n_codes: int = 256) -> bytes:
    """One expert's level-0 part (12 streams)."""
    b = [np.ascontiguousarray(x) for x in blocs3]
    bi = [np.ascontiguousarray(x, np.float32) for x in biais3]
    pb = (C.c_void_p * 3)(*[_p(x) for x in b])
    pbi = (C.c_void_p * 3)(*[_p(x) for x in bi])
    f = np.ascontiguousarray(freqs, np.uint16)
    ut = C.c_uint32()
    # rANS output is at most 1.5x its input (12-bit probabilities): one pass with room to spare,
    # a second only if a pathological input needs more.
    cap = 2 * sum(x.size for x in b) + 4 * sum(x.size for x in bi) + (1 << 16)
    out = np.zeros(cap, np.uint8)
    n = lib.trc_coder_partie(pb, pbi, C.byref(dims), _p(f), int(canonique), couche, expert, n_delta, n_codes, _p(out),
                             cap, C.byref(ut))
    if n > cap:
        out = np.zeros(int(n), np.uint8)
        n = lib.trc_coder_partie(pb, pbi, C.byref(dims), _p(f), int(canonique), couche, expert, n_delta, n_codes,
                                 _p(out), out.size, C.byref(ut))
    if n < 0:
        raise ValueError("encoding refused (a symbol absent from its table, or bad dimensions)")
    return out[:n].tobytes()


def _descs_gpu(blocs, biais, experts, sorties, capacite):
    import torch

    from . import DescCodage

    n = len(blocs)
    d = (DescCodage * n)()
    for e in range(n):
        for j in range(3):
            assert blocs[e][j].is_cuda and blocs[e][j].dtype == torch.uint8 and blocs[e][j].is_contiguous()
            assert biais[e][j].is_cuda and biais[e][j].dtype == torch.float32 and biais[e][j].is_contiguous()
            d[e].blocs[j] = blocs[e][j].data_ptr()
            d[e].biais[j] = biais[e][j].data_ptr()
        d[e].sortie = sorties[e].data_ptr() if sorties is not None else 0
        d[e].capacite = capacite
        d[e].expert = experts[e]
    brut = np.frombuffer(bytes(d), np.uint8)
    return torch.from_numpy(brut.copy()).cuda()


def comptes_gpu(blocs, dims: DimsExpert, canonique: bool = True, comptes=None):
    """trc_comptes_gpu: the symbol counts u64[3][4][256] of the experts whose blocks are the CUDA
    tensors blocs[e][j], added into `comptes` (a CUDA int64 tensor, or a new one); returns it."""
    import torch

    from . import verifier

    n = len(blocs)
    z = [[torch.zeros(1, dtype=torch.float32, device="cuda")] * 3] * n
    descs = _descs_gpu(blocs, z, [0] * n, None, 0)
    if comptes is None:
        comptes = torch.zeros(3 * 4 * 256, dtype=torch.int64, device="cuda")
    verifier(lib.trc_comptes_gpu(descs.data_ptr(), descs.numel(), n, C.byref(dims), int(canonique), comptes.data_ptr(),
                                 comptes.numel() * 8, torch.cuda.current_stream().cuda_stream))
    torch.cuda.current_stream().synchronize()
    return comptes


def coder_parties_gpu(blocs, biais, dims: DimsExpert, freqs, canonique: bool = True, couche: int = 0, experts=None,
                      n_delta: int = 256, n_codes: int = 256) -> list:
    """trc_coder_parties_gpu: the level-0 parts of the experts whose blocks and biases are the
    CUDA tensors blocs[e][j], biais[e][j], with the layer's tables `freqs` (u16[3][4][256]).
    Returns each part's bytes (synchronises)."""
    import torch

    from . import verifier

    n = len(blocs)
    experts = list(range(n)) if experts is None else experts
    cap = 2 * sum(b.numel() for b in blocs[0]) + 4 * sum(b.numel() for b in biais[0]) + (1 << 16)
    sorties = [torch.empty(cap, dtype=torch.uint8, device="cuda") for _ in range(n)]
    descs = _descs_gpu(blocs, biais, experts, sorties, cap)
    f = torch.from_numpy(np.ascontiguousarray(freqs, np.uint16).reshape(-1).view(np.int16)).cuda()
    octets = torch.zeros(2 * n, dtype=torch.int64, device="cuda")
    n_esp = int(lib.trc_coder_parties_gpu_espace(C.byref(dims), n, n_delta, n_codes))
    espace = torch.empty(n_esp + 256, dtype=torch.uint8, device="cuda")
    e0 = espace.data_ptr() + (-espace.data_ptr()) % 256
    verifier(lib.trc_coder_parties_gpu(descs.data_ptr(), descs.numel(), n, C.byref(dims), f.data_ptr(), int(canonique),
                                       couche, n_delta, n_codes, octets.data_ptr(), octets.numel() * 8, e0, n_esp,
                                       torch.cuda.current_stream().cuda_stream))
    torch.cuda.current_stream().synchronize()
    o = octets.cpu().numpy()
    parts = []
    for e in range(n):
        if o[2 * e] == 0 or o[2 * e] > cap:
            raise ValueError(f"expert {e}: encoding failed (a symbol absent from its table, or too long)")
        parts.append(sorties[e][:int(o[2 * e])].cpu().numpy().tobytes())
    return parts


def coder_partie_brute(blocs3, biais3, dims: DimsExpert, couche: int = 0, expert: int = 0) -> bytes:
    """The same expert's raw part (9 streams, origin bytes)."""
    b = [np.ascontiguousarray(x) for x in blocs3]
    bi = [np.ascontiguousarray(x, np.float32) for x in biais3]
    pb = (C.c_void_p * 3)(*[_p(x) for x in b])
    pbi = (C.c_void_p * 3)(*[_p(x) for x in bi])
    ut = C.c_uint32()
    n = lib.trc_coder_partie_brute(pb, pbi, C.byref(dims), couche, expert, None, 0, C.byref(ut))
    out = np.zeros(int(n), np.uint8)
    n2 = lib.trc_coder_partie_brute(pb, pbi, C.byref(dims), couche, expert, _p(out), out.size, C.byref(ut))
    if n2 != n:
        raise ValueError("raw encoding failed")
    return out.tobytes()


@dataclass
class Couche:
    """A synthetic MoE layer: E experts (blocks, biases), the layer's tables and LUTs, each
    expert's v1.2 part and raw part, and a router (f32 [E][C] weights, f32 biases). When only a
    share of the experts is held here, `premier` is the first one, blocs / biais hold the share
    only and the other experts' parts are None."""

    dims: DimsExpert
    experts: int
    blocs: list = field(default_factory=list)    # [j] uint8[held, R*B*17]
    biais: list = field(default_factory=list)    # [j] float32[held, R]
    freqs: np.ndarray = None
    luts: np.ndarray = None
    parties: list = field(default_factory=list)
    parties_brutes: list = field(default_factory=list)
    wr: np.ndarray = None
    br: np.ndarray = None
    premier: int = 0


def couche(graine: int, dims: DimsExpert, experts: int, canonique: bool = True, brut: bool = True,
           n_delta: int = 256, n_codes: int = 256, fils: int = 0, tenus=None, reduire=None) -> Couche:
    """A seeded layer. `tenus` = (debut, fin): draw and encode only experts [debut, fin) (an
    expert-parallel share); `reduire`: a function summing the counts u64[3][4][256] over every
    share of the layer, so that every share builds the same tables from all experts."""
    debut, fin = tenus if tenus is not None else (0, experts)
    c = Couche(dims=dims, experts=experts, premier=debut)
    for j in range(3):
        bl, bi = matrices(graine * 7 + j, dims.lignes[j], dims.colonnes[j], fin - debut, fils, premier=debut)
        c.blocs.append(bl)
        c.biais.append(bi)
    cpt = comptes(c.blocs, dims, canonique)
    if reduire is not None:
        cpt = np.ascontiguousarray(reduire(cpt), dtype=np.uint64)
    c.freqs = tables_de_comptes(cpt)
    c.luts = luts(c.freqs)
    nf = fils if fils > 0 else (os.cpu_count() or 1)

    def un(x):
        b3 = [c.blocs[j][x] for j in range(3)]
        i3 = [c.biais[j][x] for j in range(3)]
        p = coder_partie(b3, i3, dims, c.freqs, canonique, 0, debut + x, n_delta, n_codes)
        q = coder_partie_brute(b3, i3, dims, 0, debut + x) if brut else None
        return p, q

    with cf.ThreadPoolExecutor(max_workers=nf) as ex:
        res = list(ex.map(un, range(fin - debut)))
    c.parties = [None] * experts
    c.parties_brutes = [None] * experts
    for x, (p, q) in enumerate(res):
        c.parties[debut + x] = p
        c.parties_brutes[debut + x] = q
    rng = np.random.default_rng(graine)
    c.wr = (rng.standard_normal((experts, dims.colonnes[0])) * 0.02).astype(np.float32)
    c.br = np.zeros(experts, np.float32)
    return c


def slot_attendu(c: Couche, x: int, canonique: bool = True) -> np.ndarray:
    """The SoA slot an exact decoder must produce for expert x (abi.rs:69-122): codes (canonical
    when the part is v1.2), scales and biases of the three matrices."""
    d = c.dims
    total = int(lib.trc_taille_emplacement(C.byref(d)))
    out = np.zeros(total, np.uint8)
    base = 0
    for j in range(3):
        R, Cc = d.lignes[j], d.colonnes[j]
        nb = R * (Cc // 32)
        bl = c.blocs[j][x - c.premier].reshape(nb, 17)
        ech = bl[:, 0]
        qs = bl[:, 1:].reshape(-1)
        if canonique:
            lo, hi = qs & 15, qs >> 4
            lo = np.where(lo == 8, 0, lo)
            hi = np.where(hi == 8, 0, hi)
            qs = (lo | (hi << 4)).astype(np.uint8)
        e_off = (nb * 16 + 255) & ~255
        b_off = (e_off + nb + 255) & ~255
        pas = (b_off + 4 * R + 255) & ~255
        out[base:base + nb * 16] = qs
        out[base + e_off:base + e_off + nb] = ech
        out[base + b_off:base + b_off + 4 * R] = c.biais[j][x - c.premier].view(np.uint8)
        base += pas
    return out
