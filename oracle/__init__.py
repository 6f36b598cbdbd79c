"""TEST INFRASTRUCTURE — ctypes access to the CPU oracle (oracle/_build/liboracle.so).

The oracle restates, in plain C, the reference's CPU codec and format (rANS tables, LUT,
coder, normative decoder, part layout, v1.2 expert reconstruction, empreinte64) and the
single-vector numerics of the MoE layer. Only tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg may use it, as the checker or as the timed CPU baseline; the
product never does.

``ref`` gives the reference's own CUDA kernels (oracle/_ref/libtrc_ref.so, compiled from the
reference checkout by ``make ref``) when that library is present.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

ICI = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(ICI, "_build", "liboracle.so")
_REF = os.path.join(ICI, "_ref", "libtrc_ref.so")
_BANC = os.path.join(ICI, "_ref", "libtrc_banc.so")

P8 = C.POINTER(C.c_uint8)
P16 = C.POINTER(C.c_uint16)
P32 = C.POINTER(C.c_uint32)
P64 = C.POINTER(C.c_uint64)
PF = C.POINTER(C.c_float)
PD = C.POINTER(C.c_double)


class Bilan(C.Structure):
    """Integrity record of a decode (rans.rs:357-382)."""

    _fields_ = [("voies_hors_l", C.c_uint64), ("tuiles_mots_faux", C.c_uint64), ("premiere_tuile", C.c_int64)]

    def intact(self) -> bool:
        return self.voies_hors_l == 0 and self.tuiles_mots_faux == 0


def construire() -> None:
    """Builds liboracle.so (gcc) when it is missing or older than its sources."""
    sources = [os.path.join(ICI, f) for f in ("trc_oracle.c", "ordre_b200.c", "couche_cpu.c", "attention_cpu.c",
                                              "couche_synth.c")]
    if os.path.exists(_LIB) and all(os.path.getmtime(_LIB) >= os.path.getmtime(s) for s in sources):
        return
    subprocess.run(["make", "-C", ICI, "all"], check=True, capture_output=True)


def _charger() -> C.CDLL:
    construire()
    lib = C.CDLL(_LIB)
    sig = {
        "orc_sha256_octets": (None, [P8, C.c_size_t, P8]),
        "orc_empreinte64": (C.c_uint64, [P8, C.c_size_t]),
        "orc_table_depuis_comptes": (None, [P64, C.c_int, P16]),
        "orc_lut": (C.c_int, [P16, C.c_int, P32]),
        "orc_coder_g1": (C.c_size_t, [P8, C.c_uint32, C.c_uint32, P8, C.c_size_t, P16, C.c_uint32, P8, C.c_size_t]),
        "orc_flux_valide": (C.c_int, [P8, C.c_size_t]),
        "orc_decoder": (C.c_int, [P8, C.c_size_t, P8, C.c_size_t, P32, C.c_uint32, P8, C.POINTER(Bilan)]),
        "orc_trouver_flux": (C.c_int, [P8, C.c_size_t, C.c_uint8, C.c_uint8, P32, P32, P32]),
        "orc_assembler_partie": (C.c_size_t, [C.c_uint16, C.c_uint16, C.c_uint8, C.c_uint8, C.c_uint32, P8, P32, P32, P8, P8, P32]),
        "orc_preparer_matrice": (None, [P8, C.c_uint32, C.c_uint32, C.c_int, P8, P8, P8]),
        "orc_ajouter_comptes": (None, [P8, C.c_size_t, P8, C.c_size_t, P64]),
        "orc_decoder_matrice_v10": (C.c_int, [P8, C.c_size_t, C.c_uint8, C.c_uint32, C.c_uint32, P32, P8, P8, PF, C.POINTER(Bilan), C.POINTER(Bilan)]),
        "orc_decoder_expert": (C.c_int, [P8, C.c_size_t, P32, P32, P32, P8, P32]),
        "orc_disposition": (None, [C.c_uint32, C.c_uint32, P64, P64, P64]),
        "orc_f16_depuis_f32": (None, [PF, P16, C.c_uint64]),
        "orc_f32_depuis_f16": (None, [P16, PF, C.c_uint64]),
        "orc_gemv_q8_0": (None, [P8, PF, PF, C.c_uint32, C.c_uint32, PF]),
        "orc_rmsnorm": (None, [PF, PF, PF, C.c_uint32, C.c_uint32, C.c_float]),
        "orc_rope_yarn": (None, [PF, PF, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p]),
        "orc_ecrire_kv": (None, [PF, PF, P16, P16, C.c_uint32, C.c_uint32]),
        "orc_attention": (None, [PF, P16, P16, PF, PF, C.c_void_p, PF]),
        "orc_gemv_f64": (None, [P8, P8, PF, PD, C.c_uint32, C.c_uint32, PD]),
        "orc_routeur_topk": (None, [PF, C.c_uint32, C.c_uint32, P32, PF]),
        "orc_swiglu": (None, [PF, PF, PF, C.c_uint32]),
        "orc_combiner": (None, [PF, PF, C.c_uint32, PF, C.c_uint32, C.c_uint32]),
        "ord_gemv": (None, [P8, P8, PF, PF, C.c_uint32, C.c_uint32, PF]),
        "ord_gemv_f32": (None, [PF, PF, PF, C.c_uint32, C.c_uint32, PF]),
        "orc_couche_moe_cpu": (C.c_int, [C.POINTER(P8), C.POINTER(C.c_size_t), C.c_uint32, P32, P32, P32,
                                         PF, PF, PF, C.c_uint32, PF, P32, PF, C.c_int]),
        "orc_decoder_matrices_cpu": (C.c_int, [P8, C.c_size_t, P32, P32, P32, C.c_uint32, P32, C.POINTER(P8),
                                               C.POINTER(P8), C.c_int]),
        "orc_synth_matrices": (C.c_int, [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, P8, PF, C.c_int]),
        "orc_comptes_couche": (None, [C.c_void_p * 3, P32, P32, C.c_uint32, C.c_int, P64]),
        "orc_coder_couche": (None, [C.c_void_p * 3, C.c_void_p * 3, P32, P32, C.c_uint32, C.c_uint32, P16, C.c_int,
                                    C.c_uint32, C.c_uint32, P8, C.c_size_t, P64]),
    }
    for nom, (res, args) in sig.items():
        f = getattr(lib, nom)
        f.restype = res
        f.argtypes = args
    return lib


lib = _charger()


def p(a: np.ndarray, t):
    """Pointer of a C-contiguous numpy array."""
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def empreinte64(b: bytes) -> int:
    a = np.frombuffer(b, dtype=np.uint8) if len(b) else np.zeros(1, np.uint8)
    return int(lib.orc_empreinte64(p(a, P8), len(b)))


def sha256(b: bytes) -> bytes:
    a = np.frombuffer(b, dtype=np.uint8) if len(b) else np.zeros(1, np.uint8)
    out = np.zeros(32, np.uint8)
    lib.orc_sha256_octets(p(a, P8), len(b), p(out, P8))
    return out.tobytes()


def table_depuis_comptes(comptes, geometrie: int = 1) -> np.ndarray:
    n = 256 if geometrie == 1 else 16
    c = np.ascontiguousarray(comptes, dtype=np.uint64)
    assert c.size == n
    f = np.zeros(n, np.uint16)
    lib.orc_table_depuis_comptes(p(c, P64), geometrie, p(f, P16))
    return f


def lut(freq, geometrie: int = 1) -> np.ndarray:
    f = np.ascontiguousarray(freq, dtype=np.uint16)
    out = np.zeros(4096, np.uint32)
    if lib.orc_lut(p(f, P16), geometrie, p(out, P32)) != 0:
        raise ValueError("frequencies do not sum to 4096")
    return out


def coder_g1(src, freqs, kappa=None, N: int = 256) -> bytes:
    """Geometry-1 stream of `src` (padded by the caller to a multiple of 128)."""
    s = np.ascontiguousarray(src, dtype=np.uint8)
    f = np.ascontiguousarray(freqs, dtype=np.uint16).reshape(-1)
    cap = 16 + 132 * (s.size // 128 // max(N, 1) + 2) + 2 * s.size + 4096
    out = np.zeros(cap, np.uint8)
    k = None if kappa is None else np.ascontiguousarray(kappa, dtype=np.uint8)
    n = lib.orc_coder_g1(p(s, P8), s.size, N, p(k, P8) if k is not None else None, 0 if k is None else k.size,
                         p(f, P16), f.size // 256, p(out, P8), cap)
    if n == 0 or n == (1 << 64) - 1:
        raise ValueError("coding failed (symbol absent from its table, or bad size)")
    return out[:n].tobytes()


def decoder(flux: bytes, luts, kappa=None):
    """(decoded P bytes, Bilan) of a geometry-1 stream (decoder_avec, rans.rs:388-451)."""
    b = np.frombuffer(flux, np.uint8)
    P = int.from_bytes(flux[0:4], "little")
    out = np.zeros(max(P, 1), np.uint8)
    l = np.ascontiguousarray(luts, dtype=np.uint32).reshape(-1)
    k = None if kappa is None else np.ascontiguousarray(kappa, dtype=np.uint8)
    bil = Bilan()
    r = lib.orc_decoder(p(b, P8), b.size, p(k, P8) if k is not None else None, 0 if k is None else k.size,
                        p(l, P32), l.size // 4096, p(out, P8), C.byref(bil))
    if r != 0:
        raise ValueError(f"malformed stream ({r})")
    return out[:P], bil


def flux_valide(flux: bytes) -> int:
    b = np.frombuffer(flux, np.uint8)
    return int(lib.orc_flux_valide(p(b, P8), b.size))


def trouver_flux(partie: bytes, sorte: int, matrice: int):
    b = np.frombuffer(partie, np.uint8)
    d, lg, pr = C.c_uint32(), C.c_uint32(), C.c_uint32()
    r = lib.orc_trouver_flux(p(b, P8), b.size, sorte, matrice, C.byref(d), C.byref(lg), C.byref(pr))
    return r, d.value, lg.value, pr.value


def assembler_partie(couche: int, expert: int, niveau: int, n_matrices: int, flux):
    """flux: list of (sorte, matrice, contexte, produits, bytes) -> (part bytes, useful bytes)."""
    n = len(flux)
    descs = np.array([[f[0], f[1], f[2]] for f in flux], np.uint8).reshape(-1)
    lg = np.array([len(f[4]) for f in flux], np.uint32)
    pr = np.array([f[3] for f in flux], np.uint32)
    data = np.frombuffer(b"".join(f[4] for f in flux) or b"\0", np.uint8)
    ut = C.c_uint32()
    total = lib.orc_assembler_partie(couche, expert, niveau, n_matrices, n, p(descs, P8), p(lg, P32), p(pr, P32),
                                     p(data, P8), None, C.byref(ut))
    out = np.zeros(total, np.uint8)
    lib.orc_assembler_partie(couche, expert, niveau, n_matrices, n, p(descs, P8), p(lg, P32), p(pr, P32),
                             p(data, P8), p(out, P8), C.byref(ut))
    return out.tobytes(), ut.value


def preparer_matrice(blocs, R: int, B: int, canonique: bool):
    """(medians, padded delta, padded qs) of R*B 17-byte MXFP4 blocks (lib.rs:348-373)."""
    bl = np.ascontiguousarray(blocs, dtype=np.uint8).reshape(-1)
    nb = R * B
    med = np.zeros(R, np.uint8)
    delta = np.zeros((nb + 127) // 128 * 128, np.uint8)
    qs = np.zeros((16 * nb + 127) // 128 * 128, np.uint8)
    lib.orc_preparer_matrice(p(bl, P8), R, B, int(canonique), p(med, P8), p(delta, P8), p(qs, P8))
    return med, delta, qs


def ajouter_comptes(delta, qs, comptes: np.ndarray) -> None:
    lib.orc_ajouter_comptes(p(delta, P8), delta.size, p(qs, P8), qs.size, p(comptes, P64))


def decoder_matrice_v10(partie: bytes, j: int, R: int, B: int, luts4):
    b = np.frombuffer(partie, np.uint8)
    l = np.ascontiguousarray(luts4, dtype=np.uint32).reshape(-1)
    codes = np.zeros(16 * R * B, np.uint8)
    ech = np.zeros(R * B, np.uint8)
    bi = np.zeros(R, np.float32)
    bd, bc = Bilan(), Bilan()
    r = lib.orc_decoder_matrice_v10(p(b, P8), b.size, j, R, B, p(l, P32), p(codes, P8), p(ech, P8), p(bi, PF),
                                    C.byref(bd), C.byref(bc))
    if r != 0:
        raise ValueError(f"format error ({r})")
    return codes, ech, bi, bd, bc


def disposition(R: int, C_: int):
    """(scales offset, bias offset, stride) of an R x C matrix in the SoA slot (abi.rs:69-122)."""
    e, b, s = C.c_uint64(), C.c_uint64(), C.c_uint64()
    lib.orc_disposition(R, C_, C.byref(e), C.byref(b), C.byref(s))
    return e.value, b.value, s.value


def decoder_expert(partie: bytes, luts, lignes, colonnes, taille_emplacement: int):
    """(slot bytes, controle[4]) of a whole level-0 part, decoded by the CPU codec."""
    b = np.frombuffer(partie, np.uint8)
    l = np.ascontiguousarray(luts, dtype=np.uint32).reshape(-1)
    R = np.array(lignes, np.uint32)
    Cc = np.array(colonnes, np.uint32)
    e = np.zeros(taille_emplacement, np.uint8)
    ctl = np.zeros(4, np.uint32)
    lib.orc_decoder_expert(p(b, P8), b.size, p(l, P32), p(R, P32), p(Cc, P32), p(e, P8), p(ctl, P32))
    return e, ctl


def gemv_f64(codes, ech, biais, x, R: int, C_: int) -> np.ndarray:
    xd = np.ascontiguousarray(x, dtype=np.float64)
    y = np.zeros(R, np.float64)
    bi = None if biais is None else np.ascontiguousarray(biais, dtype=np.float32)
    lib.orc_gemv_f64(p(codes, P8), p(ech, P8), p(bi, PF) if bi is not None else None, p(xd, PD), R, C_, p(y, PD))
    return y


def ordre_gemv(codes, ech, biais, x, R: int, C_: int) -> np.ndarray:
    """troncons_b200's GEMV reduction order, bit for bit (oracle/ordre_b200.c)."""
    xf = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(R, np.float32)
    bi = None if biais is None else np.ascontiguousarray(biais, dtype=np.float32)
    lib.ord_gemv(p(np.ascontiguousarray(codes), P8), p(np.ascontiguousarray(ech), P8),
                 p(bi, PF) if bi is not None else None, p(xf, PF), R, C_, p(y, PF))
    return y


def ordre_gemv_f32(W, x, biais, R: int, C_: int) -> np.ndarray:
    Wf = np.ascontiguousarray(W, dtype=np.float32)
    xf = np.ascontiguousarray(x, dtype=np.float32)
    bi = None if biais is None else np.ascontiguousarray(biais, dtype=np.float32)
    y = np.zeros(R, np.float32)
    lib.ord_gemv_f32(p(Wf, PF), p(xf, PF), p(bi, PF) if bi is not None else None, R, C_, p(y, PF))
    return y


def routeur_topk(logits, k: int):
    l = np.ascontiguousarray(logits, dtype=np.float32)
    idx = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    lib.orc_routeur_topk(p(l, PF), l.size, k, p(idx, P32), p(w, PF))
    return idx, w


def swiglu(g, u) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    y = np.zeros_like(g)
    lib.orc_swiglu(p(g, PF), p(u, PF), p(y, PF), g.size)
    return y


def combiner(residu, sorties, pas: int, poids, n: int, d: int) -> np.ndarray:
    r = np.array(residu, dtype=np.float32, copy=True)
    s = np.ascontiguousarray(sorties, dtype=np.float32)
    w = None if poids is None else np.ascontiguousarray(poids, dtype=np.float32)
    lib.orc_combiner(p(r, PF), p(s, PF), pas, p(w, PF) if w is not None else None, n, d)
    return r


def couche_moe_cpu(parties, luts, lignes, colonnes, Wr, br, x, k: int, residu, n_fils: int = 0):
    """One MoE layer on host cores (lignes/colonnes: the three matrices' shapes): returns
    (residual out, indices, weights)."""
    E = len(parties)
    bufs = [np.frombuffer(q, np.uint8) for q in parties]
    ptrs = (P8 * E)(*[p(b, P8) for b in bufs])
    tailles = (C.c_size_t * E)(*[b.size for b in bufs])
    l = np.ascontiguousarray(luts, dtype=np.uint32).reshape(-1)
    res = np.array(residu, dtype=np.float32, copy=True)
    idx = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    lg = np.array(list(lignes), np.uint32)
    cl = np.array(list(colonnes), np.uint32)
    r = lib.orc_couche_moe_cpu(ptrs, tailles, E, p(l, P32), p(lg, P32), p(cl, P32), p(np.ascontiguousarray(Wr, np.float32), PF),
                               p(np.ascontiguousarray(br, np.float32), PF), p(np.ascontiguousarray(x, np.float32), PF),
                               k, p(res, PF), p(idx, P32), p(w, PF), n_fils)
    if r != 0:
        raise ValueError(f"CPU layer failed ({r})")
    return res, idx, w


def decoder_matrices_cpu(partie: bytes, luts, lignes, colonnes, mats=(0, 1), n_fils: int = 0):
    """Config 0's CPU decode of matrices `mats` of one part, parallel over (matrix, tile) on
    `n_fils` host threads (0: all): [(codes uint8[16 R B], scales uint8[R B])]."""
    b = np.frombuffer(partie, np.uint8)
    l = np.ascontiguousarray(luts, dtype=np.uint32).reshape(-1)
    lg = np.array(list(lignes), np.uint32)
    cl = np.array(list(colonnes), np.uint32)
    ms = np.array(list(mats), np.uint32)
    codes = [np.empty(16 * int(lg[j]) * (int(cl[j]) // 32), np.uint8) for j in mats]
    ech = [np.empty(int(lg[j]) * (int(cl[j]) // 32), np.uint8) for j in mats]
    pc = (P8 * len(mats))(*[p(a, P8) for a in codes])
    pe = (P8 * len(mats))(*[p(a, P8) for a in ech])
    r = lib.orc_decoder_matrices_cpu(p(b, P8), b.size, p(l, P32), p(lg, P32), p(cl, P32), len(mats), p(ms, P32), pc,
                                     pe, n_fils)
    if r != 0:
        raise ValueError(f"CPU decode failed ({r})")
    return list(zip(codes, ech))


# ---------------------------------------------------------------- attention side (passe.cuh)

def f16(x) -> np.ndarray:
    """f32 -> binary16 bits, round to nearest even."""
    a = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.zeros(a.size, np.uint16)
    lib.orc_f16_depuis_f32(p(a, PF), p(out, P16), a.size)
    return out


def gemv_q8_0(W, x, biais, R: int, C_: int) -> np.ndarray:
    w = np.ascontiguousarray(W, dtype=np.uint8).reshape(-1)
    xf = np.ascontiguousarray(x, dtype=np.float32)
    bi = None if biais is None else np.ascontiguousarray(biais, dtype=np.float32)
    y = np.zeros(R, np.float32)
    lib.orc_gemv_q8_0(p(w, P8), p(xf, PF), p(bi, PF) if bi is not None else None, R, C_, p(y, PF))
    return y


def rmsnorm(x, w, n: int, lignes: int, eps: float) -> np.ndarray:
    xf = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    wf = np.ascontiguousarray(w, dtype=np.float32)
    y = np.zeros_like(xf)
    lib.orc_rmsnorm(p(xf, PF), p(wf, PF), p(y, PF), n, lignes, eps)
    return y


def rope_yarn(q, k, tetes_q: int, tetes_k: int, position: int, params) -> tuple:
    """params: a ctypes structure with the layout of trc_params_rope."""
    qf = np.array(q, dtype=np.float32, copy=True).reshape(-1)
    kf = np.array(k, dtype=np.float32, copy=True).reshape(-1)
    lib.orc_rope_yarn(p(qf, PF), p(kf, PF), tetes_q, tetes_k, position, C.addressof(params))
    return qf, kf


def ecrire_kv(k, v, cache_k, cache_v, dkv: int, case_kv: int) -> None:
    kf = np.ascontiguousarray(k, dtype=np.float32)
    vf = np.ascontiguousarray(v, dtype=np.float32)
    lib.orc_ecrire_kv(p(kf, PF), p(vf, PF), p(cache_k, P16), p(cache_v, P16), dkv, case_kv)


def attention(q, cache_k, cache_v, puits, params) -> np.ndarray:
    """params: a ctypes structure with the layout of trc_params_attention."""
    qf = np.ascontiguousarray(q, dtype=np.float32)
    ck = np.ascontiguousarray(cache_k, dtype=np.uint16)
    cv = np.ascontiguousarray(cache_v, dtype=np.uint16)
    pf = np.ascontiguousarray(puits, dtype=np.float32)
    out = np.zeros(params.tetes * 64, np.float32)
    scores = np.zeros(max(params.fin - params.debut, 1), np.float32)
    lib.orc_attention(p(qf, PF), p(ck, P16), p(cv, P16), p(pf, PF), p(out, PF), C.addressof(params), p(scores, PF))
    return out


def ref():
    """The reference's own CUDA kernels (oracle/_ref/libtrc_ref.so), or None when absent."""
    if not os.path.exists(_REF):
        return None
    r = C.CDLL(_REF)
    vp = C.c_void_p
    for nom, args in {
        "ref_decoder_expert": [vp, vp, vp, P32, vp, vp],
        "ref_copier_brut": [vp, vp, P32, vp, vp],
        "ref_gemv": [vp, vp, vp, C.c_uint32, C.c_uint32, vp],
        "ref_gemv_lot": [vp, C.c_uint32, C.c_uint32, vp],
        "ref_decoder_lot": [vp, C.c_uint32, P32, vp],
        "ref_gemv_f32": [vp, vp, vp, vp, C.c_uint32, C.c_uint32, vp],
        "ref_routeur_topk": [vp, C.c_uint32, C.c_uint32, vp, vp, vp],
        "ref_swiglu": [vp, vp, vp, C.c_uint32, vp],
        "ref_combiner": [vp, vp, C.c_uint32, vp, C.c_uint32, C.c_uint32, vp],
        "ref_gemv_q8_0": [vp, vp, vp, vp, C.c_uint32, C.c_uint32, vp],
        "ref_rmsnorm": [vp, vp, vp, C.c_uint32, C.c_uint32, C.c_float, vp],
        "ref_rope_yarn": [vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp],
        "ref_ecrire_kv": [vp, vp, vp, vp, C.c_uint32, C.c_uint32, vp],
        "ref_attention": [vp, vp, vp, vp, vp, vp, vp],
    }.items():
        f = getattr(r, nom)
        f.restype = C.c_int
        f.argtypes = args
    return r


class Banc:
    """The reference bench's independent encoder (oracle/_ref/libtrc_banc.so, compiled from
    trc-noyaux/banc/banc_k.cu by ``make ref``): geometry-1 coder, LUT and part assembler."""

    def __init__(self, chemin: str):
        self.lib = C.CDLL(chemin)
        sz = C.c_size_t
        self.lib.refb_coder_g1.restype = sz
        self.lib.refb_coder_g1.argtypes = [P8, C.c_uint32, C.c_uint32, P16, C.c_uint32, P8, C.c_uint32, P8, sz]
        self.lib.refb_lut_g1.restype = None
        self.lib.refb_lut_g1.argtypes = [P16, P32]
        self.lib.refb_assembler_partie.restype = sz
        self.lib.refb_assembler_partie.argtypes = [C.c_uint16, C.c_uint16, C.c_uint32, P8, P32, P32, P8, P8, sz]

    def coder_g1(self, src, freqs, kappa=None, N: int = 256) -> bytes:
        s = np.ascontiguousarray(src, dtype=np.uint8)
        f = np.ascontiguousarray(freqs, dtype=np.uint16).reshape(-1)
        k = None if kappa is None else np.ascontiguousarray(kappa, dtype=np.uint8)
        cap = 16 + 132 * (s.size // 128 // N + 2) + 2 * s.size + 4096
        out = np.zeros(cap, np.uint8)
        n = self.lib.refb_coder_g1(p(s, P8), s.size, N, p(f, P16), f.size // 256, p(k, P8) if k is not None else None,
                                   0 if k is None else k.size, p(out, P8), cap)
        assert n > 0
        return out[:n].tobytes()

    def lut(self, freq) -> np.ndarray:
        f = np.ascontiguousarray(freq, dtype=np.uint16)
        out = np.zeros(4096, np.uint32)
        self.lib.refb_lut_g1(p(f, P16), p(out, P32))
        return out

    def assembler_partie(self, couche: int, expert: int, flux) -> bytes:
        """flux: list of (sorte, matrice, contexte, produits, bytes), as assembler_partie."""
        descs = np.array([[f[0], f[1], f[2]] for f in flux], np.uint8).reshape(-1)
        lg = np.array([len(f[4]) for f in flux], np.uint32)
        pr = np.array([f[3] for f in flux], np.uint32)
        data = np.frombuffer(b"".join(f[4] for f in flux) or b"\0", np.uint8)
        cap = 64 + 16 * len(flux) + int(lg.sum()) + 16 * len(flux) + 8192
        out = np.zeros(cap, np.uint8)
        n = self.lib.refb_assembler_partie(couche, expert, len(flux), p(descs, P8), p(lg, P32), p(pr, P32),
                                           p(data, P8), p(out, P8), cap)
        assert n > 0
        return out[:n].tobytes()


def banc():
    """The reference bench's encoder (Banc), or None when oracle/_ref/libtrc_banc.so is absent."""
    return Banc(_BANC) if os.path.exists(_BANC) else None


# ---------------------------------------------------------------- a synthetic layer on host cores

def synth_matrices(graine: int, lignes: int, colonnes: int, n: int, premier: int = 0, fils: int = 0):
    """The bench workload's MXFP4 matrices premier .. premier + n - 1 of `graine` (blocs
    uint8[n, R*B*17], biais float32[n, R]), drawn by the oracle (oracle/couche_synth.c)."""
    B = colonnes // 32
    blocs = np.empty((n, lignes * B * 17), np.uint8)
    biais = np.empty((n, lignes), np.float32)
    if lib.orc_synth_matrices(graine, lignes, colonnes, premier, n, p(blocs, P8), p(biais, PF), fils) != 0:
        raise ValueError("synthetic generation refused its arguments")
    return blocs, biais


class CoucheOracle:
    """A seeded MoE layer built with the oracle alone (no product library): its experts' blocks
    and biases, the layer's frequency tables and LUTs (u32[3][4][4096]), each expert's level-0
    v1.2 part, and the router (f32 [E][C] weights N(0, 0.02), zero biases). The same seeds give
    the same layer as the product's troncons_b200.synth.couche, part for part."""

    def __init__(self, graine: int, lignes, colonnes, experts: int, n_delta: int = 256, n_codes: int = 256,
                 canonique: bool = True):
        self.lignes, self.colonnes, self.experts = list(lignes), list(colonnes), experts
        self.blocs, self.biais = [], []
        for j in range(3):
            b, bi = synth_matrices(graine * 7 + j, self.lignes[j], self.colonnes[j], experts)
            self.blocs.append(b)
            self.biais.append(bi)
        lg = np.array(self.lignes, np.uint32)
        cl = np.array(self.colonnes, np.uint32)
        pb = (C.c_void_p * 3)(*[b.ctypes.data for b in self.blocs])
        pbi = (C.c_void_p * 3)(*[b.ctypes.data for b in self.biais])
        comptes = np.zeros(3 * 4 * 256, np.uint64)
        lib.orc_comptes_couche(pb, p(lg, P32), p(cl, P32), experts, int(canonique), p(comptes, P64))
        self.freqs = np.stack([table_depuis_comptes(comptes[256 * i:256 * (i + 1)]) for i in range(12)]).reshape(3, 4, 256)
        self.luts = np.concatenate([lut(self.freqs[j, t]) for j in range(3) for t in range(4)])
        cap = 2 * sum(b.shape[1] for b in self.blocs) + 4 * sum(b.shape[1] for b in self.biais) + (1 << 16)
        sorties = np.zeros((experts, cap), np.uint8)
        octets = np.zeros(experts, np.uint64)
        f = np.ascontiguousarray(self.freqs, np.uint16).reshape(-1)
        lib.orc_coder_couche(pb, pbi, p(lg, P32), p(cl, P32), experts, 0, p(f, P16), int(canonique), n_delta, n_codes,
                             p(sorties, P8), cap, p(octets, P64))
        if (octets == 0).any():
            raise ValueError(f"experts {np.where(octets == 0)[0][:8].tolist()}: encoding failed")
        self.parties = [sorties[x, :int(octets[x])].tobytes() for x in range(experts)]
        rng = np.random.default_rng(graine)
        self.wr = (rng.standard_normal((experts, self.colonnes[0])) * 0.02).astype(np.float32)
        self.br = np.zeros(experts, np.float32)


def bf16(x) -> np.ndarray:
    """f32 values rounded to bf16 (nearest, ties to even), kept as f32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


# ---------------------------------------------------------------- MXFP8 activations, MXFP4 GEMM (f64)

def e4m3(v) -> np.ndarray:
    """Values rounded to E4M3 (OCP FP8: bias 7, 3 mantissa bits, subnormals from 2^-9, largest 448),
    nearest with ties to even, saturating at +-448; returned as float64."""
    v = np.asarray(v, np.float64)
    a = np.abs(v)
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)                      # below 2^-6: the subnormal step 2^-9
    pas = np.exp2(e - 3.0)
    q = np.round(a / pas) * pas                  # numpy rounds halves to even
    return np.sign(v) * np.minimum(q, 448.0)


def mxfp8(x, ordre_mma: bool = False):
    """x [n][C] -> (values [n][C] f64 as the quantized x, scales u8 [n][C/32]): per 32-block,
    E = floor(log2 max|x|) - 8 (E = -127 for a zero block), scale byte E + 127, elements
    e4m3(x / 2^E) (the OCP MX rule with E4M3's largest exponent 8). Returns the dequantized
    values (element = e4m3(x / 2^E) * 2^E) in the natural order."""
    x = np.asarray(x, np.float64)
    n, C = x.shape
    xb = x.reshape(n, C // 32, 32)
    m = np.abs(xb).max(axis=2)
    E = np.where(m > 0, np.floor(np.log2(np.where(m > 0, m, 1.0))) - 8, -127).clip(-127, 127)
    q = e4m3(xb / np.exp2(E)[:, :, None]) * np.exp2(E)[:, :, None]
    return q.reshape(n, C), (E + 127).astype(np.uint8)


def gemm_mxfp4_f64(codes, ech, biais, x_deq, R: int, C: int) -> np.ndarray:
    """y[n][r] = sum_c W[r][c] x_deq[n][c] + b[r] in f64, W dequantized exactly from the MXFP4
    blocks (codes: 16 bytes per block, element i low nibble / 16 + i high nibble of byte i;
    value K[c] 2^(e - 128), K = {0,1,2,3,4,6,8,12} signed by bit 3)."""
    K = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], np.float64)
    B = C // 32
    cb = np.asarray(codes, np.uint8).reshape(R, B, 16)
    w = np.concatenate([K[cb & 15], K[cb >> 4]], axis=2)          # [R][B][32], elements 0..15 then 16..31
    w = w * np.exp2(np.asarray(ech, np.float64).reshape(R, B, 1) - 128.0)
    W = w.reshape(R, C)
    y = np.asarray(x_deq, np.float64) @ W.T
    if biais is not None:
        y = y + np.asarray(biais, np.float64)[None, :]
    return y
