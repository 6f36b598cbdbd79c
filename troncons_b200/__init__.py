"""troncons_b200 — B200 (sm_100a) kernels for troncons' hot path, behind a C-ABI.

The product is ``_lib/libtroncons_b200.so`` and its C interface ``include/troncons_b200.h``.
This module binds that interface with ctypes and mirrors the reference's host wrapper
(``trc_noyaux::Noyaux``, moteur/crates/trc-noyaux/src/lib.rs): the same method names, argument
meaning (device views = address + bytes) and error behaviour (``ErreurUsage`` where the
reference returns ``Erreur::Usage``). There is no fallback: importing fails loudly when the
library is missing, and every call runs the CUDA kernels.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

ICI = os.path.dirname(os.path.abspath(__file__))
CHEMIN_LIB = os.path.join(ICI, "_lib", "libtroncons_b200.so")

TRC_OK, TRC_ERR_USAGE, TRC_ERR_CUDA = 0, 1, 2


class ErreurUsage(ValueError):
    """A size, alignment or shape the kernels refuse before launching (Erreur::Usage)."""


class ErreurCuda(RuntimeError):
    """A CUDA launch error."""


class DimsExpert(C.Structure):
    """Rows and columns of an expert's three matrices (abi.rs:8-13): 24 bytes."""

    _fields_ = [("lignes", C.c_uint32 * 3), ("colonnes", C.c_uint32 * 3)]

    @classmethod
    def de(cls, lignes, colonnes) -> "DimsExpert":
        d = cls()
        for j in range(3):
            d.lignes[j] = lignes[j]
            d.colonnes[j] = colonnes[j]
        return d

    @classmethod
    def gpt_oss(cls) -> "DimsExpert":
        return cls.de([2880] * 3, [2880] * 3)


class DescGemv(C.Structure):
    """One product of a GEMV batch (abi.rs:16-27): 32 bytes."""

    _fields_ = [("matrice", C.c_uint64), ("x", C.c_uint64), ("y", C.c_uint64), ("lignes", C.c_uint32),
                ("colonnes", C.c_uint32)]


class DescCodage(C.Structure):
    """One expert of a GPU encode batch (trc_desc_codage): 72 bytes."""

    _fields_ = [("blocs", C.c_uint64 * 3), ("biais", C.c_uint64 * 3), ("sortie", C.c_uint64), ("capacite", C.c_uint64),
                ("expert", C.c_uint32), ("reserve", C.c_uint32)]


class DescDecodage(C.Structure):
    """One expert of a decode batch (abi.rs:32-53): 32 bytes."""

    _fields_ = [("partie", C.c_uint64), ("emplacement", C.c_uint64), ("luts", C.c_uint64), ("controle", C.c_uint64)]


class ParamsRope(C.Structure):
    """trc_params_rope (48 bytes; abi.rs:228-249)."""

    _fields_ = [("base", C.c_double), ("facteur", C.c_double), ("ctx_origine", C.c_double),
                ("beta_rapide", C.c_double), ("beta_lent", C.c_double), ("dim_tete", C.c_uint32),
                ("variante", C.c_uint32)]

    @classmethod
    def gpt_oss(cls) -> "ParamsRope":
        return cls(150000.0, 32.0, 4096.0, 32.0, 1.0, 64, 0)


class ParamsAttention(C.Structure):
    """trc_params_attention (32 bytes; abi.rs:254-290)."""

    _fields_ = [("tetes", C.c_uint32), ("tetes_kv", C.c_uint32), ("dim_tete", C.c_uint32), ("debut", C.c_uint32),
                ("fin", C.c_uint32), ("anneau", C.c_uint32), ("echelle", C.c_float), ("reserve", C.c_uint32)]

    @classmethod
    def gpt_oss(cls, position: int, fenetre: int) -> "ParamsAttention":
        """Position `position` of a gpt-oss layer: sliding (fenetre = 128, the even layers) or full
        (fenetre = 0) (abi.rs:278-283)."""
        fin = position + 1
        debut = max(0, fin - fenetre) if fenetre > 0 else 0
        return cls(64, 8, 64, debut, fin, fenetre, 0.125, 0)


class DescGemm(C.Structure):
    """trc_desc_gemm (56 bytes): one matrix of a batch of tensor-core GEMMs."""

    _fields_ = [("codes", C.c_uint64), ("echelles", C.c_uint64), ("biais", C.c_uint64), ("x", C.c_uint64),
                ("y", C.c_uint64), ("lignes", C.c_uint32), ("colonnes", C.c_uint32), ("n", C.c_uint32),
                ("x_bf16", C.c_uint32)]


class EchangePairs(C.Structure):
    """trc_echange_pairs: every rank's exchange buffer (device addresses in this process), this
    rank, the number of ranks."""

    _fields_ = [("tampons", C.c_uint64 * 8), ("rang", C.c_uint32), ("monde", C.c_uint32)]


class MoeCouche(C.Structure):
    """The fused MoE layer descriptor (trc_moe_couche)."""

    _fields_ = [("parties", C.c_void_p), ("parties_octets", C.c_void_p), ("experts", C.c_uint32), ("k", C.c_uint32),
                ("luts", C.c_void_p), ("dims", DimsExpert), ("indices", C.c_void_p), ("poids", C.c_void_p),
                ("x", C.c_void_p), ("x_bf16", C.c_uint32), ("brut", C.c_uint32), ("residu", C.c_void_p),
                ("controle", C.c_void_p), ("n_delta", C.c_uint32), ("n_codes", C.c_uint32),
                ("jetons", C.c_uint32), ("expert_debut", C.c_uint32), ("expert_fin", C.c_uint32),
                ("partiel", C.c_uint32), ("echange", C.c_void_p), ("deltas", C.c_void_p)]


def _charger() -> C.CDLL:
    if not os.path.exists(CHEMIN_LIB):
        raise ImportError(f"troncons_b200: {CHEMIN_LIB} is missing; build it with `python troncons_b200/construire.py` "
                          "(there is no CPU fallback)")
    lib = C.CDLL(CHEMIN_LIB)
    vp, sz, u32, u64, i32, i64 = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_int, C.c_int64
    pd = C.POINTER(DimsExpert)
    sig = {
        "trc_derniere_erreur": (C.c_char_p, []),
        "trc_taille_emplacement": (u64, [pd]),
        "trc_decoder_expert": (i32, [vp, sz, vp, sz, vp, sz, pd, vp, sz, vp]),
        "trc_decoder_lot": (i32, [vp, sz, u32, pd, vp]),
        "trc_copier_brut": (i32, [vp, sz, vp, sz, pd, vp, sz, vp]),
        "trc_gemv": (i32, [vp, sz, vp, sz, vp, sz, u32, u32, vp]),
        "trc_gemv_lot": (i32, [vp, sz, u32, u32, vp]),
        "trc_gemv_f32": (i32, [vp, sz, vp, sz, vp, sz, vp, sz, u32, u32, vp]),
        "trc_routeur_topk": (i32, [vp, sz, u32, u32, vp, sz, vp, sz, u64, u32, vp]),
        "trc_swiglu_oai": (i32, [vp, sz, vp, sz, vp, sz, u32, vp]),
        "trc_combiner": (i32, [vp, sz, vp, sz, u32, vp, sz, u32, u32, vp]),
        "trc_table_depuis_comptes": (i32, [vp, u32, vp]),
        "trc_lut_geometrie1": (i32, [vp, vp]),
        "trc_luts_couche": (i32, [vp, vp, vp]),
        "trc_comptes_matrice": (i32, [vp, u32, u32, i32, vp]),
        "trc_coder_partie": (i64, [vp, vp, pd, vp, i32, C.c_uint16, C.c_uint16, u32, u32, vp, sz, C.POINTER(u32)]),
        "trc_coder_partie_brute": (i64, [vp, vp, pd, C.c_uint16, C.c_uint16, vp, sz, C.POINTER(u32)]),
        "trc_synth_matrices": (i32, [u64, u32, u32, u32, u32, vp, vp, i32]),
        "trc_moe_espace_octets": (u64, [pd, u32]),
        "trc_moe_deltas_octets": (u64, [pd, u32]),
        "trc_moe_couche_ep": (i32, [vp, vp, sz, vp, vp]),
        "trc_gemm_mxfp4": (i32, [vp, vp, vp, u32, u32, vp, u32, u32, vp, vp, sz, vp, vp]),
        "trc_gemm_mxfp4_espace_octets": (u64, [u32, u32]),
        "trc_gemm_mxfp4_lot": (i32, [vp, u32, u32, u32, u32, vp, sz, vp, vp]),
        "trc_gemm_mxfp4_lot_espace_octets": (u64, [u32, u32, u32]),
        "trc_nccl_id": (i32, [vp, sz]),
        "trc_nccl_init": (i32, [C.POINTER(vp), u32, vp, u32]),
        "trc_nccl_fin": (i32, [vp]),
        "trc_moe_predecoder_deltas": (i32, [vp, vp, u64, vp, vp]),
        "trc_moe_espace_recouvrant_octets": (u64, [pd, u32]),
        "trc_moe_par_flux_espace_octets": (u64, [pd, u32, u32]),
        "trc_moe_couche_par_flux": (i32, [C.POINTER(MoeCouche), vp, sz, vp]),
        "trc_moe_par_flux_mma_espace_octets": (u64, [pd, u32, u32, u32]),
        "trc_moe_couche_par_flux_mma": (i32, [C.POINTER(MoeCouche), u32, vp, sz, vp, vp]),
        "trc_moe_couche_fusionnee": (i32, [C.POINTER(MoeCouche), vp, sz, vp]),
        "trc_moe_couche_chrono": (i32, [C.POINTER(MoeCouche), vp, sz, vp, C.POINTER(vp)]),
        "trc_moe_couche_sans_alloc": (i32, [C.POINTER(MoeCouche), vp]),
        "trc_echange_octets": (u64, [pd, u32, u32]),
        "trc_coder_flux_gpu_espace": (u64, [u32, u32]),
        "trc_coder_flux_gpu": (i32, [vp, u32, u32, vp, u32, vp, u32, vp, sz, vp, vp, sz, vp]),
        "trc_coder_parties_gpu_espace": (u64, [pd, u32, u32, u32]),
        "trc_coder_parties_gpu": (i32, [vp, sz, u32, pd, vp, i32, C.c_uint16, u32, u32, vp, sz, vp, sz, vp]),
        "trc_comptes_gpu": (i32, [vp, sz, u32, pd, i32, vp, sz, vp]),
        "trc_gemv_q8_0": (i32, [vp, sz, vp, sz, vp, sz, vp, sz, u32, u32, vp]),
        "trc_rmsnorm": (i32, [vp, sz, vp, sz, vp, sz, u32, u32, C.c_float, vp]),
        "trc_rope_yarn": (i32, [vp, sz, vp, sz, u32, u32, u32, C.POINTER(ParamsRope), vp]),
        "trc_ecrire_kv": (i32, [vp, sz, vp, sz, vp, sz, vp, sz, u32, u32, vp]),
        "trc_attention": (i32, [vp, sz, vp, sz, vp, sz, vp, sz, vp, sz, C.POINTER(ParamsAttention), vp]),
        "trc_routeur": (i32, [vp, vp, vp, u32, u32, u32, u32, u32, vp, vp, vp, vp]),
    }
    for nom, (res, args) in sig.items():
        f = getattr(lib, nom)
        f.restype = res
        f.argtypes = args
    return lib


lib = _charger()


def verifier(statut: int) -> None:
    """Raises the error a non-zero status stands for."""
    if statut == TRC_OK:
        return
    msg = lib.trc_derniere_erreur().decode()
    if statut == TRC_ERR_USAGE:
        raise ErreurUsage(msg)
    raise ErreurCuda(msg)


@dataclass(frozen=True)
class VueCarte:
    """A non-owning view of device memory: address and bytes (ARCHITECTURE.md 5.6 `VueCarte`)."""

    adresse: int
    octets: int

    @classmethod
    def de(cls, t) -> "VueCarte":
        """View of a CUDA torch tensor (contiguous)."""
        return cls(int(t.data_ptr()), int(t.numel() * t.element_size()))

    def vue(self, decalage: int, octets: int) -> "VueCarte":
        assert decalage + octets <= self.octets
        return VueCarte(self.adresse + decalage, octets)


def _v(x) -> VueCarte:
    if x is None:
        return VueCarte(0, 0)
    return x if isinstance(x, VueCarte) else VueCarte.de(x)


def _flux(flux) -> int:
    if flux is None:
        import torch

        return int(torch.cuda.current_stream().cuda_stream)
    return int(flux.cuda_stream) if hasattr(flux, "cuda_stream") else int(flux)


def taille_emplacement(dims: DimsExpert) -> int:
    return int(lib.trc_taille_emplacement(C.byref(dims)))


class Noyaux:
    """The reference's kernel contract (trc_noyaux::Noyaux), over the C-ABI. Views are
    ``VueCarte`` or CUDA tensors; ``flux`` is a torch stream, a raw handle, or None (torch's
    current stream)."""

    def decoder_expert(self, partie, emplacement, luts, dims: DimsExpert, controle, flux=None) -> None:
        p, e, l, c = _v(partie), _v(emplacement), _v(luts), _v(controle)
        verifier(lib.trc_decoder_expert(p.adresse, p.octets, e.adresse, e.octets, l.adresse, l.octets, C.byref(dims),
                                        c.adresse, c.octets, _flux(flux)))

    def decoder_lot(self, descs, n: int, dims: DimsExpert, flux=None) -> None:
        d = _v(descs)
        verifier(lib.trc_decoder_lot(d.adresse, d.octets, n, C.byref(dims), _flux(flux)))

    def copier_brut(self, partie, emplacement, dims: DimsExpert, controle, flux=None) -> None:
        p, e, c = _v(partie), _v(emplacement), _v(controle)
        verifier(lib.trc_copier_brut(p.adresse, p.octets, e.adresse, e.octets, C.byref(dims), c.adresse, c.octets,
                                     _flux(flux)))

    def gemv(self, matrice, x, y, lignes: int, colonnes: int, flux=None) -> None:
        m, xv, yv = _v(matrice), _v(x), _v(y)
        verifier(lib.trc_gemv(m.adresse, m.octets, xv.adresse, xv.octets, yv.adresse, yv.octets, lignes, colonnes,
                              _flux(flux)))

    def gemv_lot(self, descs, n: int, lignes_max: int, flux=None) -> None:
        d = _v(descs)
        verifier(lib.trc_gemv_lot(d.adresse, d.octets, n, lignes_max, _flux(flux)))

    def gemv_f32(self, w, x, biais, y, lignes: int, colonnes: int, flux=None) -> None:
        wv, xv, bv, yv = _v(w), _v(x), _v(biais), _v(y)
        verifier(lib.trc_gemv_f32(wv.adresse, wv.octets, xv.adresse, xv.octets, bv.adresse or None, bv.octets,
                                  yv.adresse, yv.octets, lignes, colonnes, _flux(flux)))

    def routeur_topk(self, logits, experts: int, k: int, indices, poids, boite: int = 0, sequence: int = 0,
                     flux=None) -> None:
        lv, iv, pv = _v(logits), _v(indices), _v(poids)
        verifier(lib.trc_routeur_topk(lv.adresse, lv.octets, experts, k, iv.adresse, iv.octets, pv.adresse, pv.octets,
                                      boite, sequence, _flux(flux)))

    def swiglu_oai(self, g, u, y, n: int, flux=None) -> None:
        gv, uv, yv = _v(g), _v(u), _v(y)
        verifier(lib.trc_swiglu_oai(gv.adresse, gv.octets, uv.adresse, uv.octets, yv.adresse, yv.octets, n,
                                    _flux(flux)))

    def combiner(self, residu, sorties, pas: int, poids, n: int, d: int, flux=None) -> None:
        rv, sv, pv = _v(residu), _v(sorties), _v(poids)
        verifier(lib.trc_combiner(rv.adresse, rv.octets, sv.adresse, sv.octets, pas, pv.adresse or None, pv.octets, n,
                                  d, _flux(flux)))

    # ---------------------------------------------------------------- new entry points

    def routeur(self, wr, br, x, x_bf16: bool, experts: int, colonnes: int, k: int, logits, indices, poids,
                flux=None, jetons: int = 1) -> None:
        verifier(lib.trc_routeur(_v(wr).adresse, _v(br).adresse or None, _v(x).adresse, int(x_bf16), experts, colonnes,
                                 k, jetons, _v(logits).adresse, _v(indices).adresse, _v(poids).adresse, _flux(flux)))

    def moe_couche(self, desc: MoeCouche, espace, flux=None, evenements=None) -> None:
        """The fused layer; `evenements`: 6 raw cudaEvent_t handles (ints) recorded between its
        phases (trc_moe_couche_chrono), or None."""
        e = _v(espace)
        if evenements is None:
            verifier(lib.trc_moe_couche_fusionnee(C.byref(desc), e.adresse, e.octets, _flux(flux)))
        else:
            ev = (C.c_void_p * 6)(*[int(v) if v else None for v in evenements])
            verifier(lib.trc_moe_couche_chrono(C.byref(desc), e.adresse, e.octets, _flux(flux), ev))

    # ---------------------------------------------------------------- attention side

    def gemv_q8_0(self, w, x, biais, y, lignes: int, colonnes: int, flux=None) -> None:
        wv, xv, bv, yv = _v(w), _v(x), _v(biais), _v(y)
        verifier(lib.trc_gemv_q8_0(wv.adresse, wv.octets, xv.adresse, xv.octets, bv.adresse or None, bv.octets,
                                   yv.adresse, yv.octets, lignes, colonnes, _flux(flux)))

    def rmsnorm(self, x, w, y, n: int, lignes: int, eps: float, flux=None) -> None:
        xv, wv, yv = _v(x), _v(w), _v(y)
        verifier(lib.trc_rmsnorm(xv.adresse, xv.octets, wv.adresse, wv.octets, yv.adresse, yv.octets, n, lignes, eps,
                                 _flux(flux)))

    def rope_yarn(self, q, k, tetes_q: int, tetes_k: int, position: int, p: ParamsRope, flux=None) -> None:
        qv, kv = _v(q), _v(k)
        verifier(lib.trc_rope_yarn(qv.adresse, qv.octets, kv.adresse, kv.octets, tetes_q, tetes_k, position,
                                   C.byref(p), _flux(flux)))

    def ecrire_kv(self, k, v, cache_k, cache_v, dkv: int, case_kv: int, flux=None) -> None:
        a, b, ck, cv = _v(k), _v(v), _v(cache_k), _v(cache_v)
        verifier(lib.trc_ecrire_kv(a.adresse, a.octets, b.adresse, b.octets, ck.adresse, ck.octets, cv.adresse,
                                   cv.octets, dkv, case_kv, _flux(flux)))

    def attention(self, q, cache_k, cache_v, puits, sortie, p: ParamsAttention, flux=None) -> None:
        qv, ck, cv, pv, sv = _v(q), _v(cache_k), _v(cache_v), _v(puits), _v(sortie)
        verifier(lib.trc_attention(qv.adresse, qv.octets, ck.adresse, ck.octets, cv.adresse, cv.octets, pv.adresse,
                                   pv.octets, sv.adresse, sv.octets, C.byref(p), _flux(flux)))

    def moe_couche_sans_alloc(self, desc: MoeCouche, flux=None) -> None:
        """The fused layer on the library's fixed 8 MiB device workspace (no workspace argument,
        nothing allocated), for callers that cannot allocate device memory where they run the
        layer. Calls that may overlap in time on one device race on that workspace; the first
        call on each device looks its address up, so make it before any stream capture."""
        verifier(lib.trc_moe_couche_sans_alloc(C.byref(desc), _flux(flux)))


def coder_flux_gpu(src, freqs, kappa=None, N: int = 256, flux=None) -> bytes:
    """A geometry-1 stream encoded on the GPU (trc_coder_flux_gpu): `src` a CUDA uint8 tensor of
    P bytes (P a multiple of 128), `freqs` a CUDA uint16 tensor [n_tables][256], `kappa` a CUDA
    uint8 tensor of per-16-byte-block contexts or None. Returns the stream's bytes (synchronises)."""
    import torch

    P = src.numel()
    T = (P // 128 + N - 1) // N
    cap = 16 + 132 * T + 2 * P + 4096
    sortie = torch.zeros(cap, dtype=torch.uint8, device=src.device)
    octets = torch.zeros(1, dtype=torch.int64, device=src.device)
    n_esp = int(lib.trc_coder_flux_gpu_espace(P, N))
    espace = torch.empty(n_esp + 256, dtype=torch.uint8, device=src.device)
    e = espace.data_ptr() + (-espace.data_ptr()) % 256
    n_tables = freqs.numel() // 256
    verifier(lib.trc_coder_flux_gpu(src.data_ptr(), P, N, kappa.data_ptr() if kappa is not None else None,
                                    kappa.numel() if kappa is not None else 0, freqs.data_ptr(), n_tables,
                                    sortie.data_ptr(), cap, octets.data_ptr(), e, n_esp, _flux(flux)))
    torch.cuda.current_stream().synchronize() if flux is None else flux.synchronize()
    n = int(octets.item())
    if n == 0 or n > cap:
        raise ValueError("encoding failed (a symbol absent from its table, or too long)")
    return sortie[:n].cpu().numpy().tobytes()


def echange_octets(dims: DimsExpert, jetons: int, monde: int) -> int:
    """Bytes of one rank's exchange buffer (trc_echange_octets)."""
    return int(lib.trc_echange_octets(C.byref(dims), jetons, monde))


def espace_octets(dims: DimsExpert, k: int) -> int:
    return int(lib.trc_moe_espace_octets(C.byref(dims), k))


def espace_recouvrant_octets(dims: DimsExpert, k: int) -> int:
    """The workspace with which the down projection's decode overlaps gate/up (k <= 8)."""
    return int(lib.trc_moe_espace_recouvrant_octets(C.byref(dims), k))
