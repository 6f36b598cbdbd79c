"""The whole decode step of a gpt-oss-shaped model over the C-ABI (``trc_modele_pas``), on seeded
synthetic weights drawn and encoded on the GPU: the reference's ``Modele`` (trc-modele/src/
lib.rs:342-568) with this library's kernels, the fused MoE layer in place of decode + GEMVs."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import DimsExpert, ParamsRope, lib, verifier

_u64, _u32, _vp, _sz, _i32 = C.c_uint64, C.c_uint32, C.c_void_p, C.c_size_t, C.c_int


class ModeleCouche(C.Structure):
    """trc_modele_couche: 160 bytes."""
    _fields_ = [(n, C.c_uint64) for n in ("attn_norm", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "puits",
                                            "post_norm", "wr", "br", "cache_k", "cache_v", "parties",
                                            "parties_octets", "luts")] + [("anneau", C.c_uint32), ("reserve", C.c_uint32),
                                                                          ("deltas", C.c_uint64)]


class ModeleConfig(C.Structure):
    """trc_modele_config: 176 bytes."""
    _fields_ = [(n, C.c_uint32) for n in ("couches", "d", "tetes", "tetes_kv", "dim_tete", "experts", "k", "vocab",
                                            "contexte", "brut", "n_delta", "n_codes")] + [
        ("eps", C.c_float), ("reserve", C.c_uint32), ("rope", ParamsRope), ("dims", DimsExpert),
        ("couches_desc", C.c_uint64), ("enchassement", C.c_uint64), ("norme_sortie", C.c_uint64),
        ("sortie", C.c_uint64), ("espace", C.c_uint64), ("espace_octets", C.c_uint64)]


for _n, (_r, _a) in {
    "trc_ligne_q8_0": (_i32, [_vp, _sz, _u32, _u32, _vp, _sz, _vp]),
    "trc_argmax": (_i32, [_vp, _sz, _u32, _vp, _sz, _vp]),
    "trc_modele_espace_octets": (_u64, [_vp]),
    "trc_modele_sorties": (_i32, [_vp, _vp, _vp, _vp]),
    "trc_modele_pas": (_i32, [_vp, _u32, _u32, _u32, _vp]),
    "trc_modele_debut": (_i32, [_vp, _u32, _vp]),
    "trc_modele_attention": (_i32, [_vp, _u32, _u32, _vp]),
    "trc_modele_moe": (_i32, [_vp, _u32, _vp]),
    "trc_modele_fin": (_i32, [_vp, _vp]),
    "trc_modele_etat": (_i32, [_vp, _vp, _vp]),
    "trc_modele_lot_espace_octets": (_u64, [_vp, _u32]),
    "trc_modele_attention_lot": (_i32, [_vp, _u32, _u32, _u32, _vp, _sz, _vp]),
    "trc_synth_mxfp4_gpu": (_i32, [_vp, _vp, _u32, _u32, _u64, _u64, _vp]),
    "trc_synth_q8_0_gpu": (_i32, [_vp, _u32, _u32, _u64, _u64, _vp]),
    "trc_synth_f32_gpu": (_i32, [_vp, _u64, _u64, _u64, C.c_float, C.c_float, _vp]),
    "trc_parties_brutes_gpu": (_i32, [_vp, _u32, _vp, _vp, _u32, _u64, _vp]),
}.items():
    getattr(lib, _n).restype = _r
    getattr(lib, _n).argtypes = _a


def _ident(*a) -> int:
    """A deterministic 48-bit id of a tensor's name (the stream of its draws)."""
    import hashlib

    return int.from_bytes(hashlib.blake2b(repr(a).encode(), digest_size=6).digest(), "little")


def _flux():
    import torch

    return torch.cuda.current_stream().cuda_stream


def biais_zipf(experts: int, s: float, placement: str, rangs: int, graine: int, couche: int) -> np.ndarray:
    """The router bias (f32[experts]) that gives layer `couche` Zipf(s)-shaped expert popularity:
    -s ln(1 + q) for the expert of popularity rank q (0 the most popular), experts numbered by
    `placement` (see Modele)."""
    q = np.arange(experts)
    if placement == "aleatoire":
        expert = np.random.default_rng([graine, couche, 0x5A1F]).permutation(experts)
    elif placement == "equilibre":
        if experts % rangs:
            raise ValueError(f"{experts} experts over {rangs} ranks")
        expert = (q % rangs) * (experts // rangs) + q // rangs
    else:
        raise ValueError(f"placement {placement!r}: 'aleatoire' or 'equilibre'")
    b = np.zeros(experts, np.float32)
    b[expert] = (-s * np.log1p(q)).astype(np.float32)
    return b


def synth_q8_0(R: int, C_: int, graine: int, matrice: int):
    import torch

    w = torch.empty(R * (C_ // 32) * 34, dtype=torch.uint8, device="cuda")
    verifier(lib.trc_synth_q8_0_gpu(w.data_ptr(), R, C_, graine, matrice, _flux()))
    return w


def synth_f32(n: int, graine: int, flux_id: int, moyenne: float, ecart: float):
    import torch

    y = torch.empty(n, dtype=torch.float32, device="cuda")
    verifier(lib.trc_synth_f32_gpu(y.data_ptr(), n, graine, flux_id, moyenne, ecart, _flux()))
    return y


def entete_brute(dims: DimsExpert) -> tuple:
    """The header and stream table of a raw part (trc_coder_partie_brute's layout) and the part's
    size: ECHELLES_BRUTES (0x07), CODES_BRUTS (0x06), BIAIS (0x02) per matrix, each stream at an
    offset aligned to 16, zeros up to a multiple of 4096."""
    flux = []
    for j in range(3):
        R, B = dims.lignes[j], dims.colonnes[j] // 32
        flux += [(0x07, j, R * B), (0x06, j, 16 * R * B), (0x02, j, 4 * R)]
    p = 64 + 16 * len(flux)
    dec = []
    for _, _, n in flux:
        p = (p + 15) // 16 * 16
        dec.append(p)
        p += n
    utiles, total = p, (p + 4095) // 4096 * 4096
    h = np.zeros(64 + 16 * len(flux), np.uint8)
    h[0:4] = np.frombuffer(np.uint32(0x30435254).tobytes(), np.uint8)
    h[9] = 3
    h[10:12] = np.frombuffer(np.uint16(len(flux)).tobytes(), np.uint8)
    h[12:16] = np.frombuffer(np.uint32(utiles).tobytes(), np.uint8)
    for i, ((sorte, j, n), o) in enumerate(zip(flux, dec)):
        e = 64 + 16 * i
        h[e], h[e + 1], h[e + 2] = sorte, j, 0xFF
        h[e + 4:e + 16] = np.frombuffer(np.array([o, n, n], np.uint32).tobytes(), np.uint8)
    return h, total


class Modele:
    """A synthetic gpt-oss-shaped model (seeded; every tensor drawn on the GPU): `couches` layers of
    attention (Q8_0, GQA tetes / tetes_kv, head 64, sinks, YaRN, sliding window `fenetre` on even
    layers) and a MoE of `experts` MXFP4 experts of shape `dims`, top-`k`, their parts encoded as
    .trc v1.2 on the GPU (`compresse`) and / or raw (`brut`); Q8_0 embedding and unembedding of
    `vocab` rows. `pas` runs one token through trc_modele_pas on the chosen parts."""

    def __init__(self, couches: int, d: int, tetes: int, tetes_kv: int, experts: int, k: int, vocab: int,
                 contexte: int, ffn: int, fenetre: int = 128, graine: int = 1, compresse: bool = True,
                 brut: bool = False, lot: int = 32, eps: float = 1e-5, rope: ParamsRope | None = None,
                 tenus: tuple | None = None, reduire=None, zipf: float = 0.0, placement: str = "aleatoire",
                 rangs: int = 1, deltas_predecodes: bool = False):
        """`tenus` = (debut, fin): draw and encode only the experts [debut, fin) of every layer (an
        expert-parallel share; the others' parts are absent), their rANS tables built from the
        counts of all experts when `reduire` sums the share's counts over the ranks (an
        all-reduce: parallele.reduire_comptes), so every share's parts are byte for byte those of
        the whole model.

        `zipf` = s > 0 skews the experts' popularity: every layer's router bias gets
        -s ln(1 + rank), rank the expert's place in a popularity order, so that top-k routing
        picks experts with Zipf(s)-shaped frequencies. `placement` numbers the experts in that
        order: "aleatoire" (a seeded permutation per layer) or "equilibre" (popularity rank q goes
        to expert (q mod rangs) (E / rangs) + q div rangs: each of `rangs` contiguous shares holds
        every rangs-th most popular expert, a balanced load for expert parallelism).

        `deltas_predecodes`: every layer's DELTA streams decoded once after encoding
        (trc_moe_predecoder_deltas, 3 x 259,200 bytes per expert), so the compressed step skips
        the DELTA phase (the same logits)."""
        import torch

        import troncons_b200.synth as S

        self.couches, self.d, self.tetes, self.tetes_kv, self.dt = couches, d, tetes, tetes_kv, 64
        self.experts, self.k, self.vocab, self.contexte, self.fenetre = experts, k, vocab, contexte, fenetre
        self.graine, self.eps = graine, eps
        self.rope = rope or ParamsRope.gpt_oss()
        self.dims = DimsExpert.de([ffn, ffn, d], [d, d, ffn])
        dq, dkv = tetes * 64, tetes_kv * 64
        g = graine
        ident = _ident
        self._garde = []
        self.tenseurs = []
        for l in range(couches):
            t = {
                "attn_norm": synth_f32(d, g, ident("an", l), 1.0, 0.02),
                "wq": synth_q8_0(dq, d, g, ident("wq", l)), "bq": synth_f32(dq, g, ident("bq", l), 0.0, 0.01),
                "wk": synth_q8_0(dkv, d, g, ident("wk", l)), "bk": synth_f32(dkv, g, ident("bk", l), 0.0, 0.01),
                "wv": synth_q8_0(dkv, d, g, ident("wv", l)), "bv": synth_f32(dkv, g, ident("bv", l), 0.0, 0.01),
                "wo": synth_q8_0(d, dq, g, ident("wo", l)), "bo": synth_f32(d, g, ident("bo", l), 0.0, 0.01),
                "puits": synth_f32(tetes, g, ident("pu", l), 0.0, 1.0),
                "post_norm": synth_f32(d, g, ident("pn", l), 1.0, 0.02),
                "wr": synth_f32(experts * d, g, ident("wr", l), 0.0, 0.02),
                "br": synth_f32(experts, g, ident("br", l), 0.0, 0.01),
            }
            if zipf > 0:
                t["br"] += torch.from_numpy(biais_zipf(experts, zipf, placement, rangs, graine, l)).cuda()
            cases = fenetre if (l % 2 == 0 and fenetre) else contexte
            t["anneau"] = fenetre if (l % 2 == 0 and fenetre) else 0
            t["cache_k"] = torch.zeros(cases * dkv, dtype=torch.int16, device="cuda")
            t["cache_v"] = torch.zeros(cases * dkv, dtype=torch.int16, device="cuda")
            self.tenseurs.append(t)
        self.enchassement = synth_q8_0(vocab, d, g, ident("emb"))
        self.sortie_w = synth_q8_0(vocab, d, g, ident("out"))
        self.norme_sortie = synth_f32(d, g, ident("on"), 1.0, 0.02)
        # experts: draw the held experts of a layer on the GPU, count, tables, encode in batches
        self.tenus = tuple(tenus) if tenus is not None else (0, experts)
        if not 0 <= self.tenus[0] < self.tenus[1] <= experts:
            raise ValueError(f"expert share {self.tenus} of {experts}")
        ids = list(range(*self.tenus))
        self.parties = {"compresse": [], "brut": []}
        taille_src = sum(self.dims.lignes[j] * (self.dims.colonnes[j] // 32) * 17 for j in range(3))
        blocs = [[torch.empty(self.dims.lignes[j] * (self.dims.colonnes[j] // 32) * 17, dtype=torch.uint8,
                              device="cuda") for j in range(3)] for _ in ids]
        biais = [[torch.empty(self.dims.lignes[j], dtype=torch.float32, device="cuda") for j in range(3)]
                 for _ in ids]
        self.luts = []
        entete, taille_brute = entete_brute(self.dims)
        entete_dev = torch.from_numpy(entete).cuda()
        for l in range(couches):
            for i, e in enumerate(ids):
                for j in range(3):
                    verifier(lib.trc_synth_mxfp4_gpu(blocs[i][j].data_ptr(), biais[i][j].data_ptr(),
                                                     self.dims.lignes[j], self.dims.colonnes[j], g,
                                                     ident("ex", l, e, j), _flux()))
            if compresse:
                cpt = S.comptes_gpu(blocs, self.dims).cpu().numpy().astype(np.uint64).reshape(3, 4, 256)
                if reduire is not None:
                    cpt = reduire(cpt)
                freqs = S.tables_de_comptes(cpt)
                self.luts.append(torch.from_numpy(S.luts(freqs).view(np.int32)).cuda())
                self.parties["compresse"].append(self._encoder(blocs, biais, freqs, l, lot, taille_src, ids))
            else:
                self.luts.append(torch.zeros(3 * 4 * 4096, dtype=torch.int32, device="cuda"))
            if brut:
                self.parties["brut"].append(self._bruts(blocs, biais, entete_dev, taille_brute, ids))
        del blocs, biais
        torch.cuda.synchronize()
        self.deltas = []
        if compresse and deltas_predecodes:
            self._predecoder_deltas()
        self.actifs = "compresse" if compresse else "brut"
        self._monter()

    def _predecoder_deltas(self) -> None:
        """Each layer's held experts' DELTA decoded into self.deltas[l] (device uint8)."""
        import torch

        from . import MoeCouche

        n = int(lib.trc_moe_deltas_octets(C.byref(self.dims), self.experts))
        ctl = torch.zeros(4 * self.experts, dtype=torch.int32, device="cuda")
        for l in range(self.couches):
            _, adr, tailles = self.parties["compresse"][l]
            ta = torch.from_numpy(adr.view(np.int64)).cuda()
            tt = torch.from_numpy(tailles.view(np.int64)).cuda()
            out = torch.empty(n, dtype=torch.uint8, device="cuda")
            desc = MoeCouche()
            desc.parties, desc.parties_octets = ta.data_ptr(), tt.data_ptr()
            desc.experts = self.experts
            desc.luts = self.luts[l].data_ptr()
            desc.dims = self.dims
            verifier(lib.trc_moe_predecoder_deltas(C.byref(desc), out.data_ptr(), n, ctl.data_ptr(), _flux()))
            torch.cuda.synchronize()
            self.deltas.append(out)
        if int(ctl.abs().sum().item()) != 0:
            raise RuntimeError("DELTA predecode: integrity counters set")

    def _encoder(self, blocs, biais, freqs, couche: int, lot: int, taille_src: int, ids: list):
        """The layer's held experts `ids` encoded on the GPU in batches of `lot`, then packed back to
        back (each part 4096-aligned) in one buffer: (buffer, addresses u64[E], sizes u64[E]), 0
        for the experts not held."""
        import torch

        import troncons_b200.synth as S

        f = torch.from_numpy(np.ascontiguousarray(freqs, np.uint16).reshape(-1).view(np.int16)).cuda()
        cap = (taille_src * 11 // 10 + (1 << 16) + 4095) // 4096 * 4096
        morceaux, tailles = [], []
        for e0 in range(0, len(ids), lot):
            n = min(lot, len(ids) - e0)
            sorties = torch.empty(n * cap, dtype=torch.uint8, device="cuda")
            descs = S._descs_gpu(blocs[e0:e0 + n], biais[e0:e0 + n], ids[e0:e0 + n],
                                 [sorties[i * cap:(i + 1) * cap] for i in range(n)], cap)
            octets = torch.zeros(2 * n, dtype=torch.int64, device="cuda")
            n_esp = int(lib.trc_coder_parties_gpu_espace(C.byref(self.dims), n, 256, 256))
            esp = torch.empty(n_esp + 256, dtype=torch.uint8, device="cuda")
            verifier(lib.trc_coder_parties_gpu(descs.data_ptr(), descs.numel(), n, C.byref(self.dims), f.data_ptr(), 1,
                                               couche, 256, 256, octets.data_ptr(), octets.numel() * 8,
                                               esp.data_ptr() + (-esp.data_ptr()) % 256, n_esp, _flux()))
            o = octets.cpu().numpy()
            for i in range(n):
                if o[2 * i] == 0 or o[2 * i] > cap:
                    raise RuntimeError(f"layer {couche}, expert {ids[e0 + i]}: part not encoded ({o[2 * i]} bytes)")
                morceaux.append(sorties[i * cap:i * cap + int(o[2 * i])])
                tailles.append(int(o[2 * i]))
            self._garde.append((sorties, descs, esp))
        tampon = torch.empty(sum(tailles), dtype=torch.uint8, device="cuda")
        p = 0
        adr, octets = np.zeros(self.experts, np.uint64), np.zeros(self.experts, np.uint64)
        for e, m, t in zip(ids, morceaux, tailles):
            tampon[p:p + t].copy_(m)
            adr[e], octets[e] = tampon.data_ptr() + p, t
            p += t
        self._garde = []
        return tampon, adr, octets

    def _bruts(self, blocs, biais, entete_dev, taille: int, ids: list):
        import torch

        import troncons_b200.synth as S

        n = len(ids)
        tampon = torch.empty(n * taille, dtype=torch.uint8, device="cuda")
        descs = S._descs_gpu(blocs, biais, ids, [tampon[i * taille:(i + 1) * taille] for i in range(n)], taille)
        verifier(lib.trc_parties_brutes_gpu(descs.data_ptr(), n, C.byref(self.dims), entete_dev.data_ptr(),
                                            entete_dev.numel(), taille, _flux()))
        torch.cuda.synchronize()
        adr, octets = np.zeros(self.experts, np.uint64), np.zeros(self.experts, np.uint64)
        for i, e in enumerate(ids):
            adr[e], octets[e] = tampon.data_ptr() + i * taille, taille
        return tampon, adr, octets

    def _monter(self):
        """The descriptor of the parts chosen by self.actifs, and the workspace."""
        import torch

        self._tables = []
        for l in range(self.couches):
            _, adr, tailles = self.parties[self.actifs][l]
            self._tables.append((torch.from_numpy(adr.view(np.int64)).cuda(),
                                 torch.from_numpy(tailles.view(np.int64)).cuda()))
        self.desc_couches, self.config, self.espace, self._sorties = self._config(
            [(t["cache_k"], t["cache_v"]) for t in self.tenseurs])

    def _config(self, caches):
        """(layer descriptors, trc_modele_config, workspace, output addresses) of a sequence whose
        KV caches are `caches` [(k, v)] per layer, over this model's weights and chosen parts."""
        import torch

        desc = (ModeleCouche * self.couches)()
        for l, t in enumerate(self.tenseurs):
            ta, tt = self._tables[l]
            c = desc[l]
            for n in ("attn_norm", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "puits", "post_norm", "wr", "br"):
                setattr(c, n, t[n].data_ptr())
            c.cache_k, c.cache_v = caches[l][0].data_ptr(), caches[l][1].data_ptr()
            c.parties, c.parties_octets, c.luts = ta.data_ptr(), tt.data_ptr(), self.luts[l].data_ptr()
            c.anneau = t["anneau"]
            dl = self.deltas[l] if (self.deltas and self.actifs == "compresse") else None
            c.deltas = dl.data_ptr() if dl is not None else 0
        m = ModeleConfig()
        m.couches, m.d, m.tetes, m.tetes_kv, m.dim_tete = self.couches, self.d, self.tetes, self.tetes_kv, 64
        m.experts, m.k, m.vocab, m.contexte = self.experts, self.k, self.vocab, self.contexte
        m.brut = int(self.actifs == "brut")
        m.eps = self.eps
        m.rope = self.rope
        m.dims = self.dims
        m.couches_desc = C.addressof(desc)
        m.enchassement, m.norme_sortie, m.sortie = (self.enchassement.data_ptr(), self.norme_sortie.data_ptr(),
                                                    self.sortie_w.data_ptr())
        n = int(lib.trc_modele_espace_octets(C.byref(m)))
        espace = torch.zeros(n + 256, dtype=torch.uint8, device="cuda")
        m.espace = espace.data_ptr() + (-espace.data_ptr()) % 256
        m.espace_octets = n
        lg, jt, ct = C.c_uint64(), C.c_uint64(), C.c_uint64()
        verifier(lib.trc_modele_sorties(C.byref(m), C.byref(lg), C.byref(jt), C.byref(ct)))
        return desc, m, espace, (lg.value, jt.value, ct.value)

    def choisir(self, actifs: str) -> None:
        """Run on the compressed ("compresse") or raw ("brut") parts; the KV caches are cleared."""
        if not self.parties[actifs]:
            raise ValueError(f"no {actifs} parts in this model")
        self.actifs = actifs
        for t in self.tenseurs:
            t["cache_k"].zero_()
            t["cache_v"].zero_()
        self._monter()

    def pas(self, jeton: int, position: int, sortie: bool = True, flux=None) -> None:
        verifier(lib.trc_modele_pas(C.byref(self.config), jeton, position, int(sortie),
                                    (flux.cuda_stream if flux is not None else _flux())))

    def vues(self):
        """(logits f32[vocab], token u32[1], controle u32[4k]) as torch tensors on the workspace."""
        return _vues(self.espace, self._sorties, self.vocab, self.k)


def _vues(espace, sorties, vocab: int, k: int):
    import torch

    o0, o1, o2 = (a - espace.data_ptr() for a in sorties)
    return (espace[o0:o0 + 4 * vocab].view(torch.float32), espace[o1:o1 + 4].view(torch.int32),
            espace[o2:o2 + 16 * k].view(torch.int32))


class Sequence:
    """Another sequence over a Modele's weights and parts: its own KV caches and workspace, the
    same step (trc_modele_pas and its phases) on its own descriptor. `monter` follows the model's
    current choice of parts (call it after Modele.choisir); `effacer` clears the caches."""

    def __init__(self, m: Modele):
        import torch

        self.m = m
        self.caches = [(torch.zeros_like(t["cache_k"]), torch.zeros_like(t["cache_v"])) for t in m.tenseurs]
        self.monter()

    def monter(self) -> None:
        self.desc_couches, self.config, self.espace, self._sorties = self.m._config(self.caches)

    def effacer(self) -> None:
        for k, v in self.caches:
            k.zero_()
            v.zero_()

    def pas(self, jeton: int, position: int, sortie: bool = True, flux=None) -> None:
        verifier(lib.trc_modele_pas(C.byref(self.config), jeton, position, int(sortie),
                                    (flux.cuda_stream if flux is not None else _flux())))

    def vues(self):
        return _vues(self.espace, self._sorties, self.m.vocab, self.m.k)
