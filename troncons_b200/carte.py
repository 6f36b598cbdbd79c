"""Device plumbing around the C-ABI for a synthetic MoE layer: uploads a layer's parts, LUTs and
router to HBM (PyTorch allocations), and runs the layer three ways on the same stream:

- ``fusionnee``: the fused path (trc_routeur + trc_moe_couche_fusionnee) on v1.2 parts;
- ``brute``: the same entry on the raw parts (the uncompressed MXFP4 path);
- ``decodee``: the reference's decode-then-multiply sequence (trc_decoder_lot into slots, then
  trc_gemv_lot, trc_swiglu_oai, trc_gemv_lot, trc_combiner), as trc-modele's fin_couche does.

All three give the same bits. PyTorch only provides memory and streams here.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import (DescDecodage, DescGemv, DimsExpert, MoeCouche, Noyaux, espace_octets, espace_recouvrant_octets,
               taille_emplacement)
from .synth import Couche


def _octets(b: bytes, alignement: int = 4096) -> int:
    return (len(b) + alignement - 1) // alignement * alignement


class CoucheCarte:
    """A layer on the device. `jetons`: tokens per call (x [jetons][d], residual [jetons][d],
    jetons * k activations). `tenus`: the experts [debut, fin) this device holds (an
    expert-parallel share: the other experts' parts may be None and are never read); None: all.
    `recouvrement`: a workspace large enough for the fastest schedule (decode-only launches whose
    GEMVs follow, up to 32 activations); else the sequential schedule's. `espace`: a workspace of
    exactly that many bytes instead (the schedule follows from its size). `deltas_predecodes`:
    decode every expert's DELTA streams once here, and skip that phase at each step."""

    def __init__(self, c: Couche, k: int = 4, brut: bool = True, device: str = "cuda", n_delta: int = 0,
                 n_codes: int = 0, jetons: int = 1, tenus=None, recouvrement: bool = True, espace: int = 0,
                 deltas_predecodes: bool = False):
        self.c = c
        self.k = k
        self.jetons = jetons
        self.tenus = tenus
        self.dims = c.dims
        self.dev = torch.device(device)
        self.n = Noyaux()
        E = c.experts
        self.parties, self.adresses, self.tailles = self._monter(c.parties)
        if brut and any(p is not None for p in c.parties_brutes):
            self.parties_b, self.adresses_b, self.tailles_b = self._monter(c.parties_brutes)
        else:
            self.parties_b = None
        self.octets_compresses = [len(p) if p is not None else 0 for p in c.parties]
        self.luts = torch.from_numpy(c.luts.view(np.int32).copy()).to(self.dev)
        self.wr = torch.from_numpy(c.wr).to(self.dev)
        self.br = torch.from_numpy(c.br).to(self.dev)
        self.logits = torch.zeros(jetons, E, dtype=torch.float32, device=self.dev)
        self.idx = torch.zeros(jetons * k, dtype=torch.int32, device=self.dev)
        self.poids = torch.zeros(jetons * k, dtype=torch.float32, device=self.dev)
        self.controle = torch.zeros(4 * jetons * k, dtype=torch.int32, device=self.dev)
        taille = espace or (espace_recouvrant_octets if recouvrement else espace_octets)(self.dims, jetons * k)
        self.espace = torch.empty(taille + 256, dtype=torch.uint8, device=self.dev)
        self.n_delta, self.n_codes = n_delta, n_codes
        d = self.dims
        self.R0, self.C0, self.R2 = d.lignes[0], d.colonnes[0], d.lignes[2]
        self.deltas = None
        if deltas_predecodes:
            self.predecoder_deltas()

    def predecoder_deltas(self, flux=None) -> None:
        """Decodes every held expert's DELTA streams once (trc_moe_predecoder_deltas); the compressed
        layer then reads those bytes instead of decoding DELTA at each step (the same results)."""
        from . import lib, verifier

        n = int(lib.trc_moe_deltas_octets(C.byref(self.dims), self.c.experts))
        self.deltas = torch.empty(n, dtype=torch.uint8, device=self.dev)
        self.controle_deltas = torch.zeros(4 * self.c.experts, dtype=torch.int32, device=self.dev)
        desc = MoeCouche()
        desc.parties, desc.parties_octets = self.adresses.data_ptr(), self.tailles.data_ptr()
        desc.experts = self.c.experts
        desc.luts = self.luts.data_ptr()
        desc.dims = self.dims
        desc.n_delta = self.n_delta
        f = (flux or torch.cuda.current_stream()).cuda_stream
        verifier(lib.trc_moe_predecoder_deltas(C.byref(desc), self.deltas.data_ptr(), n, self.controle_deltas.data_ptr(),
                                               f))

    def _monter(self, parties):
        """Uploads the parts (None: an expert not held here, address and size 0)."""
        parties = [p if p is not None else b"" for p in parties]
        tailles = [len(p) for p in parties]
        decal = np.cumsum([0] + [_octets(p) for p in parties])
        buf = np.zeros(max(int(decal[-1]), 1), np.uint8)
        for i, p in enumerate(parties):
            buf[decal[i]:decal[i] + len(p)] = np.frombuffer(p, np.uint8)
        t = torch.from_numpy(buf).to(self.dev)
        base = t.data_ptr()
        adresses = torch.tensor([base + int(o) if len(p) else 0 for o, p in zip(decal[:-1], parties)],
                                dtype=torch.int64, device=self.dev)
        tl = torch.tensor(tailles, dtype=torch.int64, device=self.dev)
        return t, adresses, tl

    def partie(self, x: int, brute: bool = False) -> torch.Tensor:
        """Device view (tensor slice) of expert x's part."""
        src = self.c.parties_brutes if brute else self.c.parties
        buf = self.parties_b if brute else self.parties
        o = sum(_octets(p) for p in src[:x] if p is not None)
        return buf[o:o + len(src[x])]

    def routeur(self, x: torch.Tensor, flux=None) -> None:
        """The router of every token of x ([jetons][d] or [d]): logits, top-k, weights."""
        self.n.routeur(self.wr, self.br, x, x.dtype == torch.bfloat16, self.c.experts, self.C0, self.k, self.logits,
                       self.idx, self.poids, flux, jetons=self.jetons)

    def descripteur(self, x: torch.Tensor, residu: torch.Tensor, brute: bool, partiel: bool = False,
                    echange=None) -> MoeCouche:
        if x.numel() != self.jetons * self.C0 or not x.is_contiguous() or x.device.type != "cuda":
            raise ValueError(f"x: {self.jetons} x {self.C0} contiguous elements on the device expected")
        if residu.numel() != self.jetons * self.R2 or residu.dtype != torch.float32 or not residu.is_contiguous():
            raise ValueError(f"residual: {self.jetons} x {self.R2} contiguous f32 expected")
        desc = MoeCouche()
        if brute:
            desc.parties, desc.parties_octets = self.adresses_b.data_ptr(), self.tailles_b.data_ptr()
        else:
            desc.parties, desc.parties_octets = self.adresses.data_ptr(), self.tailles.data_ptr()
        desc.experts = self.c.experts
        desc.k = self.k
        desc.luts = self.luts.data_ptr()
        desc.dims = self.dims
        desc.indices = self.idx.data_ptr()
        desc.poids = self.poids.data_ptr()
        desc.x = x.data_ptr()
        desc.x_bf16 = int(x.dtype == torch.bfloat16)
        desc.brut = int(brute)
        desc.residu = residu.data_ptr()
        desc.controle = self.controle.data_ptr()
        desc.n_delta, desc.n_codes = self.n_delta, self.n_codes
        desc.jetons = self.jetons
        if self.tenus is not None:
            desc.expert_debut, desc.expert_fin = self.tenus
        desc.partiel = int(partiel)
        desc.echange = C.addressof(echange) if echange is not None else None
        desc.deltas = self.deltas.data_ptr() if (self.deltas is not None and not brute) else None
        return desc

    def _espace(self):
        a = self.espace.data_ptr()
        d = (-a) % 256
        return self.espace[d:]

    def couche(self, x: torch.Tensor, residu: torch.Tensor, brute: bool = False, flux=None, routeur: bool = True,
               evenements=None, partiel: bool = False, echange=None):
        """Router then the fused layer; `residu` (f32) is updated in place (partiel: overwritten
        with this device's share of the combine; echange: an EchangePairs, the shares of every
        GPU summed by the combine kernel over peer memory)."""
        if routeur:
            self.routeur(x, flux)
        self._desc = self.descripteur(x, residu, brute, partiel, echange)  # alive while the launch reads it
        self.n.moe_couche(self._desc, self._espace(), flux, evenements)

    def couche_ep(self, x: torch.Tensor, residu: torch.Tensor, comm: int, flux=None, routeur: bool = True) -> None:
        """Router then this rank's step of the expert-parallel layer through the C-ABI
        (trc_moe_couche_ep): the fused layer on the experts held here (`tenus`), then the NCCL
        SUM all-reduce of the residual over the communicator `comm` (an ncclComm_t, e.g. from
        trc_nccl_init): every rank ends with the whole layer's result."""
        from . import lib, verifier

        if routeur:
            self.routeur(x, flux)
        self._desc = self.descripteur(x, residu, False)
        e = self._espace()
        f = (flux or torch.cuda.current_stream()).cuda_stream
        verifier(lib.trc_moe_couche_ep(C.byref(self._desc), e.data_ptr(), e.numel(), C.c_void_p(comm), f))

    def couche_par_flux(self, x: torch.Tensor, residu: torch.Tensor, flux=None, routeur: bool = True,
                        partiel: bool = False, mma_seuil: int = 0, brute: bool = False):
        """Router then the layer "par flux" (trc_moe_couche_par_flux): each distinct routed expert
        decoded once for the batch; the residuals are the fused layer's bits (also on the share
        `tenus`, and with `partiel`: the share's sum written alone). `mma_seuil` > 0: the experts
        with at least that many activations on the tensor cores (trc_moe_couche_par_flux_mma;
        within the quantization's tolerance, one wait on the stream for the routing)."""
        from . import lib, verifier

        if routeur:
            self.routeur(x, flux)
        cle = ("_espace_pf", mma_seuil)
        if getattr(self, "_cle_pf", None) != cle:
            if mma_seuil:
                n = int(lib.trc_moe_par_flux_mma_espace_octets(C.byref(self.dims), self.c.experts, self.jetons * self.k,
                                                                mma_seuil))
            else:
                n = int(lib.trc_moe_par_flux_espace_octets(C.byref(self.dims), self.c.experts, self.jetons * self.k))
            self._espace_pf = torch.empty(n + 256, dtype=torch.uint8, device=self.dev)
            self._n_pf = n
            self._cle_pf = cle
            self.erreur_pf = torch.zeros(1, dtype=torch.int32, device=self.dev)
        e = self._espace_pf.data_ptr() + (-self._espace_pf.data_ptr()) % 256
        self._desc_pf = self.descripteur(x, residu, brute, partiel)
        f = (flux or torch.cuda.current_stream()).cuda_stream
        if mma_seuil:
            verifier(lib.trc_moe_couche_par_flux_mma(C.byref(self._desc_pf), mma_seuil, e, self._n_pf,
                                                     self.erreur_pf.data_ptr(), f))
        else:
            verifier(lib.trc_moe_couche_par_flux(C.byref(self._desc_pf), e, self._n_pf, f))

    # ---------------------------------------------------------------- decode-then-multiply

    def preparer_decodee(self):
        """Slots and descriptors for the decode-then-multiply sequence (k slots)."""
        te = taille_emplacement(self.dims)
        self.te = (te + 255) // 256 * 256
        self.emplacements = torch.empty(self.k * self.te + 256, dtype=torch.uint8, device=self.dev)
        self.ctl_d = torch.zeros(4 * self.k, dtype=torch.int32, device=self.dev)
        self.g = torch.zeros(self.k, self.R0, dtype=torch.float32, device=self.dev)
        self.u = torch.zeros_like(self.g)
        self.h = torch.zeros_like(self.g)
        self.s = torch.zeros(self.k, self.R2, dtype=torch.float32, device=self.dev)
        self.x32 = torch.zeros(self.C0, dtype=torch.float32, device=self.dev)
        self.adresses_hote = self.adresses.cpu().numpy()

    def descripteurs_decodee(self, idx) -> tuple:
        """Device descriptors of the decode-then-multiply sequence for the routed experts `idx`
        (host integers, k of them): decoder_lot into the k slots, gemv_lot of gate and up on
        x32, gemv_lot of down on h. Returns (decode, gate/up, down) descriptor tensors."""
        base = self.emplacements.data_ptr()
        base += (-base) % 256
        d = self.dims
        descs = (DescDecodage * self.k)()
        for i, e in enumerate(idx):
            descs[i] = DescDecodage(int(self.adresses_hote[int(e)]), base + i * self.te, self.luts.data_ptr(),
                                    self.ctl_d.data_ptr() + 16 * i)
        dd = torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).to(self.dev)
        pas = [0, 0, 0]
        for j in range(3):
            R, Cc = d.lignes[j], d.colonnes[j]
            nb = R * (Cc // 32)
            eo = (nb * 16 + 255) & ~255
            bo = (eo + nb + 255) & ~255
            pas[j] = (bo + 4 * R + 255) & ~255
        off = [0, pas[0], pas[0] + pas[1]]
        gu = (DescGemv * (2 * self.k))()
        for i in range(self.k):
            for j in range(2):
                gu[2 * i + j] = DescGemv(base + i * self.te + off[j], self.x32.data_ptr(),
                                         (self.g if j == 0 else self.u)[i].data_ptr(), d.lignes[j], d.colonnes[j])
        dg = torch.frombuffer(bytearray(bytes(gu)), dtype=torch.uint8).to(self.dev)
        dn = (DescGemv * self.k)()
        for i in range(self.k):
            dn[i] = DescGemv(base + i * self.te + off[2], self.h[i].data_ptr(), self.s[i].data_ptr(), d.lignes[2],
                             d.colonnes[2])
        ddn = torch.frombuffer(bytearray(bytes(dn)), dtype=torch.uint8).to(self.dev)
        return dd, dg, ddn

    def sequence_decodee(self, descs, x: torch.Tensor, residu: torch.Tensor, flux=None) -> None:
        """The sequence itself on `descs` (descripteurs_decodee), with this library's kernels:
        decoder_lot, gemv_lot (gate, up), swiglu_oai, gemv_lot (down), combiner with the router's
        weights (self.poids)."""
        dd, dg, ddn = descs
        self.x32.copy_(x.float())
        self.n.decoder_lot(dd, self.k, self.dims, flux)
        self.n.gemv_lot(dg, 2 * self.k, self.R0, flux)
        self.n.swiglu_oai(self.g, self.u, self.h, self.k * self.R0, flux)
        self.n.gemv_lot(ddn, self.k, self.R2, flux)
        self.n.combiner(residu, self.s, self.R2, self.poids, self.k, self.R2, flux)

    def decodee(self, x: torch.Tensor, residu: torch.Tensor, flux=None):
        """Router, then decoder_lot into slots, gemv_lot (gate, up), swiglu, gemv_lot (down),
        combiner. Reads the router's indices on the host, as the reference's scheduler does."""
        self.routeur(x, flux)
        idx = self.idx.cpu().numpy()
        self._garde = self.descripteurs_decodee(idx)
        self.sequence_decodee(self._garde, x, residu, flux)
