"""Expert parallelism for the fused MoE layer: one process per GPU, each holding a contiguous
share of a layer's experts (16 of 128 per GPU at 8 GPUs).

Per step every rank runs the router on the same tokens (replicated weights, identical
results), then the fused layer on its share only: activations whose expert it does not hold are
skipped. The layer's one exchange is the weighted combine: rank 0 adds its share's weighted sum
into the residual, every other rank writes its share's sum alone (a partial combine), and one
SUM all-reduce of [tokens][d] f32 over NCCL (NVLink) leaves residual + the sum over all experts
on every rank. This replaces the reference's single-GPU `combiner` over the k experts
(trc-modele/src/lib.rs:533-553, noyaux/passe.cuh:611-622): the terms are the same, summed in
another order, so results agree within f32 rounding, not bit for bit, across GPU counts.

Two forms of the exchange: "nccl" (rank 0 adds its share into the residual, the others write
theirs alone, then one NCCL all-reduce), and "pairs" (the default: the combine kernel itself
writes its share into every rank's exchange buffer over NVLink peer stores, waits for the others'
flags and sums the shares in rank order: one kernel, no collective launch, and the same residual
bits on every rank). The exchange buffers are symmetric memory (torch.distributed's, one buffer
per rank mapped in every rank's address space).

The synthetic layer is drawn the same way: each rank draws and encodes only its experts, and
the layer's rANS tables come from the counts of all experts, summed by an all-reduce."""
from __future__ import annotations

import ctypes as C

import numpy as np


def partage(experts: int, rang: int, monde: int) -> tuple[int, int]:
    """The experts [debut, fin) of rank `rang` among `monde`: contiguous shares whose sizes
    differ by at most one (16 each for 128 experts on 8 ranks)."""
    if not 0 <= rang < monde or experts < monde:
        raise ValueError(f"rank {rang} of {monde} for {experts} experts")
    q, r = divmod(experts, monde)
    debut = rang * q + min(rang, r)
    return debut, debut + q + (1 if rang < r else 0)


def reduire_comptes(groupe=None, device=None):
    """A function summing a u64 count array over the ranks of `groupe` (all-reduce): pass it to
    synth.couche(reduire=...) so that every share builds the layer's tables from all experts."""
    import torch
    import torch.distributed as dist

    def reduire(c: np.ndarray) -> np.ndarray:
        t = torch.from_numpy(np.ascontiguousarray(c).astype(np.int64))
        if device is not None:
            t = t.to(device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=groupe)
        return t.cpu().numpy().astype(np.uint64)

    return reduire


ECHANGES = ("pairs", "nccl")
FORMES_MOE = ("fusionnee", "par_flux")


def verifier_arguments_ep(experts: int, rang: int, monde: int, k: int, jetons: int, echange: str,
                          moe: str) -> None:
    """Refuses a bad expert-parallel configuration before any device work (ValueError): the rank
    and share, k in 1..8, at least one token, a known exchange, and a known MoE form (par flux
    only with the NCCL exchange when several ranks share the layer)."""
    partage(experts, rang, monde)
    if not 1 <= k <= 8:
        raise ValueError(f"k = {k}: 1 to 8 routed experts per token")
    if jetons < 1:
        raise ValueError(f"{jetons} tokens per step")
    if echange not in ECHANGES:
        raise ValueError(f"exchange {echange!r}: one of {ECHANGES}")
    if moe not in FORMES_MOE or (moe == "par_flux" and echange == "pairs" and monde > 1):
        raise ValueError(f"MoE form {moe!r}: 'fusionnee', or 'par_flux' (with the NCCL exchange)")


def etape_ep(calcul_local, residu, rang: int, groupe=None) -> None:
    """One expert-parallel step: `calcul_local(residu, partiel)` runs this rank's share of the
    layer on `residu` ([tokens][d] f32; rank 0 adds into it, the others overwrite it with their
    share, partiel = True), then a SUM all-reduce gives every rank the whole layer's result."""
    import torch.distributed as dist

    calcul_local(residu, rang != 0)
    dist.all_reduce(residu, op=dist.ReduceOp.SUM, group=groupe)


def monter_paires(dims, jetons: int, rang: int, monde: int, groupe=None):
    """The combine's exchange buffers: one symmetric-memory buffer per rank (torch.distributed's),
    mapped in every rank's address space, zeroed on every rank before any exchange. Returns
    (buffer, handle, EchangePairs) (keep the first two alive as long as the third is used)."""
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm

    from . import EchangePairs, echange_octets

    g = groupe if groupe is not None else dist.group.WORLD
    n = echange_octets(dims, jetons, monde)
    tampon = symm.empty(n, dtype=torch.uint8, device=torch.device("cuda", torch.cuda.current_device()))
    tampon.zero_()
    poignee = symm.rendezvous(tampon, g)
    ptrs = [int(p) for p in poignee.buffer_ptrs]
    if len(ptrs) != monde or any(p % 256 for p in ptrs):
        raise RuntimeError(f"symmetric memory: {len(ptrs)} buffers for {monde} ranks, or misaligned")
    paires = EchangePairs((C.c_uint64 * 8)(*(ptrs + [0] * (8 - len(ptrs)))), rang, monde)
    torch.cuda.synchronize()
    dist.barrier(group=groupe)  # every buffer zeroed before any rank's first exchange
    return tampon, poignee, paires


class CoucheEP:
    """This rank's share of a layer on its GPU: the parts of its experts, the layer's LUTs and
    the router; `etape` runs router + fused share + the combine's exchange on the current stream."""

    def __init__(self, c, rang: int, monde: int, k: int = 4, jetons: int = 1, groupe=None, echange: str = "pairs",
                 moe: str = "fusionnee"):
        verifier_arguments_ep(c.experts, rang, monde, k, jetons, echange, moe)
        from .carte import CoucheCarte

        self.rang, self.monde, self.groupe = rang, monde, groupe
        self.tenus = partage(c.experts, rang, monde)
        self.moe = moe
        self.echange = echange if monde > 1 else "aucun"
        self.carte = CoucheCarte(c, k=k, brut=False, jetons=jetons, tenus=self.tenus)
        self.paires = None
        if self.echange == "pairs":
            self._monter_paires(c, jetons)

    def _monter_paires(self, c, jetons: int) -> None:
        self.tampon, self.poignee, self.paires = monter_paires(c.dims, jetons, self.rang, self.monde, self.groupe)

    def local(self, x, residu, partiel: bool, flux=None) -> None:
        if self.moe == "par_flux":
            self.carte.couche_par_flux(x, residu, flux=flux, partiel=partiel)
        else:
            self.carte.couche(x, residu, flux=flux, partiel=partiel)

    def etape(self, x, residu, flux=None) -> None:
        """One step: every rank ends with the whole layer's residual."""
        if self.echange == "pairs":
            self.carte.couche(x, residu, flux=flux, echange=self.paires)
        elif self.echange == "nccl":
            etape_ep(lambda r, p: self.local(x, r, p, flux), residu, self.rang, self.groupe)
        else:
            self.local(x, residu, False, flux)


class ModeleEP:
    """The expert-parallel decode step of a whole gpt-oss model: one process per GPU, `par_rang`
    sequences per rank (a batch of monde x par_rang), each rank holding its contiguous share of
    every layer's experts (16 of 128 at 8 GPUs) and a replica of the dense weights.

    Per layer (the phases of trc_modele_pas, with the exchange between them): the attention side
    of the rank's tokens (trc_modele_attention, or trc_modele_attention_lot for several sequences:
    their Q8_0 GEMVs launched once for all of them; the KV caches stay on the rank's GPU); an all-gather of the MoE inputs h2 ([monde x par_rang][d] f32, NCCL); the router
    on every token (replicated, identical on every rank); the fused layer on the rank's share for
    every token (or, with moe="par_flux", the layer par flux: each held expert routed to by any of
    the step's tokens decoded once, the same bits); then the combine's exchange. "nccl" (the default): each token's share written
    alone (partiel), a SUM reduce-scatter, added into each sequence's x. "pairs": the combine
    kernel writes each token's share into every rank's symmetric buffer over NVLink peer stores
    and adds all ranks' shares in rank order into [tokens][d] rows, this rank's rows holding its
    sequences' x (copied in before, out after); measured 3 % slower on the whole model at 2 GPUs
    (the copies and the zeroing; the step waits on the busiest rank's share either way). Then each
    sequence's unembedding and greedy token.

    The weighted experts' sum is the single-GPU combine's terms in another order (the shares
    summed across ranks), so the logits agree with the one-GPU model within f32 rounding, not
    bit for bit; with one rank and one sequence the step is trc_modele_pas's bits."""

    def __init__(self, rang: int, monde: int, groupe=None, echange: str = "nccl", par_rang: int = 1,
                 moe: str = "fusionnee", **modele):
        import torch

        from . import espace_recouvrant_octets
        from .modele import Modele, Sequence

        self.rang, self.monde, self.groupe, self.b = rang, monde, groupe, par_rang
        if not 1 <= par_rang or monde * par_rang > 128:
            raise ValueError(f"{par_rang} sequences per rank on {monde} ranks: 1 to 128 tokens per step")
        verifier_arguments_ep(modele["experts"], rang, monde, modele.get("k", 4), monde * par_rang, echange, moe)
        self.moe = moe
        self.echange = echange if monde > 1 else "aucun"
        self.tenus = partage(modele["experts"], rang, monde)
        modele.setdefault("rangs", monde)  # the balanced placement of a skewed popularity
        dev = torch.device("cuda", torch.cuda.current_device())
        self.m = Modele(**modele, tenus=self.tenus, reduire=reduire_comptes(groupe, dev) if monde > 1 else None)
        self.sequences = [self.m] + [Sequence(self.m) for _ in range(par_rang - 1)]
        m, n_tok = self.m, monde * par_rang
        f32 = torch.float32
        self.h2_locaux = torch.empty(par_rang * m.d, dtype=f32, device=dev)
        self.h2_tous = torch.empty(n_tok * m.d, dtype=f32, device=dev)
        self.y_tous = torch.empty(n_tok * m.d, dtype=f32, device=dev)
        self.y = torch.empty(par_rang * m.d, dtype=f32, device=dev)
        self.logits_routeur = torch.empty(n_tok * m.experts, dtype=f32, device=dev)
        self.idx = torch.empty(n_tok * m.k, dtype=torch.int32, device=dev)
        self.poids = torch.empty(n_tok * m.k, dtype=f32, device=dev)
        self.controle = torch.zeros(n_tok * m.k * 4, dtype=torch.int32, device=dev)
        if moe == "par_flux":
            from . import lib as _l

            n = int(_l.trc_moe_par_flux_espace_octets(C.byref(m.dims), m.experts, n_tok * m.k))
        else:
            n = espace_recouvrant_octets(m.dims, n_tok * m.k)
        self._espace = torch.empty(n + 256, dtype=torch.uint8, device=dev)
        self.espace_octets = n
        if self.echange == "pairs":
            self.tampon, self.poignee, self.paires = monter_paires(m.dims, n_tok, rang, monde, groupe)
        if par_rang > 1:
            from .modele import lib as _lib

            n_lot = int(_lib.trc_modele_lot_espace_octets(C.byref(m.config), par_rang))
            self._lot = torch.empty(n_lot + 256, dtype=torch.uint8, device=dev)
            self._lot_octets = n_lot
        self._monter()

    def _monter(self) -> None:
        import torch

        from . import MoeCouche, lib, verifier

        m, d_ = self.m, self.m.d
        self.x, self.h2 = [], []
        for q in self.sequences:
            x, h2 = C.c_uint64(), C.c_uint64()
            verifier(lib.trc_modele_etat(C.byref(q.config), C.byref(x), C.byref(h2)))
            base = q.espace.data_ptr()
            self.x.append(q.espace[x.value - base:x.value - base + 4 * d_].view(torch.float32))
            self.h2.append(q.espace[h2.value - base:h2.value - base + 4 * d_].view(torch.float32))
        # the MoE's input: this rank's h2 itself (one rank, one sequence), its sequences' h2
        # side by side (one rank), or every rank's (gathered)
        self._entree = self.h2[0] if (self.monde, self.b) == (1, 1) else (
            self.h2_locaux if self.monde == 1 else self.h2_tous)
        self.descs = []
        for l in range(m.couches):
            ta, tt = m._tables[l]
            d = MoeCouche()
            d.parties, d.parties_octets = ta.data_ptr(), tt.data_ptr()
            d.experts, d.k, d.luts, d.dims = m.experts, m.k, m.luts[l].data_ptr(), m.dims
            d.indices, d.poids = self.idx.data_ptr(), self.poids.data_ptr()
            d.x, d.x_bf16, d.brut = self._entree.data_ptr(), 0, int(m.actifs == "brut")
            d.residu, d.controle = self.y_tous.data_ptr(), self.controle.data_ptr()
            d.n_delta = d.n_codes = 0
            d.jetons = self.monde * self.b
            d.expert_debut, d.expert_fin = self.tenus
            if m.deltas and m.actifs == "compresse":  # DELTA decoded at load
                d.deltas = m.deltas[l].data_ptr()
            if self.echange == "pairs":
                d.partiel, d.echange = 0, C.addressof(self.paires)
            else:
                d.partiel = 1
            self.descs.append(d)
        rangs = self.y_tous.view(self.monde * self.b, d_)
        self._lignes = [rangs[self.rang * self.b + i] for i in range(self.b)]
        self._configs = (C.c_void_p * self.b)(*[C.addressof(q.config) for q in self.sequences])

    def choisir(self, actifs: str) -> None:
        """Run on the compressed or raw parts; every sequence's KV caches are cleared."""
        self.m.choisir(actifs)
        for q in self.sequences[1:]:
            q.effacer()
            q.monter()
        self._monter()

    def vues(self, i: int = 0):
        """(logits, greedy token, controle) of this rank's sequence i (see Modele.vues)."""
        return self.sequences[i].vues()

    def pas(self, jetons, position: int, sortie: bool = True, flux=None, journal: list | None = None) -> None:
        """This rank's tokens (an int, or one per sequence) at `position` (the same for all of the
        rank's sequences); every rank calls it once per step (the collectives pair them up).
        `journal`: a list that receives a device copy of every layer's routed experts."""
        import torch
        import torch.distributed as dist

        from . import lib, verifier

        jetons = [int(jetons)] if np.isscalar(jetons) else [int(j) for j in jetons]
        if len(jetons) != self.b:
            raise ValueError(f"{len(jetons)} tokens for {self.b} sequences")
        m, d_ = self.m, self.m.d
        cfgs = [C.byref(q.config) for q in self.sequences]
        s = flux or torch.cuda.current_stream()
        f = s.cuda_stream
        e = self._espace.data_ptr()
        e += (-e) % 256
        for cfg, j in zip(cfgs, jetons):
            verifier(lib.trc_modele_debut(cfg, j, f))
        with torch.cuda.stream(s):
            if self.echange == "pairs":
                # the exchange adds every rank's shares into all rows of y_tous; this rank's rows
                # carry its sequences' x through the layer, the other rows restart from 0 every step
                self.y_tous.zero_()
            lot = 0
            if self.b > 1:
                lot = self._lot.data_ptr()
                lot += (-lot) % 256
            for l in range(m.couches):
                t = m.tenseurs[l]
                if self.b > 1:  # the sequences' attention sides together (weights read once)
                    verifier(lib.trc_modele_attention_lot(self._configs, self.b, l, position, lot, self._lot_octets, f))
                else:
                    verifier(lib.trc_modele_attention(cfgs[0], l, position, f))
                if self._entree is not self.h2[0]:
                    for i in range(self.b):
                        self.h2_locaux[i * d_:(i + 1) * d_].copy_(self.h2[i])
                if self.monde > 1:
                    dist.all_gather_into_tensor(self.h2_tous, self.h2_locaux, group=self.groupe)
                verifier(lib.trc_routeur(t["wr"].data_ptr(), t["br"].data_ptr(), self._entree.data_ptr(), 0, m.experts,
                                         d_, m.k, self.monde * self.b, self.logits_routeur.data_ptr(),
                                         self.idx.data_ptr(), self.poids.data_ptr(), f))
                if journal is not None:
                    journal.append(self.idx.clone())
                if self.echange == "pairs":
                    for i in range(self.b):
                        self._lignes[i].copy_(self.x[i])
                    verifier(lib.trc_moe_couche_fusionnee(C.byref(self.descs[l]), e, self.espace_octets, f))
                    for i in range(self.b):
                        self.x[i].copy_(self._lignes[i])
                    continue
                couche = lib.trc_moe_couche_par_flux if self.moe == "par_flux" else lib.trc_moe_couche_fusionnee
                verifier(couche(C.byref(self.descs[l]), e, self.espace_octets, f))
                if self.monde > 1:
                    dist.reduce_scatter_tensor(self.y, self.y_tous, op=dist.ReduceOp.SUM, group=self.groupe)
                    for i in range(self.b):
                        self.x[i].add_(self.y[i * d_:(i + 1) * d_])
                else:
                    for i in range(self.b):
                        self.x[i].add_(self._lignes[i])
        if sortie:
            for cfg in cfgs:
                verifier(lib.trc_modele_fin(cfg, f))
