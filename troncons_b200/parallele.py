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


def etape_ep(calcul_local, residu, rang: int, groupe=None) -> None:
    """One expert-parallel step: `calcul_local(residu, partiel)` runs this rank's share of the
    layer on `residu` ([tokens][d] f32; rank 0 adds into it, the others overwrite it with their
    share, partiel = True), then a SUM all-reduce gives every rank the whole layer's result."""
    import torch.distributed as dist

    calcul_local(residu, rang != 0)
    dist.all_reduce(residu, op=dist.ReduceOp.SUM, group=groupe)


class CoucheEP:
    """This rank's share of a layer on its GPU: the parts of its experts, the layer's LUTs and
    the router; `etape` runs router + fused share + the combine's exchange on the current stream."""

    def __init__(self, c, rang: int, monde: int, k: int = 4, jetons: int = 1, groupe=None, echange: str = "pairs"):
        from .carte import CoucheCarte

        self.rang, self.monde, self.groupe = rang, monde, groupe
        self.tenus = partage(c.experts, rang, monde)
        self.carte = CoucheCarte(c, k=k, brut=False, jetons=jetons, tenus=self.tenus)
        self.echange = echange if monde > 1 else "aucun"
        self.paires = None
        if self.echange == "pairs":
            self._monter_paires(c, jetons)

    def _monter_paires(self, c, jetons: int) -> None:
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        from . import EchangePairs, echange_octets

        groupe = self.groupe if self.groupe is not None else dist.group.WORLD
        n = echange_octets(c.dims, jetons, self.monde)
        self.tampon = symm.empty(n, dtype=torch.uint8, device=torch.device("cuda", torch.cuda.current_device()))
        self.tampon.zero_()
        self.poignee = symm.rendezvous(self.tampon, groupe)
        ptrs = [int(p) for p in self.poignee.buffer_ptrs]
        if len(ptrs) != self.monde or any(p % 256 for p in ptrs):
            raise RuntimeError(f"symmetric memory: {len(ptrs)} buffers for {self.monde} ranks, or misaligned")
        tampons = (C.c_uint64 * 8)(*(ptrs + [0] * (8 - len(ptrs))))
        self.paires = EchangePairs(tampons, self.rang, self.monde)
        torch.cuda.synchronize()
        dist.barrier(group=self.groupe)  # every buffer zeroed before any rank's first exchange

    def local(self, x, residu, partiel: bool, flux=None) -> None:
        self.carte.couche(x, residu, flux=flux, partiel=partiel)

    def etape(self, x, residu, flux=None) -> None:
        """One step: every rank ends with the whole layer's residual."""
        if self.echange == "pairs":
            self.carte.couche(x, residu, flux=flux, echange=self.paires)
        elif self.echange == "nccl":
            etape_ep(lambda r, p: self.local(x, r, p, flux), residu, self.rang, self.groupe)
        else:
            self.carte.couche(x, residu, flux=flux)
