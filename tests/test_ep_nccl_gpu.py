"""GPU, two or more devices: the expert-parallel layer against the single-GPU layer.

Two ranks (one process per GPU) each draw and encode only their half of a layer's experts,
build the layer's tables from the counts summed over NCCL, then run expert-parallel steps on a
batch of 2 tokens: router on every rank, the fused layer on the rank's share, and the combine's
exchange, either NCCL (rank 0 adds into the residual, rank 1 writes its share alone, one SUM
all-reduce) or "pairs" (the combine kernel writes its share into every rank's symmetric buffer
over NVLink and sums the shares in rank order itself). Rank 0 also runs the whole layer on one
GPU; they agree within 1e-5 max|residual| (the same terms summed in another order) and route
the same experts. With "pairs" both ranks hold the same residual bits, step after step, also
when the step is replayed from a CUDA graph. Skipped with fewer than two GPUs."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _port_libre() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rang(rang, monde, port, echange="nccl"):
    import torch.distributed as dist

    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.carte import CoucheCarte
    from troncons_b200.parallele import CoucheEP, partage, reduire_comptes

    torch.cuda.set_device(rang)
    dev = torch.device("cuda", rang)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rang, world_size=monde,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        dims = T.DimsExpert.de([256, 256, 512], [512, 512, 256])
        part = S.couche(77, dims, 8, brut=False, tenus=partage(8, rang, monde), reduire=reduire_comptes(device=dev))
        ep = CoucheEP(part, rang, monde, k=4, jetons=2, echange=echange)
        toute = CoucheCarte(S.couche(77, dims, 8, brut=False), k=4, brut=False, jetons=2) if rang == 0 else None
        rng = np.random.default_rng(3)
        for _ in range(6):
            x = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
            r0 = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).cuda()
            r = r0.clone()
            ep.carte.controle.zero_()
            ep.etape(x, r)
            torch.cuda.synchronize()
            assert (ep.carte.controle == 0).all()
            if rang == 0:
                rt = r0.clone()
                toute.couche(x, rt)
                torch.cuda.synchronize()
                assert torch.equal(toute.idx, ep.carte.idx)
                a, b = r.cpu().numpy(), rt.cpu().numpy()
                assert np.abs(a - b).max() <= 1e-5 * max(1.0, np.abs(b).max())
            if echange == "pairs":
                tous = [torch.zeros_like(r) for _ in range(monde)]
                dist.all_gather(tous, r)
                assert all(torch.equal(tous[0].view(torch.int32), t.view(torch.int32)) for t in tous)
        if echange == "pairs":
            # the same step replayed from a CUDA graph: the exchange's sequence lives on the device
            xs = torch.zeros(2, 512, dtype=torch.bfloat16, device="cuda")
            rs = torch.zeros(2, 512, dtype=torch.float32, device="cuda")
            graphe = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graphe):
                ep.etape(xs, rs)
            for _ in range(3):
                x = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
                r0 = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).cuda()
                xs.copy_(x)
                rs.copy_(r0)
                graphe.replay()
                torch.cuda.synchronize()
                assert (ep.carte.controle == 0).all()
                if rang == 0:
                    rt = r0.clone()
                    toute.couche(x, rt)
                    torch.cuda.synchronize()
                    a, b = rs.cpu().numpy(), rt.cpu().numpy()
                    assert np.abs(a - b).max() <= 1e-5 * max(1.0, np.abs(b).max())
            del graphe
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("echange", ["nccl", "pairs"])
def test_ep_deux_gpus_egale_un_gpu(echange):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_rang, args=(2, _port_libre(), echange), nprocs=2, join=True, start_method="spawn")


@pytest.mark.parametrize("moe", ["fusionnee", "par_flux"])
def test_ep_un_rang_egale_la_couche(moe):
    """One rank holding every expert (no process group, no exchange): the expert-parallel layer's
    step is the fused layer's (trc_moe_couche_fusionnee) bit for bit, for either MoE form (par
    flux gives the fused layer's bits), step after step. Runs on a one-GPU box, so a fault in the
    layer's construction or step cannot hide behind the two-GPU skip."""
    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.carte import CoucheCarte
    from troncons_b200.parallele import CoucheEP

    torch.cuda.set_device(0)
    dims = T.DimsExpert.de([256, 256, 512], [512, 512, 256])
    c = S.couche(78, dims, 8, brut=False)
    ep = CoucheEP(c, 0, 1, k=4, jetons=3, moe=moe)
    assert ep.echange == "aucun" and ep.carte.tenus == (0, 8)
    toute = CoucheCarte(c, k=4, brut=False, jetons=3)
    rng = np.random.default_rng(5)
    for _ in range(4):
        x = torch.from_numpy(rng.standard_normal((3, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
        r0 = torch.from_numpy(rng.standard_normal((3, 512)).astype(np.float32)).cuda()
        r, rt = r0.clone(), r0.clone()
        ep.etape(x, r)
        toute.couche(x, rt)
        torch.cuda.synchronize()
        assert (ep.carte.controle == 0).all() and (toute.controle == 0).all()
        assert torch.equal(ep.carte.idx, toute.idx)
        assert torch.equal(r.view(torch.int32), rt.view(torch.int32))
