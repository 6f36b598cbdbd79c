"""GPU: the expert-parallel layer through the C-ABI alone (trc_moe_couche_ep over an NCCL
communicator made by trc_nccl_id / trc_nccl_init), the path a host with no PyTorch takes (a Rust
engine): no torch.distributed anywhere, the unique id passed between the processes by a pipe.
PyTorch only allocates device memory here.

- one rank (a communicator of one, runs on a one-GPU box): the step is the fused layer's, bit
  for bit, step after step;
- two ranks (two GPUs, skipped otherwise): each holds half of the experts; after the step both
  ranks hold the same residual bits, within 1e-5 of max|r| of the whole layer on one GPU (the
  same terms summed in another order), with the same routing."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DIMS = ([256, 256, 512], [512, 512, 256])


def _comm(monde: int, rang: int, id_octets: bytes):
    import troncons_b200 as T

    comm = C.c_void_p()
    b = (C.c_uint8 * 128).from_buffer_copy(id_octets)
    assert T.lib.trc_nccl_init(C.byref(comm), monde, b, rang) == T.TRC_OK, T.lib.trc_derniere_erreur()
    return comm


def _nouvel_id() -> bytes:
    import troncons_b200 as T

    b = (C.c_uint8 * 128)()
    assert T.lib.trc_nccl_id(b, 128) == T.TRC_OK, T.lib.trc_derniere_erreur()
    return bytes(b)


def test_un_rang_egale_la_couche():
    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.carte import CoucheCarte

    torch.cuda.set_device(0)
    c = S.couche(77, T.DimsExpert.de(*DIMS), 8, brut=False)
    comm = _comm(1, 0, _nouvel_id())
    try:
        ep = CoucheCarte(c, k=4, brut=False, jetons=2)
        toute = CoucheCarte(c, k=4, brut=False, jetons=2)
        rng = np.random.default_rng(12)
        for _ in range(4):
            x = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
            r0 = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).cuda()
            a, b = r0.clone(), r0.clone()
            ep.couche_ep(x, a, comm.value)
            toute.couche(x, b)
            torch.cuda.synchronize()
            assert (ep.controle == 0).all()
            assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    finally:
        assert T.lib.trc_nccl_fin(comm) == T.TRC_OK


def _rang(rang: int, monde: int, tuyau, sortie):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.carte import CoucheCarte
    from troncons_b200.parallele import partage

    torch.cuda.set_device(rang)
    if rang == 0:
        ident = _nouvel_id()
        for _ in range(monde - 1):
            tuyau.put(ident)
    else:
        ident = tuyau.get(timeout=120)
    comm = _comm(monde, rang, ident)
    try:
        c = S.couche(77, T.DimsExpert.de(*DIMS), 8, brut=False)
        ep = CoucheCarte(c, k=4, brut=False, jetons=2, tenus=partage(8, rang, monde))
        toute = CoucheCarte(c, k=4, brut=False, jetons=2)
        rng = np.random.default_rng(21)
        res = []
        for _ in range(4):
            x = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
            r0 = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).cuda()
            a, b = r0.clone(), r0.clone()
            ep.couche_ep(x, a, comm.value)
            toute.couche(x, b)
            torch.cuda.synchronize()
            assert (ep.controle == 0).all() and torch.equal(ep.idx, toute.idx)
            ga, gb = a.cpu().numpy(), b.cpu().numpy()
            assert np.abs(ga - gb).max() <= 1e-5 * max(1.0, np.abs(gb).max())
            res.append(ga.view(np.uint32).copy())
        sortie.put((rang, np.stack(res)))
    finally:
        T.lib.trc_nccl_fin(comm)


def test_deux_rangs_sans_pytorch_distribue():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    tuyau, sortie = ctx.Queue(), ctx.Queue()
    ps = [ctx.Process(target=_rang, args=(r, 2, tuyau, sortie)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(sortie.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(res[0], res[1]), "the ranks' residuals differ"
