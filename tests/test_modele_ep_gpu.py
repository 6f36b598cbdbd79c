"""GPU: the expert-parallel whole model (troncons_b200.parallele.ModeleEP), on a small synthetic
gpt-oss-shaped model (2 layers, 8 experts top-4).

- one rank: the phased step (trc_modele_debut / attention / moe-on-a-share / fin, the router and
  the fused layer called for the batch, the share's sum added on the host side's stream) gives
  trc_modele_pas's logits bit for bit, 24 greedy steps (past the sliding layers' ring), from the
  .trc parts and from the raw parts;
- two ranks (one process per GPU, NCCL for the MoE inputs' all-gather; the combine's exchange by
  NVLink peer stores in the combine kernel, or by an NCCL reduce-scatter): each rank holds half
  of every layer's experts and runs its own sequence; its logits agree with the one-GPU model run on that sequence within 1e-4 of
  max|z| (the same experts' terms summed in another order across the GPUs) with the same greedy
  token; the shares' parts are byte for byte the whole model's (tables from the counts summed
  over NCCL); the same with two sequences per rank (a batch of 4). Skipped with fewer than two
  GPUs;
- several sequences on one rank (the router and the fused layer called for the batch): each
  sequence's logits are the model's on that sequence alone, bit for bit."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FORME = dict(couches=2, d=256, tetes=8, tetes_kv=2, experts=8, k=4, vocab=512, contexte=64, ffn=256, fenetre=16,
             graine=13, compresse=True, brut=True)


# Two ranks against one GPU: each layer's expert terms are summed in another order across the
# GPUs (f32 rounding, ~1e-7 of a layer's output), and the difference is carried from step to step
# through the KV caches: measured up to 1.6e-5 of max|z| after 12 steps of a batch of two
# sequences per rank; the bound leaves a margin over that, and the greedy tokens must agree.
TOLERANCE_EP = 1e-4


def _suite(m_pas, vues, jetons):
    lg, jt, ct = vues()
    ct.zero_()
    out = []
    for t, j in enumerate(jetons):
        m_pas(int(j), t)
        torch.cuda.synchronize()
        out.append((lg.cpu().numpy().copy(), int(jt.cpu().numpy()[0])))
    assert (ct.cpu().numpy() == 0).all()
    return out


def test_un_rang_egale_le_pas():
    import troncons_b200.modele as M
    from troncons_b200.parallele import ModeleEP

    ep = ModeleEP(0, 1, **FORME)
    m = M.Modele(**FORME)
    jetons = np.random.default_rng(4).integers(0, 512, 24)
    for actifs in ("compresse", "brut"):
        ep.choisir(actifs)
        m.choisir(actifs)
        ep.controle.zero_()
        a = _suite(ep.pas, ep.m.vues, jetons)
        assert (ep.controle == 0).all()
        b = _suite(m.pas, m.vues, jetons)
        for t, ((za, ja), (zb, jb)) in enumerate(zip(a, b)):
            assert np.array_equal(za.view(np.int32), zb.view(np.int32)) and ja == jb, f"{actifs} step {t}"


@pytest.mark.parametrize("b,moe", [(3, "fusionnee"), (9, "fusionnee"), (9, "par_flux")])
def test_un_rang_plusieurs_sequences(b, moe):
    """b sequences on one rank (their attention sides batched: trc_modele_attention_lot, the Q8_0
    GEMVs by launches of up to 8 tokens; the router and the fused layer, or the layer par flux,
    called for the b tokens): each sequence's logits are those of the model run on that sequence
    alone, bit for bit."""
    import troncons_b200.modele as M
    from troncons_b200.parallele import ModeleEP

    ep = ModeleEP(0, 1, par_rang=b, moe=moe, **FORME)
    m = M.Modele(**FORME)
    jetons = np.random.default_rng(8).integers(0, 512, (b, 20))
    ep.choisir("compresse")
    vues = [ep.vues(i) for i in range(b)]
    z = [[] for _ in range(b)]
    for t in range(20):
        ep.pas(jetons[:, t], t)
        torch.cuda.synchronize()
        for i in range(b):
            z[i].append(vues[i][0].cpu().numpy().copy())
    assert (ep.controle == 0).all()
    for i in range(b):
        m.choisir("compresse")
        b = _suite(m.pas, m.vues, jetons[i])
        for t in range(20):
            assert np.array_equal(z[i][t].view(np.int32), b[t][0].view(np.int32)), f"sequence {i} step {t}"


def _port_libre() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _journal(rang, t0, *quoi):
    """A rank's progress on stderr (shown by pytest when a rank fails or times out)."""
    import sys
    import time

    print(f"[{time.time() - t0:7.2f} s] rank {rang}:", *quoi, file=sys.stderr, flush=True)


def _rang(rang, monde, port, echange, moe):
    import time

    import torch.distributed as dist

    import troncons_b200.modele as M
    from troncons_b200.parallele import ModeleEP

    torch.cuda.set_device(rang)
    dev = torch.device("cuda", rang)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rang, world_size=monde,
                            timeout=timedelta(seconds=60), device_id=dev)
    t0 = time.time()
    try:
        ep = ModeleEP(rang, monde, echange=echange, moe=moe, **FORME)
        _journal(rang, t0, "expert-parallel model built")
        seul = M.Modele(**FORME)
        _journal(rang, t0, "one-GPU model built")
        # the share's parts are the whole model's, byte for byte
        for l in range(FORME["couches"]):
            tp, adr, tailles = ep.m.parties["compresse"][l]
            tt, adr_t, tailles_t = seul.parties["compresse"][l]
            for e in range(*ep.tenus):
                a = tp[int(adr[e]) - tp.data_ptr():int(adr[e]) - tp.data_ptr() + int(tailles[e])]
                b = tt[int(adr_t[e]) - tt.data_ptr():int(adr_t[e]) - tt.data_ptr() + int(tailles_t[e])]
                assert torch.equal(a, b), (l, e)
            assert all(adr[e] == 0 for e in range(FORME["experts"]) if not ep.tenus[0] <= e < ep.tenus[1])
        jetons = np.random.default_rng(100 + rang).integers(0, 512, 20)  # each rank its own sequence
        for actifs in ("compresse", "brut"):
            ep.choisir(actifs)
            seul.choisir(actifs)
            a = _suite(ep.pas, ep.m.vues, jetons)
            _journal(rang, t0, actifs, "expert-parallel steps done")
            b = _suite(seul.pas, seul.vues, jetons)
            _journal(rang, t0, actifs, "one-GPU steps done")
            for t, ((za, ja), (zb, jb)) in enumerate(zip(a, b)):
                assert np.abs(za - zb).max() <= TOLERANCE_EP * np.abs(zb).max(), f"rank {rang} {actifs} step {t}"
                assert ja == jb, f"rank {rang} {actifs} step {t}"
        assert (ep.controle == 0).all()
        # two sequences per rank: a batch of 4 tokens over 2 GPUs
        del ep
        ep = ModeleEP(rang, monde, echange=echange, par_rang=2, moe=moe, **FORME)
        _journal(rang, t0, "two sequences per rank: model built")
        ep.choisir("compresse")
        seul.choisir("compresse")
        jetons = np.random.default_rng(200 + rang).integers(0, 512, (2, 16))
        vues = [ep.vues(i) for i in range(2)]
        z = [[] for _ in range(2)]
        for t in range(16):
            ep.pas(jetons[:, t], t)
            torch.cuda.synchronize()
            for i in range(2):
                z[i].append(vues[i][0].cpu().numpy().copy())
        for i in range(2):
            seul.choisir("compresse")
            b = _suite(seul.pas, seul.vues, jetons[i])
            for t in range(16):
                ecart = np.abs(z[i][t] - b[t][0]).max() / np.abs(b[t][0]).max()
                assert ecart <= TOLERANCE_EP, f"rank {rang} seq {i} step {t}: {ecart:.3g} of max|z|"
        assert (ep.controle == 0).all()
        _journal(rang, t0, "done, final barrier")
        dist.barrier()
    except BaseException as erreur:  # shown at once: the other rank may be waiting in a collective
        _journal(rang, t0, "FAILED:", repr(erreur)[:2000])
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("echange,moe", [("pairs", "fusionnee"), ("nccl", "fusionnee"), ("nccl", "par_flux")])
def test_deux_rangs_egalent_un_gpu(echange, moe):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_rang, args=(2, _port_libre(), echange, moe), nprocs=2, join=True, start_method="spawn")
