#!/usr/bin/env python
"""bench.py — the fused rANS-decode + MXFP4 MoE layer on B200.

Workload (one "step"): one gpt-oss-120b MoE layer for one token. 128 experts (gate, up, down
2880 x 2880 MXFP4 each, seeded synthetic weights, see troncons_b200/synth.py) are resident in
HBM as `.trc` v1.2 parts; x is bf16[2880]; the router (f32 128 x 2880) picks 4 experts; the
layer decodes their DELTA and CODES_CTX streams fused into the gate/up GEMV, applies the clamped
SwiGLU, the fused down projection, and adds the weighted combine to the f32 residual.

Metric: GB/s of algorithmic bytes per step = the useful bytes of the 4 routed experts' parts
(what the layer must read) + the router's f32 weights and biases + the layer's LUTs + x and
the residual read and written. `value`: inputs already in HBM, L2 flushed (256 MB written)
between steps, each step timed with CUDA events on its stream. `e2e`: the same through the C-ABI
from pinned host buffers (x and residual copied in, residual copied out, inside the timing).
`--impl reference`: the reference's path on host cores (the oracle's C port of trc-codec's
decoder and the layer's numerics; the reference's Rust CPU codec cannot be built here).

Multi-GPU (torchrun): one process per GPU, each runs its own replica of the workload (weak
scaling, no collective on the data path yet); times are the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

RACINE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, RACINE)

METRIQUE = "fused rANS+MXFP4 GEMV GB/s vs HBM peak; gpt-oss-120b tok/s at 1/2/4/8 B200"
UNITE = "GB/s"


def arguments(argv=None):
    a = argparse.ArgumentParser()
    a.add_argument("--gpus", type=int, default=1)
    a.add_argument("--steps", type=int, default=30)
    a.add_argument("--warmup", type=int, default=5)
    a.add_argument("--impl", choices=["ours", "reference"], default="ours")
    a.add_argument("--experts", type=int, default=128)
    a.add_argument("--k", type=int, default=4)
    a.add_argument("--graine", type=int, default=20261201)
    a.add_argument("--n-delta", type=int, default=256, help="macro-steps per DELTA tile the parts are encoded with")
    a.add_argument("--n-codes", type=int, default=256, help="macro-steps per CODES_CTX tile")
    a.add_argument("--no-cpu-baseline", action="store_true")
    a.add_argument("--sans-legs", action="store_true",
                   help="skip config 1's other measurements (raw layer, DELTA decoded ahead, decode then multiply "
                        "with ours and the reference's kernels, all experts at once)")
    a.add_argument("--sequentiel", action="store_true",
                   help="the sequential schedule (down decoded after SwiGLU, fused into its GEMV) instead of "
                        "the one that decodes down alongside gate/up")
    a.add_argument("--flux", action="store_true",
                   help="measure the streaming executor on the reference engine's gpt-oss-120b routing trace "
                        "(parts in pinned host memory, --emplacements device slots)")
    a.add_argument("--emplacements", type=int, default=326,
                   help="device part slots of the streaming executor (326: the reference engine's run)")
    a.add_argument("--prefill", type=int, default=0,
                   help="measure a batch of this many positions (1..128) through the fused layer and "
                        "through the layer par flux (each routed expert decoded once for the batch)")
    a.add_argument("--modele", action="store_true",
                   help="the whole gpt-oss-120b decode step (config 2): tokens/s after a context of --contexte "
                        "tokens; with --exactitude N, N greedy steps from .trc v1.2 then from raw parts (config 4)")
    a.add_argument("--contexte", type=int, default=2048)
    a.add_argument("--sans-modele", action="store_true", help="skip the whole-model tokens/s in the default line")
    a.add_argument("--exactitude", type=int, default=0)
    a.add_argument("--sans-predecodage", action="store_true",
                   help="whole model: decode DELTA at every step instead of once at load")
    a.add_argument("--couches", type=int, default=36)
    a.add_argument("--gemm", type=int, default=0,
                   help="measure the tensor-core expert GEMM on a 16-expert share with this many tokens per expert")
    a.add_argument("--codeur", action="store_true",
                   help="measure the GPU .trc encoder instead (a layer's experts: counts, then parts)")
    a.add_argument("--par-rang", type=int, default=1,
                   help="sequences per GPU in the expert-parallel whole-model measurement (batch = GPUs x this); "
                        "with --modele on one GPU, a batch of this many sequences")
    a.add_argument("--sans-couche", action="store_true",
                   help="N > 1: measure the expert-parallel whole model only (its own line)")
    a.add_argument("--moe", choices=["fusionnee", "par_flux"], default="fusionnee",
                   help="expert-parallel whole model: the fused layer, or the layer par flux (each held expert "
                        "decoded once per step)")
    a.add_argument("--zipf", type=float, default=0.0,
                   help="whole model: Zipf(s)-shaped expert popularity from a seeded router bias (0: uniform)")
    a.add_argument("--placement", choices=["aleatoire", "equilibre"], default="aleatoire",
                   help="with --zipf: the popular experts numbered at random, or interleaved over the GPUs' shares")
    a.add_argument("--echange", choices=["pairs", "nccl"], default="pairs",
                   help="N > 1: the combine's exchange in the combine kernel over NVLink (pairs) or by NCCL")
    return a.parse_args(argv)


def rang():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def pics():
    try:
        with open(os.path.join(RACINE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# DRAM bytes (read + write) of the dominant launch measured by ncu on the same launch shape (4
# routed experts of 2880 x 2880): the decode launch of the overlapped schedule (every tile of the
# 3 x 4 CODES_CTX streams decoded, the words stored for the row-group GEMVs; 51.27 MB read,
# 9.50 MB of the stored words written back from L2, for 47.64 MB of streams,
# profiles/k_moe_codes_plat_config1_4experts.md), and the sequential schedule's gate/up launch
# (34.03 MB read, 13 KB written for 31.76 MB of streams, an earlier capture of that launch shape).
TRAFIC_CODES = {"recouvrant": 60_769_792, "sequentiel": 34_041_856}


class Horloges:
    """SM clock and clock-event reasons of this GPU (found by its UUID) sampled through NVML
    while the timed region runs (read-only queries): one sample on entry, one every `periode`
    seconds, one on exit. NVML queries take the driver's locks, so only one process samples
    (`actif`), and not faster than needed: CUDA calls of the timed loop must not wait on them."""

    RAISONS = [("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80)]

    def __init__(self, uuid: str, index: int, actif: bool = True, periode: float = 0.02):
        self.uuid, self.index, self.actif, self.periode = uuid, index, actif, periode
        self.echantillons = []
        self.max_mhz = None
        self.arret = threading.Event()
        self.t = None

    def __enter__(self):
        if not self.actif:
            return self
        try:
            import pynvml as N

            N.nvmlInit()
            try:
                h = N.nvmlDeviceGetHandleByUUID(self.uuid)
            except Exception:
                h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)

            def lire():
                while True:
                    try:
                        self.echantillons.append((N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM),
                                                  N.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except Exception:
                        return
                    if self.arret.wait(self.periode):
                        return

            self.h, self.N = h, N
            self.echantillons.append((N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM),
                                      N.nvmlDeviceGetCurrentClocksEventReasons(h)))
            self.t = threading.Thread(target=lire, daemon=True)
            self.t.start()
        except Exception:
            self.t = None
        return self

    def __exit__(self, *a):
        self.arret.set()
        if self.t is not None:
            self.t.join(timeout=2)
            try:
                self.echantillons.append((self.N.nvmlDeviceGetClockInfo(self.h, self.N.NVML_CLOCK_SM),
                                          self.N.nvmlDeviceGetCurrentClocksEventReasons(self.h)))
            except Exception:
                pass

    def resume(self):
        if not self.echantillons:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(e[0] for e in self.echantillons)
        raisons = sorted({nom for _, r in self.echantillons for nom, bit in self.RAISONS if r & bit})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": self.max_mhz, "reasons": raisons,
                "samples": len(sm), "source": "NVML"}


def config_couche(args, ordo: str, parallelisme: str) -> dict:
    """Config 1's `config` object, the same keys in both arms."""
    return {
        "workload": "config 1: one gpt-oss-120b MoE layer, batch 1, 128 experts, top-4, x bf16[2880], "
                    "router f32 128x2880, SwiGLU alpha 1.702 limit 7, weights resident as .trc v1.2 parts",
        "experts": args.experts, "k": args.k, "n_delta": args.n_delta, "n_codes": args.n_codes,
        "schedule": ordo, "l2": "flushed between steps (256 MB written)", "parallelism": parallelisme,
    }


def entrees_couche(args, C0: int, R2: int, rang_: int = 0):
    """The steps' inputs, the same draws in both arms: x f32 values already rounded to bf16
    ([steps][C0]) and the residuals ([steps][R2])."""
    import numpy as np

    rng = np.random.default_rng(args.graine + rang_)
    n_pas = args.warmup + args.steps
    xs = rng.standard_normal((n_pas, C0)).astype(np.float32)
    res0 = rng.standard_normal((n_pas, R2)).astype(np.float32)
    u = xs.view(np.uint32).astype(np.uint64)
    xs = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    return xs, res0


def construire_couche(args, brut: bool = False):
    import troncons_b200 as T
    import troncons_b200.synth as S

    t0 = time.time()
    c = S.couche(args.graine, T.DimsExpert.gpt_oss(), args.experts, brut=brut, n_delta=args.n_delta,
                 n_codes=args.n_codes)
    return c, time.time() - t0


def octets_pas(c, idx, k):
    """Algorithmic bytes of one step with experts `idx` routed."""
    utiles = sum(int.from_bytes(c.parties[int(e)][12:16], "little") for e in idx[:k])
    E, C = c.experts, c.dims.colonnes[0]
    return utiles + 4 * E * C + 4 * E + 3 * 4 * 4 * 4096 + 2 * C + 2 * 4 * c.dims.lignes[2]


def octets_codes_dominant(c, idx, k, matrices=(0, 1, 2)):
    """Compressed CODES_CTX bytes of `matrices` of the routed experts: what the dominant launch
    (the decode launch: k_moe_codes_plat in the overlapped schedule, k_moe_codes / _dense with
    gate/up decoded into the GEMV in the sequential one) must stream from HBM."""
    total = 0
    for e in idx[:k]:
        p = c.parties[int(e)]
        n = int.from_bytes(p[10:12], "little")
        for i in range(n):
            d = p[64 + 16 * i:80 + 16 * i]
            if d[0] == 0x04 and d[1] in matrices:
                total += int.from_bytes(d[8:12], "little")
    return total


def notre_bras(args):
    import numpy as np
    import torch

    r, w, lr = rang()
    torch.cuda.set_device(lr)
    dist = None
    if w > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    import troncons_b200 as T  # noqa: F401
    from troncons_b200.carte import CoucheCarte

    c, t_gen = construire_couche(args, brut=not args.sans_legs)
    cc = CoucheCarte(c, k=args.k, brut=not args.sans_legs, n_delta=args.n_delta, n_codes=args.n_codes,
                     recouvrement=not args.sequentiel)
    n_pas = args.warmup + args.steps
    xs_np, res_np = entrees_couche(args, c.dims.colonnes[0], c.dims.lignes[2], r)
    xs = torch.from_numpy(xs_np).to(torch.bfloat16)  # exact: the values are bf16 already
    xs_dev = xs.cuda()
    x_hote = xs.pin_memory()
    res0 = torch.from_numpy(res_np)
    res_hote = res0.pin_memory()
    res_sortie = torch.empty_like(res_hote).pin_memory()
    residu = torch.empty(c.dims.lignes[2], dtype=torch.float32, device="cuda")
    x_dev = torch.empty(c.dims.colonnes[0], dtype=torch.bfloat16, device="cuda")
    vidange = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB > L2 (126 MB)
    flux = torch.cuda.current_stream()
    idx_journal = torch.zeros(n_pas, args.k, dtype=torch.int32, device="cuda")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
    for e in ev:
        e.record()
    torch.cuda.synchronize()
    phases = [e.cuda_event for e in ev[1:7]]

    x_buf = torch.empty(c.dims.colonnes[0], dtype=torch.bfloat16, device="cuda")
    res_dev = res0.cuda()

    # The step (router + fused layer: 7 kernels) is captured once in a CUDA graph and replayed:
    # the launches reach the GPU back to back, with no host gap between kernels.
    x_buf.copy_(xs_dev[0])
    residu.copy_(res_dev[0])
    for _ in range(3):  # first calls set the kernels' shared-memory attributes, before capture
        cc.couche(x_buf, residu)
    torch.cuda.synchronize()
    graphe = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graphe):
        cc.couche(x_buf, residu)
    torch.cuda.synchronize()

    def pas_carte(s):
        vidange.zero_()
        x_buf.copy_(xs_dev[s])
        residu.copy_(res_dev[s])
        ev[0].record()
        graphe.replay()
        ev[7].record()
        idx_journal[s].copy_(cc.idx)

    # ---- device-timed region
    torch.cuda.synchronize()
    for s in range(args.warmup):
        pas_carte(s)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t_pas = []
    uuid = str(getattr(torch.cuda.get_device_properties(lr), "uuid", ""))
    with Horloges(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}", lr) as horl:
        t0 = time.time()
        for s in range(args.warmup, n_pas):
            pas_carte(s)
            torch.cuda.synchronize()
            t_pas.append(ev[0].elapsed_time(ev[7]))
        mur = time.time() - t0
    assert (cc.controle.cpu().numpy() == 0).all(), "integrity counters set during the bench"
    idx = idx_journal.cpu().numpy()
    octets = sum(octets_pas(c, idx[s], args.k) for s in range(args.warmup, n_pas))
    ordo = "sequentiel" if args.sequentiel else "recouvrant"
    matrices_dom = (0, 1) if args.sequentiel else (0, 1, 2)
    octets_dom = sum(octets_codes_dominant(c, idx[s], args.k, matrices_dom) for s in range(args.warmup, n_pas))
    t_total_ms = sum(t_pas)

    # ---- phases: the same steps launched eagerly, events recorded between the layer's kernels
    t_phase = [[] for _ in range(6)]
    for s in range(n_pas):
        vidange.zero_()
        x_buf.copy_(xs_dev[s])
        residu.copy_(res_dev[s])
        ev[0].record()
        cc.couche(x_buf, residu, evenements=phases)
        torch.cuda.synchronize()
        if s >= args.warmup:
            t_phase[0].append(ev[0].elapsed_time(ev[1]))
            for i in range(5):
                t_phase[1 + i].append(ev[1 + i].elapsed_time(ev[2 + i]))

    # ---- end to end through the C-ABI with host buffers (pinned), copies inside the timing
    torch.cuda.synchronize()
    e2e = []
    for s in range(n_pas):
        vidange.zero_()
        ev[0].record()
        x_buf.copy_(x_hote[s], non_blocking=True)
        residu.copy_(res_hote[s], non_blocking=True)
        graphe.replay()
        res_sortie[s].copy_(residu, non_blocking=True)
        ev[7].record()
        torch.cuda.synchronize()
        if s >= args.warmup:
            e2e.append(ev[0].elapsed_time(ev[7]))
    t_e2e_ms = sum(e2e)
    del graphe

    if dist:
        tt = torch.tensor([t_total_ms, t_e2e_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_total_ms, t_e2e_ms = float(tt[0]), float(tt[1])
    pic, sorte_pic = pics()
    dom_ms = sum(t_phase[2]) / len(t_phase[2])
    atteint = (octets_dom / args.steps) / (dom_ms * 1e-3) / 1e9
    ligne = {
        "metric": METRIQUE,
        "value": round(w * octets / (t_total_ms * 1e-3) / 1e9, 2),
        "unit": UNITE,
        "n_gpus": w,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic (seeded gpt-oss-120b-shaped MXFP4 experts, .trc v1.2 parts)",
        "config": dict(config_couche(args, ordo, f"replicas x{w}"), bytes_per_step=round(octets / args.steps)),
        "e2e": {"value": round(w * octets / (t_e2e_ms * 1e-3) / 1e9, 2), "unit": UNITE,
                "h2d_bytes_per_step": 2 * c.dims.colonnes[0] + 4 * c.dims.lignes[2],
                "d2h_bytes_per_step": 4 * c.dims.lignes[2]},
        "gpu_launches": args.steps * (7 if args.sequentiel else 8),
        "roofline": {"bound": "hbm",
                     "kernel": ("k_moe_codes / k_moe_codes_dense (gate/up: CODES_CTX decode fused into the GEMV)"
                                if args.sequentiel else
                                "k_moe_codes_plat (every CODES_CTX tile of the routed experts decoded, the tiles "
                                "spread evenly over the SMs, the words stored for the row-group GEMVs)"),
                     "achieved": round(atteint, 2), "peak": pic, "unit": "GB/s", "frac": round(atteint / pic, 4),
                     "peak_source": sorte_pic, "frac_8tbs": round(atteint / 8000.0, 4),
                     # DRAM read + write bytes of that launch, from ncu on the same launch shape
                     # (4 routed experts of 2880 x 2880), summarised under profiles/.
                     "traffic": TRAFIC_CODES[ordo], "traffic_source": "ncu dram__bytes_read.sum + "
                     "dram__bytes_write.sum, one launch of the same shape (summary under profiles/)",
                     "algorithmic_bytes_per_launch": round(octets_dom / args.steps)},
        "phases_ms": {n: round(sum(v) / len(v), 4) for n, v in
                      zip(["router", "delta", "gate_up", "swiglu", "down", "combine"] if args.sequentiel else
                          ["router", "delta", "decode", "gate_up_gemv_swiglu", "down_gemv", "combine"], t_phase)},
        "clocks": horl.resume(),
        "wall_s_timed_region": round(mur, 3),
        "generation_s": round(t_gen, 1),
    }
    ligne["step_frac_of_peak"] = round(octets / (t_total_ms * 1e-3) / 1e9 / pic, 4)
    ligne["step_frac_of_8tbs"] = round(octets / (t_total_ms * 1e-3) / 1e12 / 8.0, 4)
    if w == 1 and not args.sans_legs:
        ligne.update(legs_couche(args, c, cc, xs_dev, res_dev, idx, vidange, pic))
    if r == 0 and w == 1 and not args.no_cpu_baseline:
        ligne["cpu_baseline"] = base_cpu(c, args, bornes_s=12.0)
        ligne["config0"] = config0_cpu(c.parties, c.luts, list(c.dims.lignes), list(c.dims.colonnes))
    if w == 1 and not args.sans_modele:
        # The headline metric's second half: the whole gpt-oss-120b decode step (config 2).
        del cc, c
        torch.cuda.empty_cache()
        try:
            mod = mesurer_modele(args, 16, 3, 512)
            ligne["modele"] = {k: mod[k] for k in ("metric", "value", "unit", "ms_per_step", "config", "roofline",
                                                    "generation_s", "context_s", "exactitude")}
        except Exception as ex:  # reported, not hidden: the layer's line stands on its own
            ligne["modele"] = {"unavailable": f"{type(ex).__name__}: {ex}"[:300]}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if r == 0:
        print(json.dumps(ligne), flush=True)


def octets_flux(p: bytes, sortes, matrices) -> int:
    """Bytes of the streams of a part whose kind is in `sortes` and matrix in `matrices`."""
    n = int.from_bytes(p[10:12], "little")
    total = 0
    for i in range(n):
        d = p[64 + 16 * i:80 + 16 * i]
        if d[0] in sortes and d[1] in matrices:
            total += int.from_bytes(d[8:12], "little")
    return total


def chrono_etapes(etape, preparer, n_pas: int, warmup: int, vidange, graphe: bool = True):
    """Device time (ms) of `etape()` per step, after `preparer(s)` set step s's inputs and L2
    was flushed; the step is captured in a CUDA graph when `graphe`. Returns per-step times of
    the n_pas - warmup timed steps."""
    import torch

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    preparer(0)
    for _ in range(2):
        etape()
    torch.cuda.synchronize()
    g = None
    if graphe:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            etape()
        torch.cuda.synchronize()
    t = []
    for s in range(n_pas):
        vidange.zero_()
        preparer(s)
        ev[0].record()
        g.replay() if g is not None else etape()
        ev[1].record()
        torch.cuda.synchronize()
        if s >= warmup:
            t.append(ev[0].elapsed_time(ev[1]))
    del g
    return t


def legs_couche(args, c, cc, xs_dev, res_dev, idx, vidange, pic: float) -> dict:
    """The other measurements of config 1, on the same layer, inputs and routed experts, L2
    flushed between steps (each a named object of the default line):
    - raw_layer: the fused layer on the raw parts (k_moe_brut), with the roofline of its gate/up
      launch (CODES_BRUTS + ECHELLES_BRUTES of gate and up: a pure HBM stream);
    - delta_predecoded: the compressed layer with every expert's DELTA decoded once ahead
      (trc_moe_predecoder_deltas), its bytes counted instead of the DELTA streams;
    - decode_then_gemv: the reference's operator sequence (decoder_lot into slots, gemv_lot,
      swiglu_oai, gemv_lot, combiner) on the step's routed experts, with this library's kernels
      and with the reference's own kernels compiled for sm_100a (oracle/_ref, a reported
      baseline like cpu_baseline), against the fused layer without its router;
    - throughput_all_experts: every one of the layer's 128 experts active in one call (32
      tokens x top-4, one activation per expert), the decode launches in throughput mode."""
    import numpy as np
    import torch

    import troncons_b200 as T
    from troncons_b200.carte import CoucheCarte

    n_pas = args.warmup + args.steps
    k = args.k
    x_buf = torch.empty(c.dims.colonnes[0], dtype=torch.bfloat16, device="cuda")
    residu = torch.empty(c.dims.lignes[2], dtype=torch.float32, device="cuda")

    def prep(s):
        x_buf.copy_(xs_dev[s])
        residu.copy_(res_dev[s])

    fixe = 4 * c.experts * c.dims.colonnes[0] + 4 * c.experts + 2 * c.dims.colonnes[0] + 8 * c.dims.lignes[2]
    out = {}
    steps = range(args.warmup, n_pas)

    # -- raw parts
    t = chrono_etapes(lambda: cc.couche(x_buf, residu, brute=True), prep, n_pas, args.warmup, vidange)
    octets = sum(sum(int.from_bytes(c.parties_brutes[int(e)][12:16], "little") for e in idx[s]) + fixe for s in steps)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    for e in ev:  # torch creates the CUDA event at its first record
        e.record()
    torch.cuda.synchronize()
    ph = []
    for s in range(n_pas):
        vidange.zero_()
        prep(s)
        ev[0].record()
        cc.couche(x_buf, residu, brute=True, evenements=[e.cuda_event for e in ev[1:7]])
        torch.cuda.synchronize()
        if s >= args.warmup:
            ph.append(ev[2].elapsed_time(ev[3]))
    brut_gu = sum(octets_flux(c.parties_brutes[int(e)], (0x06, 0x07), (0, 1)) for s in steps for e in idx[s])
    ach = brut_gu / args.steps / (np.mean(ph) * 1e-3) / 1e9
    out["raw_layer"] = {
        "value": round(octets / (sum(t) * 1e-3) / 1e9, 2), "unit": UNITE, "ms_per_step": round(sum(t) / args.steps, 4),
        "bytes_per_step": round(octets / args.steps),
        "roofline": {"bound": "hbm", "kernel": "k_moe_brut_groupes (gate/up: CODES_BRUTS + ECHELLES_BRUTES of the routed experts)",
                     "achieved": round(ach, 1), "peak": pic, "unit": "GB/s", "frac": round(ach / pic, 4),
                     "frac_8tbs": round(ach / 8000.0, 4), "ms": round(float(np.mean(ph)), 4),
                     "algorithmic_bytes_per_launch": round(brut_gu / args.steps)}}

    # -- DELTA decoded ahead
    cc.predecoder_deltas()
    torch.cuda.synchronize()
    assert (cc.controle_deltas == 0).all()
    t = chrono_etapes(lambda: cc.couche(x_buf, residu), prep, n_pas, args.warmup, vidange)
    octets = sum(sum(int.from_bytes(c.parties[int(e)][12:16], "little") - octets_flux(c.parties[int(e)], (0x03,), (0, 1, 2))
                     for e in idx[s]) + k * sum(c.dims.lignes[j] * (c.dims.colonnes[j] // 32) for j in range(3)) + fixe
                 for s in steps)
    out["delta_predecoded"] = {
        "value": round(octets / (sum(t) * 1e-3) / 1e9, 2), "unit": UNITE, "ms_per_step": round(sum(t) / args.steps, 4),
        "bytes_per_step": round(octets / args.steps),
        "note": "DELTA streams replaced by the decoded delta bytes (one per 32-block), decoded once at load: "
                "99.5 MB per 128-expert layer resident"}
    cc.deltas = None

    # -- decode then multiply: ours and the reference's kernels, the fused layer without router
    cc.preparer_decodee()
    descs = [cc.descripteurs_decodee(idx[s]) for s in range(n_pas)]
    cc.routeur(x_buf)
    cour = [None]

    def prep_d(s):
        prep(s)
        cour[0] = descs[s]

    t_nous = chrono_etapes(lambda: cc.sequence_decodee(cour[0], x_buf, residu), prep_d, n_pas, args.warmup, vidange,
                           graphe=False)
    t_fus = chrono_etapes(lambda: cc.couche(x_buf, residu, routeur=False), prep, n_pas, args.warmup, vidange)
    octets = sum(sum(int.from_bytes(c.parties[int(e)][12:16], "little") for e in idx[s]) + fixe for s in steps)
    d = {"fused_layer_ms": round(sum(t_fus) / args.steps, 4), "ours_ms": round(sum(t_nous) / args.steps, 4),
         "ours_value": round(octets / (sum(t_nous) * 1e-3) / 1e9, 2),
         "fused_value": round(octets / (sum(t_fus) * 1e-3) / 1e9, 2), "unit": UNITE,
         "note": "the step's routed experts known on the host; no router in either time"}
    try:
        import oracle as O

        ref = O.ref()
    except Exception:
        ref = None
    if ref is not None:
        dims6 = np.array(list(c.dims.lignes) + list(c.dims.colonnes), np.uint32)
        f = torch.cuda.current_stream().cuda_stream
        p6 = dims6.ctypes.data_as(O.P32)

        def ref_seq():
            dd, dg, ddn = cour[0]
            cc.x32.copy_(x_buf.float())
            assert ref.ref_decoder_lot(dd.data_ptr(), k, p6, f) == 0
            assert ref.ref_gemv_lot(dg.data_ptr(), 2 * k, cc.R0, f) == 0
            assert ref.ref_swiglu(cc.g.data_ptr(), cc.u.data_ptr(), cc.h.data_ptr(), k * cc.R0, f) == 0
            assert ref.ref_gemv_lot(ddn.data_ptr(), k, cc.R2, f) == 0
            assert ref.ref_combiner(residu.data_ptr(), cc.s.data_ptr(), cc.R2, cc.poids.data_ptr(), k, cc.R2, f) == 0

        t_ref = chrono_etapes(ref_seq, prep_d, n_pas, args.warmup, vidange, graphe=False)
        d["reference_kernels_ms"] = round(sum(t_ref) / args.steps, 4)
        d["reference_kernels_value"] = round(octets / (sum(t_ref) * 1e-3) / 1e9, 2)
        d["reference_kernels"] = "trc-noyaux/noyaux/noyaux.cu compiled unchanged for sm_100a (oracle/_ref)"
    else:
        d["reference_kernels"] = "unavailable: oracle/_ref/libtrc_ref.so not built"
    out["decode_then_gemv"] = d

    # -- throughput mode: the 128 experts active at once
    E = c.experts
    if E % k == 0 and E // k <= 128:
        jt = E // k
        ct = CoucheCarte(c, k=k, brut=False, jetons=jt)
        perm = np.random.default_rng(args.graine).permutation(E).astype(np.int32)
        ct.idx.copy_(torch.from_numpy(perm))
        ct.poids.fill_(1.0 / k)
        xt = torch.zeros(jt, c.dims.colonnes[0], dtype=torch.bfloat16, device="cuda")
        rt = torch.zeros(jt, c.dims.lignes[2], dtype=torch.float32, device="cuda")

        def prep_t(s):
            xt.copy_(xs_dev[s].expand(jt, -1))
            rt.copy_(res_dev[s].expand(jt, -1))

        t = chrono_etapes(lambda: ct.couche(xt, rt, routeur=False), prep_t, n_pas, args.warmup, vidange)
        assert (ct.controle == 0).all()
        tout = sum(int.from_bytes(p[12:16], "little") for p in c.parties)
        codes = sum(octets_flux(p, (0x04,), (0, 1, 2)) for p in c.parties)
        ms = sum(t) / args.steps
        out["throughput_all_experts"] = {
            "value": round(tout / (ms * 1e-3) / 1e9, 2), "unit": UNITE, "ms_per_step": round(ms, 4),
            "activations": E, "bytes_per_step": tout, "codes_ctx_bytes": codes,
            "frac": round(tout / (ms * 1e-3) / 1e9 / pic, 4), "frac_8tbs": round(tout / (ms * 1e-3) / 1e12 / 8.0, 4),
            "note": "every expert of the layer decoded and multiplied in one call (sequential schedule, one warp "
                    "per tile): where the rANS decode chain sits when the GPU is full of tiles"}
        del ct
    return out


def couche_ep(args, c, r: int, w: int):
    """This rank's share of the layer for the expert-parallel arm: the bench's arguments (k,
    exchange, MoE form) checked and passed through; a batch of w tokens (one per GPU on average)."""
    from troncons_b200.parallele import CoucheEP

    return CoucheEP(c, r, w, k=args.k, jetons=w, echange=args.echange, moe=args.moe)


def bras_ep(args):
    """N > 1: the expert-parallel layer (config 3). Rank r holds experts partage(128, r, N) (16
    per GPU at 8); a step is a batch of N tokens (one per GPU on average: weak scaling), the
    router replicated on every rank, the fused layer on the rank's share, then the combine's SUM
    all-reduce over NCCL. Times are the max over ranks; bytes are what all ranks read."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.parallele import partage, reduire_comptes

    r, w, lr = rang()
    torch.cuda.set_device(lr)
    dev = torch.device("cuda", lr)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if args.sans_couche:  # the expert-parallel whole model alone, its own line
        modele = mesurer_modele_ep(args, args.steps, args.warmup)
        dist.barrier()
        dist.destroy_process_group()
        if r == 0:
            print(json.dumps(modele), flush=True)
        return
    jetons = w
    t0 = time.time()
    c = S.couche(args.graine, T.DimsExpert.gpt_oss(), args.experts, brut=False, n_delta=args.n_delta,
                 n_codes=args.n_codes, tenus=partage(args.experts, r, w), reduire=reduire_comptes(device=dev))
    t_gen = time.time() - t0
    ep = couche_ep(args, c, r, w)
    C0, R2 = c.dims.colonnes[0], c.dims.lignes[2]
    n_pas = args.warmup + args.steps
    rng = np.random.default_rng(args.graine)  # the same tokens on every rank
    xs = torch.from_numpy(rng.standard_normal((n_pas, jetons, C0)).astype(np.float32)).to(torch.bfloat16)
    res0 = torch.from_numpy(rng.standard_normal((n_pas, jetons, R2)).astype(np.float32))
    xs_dev, res_dev = xs.cuda(), res0.cuda()
    x_hote, res_hote = xs.pin_memory(), res0.pin_memory()
    res_sortie = torch.empty_like(res_hote).pin_memory()
    x_buf = torch.empty(jetons, C0, dtype=torch.bfloat16, device="cuda")
    residu = torch.empty(jetons, R2, dtype=torch.float32, device="cuda")
    vidange = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB > L2 (126 MB)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    idx_journal = torch.zeros(n_pas, jetons * args.k, dtype=torch.int32, device="cuda")
    partiel = r != 0

    # The step is captured in a CUDA graph: with the "pairs" exchange the whole step (router,
    # fused share, combine and exchange in one kernel); with "nccl", the local part, and the
    # all-reduce is issued after each replay.
    paires = ep.echange == "pairs"
    x_buf.copy_(xs_dev[0])
    residu.copy_(res_dev[0])
    for _ in range(3):
        ep.etape(x_buf, residu) if paires else ep.local(x_buf, residu, partiel)
    torch.cuda.synchronize()
    dist.barrier()
    graphe = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graphe):
        ep.etape(x_buf, residu) if paires else ep.local(x_buf, residu, partiel)
    torch.cuda.synchronize()

    def pas(s, hote=False):
        vidange.zero_()
        ev[0].record()
        if hote:
            x_buf.copy_(x_hote[s], non_blocking=True)
            residu.copy_(res_hote[s], non_blocking=True)
        else:
            x_buf.copy_(xs_dev[s])
            residu.copy_(res_dev[s])
        graphe.replay()
        if not paires:
            dist.all_reduce(residu, op=dist.ReduceOp.SUM)
        if hote:
            res_sortie[s].copy_(residu, non_blocking=True)
        ev[1].record()
        idx_journal[s].copy_(ep.carte.idx)

    for s in range(args.warmup):
        pas(s)
    torch.cuda.synchronize()
    t_pas = []
    uuid = str(getattr(torch.cuda.get_device_properties(lr), "uuid", ""))
    with Horloges(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}", lr, actif=(r == 0)) as horl:
        # The sampler starts (NVML initialisation) before the barrier: every rank enters the
        # timed steps together.
        dist.barrier()
        torch.cuda.synchronize()
        for s in range(args.warmup, n_pas):
            pas(s)
            torch.cuda.synchronize()
            t_pas.append(ev[0].elapsed_time(ev[1]))
    assert (ep.carte.controle.cpu().numpy() == 0).all(), "integrity counters set during the bench"
    dist.barrier()
    e2e = []
    for s in range(n_pas):
        pas(s, hote=True)
        torch.cuda.synchronize()
        if s >= args.warmup:
            e2e.append(ev[0].elapsed_time(ev[1]))
    del graphe

    # Bytes this rank read per step: the parts of its held activations, the router (read by
    # every rank), LUTs, x and the residual's read and write.
    idx = idx_journal.cpu().numpy()
    debut, fin = ep.tenus
    E = c.experts
    fixe = 4 * E * C0 + 4 * E + 3 * 4 * 4 * 4096 + jetons * (2 * C0 + 2 * 4 * R2)
    octets = sum(sum(int.from_bytes(c.parties[int(e)][12:16], "little") for e in idx[s] if debut <= e < fin) + fixe
                 for s in range(args.warmup, n_pas))
    tt = torch.tensor([sum(t_pas), sum(e2e)], dtype=torch.float64, device="cuda")
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    oc = torch.tensor([float(octets)], dtype=torch.float64, device="cuda")
    dist.all_reduce(oc, op=dist.ReduceOp.SUM)
    t_total_ms, t_e2e_ms, octets_tous = float(tt[0]), float(tt[1]), float(oc[0])
    clocks = horl.resume()
    dist.barrier()
    modele = None
    echange = ep.echange
    if not args.sans_modele:
        del ep, c, xs_dev, res_dev, vidange
        torch.cuda.empty_cache()
        modele = mesurer_modele_ep(args, 16, 3)
    dist.destroy_process_group()
    if r != 0:
        return
    ligne = {
        "metric": METRIQUE,
        "value": round(octets_tous / (t_total_ms * 1e-3) / 1e9, 2),
        "unit": UNITE,
        "n_gpus": w,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic (seeded gpt-oss-120b-shaped MXFP4 experts, .trc v1.2 parts)",
        "config": {
            "workload": f"config 3: expert-parallel gpt-oss-120b MoE layer, {args.experts} experts "
                        f"({fin - debut} per GPU), top-{args.k}, batch {jetons} tokens (one per GPU), x bf16[2880], "
                        "router f32 replicated, " + ("combine and its exchange in one kernel over NVLink peer "
                        "memory" if paires else "combine by NCCL all-reduce of the batch's f32 residual"),
            "experts": args.experts, "k": args.k, "tokens_per_step": jetons, "n_delta": args.n_delta,
            "n_codes": args.n_codes, "l2": "flushed between steps (256 MB written)",
            "bytes_per_step": round(octets_tous / args.steps), "parallelism": f"ep{w}", "exchange": echange,
        },
        "e2e": {"value": round(octets_tous / (t_e2e_ms * 1e-3) / 1e9, 2), "unit": UNITE,
                "h2d_bytes_per_step": jetons * (2 * C0 + 4 * R2), "d2h_bytes_per_step": jetons * 4 * R2},
        "gpu_launches": args.steps * (2 * jetons + 5),  # the all-reduce (nccl) is NCCL's
        "roofline": None,
        "clocks": clocks,
        "generation_s": round(t_gen, 1),
    }
    if modele is not None:
        ligne["modele"] = modele
    print(json.dumps(ligne), flush=True)


def mesurer_modele_ep(args, steps: int, warmup: int) -> dict:
    """Config 3, the whole model expert-parallel (every rank of the torchrun group calls it): a
    seeded synthetic gpt-oss-120b, each rank holding its share of every layer's experts
    (partage: 16 of 128 at 8 GPUs, drawn and encoded on its GPU, the tables from the counts summed
    over NCCL) and a replica of the dense weights; --par-rang sequences per rank (a batch of N x
    par-rang; one GPU and par-rang > 1: the batch on that GPU), each its own --contexte seeded
    tokens through the step, then `steps` greedy steps timed with CUDA events after `warmup`,
    every rank in step (two NCCL collectives per layer: the MoE inputs gathered, the shares' sums
    scattered back), the MoE by the fused layer or par flux (--moe), the router biased for Zipf
    popularity with --zipf. tokens/s = batch x steps / the max over ranks of the timed region;
    after the timing, one more step records each GPU's activations per layer ("load")."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from troncons_b200.parallele import ModeleEP, partage

    r, w, _ = rang()
    b = args.par_rang
    t0 = time.time()
    ep = ModeleEP(r, w, echange="nccl", par_rang=b, moe=args.moe, couches=args.couches, d=2880, tetes=64, tetes_kv=8,
                  experts=args.experts, k=args.k, vocab=201088, contexte=args.contexte + warmup + steps + 2, ffn=2880,
                  fenetre=128, graine=args.graine, compresse=True, brut=False, zipf=args.zipf,
                  placement=args.placement, deltas_predecodes=not args.sans_predecodage)
    torch.cuda.synchronize()
    t_gen = time.time() - t0
    # each sequence its own seeded context
    contexte = np.random.default_rng(args.graine + 1000 * r).integers(0, 201088, (b, args.contexte))
    vues = [ep.vues(i) for i in range(b)]
    for _, _, ct in vues:
        ct.zero_()
    ep.controle.zero_()

    def barriere():
        if w > 1:
            dist.barrier()

    barriere()
    t1 = time.time()
    for p in range(args.contexte):
        ep.pas(contexte[:, p], p, sortie=False)
    torch.cuda.synchronize()
    t_ctx = time.time() - t1
    pos, j = args.contexte, contexte[:, -1].copy()
    for _ in range(warmup):
        ep.pas(j, pos)
        j = np.array([int(v[1].cpu().numpy()[0]) for v in vues])
        pos += 1
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    barriere()
    ev[0].record()
    for _ in range(steps):
        ep.pas(j, pos)  # the greedy tokens stay on the device: the same tokens are fed (no host sync)
        pos += 1
    ev[1].record()
    torch.cuda.synchronize()
    t = torch.tensor([ev[0].elapsed_time(ev[1])], dtype=torch.float64, device="cuda")
    ok = torch.tensor([int((ep.controle.cpu().numpy() == 0).all())], device="cuda")
    if w > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    ms = float(t[0]) / steps
    if not int(ok[0]):
        raise RuntimeError("integrity counters set during the expert-parallel model steps")
    # one more step, untimed, with every layer's routing kept: the activations each GPU's share
    # holds, per layer (the busiest GPU's count against the mean)
    journal = []
    ep.pas(j, pos, journal=journal)
    torch.cuda.synchronize()
    parts = np.array([np.bincount(np.array([partage(args.experts, q, w)[0] for q in range(w)]).searchsorted(
        x.cpu().numpy(), side="right") - 1, minlength=w) for x in journal])
    charge = {"activations_per_layer": int(parts.sum(1)[0]), "busiest_gpu_mean": round(float(parts.max(1).mean()), 2),
              "mean_per_gpu": round(float(parts.sum(1)[0]) / w, 2)}
    debut, fin = ep.tenus
    del ep
    torch.cuda.empty_cache()
    return {"metric": f"gpt-oss-120b decode tokens/s (whole step, expert-parallel over {w} GPUs, batch {w * b})",
            "value": round(w * b * 1000.0 / ms, 2), "unit": "tokens/s", "ms_per_step": round(ms, 4), "steps": steps,
            "warmup": warmup, "batch": w * b, "sequences_per_gpu": b, "experts_per_gpu": fin - debut, "n_gpus": w,
            "popularity": ({"zipf": args.zipf, "placement": args.placement} if args.zipf > 0 else "uniform"),
            "moe": args.moe,
            "load": charge,
            "workload": f"config 3: {args.couches} layers, {args.experts} experts top-{args.k} ({fin - debut} per GPU), "
                        f"{b} sequence(s) per GPU, context {args.contexte} seeded tokens, attention on each sequence's "
                        "GPU, MoE inputs all-gathered and the shares' sums reduce-scattered over NCCL per layer",
            "exchange": "nccl", "delta_predecoded": not args.sans_predecodage,
            "generation_s": round(t_gen, 1), "context_s": round(t_ctx, 1)}


def modele_cpu() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            return next((l.split(":", 1)[1].strip() for l in f if l.startswith("model name")), "")
    except Exception:
        return ""


def octets_pas_parties(parties, idx, k, E, C, R2):
    """octets_pas for a list of parts (the reference arm has no product layer object)."""
    utiles = sum(int.from_bytes(parties[int(e)][12:16], "little") for e in idx[:k])
    return utiles + 4 * E * C + 4 * E + 3 * 4 * 4 * 4096 + 2 * C + 2 * 4 * R2


def pas_cpu(parties, luts, lignes, colonnes, wr, br, args, bornes_s: float, pas_min: int, n_pas: int = 0):
    """The reference's path on host cores (oracle/couche_cpu.c: router, decode of the routed
    experts, GEMVs, SwiGLU, combine), all threads, on the bench's bf16 inputs: (seconds, bytes,
    steps). n_pas: exactly that many steps after args.warmup; else at least pas_min steps and
    bornes_s seconds (at most 200)."""
    import oracle as O

    n_fils = os.cpu_count() or 1
    total = n_pas + args.warmup if n_pas else 200 + args.warmup
    xs, res0 = entrees_couche(args, colonnes[0], lignes[2])
    t, octets, n = 0.0, 0, 0
    for s in range(total):
        i = s % len(xs)
        t0 = time.perf_counter()
        _, idx, _ = O.couche_moe_cpu(parties, luts, lignes, colonnes, wr, br, xs[i], args.k, res0[i], n_fils)
        dt = time.perf_counter() - t0
        if s < args.warmup:
            continue
        t += dt
        octets += octets_pas_parties(parties, idx, args.k, len(parties), colonnes[0], lignes[2])
        n += 1
        if not n_pas and n >= pas_min and t >= bornes_s:
            break
    return t, octets, n


def base_cpu(c, args, bornes_s: float, pas_min: int = 3):
    """cpu_baseline of the GPU arm's line: pas_cpu on the same parts, a bounded sample."""
    t, octets, n = pas_cpu(c.parties, c.luts, list(c.dims.lignes), list(c.dims.colonnes), c.wr, c.br, args, bornes_s,
                           pas_min)
    return {"value": round(octets / t / 1e9, 3), "unit": UNITE, "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{n} layer steps on the bench's bf16 inputs (router, decode of the 4 routed experts, GEMVs, "
                      f"SwiGLU, combine), {round(t, 1)} s; CPU: {modele_cpu()}"}


def config0_cpu(parties, luts, lignes, colonnes, bornes_s: float = 6.0) -> dict:
    """Config 0: the reference's CPU decoder (decoder_avec per tile, decoder_matrice_v10 per
    matrix, restated in oracle/couche_cpu.c) on one gate + up pair (matrices 0 and 1 of expert 0),
    parallel over (matrix, tile) on every host thread; decoded GB/s = 2 x (16 nb + nb) bytes of
    MXFP4 codes and scales per pair (8,812,800 B for 2880 x 2880)."""
    import oracle as O

    n_fils = os.cpu_count() or 1
    decodes = sum(17 * lignes[j] * (colonnes[j] // 32) for j in (0, 1))
    lus = 0
    p = parties[0]
    nf = int.from_bytes(p[10:12], "little")
    for i in range(nf):
        d = p[64 + 16 * i:80 + 16 * i]
        if d[0] in (0x03, 0x04) and d[1] in (0, 1):
            lus += int.from_bytes(d[8:12], "little")
    O.decoder_matrices_cpu(p, luts, lignes, colonnes, (0, 1), n_fils)  # warm-up
    t, n = 0.0, 0
    while n < 3 or t < bornes_s:
        t0 = time.perf_counter()
        O.decoder_matrices_cpu(p, luts, lignes, colonnes, (0, 1), n_fils)
        t += time.perf_counter() - t0
        n += 1
    return {"metric": "decoded GB/s on host cores (config 0: one gate+up pair, .trc v1.2)",
            "value": round(n * decodes / t / 1e9, 3), "unit": "GB/s", "decoded_bytes_per_pair": decodes,
            "compressed_bytes_per_pair": lus, "passes": n, "seconds": round(t, 2), "cores": n_fils,
            "nproc": os.cpu_count(), "cpu": modele_cpu(), "kind": "port",
            "source": "oracle/couche_cpu.c orc_decoder_matrices_cpu (rans.rs:388-451, trc-codec/src/lib.rs:190-218)"}


def bras_reference(args):
    """The reference arm: the reference's CPU path (restated in oracle/) on host cores, on the
    GPU arm's config-1 workload. Its layer is built by the oracle alone (oracle.CoucheOracle:
    the same weights, tables and parts as the product's generator, byte for byte), so no product
    library is loaded; x is the GPU arm's bf16 input."""
    r, w, _ = rang()
    if r != 0:
        return
    import oracle as O

    t0 = time.time()
    d = [2880, 2880, 2880]
    c = O.CoucheOracle(args.graine, d, d, args.experts, args.n_delta, args.n_codes)
    t_gen = time.time() - t0
    n_fils = os.cpu_count() or 1
    t, octets, n = pas_cpu(c.parties, c.luts, c.lignes, c.colonnes, c.wr, c.br, args, 0.0, 0, n_pas=args.steps)
    v = round(octets / t / 1e9, 3)
    ligne = {
        "impl": "reference", "metric": METRIQUE, "value": v, "unit": UNITE, "n_gpus": w, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * t / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded gpt-oss-120b-shaped MXFP4 experts, .trc v1.2 parts)",
        "config": dict(config_couche(args, "reference CPU path: decode then multiply, OpenMP over tiles and rows",
                                     f"{n_fils} host threads"), bytes_per_step=round(octets / args.steps)),
        "cpu_baseline": {"value": v, "unit": UNITE, "cores": n_fils, "kind": "port",
                         "sample": f"{n} layer steps after {args.warmup} warm-up, {round(t, 2)} s; CPU: {modele_cpu()}"},
        "e2e": {"value": v, "unit": UNITE, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "config0": config0_cpu(c.parties, c.luts, c.lignes, c.colonnes),
        "generation_s": round(t_gen, 1),
    }
    print(json.dumps(ligne), flush=True)


def bras_codeur(args):
    """The GPU `.trc` encoder on `--experts` gpt-oss-shaped experts (one process, one GPU): the
    layer's symbol counts (trc_comptes_gpu), then every expert's level-0 part in one call
    (trc_coder_parties_gpu), timed with CUDA events over --steps calls after --warmup; expert
    0's part checked byte for byte against the CPU encoder, which is timed on one expert."""
    import ctypes as C

    import numpy as np
    import torch

    import troncons_b200 as T
    import troncons_b200.synth as S

    dims = T.DimsExpert.gpt_oss()
    n = args.experts
    hote = [S.matrices(args.graine + j, dims.lignes[j], dims.colonnes[j], n) for j in range(3)]
    blocs = [[torch.from_numpy(hote[j][0][e]).cuda() for j in range(3)] for e in range(n)]
    biais = [[torch.from_numpy(hote[j][1][e]).cuda() for j in range(3)] for e in range(n)]
    source = sum(b.numel() for b in blocs[0]) * n
    cap = 2 * sum(b.numel() for b in blocs[0]) + (1 << 16)
    sorties = [torch.empty(cap, dtype=torch.uint8, device="cuda") for _ in range(n)]
    descs = S._descs_gpu(blocs, biais, list(range(n)), sorties, cap)
    comptes = torch.zeros(3 * 4 * 256, dtype=torch.int64, device="cuda")
    fl = torch.cuda.current_stream().cuda_stream

    def compter():
        T.verifier(T.lib.trc_comptes_gpu(descs.data_ptr(), descs.numel(), n, C.byref(dims), 1, comptes.data_ptr(),
                                         comptes.numel() * 8, fl))

    compter()
    torch.cuda.synchronize()
    freqs = S.tables_de_comptes(comptes.cpu().numpy().astype(np.uint64).reshape(3, 4, 256))
    f = torch.from_numpy(freqs.reshape(-1).view(np.int16)).cuda()
    octets = torch.zeros(2 * n, dtype=torch.int64, device="cuda")
    n_esp = int(T.lib.trc_coder_parties_gpu_espace(C.byref(dims), n, 256, 256))
    esp = torch.empty(n_esp + 256, dtype=torch.uint8, device="cuda")
    e0 = esp.data_ptr() + (-esp.data_ptr()) % 256

    def coder():
        T.verifier(T.lib.trc_coder_parties_gpu(descs.data_ptr(), descs.numel(), n, C.byref(dims), f.data_ptr(), 1, 0,
                                               256, 256, octets.data_ptr(), octets.numel() * 8, e0, n_esp, fl))

    def chrono(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps

    ms_comptes, ms_coder = chrono(compter), chrono(coder)
    o = octets.cpu().numpy()
    t0 = time.perf_counter()
    attendu = S.coder_partie([hote[j][0][0] for j in range(3)], [hote[j][1][0] for j in range(3)], dims, freqs, expert=0)
    cpu_s = time.perf_counter() - t0
    assert sorties[0][:int(o[0])].cpu().numpy().tobytes() == attendu, "GPU part differs from the CPU encoder's"
    print(json.dumps({
        "metric": "GPU .trc encoder: MXFP4 source bytes encoded into level-0 v1.2 parts per second",
        "value": round(source / (ms_coder * 1e-3) / 1e9, 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_coder, 4), "higher_is_better": True,
        "dtype": "u8", "data": "synthetic (seeded gpt-oss-120b-shaped MXFP4 experts)",
        "config": {"workload": f"{n} experts of 3 x 2880 x 2880 MXFP4 (one call), tiles of 256 macro-steps",
                   "source_bytes": source, "part_bytes": int(o[0::2].sum())},
        "comptes": {"ms": round(ms_comptes, 4), "GBps": round(source / (ms_comptes * 1e-3) / 1e9, 2)},
        "cpu_encoder_one_expert_s": round(cpu_s, 4), "gpu_ms_per_expert": round(ms_coder / n, 4),
        "identical_to_cpu_encoder": True}), flush=True)


def bras_flux(args):
    """The streaming executor (trc_flux_*) on the gpt-oss-120b routing trace the reference's engine
    wrote (708 tokens x 36 layers x top-4 of 128 experts, tests/golden/traces_boucle.npz): every
    layer's parts in pinned host memory (one layer's 128 synthetic gpt-oss experts, shared by the 36
    layers: each (layer, expert) is still its own cache entry and its own copy), --emplacements
    device slots managed by the LRU expert cache, routing imposed from the trace (weights 1/4).
    Timed with CUDA events on the compute stream over the whole trace, from a cold cache, as the
    reference's run was; the cache counts are compared with that run's counters."""
    import numpy as np
    import torch

    import troncons_b200.flux as F

    c, t_gen = construire_couche(args)
    with open(os.path.join(RACINE, "tests", "golden", "traces_boucle.json")) as f:
        gold = json.load(f)["t120-boucle"]
    choix = np.load(os.path.join(RACINE, "tests", "golden", "traces_boucle.npz"))["t120_boucle"]
    T_, L, k = choix.shape
    if args.steps < T_:
        T_ = args.steps
    tampon, adr, tailles = F.tiers_hote(c.parties)
    luts = torch.from_numpy(np.tile(c.luts.view(np.int32), L)).cuda()
    fl = F.Flux(c.dims, L, c.experts, k, args.emplacements, np.tile(adr, L), np.tile(tailles, L), luts)
    x = torch.zeros(1, c.dims.colonnes[0], dtype=torch.bfloat16, device="cuda")
    r = torch.zeros(1, c.dims.lignes[2], dtype=torch.float32, device="cuda")
    w = np.full((1, k), 0.25, np.float32)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    octets, t0 = 0, time.time()
    a.record()
    for t in range(T_):
        for l in range(L):
            octets += fl.couche(l, x, r, choix[t, l].reshape(1, k), w).octets_copies
    b.record()
    torch.cuda.synchronize()
    mur = time.time() - t0
    ms = a.elapsed_time(b)
    cpt = fl.compteurs()
    assert (fl.controle() == 0).all(), "integrity counters set"
    # The copy engine's own rate: one pinned 1 GiB host-to-device copy, best of 3.
    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    pic = 0.0
    for _ in range(3):
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        pic = max(pic, (1 << 30) / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    ligne = {
        "metric": "streaming MoE layers: tokens per second over the reference engine's gpt-oss-120b routing trace",
        "value": round(T_ / (ms * 1e-3), 2), "unit": "tokens/s", "n_gpus": 1, "steps": T_, "warmup": 0,
        "ms_per_step": round(ms / T_, 4), "higher_is_better": True, "dtype": "u8",
        "data": "synthetic gpt-oss-120b-shaped experts (.trc v1.2) in pinned host memory; routing from the "
                "reference engine's trace",
        "config": {"workload": f"{T_} tokens x {L} MoE layers, top-{k} of {c.experts}, {args.emplacements} device "
                               "part slots (LRU), cold start", "emplacements": args.emplacements},
        "ms_per_layer": round(ms / (T_ * L), 4),
        "h2d": {"bytes": int(octets), "GBps": round(octets / (ms * 1e-3) / 1e9, 2),
                "peak_GBps": round(pic, 2), "peak_source": "one pinned 1 GiB host-to-device copy, best of 3",
                "frac": round(octets / (ms * 1e-3) / 1e9 / pic, 4)},
        "cache": {"acces": cpt.acces(), "succes": cpt.succes_vram, "defauts": cpt.defauts_disque,
                  "evictions": cpt.evictions},
        "wall_s": round(mur, 3), "generation_s": round(t_gen, 1),
    }
    if T_ == choix.shape[0]:
        ref = next((x for x in gold["resultats"] if x["emplacements"] == args.emplacements), None)
        if ref is not None:
            ligne["cache_equals_reference_engine"] = (cpt.succes_vram, cpt.defauts_disque, cpt.evictions) == (
                ref["succes_vram"], ref["defauts_disque"], ref["evictions"])
    print(json.dumps(ligne), flush=True)


def bras_gemm(args):
    """The tensor-core expert GEMM (trc_gemm_mxfp4_lot) on an expert-parallel share: 16 experts
    of 3 x 2880 x 2880 MXFP4 matrices (raw parts' CODES_BRUTS / ECHELLES_BRUTES, as resident),
    --gemm tokens per expert (16 at batch 64 over 8 GPUs with uniform top-4), x f32; all 48
    GEMMs in one batched call (quantization launch + MMA launch), timed with CUDA events, L2
    flushed between steps. Beside it the same products token by token with the row-group GEMV
    (trc_gemv_lot over the 48 matrices, one launch per token). Roofline: HBM, the matrices'
    bytes (0.53 B per weight) per call; FLOP/s reported beside it."""
    import ctypes as C

    import numpy as np
    import torch

    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.carte import CoucheCarte

    torch.cuda.set_device(rang()[2])
    n, E = args.gemm, 16
    t0 = time.time()
    c = S.couche(args.graine, T.DimsExpert.gpt_oss(), E, brut=True)
    t_gen = time.time() - t0
    cc = CoucheCarte(c, k=args.k, brut=True)
    R = Cc = 2880
    rng = np.random.default_rng(args.graine)
    x = torch.from_numpy(rng.standard_normal((E * 3, n, Cc)).astype(np.float32)).cuda()
    y = torch.zeros(E * 3, n, R, dtype=torch.float32, device="cuda")
    # the experts resident as SoA slots (codes of each matrix 256-aligned: the weight tiles come
    # by TMA), copied from the raw parts; the same GEMMs on the raw parts' streams (their codes
    # 16 mod 32 here: the tiles by 8-byte copies) as a second leg
    te = T.taille_emplacement(c.dims)
    slots = torch.empty(E * te + 256, dtype=torch.uint8, device="cuda")
    sb = slots.data_ptr() + (-slots.data_ptr()) % 256
    te256 = (te + 255) // 256 * 256
    ctl = torch.zeros(4 * E, dtype=torch.int32, device="cuda")
    for e in range(E):
        cc.n.copier_brut(cc.partie(e, brute=True), slots[(sb - slots.data_ptr()) + e * te256:][:te], c.dims,
                         ctl[4 * e:4 * e + 4])
    torch.cuda.synchronize()
    assert (ctl == 0).all()
    nbj = R * (Cc // 32)
    eo = (nbj * 16 + 255) & ~255
    bo = (eo + nbj + 255) & ~255
    descs, descs_p = [], []
    for e in range(E):
        p = c.parties_brutes[e]
        base = cc.partie(e, brute=True).data_ptr()
        nf = int.from_bytes(p[10:12], "little")
        flux = {}
        for i in range(nf):
            d = p[64 + 16 * i:80 + 16 * i]
            flux[(d[0], d[1])] = int.from_bytes(d[4:8], "little")
        for j in range(3):
            m = 3 * e + j
            s0 = sb + e * te256 + j * ((bo + 4 * R + 255) & ~255)
            descs.append(T.DescGemm(s0, s0 + eo, s0 + bo, x[m].data_ptr(), y[m].data_ptr(), R, Cc, n, 0))
            cod, ech, bia = base + flux[(0x06, j)], base + flux[(0x07, j)], base + flux[(0x02, j)]
            descs_p.append(T.DescGemm(cod, ech, bia, x[m].data_ptr(), y[m].data_ptr(), R, Cc, n, 0))
    nb = len(descs)
    hote = (T.DescGemm * nb)(*descs)  # host descriptors (copied into the launches' parameters)
    hote_p = (T.DescGemm * nb)(*descs_p)
    par_tma = sum(1 for d in descs if d.codes % 32 == 0)  # weight tiles by TMA (else 8-byte copies)
    par_tma_p = sum(1 for d in descs_p if d.codes % 32 == 0)
    octets = int(T.lib.trc_gemm_mxfp4_lot_espace_octets(Cc, n, nb))
    esp = torch.empty(octets + 256, dtype=torch.uint8, device="cuda")
    e0 = esp.data_ptr() + (-esp.data_ptr()) % 256
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    vidange = torch.empty(64 << 20, dtype=torch.float32, device="cuda")

    def gemm(h=hote):
        T.verifier(T.lib.trc_gemm_mxfp4_lot(C.addressof(h), nb, R, Cc, n, e0, octets, err.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))

    t_p = chrono_etapes(lambda: gemm(hote_p), lambda s: None, args.warmup + args.steps, args.warmup, vidange)
    y_p = y.clone()
    t = chrono_etapes(gemm, lambda s: None, args.warmup + args.steps, args.warmup, vidange)
    assert int(err.item()) == 0, "a bounded wait of the GEMM gave up"
    assert torch.equal(y.view(torch.int32), y_p.view(torch.int32)), "slots and raw parts: different bits"
    # the same products token by token over the slots (the row-group GEMV batch)
    pas_m = (bo + 4 * R + 255) & ~255
    off = [0, pas_m, 2 * pas_m]
    yg = torch.zeros(n, E * 3, R, dtype=torch.float32, device="cuda")
    xg = x.transpose(0, 1).contiguous()  # [n][48][C]
    lots = []
    for tk in range(n):
        dg = (T.DescGemv * nb)(*[T.DescGemv(sb + (m // 3) * te256 + off[m % 3], xg[tk, m].data_ptr(), yg[tk, m].data_ptr(),
                                            R, Cc) for m in range(nb)])
        lots.append(torch.frombuffer(bytearray(bytes(dg)), dtype=torch.uint8).cuda())

    def gemv():
        for tk in range(n):
            cc.n.gemv_lot(lots[tk], nb, R)

    t_v = chrono_etapes(gemv, lambda s: None, args.warmup + args.steps, args.warmup, vidange)
    torch.cuda.synchronize()
    # agreement of the two (x quantized to MXFP8 on the tensor-core side)
    a = y.cpu().numpy()
    b = yg.transpose(0, 1).cpu().numpy()
    ecart = float(np.abs(a - b).max() / max(1.0, np.abs(b).max()))
    octets_w = nb * (R * Cc // 32 * 17)
    ms, ms_v = sum(t) / args.steps, sum(t_v) / args.steps
    pic, sorte = pics()
    flops = 2.0 * nb * R * Cc * n
    ligne = {
        "metric": "tensor-core MXFP4 expert GEMM (tcgen05 block-scaled), GB/s of weights",
        "value": round(octets_w / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "steps": args.steps, "warmup": args.warmup, "n_gpus": 1, "higher_is_better": True, "dtype": "e2m1 x e4m3 -> f32",
        "config": {"workload": f"config 3 share: {E} experts x 3 matrices 2880 x 2880 MXFP4, {n} tokens per expert "
                               "(x f32, quantized to MXFP8 in the call)", "tokens_per_expert": n, "matrices": nb,
                               "weights": "resident as SoA slots (codes 256-aligned)",
                               "weight_tiles_by_tma": par_tma,
                   "l2": "flushed between steps (256 MB written)"},
        "tflops": round(flops / (ms * 1e-3) / 1e12, 2),
        "roofline": {"bound": "hbm", "achieved": round(octets_w / (ms * 1e-3) / 1e9, 1), "peak": pic, "unit": "GB/s",
                     "frac": round(octets_w / (ms * 1e-3) / 1e9 / pic, 4), "peak_source": sorte,
                     "algorithmic_bytes_per_launch": octets_w},
        "gemv_token_by_token": {"ms": round(ms_v, 4), "value": round(n * octets_w / (ms_v * 1e-3) / 1e9, 1),
                                "unit": "GB/s (weight bytes read per token pass)",
                                "speedup_of_gemm": round(ms_v / ms, 2)},
        "from_raw_parts": {"ms": round(sum(t_p) / args.steps, 4),
                           "value": round(octets_w / (sum(t_p) / args.steps * 1e-3) / 1e9, 1), "unit": "GB/s",
                           "weight_tiles_by_tma": par_tma_p,
                           "note": "the same GEMMs on the raw parts' CODES_BRUTS / ECHELLES_BRUTES streams, same bits"},
        "max_rel_diff_vs_gemv": ecart,
        "generation_s": round(t_gen, 1),
    }
    print(json.dumps(ligne), flush=True)


def bras_prefill(args):
    """One gpt-oss-120b MoE layer (128 resident experts, top-4) on a batch of --prefill positions:
    router then the fused layer (each activation decodes its expert's tiles), and router then the
    layer par flux (each distinct routed expert decoded once for the batch), both captured in a
    CUDA graph, timed with CUDA events over --steps replays after --warmup, L2 flushed between
    replays; the two residuals are checked bit for bit on every step."""
    import numpy as np
    import torch

    from troncons_b200.carte import CoucheCarte

    P = args.prefill
    c, t_gen = construire_couche(args)
    cc = CoucheCarte(c, k=args.k, brut=False, jetons=P, n_delta=args.n_delta, n_codes=args.n_codes)
    d, R2 = c.dims.colonnes[0], c.dims.lignes[2]
    rng = np.random.default_rng(args.graine)
    x = torch.from_numpy(rng.standard_normal((P, d)).astype(np.float32)).to(torch.bfloat16).cuda()
    r0 = torch.from_numpy(rng.standard_normal((P, R2)).astype(np.float32)).cuda()
    rf, rp = r0.clone(), r0.clone()
    vidange = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    legs = ("fusionnee", "par_flux") if P <= 128 else ("par_flux",)  # the fused layer takes 128 tokens at most
    for _ in range(2):
        if P <= 128:
            cc.couche(x, rf)
        cc.couche_par_flux(x, rp)
    torch.cuda.synchronize()
    graphes = {}
    for nom, f in (("fusionnee", lambda: cc.couche(x, rf)), ("par_flux", lambda: cc.couche_par_flux(x, rp))):
        if nom not in legs:
            continue
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            f()
        graphes[nom] = g
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    temps = {n: [] for n in legs}
    egaux = True
    for s in range(args.warmup + args.steps):
        for nom in legs:
            (rf if nom == "fusionnee" else rp).copy_(r0)
            vidange.zero_()
            a.record()
            graphes[nom].replay()
            b.record()
            torch.cuda.synchronize()
            if s >= args.warmup:
                temps[nom].append(a.elapsed_time(b))
        if P <= 128:
            egaux &= bool(torch.equal(rf.view(torch.int32), rp.view(torch.int32)))
    assert (cc.controle.cpu().numpy() == 0).all()
    # the same with the experts of >= 16 activations on the tensor cores (trc_moe_couche_par_flux_mma):
    # not capturable (one wait for the routing), timed eagerly, router included
    rm = r0.clone()
    t_mma = []
    for s in range(args.warmup + args.steps):
        rm.copy_(r0)
        vidange.zero_()
        a.record()
        cc.couche_par_flux(x, rm, mma_seuil=16)
        b.record()
        torch.cuda.synchronize()
        if s >= args.warmup:
            t_mma.append(a.elapsed_time(b))
    assert int(cc.erreur_pf.item()) == 0 and (cc.controle.cpu().numpy() == 0).all()
    dp, dm = (rp - r0).cpu().numpy(), (rm - r0).cpu().numpy()
    ecart_mma = float(np.abs(dm - dp).max() / max(1e-30, np.abs(dp).max()))
    ms = {n: sum(v) / len(v) for n, v in temps.items()}
    ms_mma = sum(t_mma) / len(t_mma)
    idx = cc.idx.cpu().numpy()
    comptes = np.bincount(idx, minlength=c.experts)
    print(json.dumps({
        "metric": "MoE layer over a batch of positions: positions per second, layer par flux",
        "value": round(P / (ms["par_flux"] * 1e-3), 1), "unit": "positions/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms["par_flux"], 4), "higher_is_better": True, "dtype": "u8",
        "data": "synthetic (seeded gpt-oss-120b-shaped MXFP4 experts, .trc v1.2 parts)",
        "config": {"workload": f"one gpt-oss-120b MoE layer, {P} positions, 128 experts, top-{args.k}",
                   "distinct_experts": int(len(np.unique(idx))), "l2": "flushed between replays"},
        "fused_ms_per_step": round(ms["fusionnee"], 4) if P <= 128 else None,
        "fused_positions_per_s": round(P / (ms["fusionnee"] * 1e-3), 1) if P <= 128 else None,
        "speedup_vs_fused": round(ms["fusionnee"] / ms["par_flux"], 3) if P <= 128 else None,
        "bit_identical_to_fused": egaux if P <= 128 else None,
        "tensor_cores": {"ms_per_step": round(ms_mma, 4), "positions_per_s": round(P / (ms_mma * 1e-3), 1),
                         "speedup_vs_par_flux": round(ms["par_flux"] / ms_mma, 3),
                         "experts_on_tensor_cores": int((comptes >= 16).sum()),
                         "activations_on_tensor_cores": int(comptes[comptes >= 16].sum()),
                         "max_rel_diff_vs_exact": ecart_mma,
                         "note": "trc_moe_couche_par_flux_mma, experts with >= 16 activations as tcgen05 GEMMs "
                                 "(x and h quantized to MXFP8); eager, router included, one wait for the routing"},
        "generation_s": round(t_gen, 1)}), flush=True)
    del graphes


def bras_modele(args):
    """Prints mesurer_modele's line (see there); with --par-rang B > 1, mesurer_modele_ep's
    measurement of a batch of B sequences on this one GPU."""
    if args.par_rang > 1:
        print(json.dumps(mesurer_modele_ep(args, args.steps, args.warmup)), flush=True)
        return
    print(json.dumps(mesurer_modele(args, args.steps, args.warmup, args.exactitude)), flush=True)


def mesurer_modele(args, steps: int, warmup: int, exactitude: int) -> dict:
    """Config 2 (and 4): a seeded synthetic gpt-oss-120b (36 layers, d 2880, 64 / 8 heads of 64,
    sinks, YaRN, even layers sliding over 128, 128 experts top-4 of 2880 x 2880 MXFP4 as .trc v1.2
    parts, Q8_0 attention, embedding and unembedding of 201,088 rows) drawn and encoded on the GPU,
    all resident in HBM. The context: --contexte seeded token ids through the step (no
    unembedding), then --steps greedy steps timed with CUDA events after --warmup. With
    --exactitude N: N greedy steps from the context on the .trc parts, then on the raw parts of
    the same weights; every step's logits compared bit for bit (the exactness invariant)."""
    import hashlib

    import numpy as np
    import torch

    import troncons_b200.modele as M

    t0 = time.time()
    m = M.Modele(couches=args.couches, d=2880, tetes=64, tetes_kv=8, experts=args.experts, k=args.k, vocab=201088,
                 contexte=args.contexte + warmup + max(steps, exactitude) + 1, ffn=2880, fenetre=128,
                 graine=args.graine, compresse=True, brut=exactitude > 0, deltas_predecodes=not args.sans_predecodage)
    torch.cuda.synchronize()
    t_gen = time.time() - t0
    rng = np.random.default_rng(args.graine)
    contexte = rng.integers(0, 201088, args.contexte)
    lg, jt, ct = m.vues()

    def prefixe():
        for p, j in enumerate(contexte):
            m.pas(int(j), p, sortie=False)
        torch.cuda.synchronize()

    t1 = time.time()
    prefixe()
    t_ctx = time.time() - t1
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    pos = args.contexte
    j = int(contexte[-1])
    for _ in range(warmup):
        m.pas(j, pos)
        pos += 1
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(steps):
        m.pas(j, pos)
        pos += 1
    ev[1].record()
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / steps
    assert (ct.cpu().numpy() == 0).all(), "integrity counters set"
    # algorithmic bytes of a token at the timed positions: 4 routed experts' parts per layer (the
    # mean part), the attention's Q8_0 and f32 tensors, the router, the KV cache read, the
    # unembedding
    parts = [float(np.mean(m.parties["compresse"][l][2])) for l in range(m.couches)]
    if m.deltas:
        # DELTA decoded ahead: the step reads the decoded delta bytes instead of the DELTA streams
        # (the streams' size from expert 0's part table of each layer, taken as the layer's mean).
        nbd = sum(m.dims.lignes[j] * (m.dims.colonnes[j] // 32) for j in range(3))
        for l in range(m.couches):
            buf, adr, _ = m.parties["compresse"][l]
            e0 = int(np.flatnonzero(adr)[0])
            o = int(adr[e0]) - buf.data_ptr()
            tete = buf[o:o + 64 + 16 * 16].cpu().numpy().tobytes()
            parts[l] += nbd - octets_flux(tete, (0x03,), (0, 1, 2))
    dq, dkv = 64 * 64, 8 * 64
    att = (dq + 2 * dkv) * 2880 // 32 * 34 + 2880 * dq // 32 * 34 + 4 * (dq + 2 * dkv + 2880 + 64 + 2 * 2880)
    routeur = 4 * 128 * 2880 + 4 * 128
    kv = sum(2 * 2 * dkv * (min(128, pos) if l % 2 == 0 else pos) for l in range(m.couches))
    octets = m.k * sum(parts) + m.couches * (att + routeur) + kv + 201088 * 2880 // 32 * 34 + 4 * 2880
    pic, sorte_pic = pics()
    ligne = {
        "metric": "gpt-oss-120b decode tokens/s (whole step, batch 1, synthetic weights)",
        "value": round(1000.0 / ms, 2), "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "u8",
        "data": "synthetic seeded gpt-oss-120b-shaped weights drawn and encoded on the GPU (.trc v1.2 parts)",
        "config": {"workload": f"config 2: {m.couches} layers, 128 experts top-4, vocab 201,088, context "
                               f"{args.contexte} seeded tokens, greedy", "positions": [args.contexte, pos],
                   "delta_predecoded": not args.sans_predecodage},
        "roofline": {"bound": "hbm", "algorithmic_bytes_per_token": int(octets),
                     "achieved": round(octets / (ms * 1e-3) / 1e9, 2), "peak": pic, "unit": "GB/s",
                     "frac": round(octets / (ms * 1e-3) / 1e9 / pic, 4), "peak_source": sorte_pic},
        "generation_s": round(t_gen, 1), "context_s": round(t_ctx, 1),
    }
    if exactitude:
        empreintes, jetons = {}, {}
        for actifs in ("compresse", "brut"):
            m.choisir(actifs)
            lg, jt, ct = m.vues()
            ct.zero_()
            prefixe()
            h = hashlib.sha256()
            j, js = int(contexte[-1]), []
            for s in range(exactitude):
                m.pas(j, args.contexte + s)
                z = lg.cpu().numpy()
                h.update(z.tobytes())
                j = int(jt.cpu().numpy()[0])
                js.append(j)
            assert (ct.cpu().numpy() == 0).all()
            empreintes[actifs], jetons[actifs] = h.hexdigest(), js
        ligne["exactitude"] = {"steps": exactitude, "logits_sha256_compresse": empreintes["compresse"],
                               "logits_sha256_brut": empreintes["brut"],
                               "bit_identical": empreintes["compresse"] == empreintes["brut"],
                               "tokens_identical": jetons["compresse"] == jetons["brut"]}
    del m
    torch.cuda.empty_cache()
    return ligne


def main():
    args = arguments()
    if args.modele:
        bras_modele(args)
        return
    if args.prefill:
        bras_prefill(args)
        return
    if args.flux:
        bras_flux(args)
        return
    if args.codeur:
        bras_codeur(args)
        return
    if args.gemm:
        bras_gemm(args)
        return
    if args.impl == "reference":
        bras_reference(args)
    elif rang()[1] > 1:
        bras_ep(args)
    else:
        notre_bras(args)


if __name__ == "__main__":
    main()
