#!/usr/bin/env python
"""Benchmark of the DS-MeZO zeroth-order optimizer step on B200.

One step = power iteration of every unique activation (3 iterations), AGZO perturbation
with Philox-regenerated draws, pos/neg copies, Kalman/SPSA update and ZO-Muon
Newton-Schulz of every adapter factor of every layer (ds_mezo/controller.py:165-292),
plus, on N > 1 GPUs, the all-reduce of the Kalman sums and the all-gather of the updated
factors. Synthetic seeded inputs of the named shapes stand in for a model's adapters and
rollout activations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 7b|1.5b|toy|70b] [--impl ours|reference]

Prints one JSON line (rank 0). N > 1 runs under torch.distributed.run, one rank per GPU,
layers sharded in contiguous ranges.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ds-mezo_b200"))

CONFIGS = {
    # name: layers, hidden, intermediate, kv_out, rank, tokens, factor dtype, act dtype, schedule, seed
    "toy": dict(layers=4, hidden=512, inter=1408, kv=128, rank=8, tokens=256, fdt="f32", adt="f32",
                schedule="quintic", seed=0, workload="toy adapter set (4 layers x 7 modules, rank 8)"),
    "1.5b": dict(layers=28, hidden=1536, inter=8960, kv=256, rank=16, tokens=2048, fdt="bf16", adt="bf16",
                 schedule="quintic", seed=1, workload="Qwen2.5-1.5B-shaped adapter set (28 x 7 modules, rank 16)"),
    "7b": dict(layers=28, hidden=3584, inter=18944, kv=512, rank=64, tokens=4096, fdt="bf16", adt="bf16",
               schedule="cubic", seed=2, workload="Qwen2.5-7B-shaped adapter set (28 x 7 modules, rank 64)"),
    "70b": dict(layers=80, hidden=8192, inter=28672, kv=1024, rank=128, tokens=8192, fdt="bf16", adt="bf16",
                schedule="cubic", seed=3, workload="Llama-3-70B-shaped adapter set (80 x 7 modules, rank 128)"),
    # 16 SPSA directions per step: 32 +/- copies, per direction 8 Bernoulli(0.4) rollout
    # rewards (4 per copy) turned into dd_k by the RLOO baseline, one joint Kalman update
    "7b-k16": dict(layers=28, hidden=3584, inter=18944, kv=512, rank=64, tokens=4096, fdt="bf16", adt="bf16",
                   schedule="cubic", seed=4, directions=16, rollouts=8,
                   workload="Qwen2.5-7B-shaped adapter set (28 x 7 modules, rank 64), 16 SPSA directions"),
}
DT = {"f32": torch.float32, "bf16": torch.bfloat16}
METRIC = "ZO optimizer step ms (all adapters, 7B/70B shape) at 1/2/4/8 B200; % HBM roofline"
EPS = 1e-3
TOTAL_STEPS = 1000


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clocks and clock-event reasons during the timed region through NVML
    (read-only queries, every ~2 ms from a thread, so even a short timed region has
    samples); reports no samples when NVML is not importable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, gpus):
        self.gpus = gpus
        self.samples = []          # (sm_mhz, sm_max_mhz, reason bits)
        self.reasons = set()
        self._stop = False
        self._thread = None
        self._nvml = None

    def _run(self, handles):
        nv = self._nvml
        bits = [(name, getattr(nv, attr, 0)) for name, attr in self.REASONS]
        while not self._stop:
            for h in handles:
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                except Exception:
                    continue
                self.samples.append((sm, smax))
                for name, bit in bits:
                    if bit and (r & bit):
                        self.reasons.add(name)
            time.sleep(0.002)

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self._nvml = nv
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            ids = [int(x) for x in vis.split(",")] if vis else None
            handles = [nv.nvmlDeviceGetHandleByIndex(ids[g] if ids and g < len(ids) else g) for g in self.gpus]
            import threading
            self._thread = threading.Thread(target=self._run, args=(handles,), daemon=True)
            self._thread.start()
        except Exception:
            self._nvml = None
        return self

    def __exit__(self, *a):
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=2)
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples (NVML unavailable)"]}
        sm = sorted(x[0] for x in self.samples)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(x[1] for x in self.samples),
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "NVML, 2 ms period"}


def config_of(cfg, world, act_gb_per_gpu=None):
    """The workload description both arms print (same keys, so the lines compare)."""
    act = act_gb_per_gpu
    if act is None:
        act = cfg["tokens"] * (3 * cfg["hidden"] + cfg["inter"]) * (2 if cfg["adt"] == "bf16" else 4) * \
            cfg["layers"] / max(world, 1) / 1e9
    return {"workload": cfg["workload"], "layers": cfg["layers"], "hidden": cfg["hidden"],
            "intermediate": cfg["inter"], "kv_out": cfg["kv"], "rank": cfg["rank"], "tokens": cfg["tokens"],
            "copy_dtype": cfg["fdt"], "activation_dtype": cfg["adt"], "ns_schedule": cfg["schedule"],
            "directions": cfg.get("directions", 1), "power_iters": 3,
            "parallelism": f"layer-sharded x{world}" if world > 1 else "single GPU",
            "l2": ("inputs larger than L2 (activations %.2f GB per step per GPU)" % act) if act >= 0.256 else
                  ("L2 flushed between timed steps (a 256 MB write outside the timing; activations %.3f GB)" % act)}


# ----------------------------------------------------------------------------- setup
def init_set(aset, cfg, device, layer0):
    """Seeded synthetic state: factors and momentum ~ N(0,1) (the factors rounded to the copy
    dtype and held as fp32 masters), var = eps^2, bases = QR of a Gaussian, activations
    N(0,1) x lognormal(0,1) channel scales."""
    g = torch.Generator(device=device)
    g.manual_seed(cfg["seed"] * 1000 + layer0)
    aset.factors[: aset.numel].copy_(torch.randn(aset.numel, generator=g, device=device).to(DT[cfg["fdt"]]))
    aset.sync_shadow()
    aset.mu.normal_(generator=g)
    aset.var.fill_(EPS ** 2)
    for b, s in enumerate(aset.bases):
        aset.V(b).copy_(torch.linalg.qr(torch.randn(s.D, cfg["rank"], generator=g, device=device))[0])
        scale = torch.exp(torch.randn(s.D, generator=g, device=device))
        aset.H(b).copy_(torch.randn(s.T, s.D, generator=g, device=device) * scale)


def alg_bytes(aset, cfg):
    """Algorithmic bytes per launch of each streaming kernel (whole set). Masters, momentum,
    variance and z are fp32; f is the copy dtype's size (the +/- copies and the shadow)."""
    f = aset.pos.element_size()
    fs = f if aset.shadow is not None else 0
    N = aset.numel
    K = aset.directions
    hb = sum(b.T * b.D for b in aset.bases) * aset.H_arena.element_size()
    R = cfg["rank"]
    vr = sum(b.D * R for b in aset.bases) * 4
    yr = sum(b.T * R for b in aset.bases) * 4
    nB = sum(R * m.d_in for m in aset.modules)
    # fused W Gram (tensor-core path, R <= 64): per 128-row W tile its upper 8 x 8 blocks
    nq = (R // 8) * (R // 8 + 1) // 2
    gp = sum((b.D + 127) // 128 for b in aset.bases) * nq * 64 * 8
    return {
        # single pass: read H once, [V_hi|V_lo]; write and read back [Y_hi|Y_lo]; write W and
        # the W-tile Gram partials
        "pi_fused": hb + 2 * vr + 2 * yr + (gp if R <= 64 else 0),
        "pi_y": hb + vr + yr,                      # read H, bf16 [V_hi|V_lo]; write bf16 [Y_hi|Y_lo]
        "pi_w": hb + yr + vr,                      # read H, [Y_hi|Y_lo]; write W (fp32)
        "pi_gram": gp if R <= 64 else vr,          # read the per-tile Gram partials (else W)
        "pi_apply": 3 * vr,                        # read W; write V (fp32) and [V_hi|V_lo]^T (bf16)
        "pi_split": 2 * vr,                        # read V, write bf16 [V_hi | V_lo]^T
        "bside": nB * 12,                          # read B, var_B and the basis rows
        "perturb": N * (2 * f + 20),               # read p, mu, var, K-operand rows; write pos, neg, z
        "gram": N * 20 if K == 1 else N * 4,       # read mu, var, z, write mu, var (K > 1: read mu2)
        "kalman_dirs": N * (16 + 4 * K),           # read mu, var, K z; write mu, var
        "apply": N * (12 + fs),                    # read p, mu2; write p and its shadow
    }


# DRAM bytes per algorithmic byte of each kernel, from ncu (dram__bytes_read.sum +
# dram__bytes_write.sum) on the 4-layer cut of the 7B workload, whose launches read more
# than L2 holds; the full workload's launches do the same work per unit, so traffic scales
# with the algorithmic bytes (the k_pi_yp / k_pi_w and adapter-kernel summaries under profiles/).
TRAFFIC_PER_ALG_BYTE = {"pi_y": 1.002, "pi_w": 1.002, "perturb": 0.925, "gram": 0.899, "apply": 0.862,
                        "bside": 0.981}


# ----------------------------------------------------------------------------- CPU oracle
def cpu_oracle_sample(cfg, layers_in_sample=1, steps=1, warmup=0):
    """The oracle (reference algorithm restated on CPU, fp32) on `layers_in_sample` layers
    of the workload; returns seconds per step for the sample. With K directions the
    perturbation runs K times and the joint update observes all K."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle import reference_ops as ref
    from step_harness import make_inputs, oracle_state
    torch.set_num_threads(os.cpu_count() or 1)
    mods, bases, A, B, V0, H = make_inputs(layers_in_sample, cfg["hidden"], cfg["inter"], cfg["kv"], cfg["rank"],
                                           cfg["tokens"], cfg["seed"], torch.float32, torch.float32)
    st = oracle_state(mods, A, B, V0, EPS, TOTAL_STEPS, schedule=ref.get_schedule(cfg["schedule"]))
    g = torch.Generator().manual_seed(cfg["seed"])
    rca = cfg["rank"]
    times = []
    K = cfg.get("directions", 1)
    for i in range(warmup + steps):
        dirs = []
        for _ in range(K):
            draws = []
            for m in mods:
                draws.append(torch.randn(cfg["rank"], cfg["rank"], generator=g))
                draws.append(torch.randn(m.d_out, rca, generator=g))
            dirs.append(draws)
        t0 = time.perf_counter()
        st.step_count += 1
        if K == 1:
            perts = ref.perturb_phase(st, H, dirs[0], 3)
            ref.update_phase(st, perts, 1.0)
        else:
            perts = ref.perturb_phase_directions(st, H, dirs, 3)
            ref.update_phase_directions(st, perts, [1.0] * K)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return sum(times) / len(times), torch.get_num_threads()


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="7b", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small profiling cases)")
    ap.add_argument("--perturb", default="tensor-cores", choices=["tensor-cores", "cuda-cores"],
                    help="row products of the perturbation: the tcgen05 kernel (default, rank <= 64), or the "
                         "CUDA cores inside the streaming kernel")
    ap.add_argument("--power-iter", default="two-pass", choices=["two-pass", "single-pass"],
                    help="tensor-core power iteration: two products per iteration (default), or the single-pass "
                         "kernel that reads each activation from HBM once per iteration")
    ap.add_argument("--factor-gather", default=None, choices=["copy-engine", "fused", "nccl"],
                    help="N > 1: how the updated factors reach every rank: one copy-engine copy per peer beside "
                         "the next power iteration, peer stores inside the update kernel, or NCCL (default: "
                         "copy engines on 2 GPUs, peer stores on more)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.layers > 0:
        cfg["layers"] = args.layers
        cfg["workload"] += f" [first {args.layers} layers only]"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, cfg, world, rank)

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        pg = dist.group.WORLD
    from dsmezo_b200 import ShardedStep
    from dsmezo_b200._lib import KERNEL_IDS, lib
    gen = torch.Generator(device=device)
    gen.manual_seed(cfg["seed"])
    K = cfg.get("directions", 1)
    sstep = ShardedStep(cfg["layers"], cfg["hidden"], cfg["inter"], cfg["kv"], cfg["rank"], cfg["tokens"], eps=EPS,
                        total_steps=TOTAL_STEPS, generator=gen, copy_dtype=DT[cfg["fdt"]], act_dtype=DT[cfg["adt"]],
                        schedule=cfg["schedule"], device=device, process_group=pg, directions=K,
                        single_pass_power_iter=args.power_iter == "single-pass",
                        tensor_core_perturb=args.perturb == "tensor-cores", factor_gather=args.factor_gather)
    aset = sstep.aset
    init_set(aset, cfg, device, sstep.layout.ranges[rank].start)
    dd_gen = torch.Generator().manual_seed(cfg["seed"])

    def next_dd():
        """The step's projected-gradient scalar(s): seeded N(0,1) x 10 for one direction; for K
        directions the RLOO scalars of seeded Bernoulli(0.4) rollout rewards."""
        if K == 1:
            return float(torch.randn((), generator=dd_gen)) * 10.0
        from dsmezo_b200 import rloo_direction_scalars
        rewards = torch.bernoulli(torch.full((K, cfg["rollouts"]), 0.4), generator=dd_gen)
        return rloo_direction_scalars(rewards, EPS)

    def step(record=False, gathers=True):
        sstep.perturb()
        if world > 1 and gathers:
            sstep.gather("pos", "neg")              # the +/- adapters the scoring pass needs
        dd = sstep.broadcast_dd(next_dd())
        sstep.update(dd)
        if world > 1 and gathers:
            sstep.gather("factors")                 # updated adapters for the next rollout; it
                                                    # overlaps the next step's power iteration

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local_rank])

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()

    # per-kernel probes over the timed region
    per_step = {"pi_fused": 3, "pi_y": 3, "pi_w": 3, "pi_gram": 6, "pi_chol": 6, "pi_apply": 3, "pi_split": 3, "bside": 1,
                "coef": K, "draw": K, "perturb": K, "kalman_sum": K, "kalman_dirs": 1, "gram": 1, "ns_solve": 1,
                "apply": 1}
    probes = {}
    for name, n in per_step.items():
        cap = n * args.steps
        st_ev = [torch.cuda.Event(enable_timing=True) for _ in range(cap)]
        sp_ev = [torch.cuda.Event(enable_timing=True) for _ in range(cap)]
        for e in st_ev + sp_ev:
            e.record()                               # creates the underlying cudaEvent_t
        probes[name] = [st_ev, sp_ev]
    torch.cuda.synchronize()
    for name, pr in probes.items():
        st_ev, sp_ev = pr
        arr_s = (ctypes_void_array(len(st_ev)))(*[e.cuda_event for e in st_ev])
        arr_p = (ctypes_void_array(len(sp_ev)))(*[e.cuda_event for e in sp_ev])
        pr += [arr_s, arr_p]                         # keep the arrays alive while probed
        lib().dsmz_plan_set_probe(aset._plan, KERNEL_IDS[name], arr_s, arr_p, len(st_ev))

    # A step whose activations fit in L2 (the toy set) would find the previous step's data
    # there: such runs write a buffer larger than L2 between timed steps, outside the timing.
    act_bytes = sum(b.T * b.D for b in aset.bases) * aset.H_arena.element_size()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device) if act_bytes < (256 << 20) else None
    t_start = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_stop = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    launches0 = aset.launches
    with ClockSampler([local_rank] if world == 1 else list(range(world))) as clk:
        for i in range(args.steps):
            if flush is not None:
                flush.fill_(i & 255)
            t_start[i].record()
            step(record=True)
            t_stop[i].record()
        if world > 1:
            sstep.synchronize()                     # the last factors gather is part of the run
            t_stop[-1].record()
        torch.cuda.synchronize()
        barrier()
    ms_local = sum(a.elapsed_time(b) for a, b in zip(t_start, t_stop)) / args.steps
    launches_timed = aset.launches - launches0
    kern = {}
    for name, (st_ev, sp_ev, _, _) in probes.items():
        cnt = lib().dsmz_plan_probe_count(aset._plan, KERNEL_IDS[name])
        lib().dsmz_plan_set_probe(aset._plan, KERNEL_IDS[name], None, None, 0)
        if cnt:
            tot = sum(st_ev[i].elapsed_time(sp_ev[i]) for i in range(cnt))
            kern[name] = {"launches": cnt, "total_ms": tot, "avg_ms": tot / cnt}
    # the all-gathers on their own (each timed alone, between synchronisations), and the step
    # without them: what the gathers add to the step beyond what overlaps
    gathers = None
    if world > 1:
        import torch.distributed as dist
        g_ms = {}
        for names in (("pos", "neg"), ("factors",)):
            ev = []
            for _ in range(3):
                barrier()
                a0 = torch.cuda.Event(enable_timing=True)
                a1 = torch.cuda.Event(enable_timing=True)
                a0.record()
                sstep.gather(*names)
                sstep.synchronize()
                a1.record()
                torch.cuda.synchronize()
                ev.append(a0.elapsed_time(a1))
            g_ms["+".join(names)] = sorted(ev)[1]
        barrier()
        torch.cuda.synchronize()
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(args.steps):
            step(gathers=False)
        c1.record()
        torch.cuda.synchronize()
        barrier()
        t = torch.tensor([c0.elapsed_time(c1) / args.steps] + list(g_ms.values()), device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = t.tolist()
        gathers = {"compute_ms_per_step": vals[0], "allgather_ms": dict(zip(g_ms.keys(), vals[1:])),
                   "bytes_received_per_rank": {k: (world - 1) * sstep.layout.capacity * aset.pos.element_size() *
                                               (K if k.startswith("pos") else 1) * (2 if k.startswith("pos") else 1)
                                               for k in g_ms},
                   "fused_pos_neg": sstep.fused_gather, "factor_gather": sstep.factor_gather,
                   "note": "compute_ms_per_step: the same steps without the all-gathers (Kalman all-reduce and dd "
                           "broadcast kept); allgather_ms: each gather alone; the factors gather overlaps the next "
                           "step's power iteration in the timed steps" +
                           ("; +/- copies: stored into every rank's buffers by the perturbation itself (NVLink "
                            "peer stores), so their gather is part of compute_ms_per_step" if sstep.fused_gather
                            else "") +
                           ("; factors: the update stores the bf16 shadow into every rank's buffer (NVLink peer "
                            "stores); their 'gather' is a one-integer barrier" if sstep.factor_gather == "fused"
                            else "") +
                           ("; factors: a barrier, then one copy-engine copy per peer of this rank's shadow on its "
                            "own stream, beside the next step's power iteration; the timed run ends with a barrier "
                            "after the last copies" if sstep.factor_gather == "copy-engine" else "")}
    gather_ms = sum(gathers["allgather_ms"].values()) if gathers else 0.0
    ms = ms_local
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms_local], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # end to end through the public API: activations from pinned host memory each step,
    # Kalman scalars read back each step
    e2e = None
    if not args.no_e2e:
        host_H = torch.empty(aset.H_arena.numel(), dtype=aset.H_arena.dtype, pin_memory=True)
        host_H.copy_(aset.H_arena)
        host_out = torch.empty(aset.kalman_sums().numel(), dtype=torch.float64, pin_memory=True)
        n_e2e = max(1, min(args.steps, 5))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n_e2e):
            aset.H_arena.copy_(host_H, non_blocking=True)
            sstep.perturb()
            host_out.copy_(aset.kalman_sums(), non_blocking=True)
            if world > 1:
                sstep.gather("pos", "neg")
            dd = sstep.broadcast_dd(next_dd())
            sstep.update(dd)
            if world > 1:
                sstep.gather("factors")
        if world > 1:
            sstep.synchronize()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / n_e2e
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": e2e_ms, "unit": "ms", "h2d_bytes_per_step": host_H.numel() * host_H.element_size(),
               "d2h_bytes_per_step": host_out.numel() * 8, "steps": n_e2e}

    # device-resident activation handoff: every basis's fp32 forward-hook capture converted
    # into the bf16 activation buffer on the device (a distinct capture per basis, so nothing
    # is served from L2), against the reference's pinned-host round trip of the same bytes
    # (timed on the largest capture and scaled by bytes)
    handoff = None
    if not args.no_e2e and world == 1:
        hgen = torch.Generator(device=device).manual_seed(cfg["seed"] + 1)
        # fp32 captures of the first bases that fit in a quarter of the free memory (all of
        # them up to the 7B set; a subset of the 70B set, whose captures exceed HBM)
        budget = torch.cuda.mem_get_info(device)[0] // 4
        nb_h, tot = 0, 0
        for b in aset.bases:
            if tot + b.T * b.D * 4 > budget:
                break
            tot += b.T * b.D * 4
            nb_h += 1
        caps = [torch.randn(b.T, b.D, generator=hgen, device=device) for b in aset.bases[:nb_h]]
        hbytes = sum(c.numel() * (4 + aset.H_arena.element_size()) for c in caps)
        for i, c in enumerate(caps):
            aset.load_activations(i, c)
        h0 = torch.cuda.Event(enable_timing=True)
        h1 = torch.cuda.Event(enable_timing=True)
        n_h = 3
        torch.cuda.synchronize()
        h0.record()
        for _ in range(n_h):
            for i, c in enumerate(caps):
                aset.load_activations(i, c)
        h1.record()
        torch.cuda.synchronize()
        h_ms = h0.elapsed_time(h1) / n_h
        big = max(caps, key=lambda c: c.numel())
        pinned = torch.empty(big.shape, dtype=big.dtype, pin_memory=True)
        r0 = torch.cuda.Event(enable_timing=True)
        r1 = torch.cuda.Event(enable_timing=True)
        pinned.copy_(big, non_blocking=True)
        big.copy_(pinned, non_blocking=True)
        torch.cuda.synchronize()
        r0.record()
        pinned.copy_(big, non_blocking=True)       # ds_mezo/backend.py:85-86
        big.copy_(pinned, non_blocking=True)       # ds_mezo/controller.py:171
        r1.record()
        torch.cuda.synchronize()
        ref_ms = r0.elapsed_time(r1) * sum(c.numel() for c in caps) / big.numel()
        # the step end to end with its activations handed over on the device (the product's
        # path: forward-hook captures already in HBM), the Kalman sums read back each step
        host_out = torch.empty(aset.kalman_sums().numel(), dtype=torch.float64, pin_memory=True)
        d0 = torch.cuda.Event(enable_timing=True)
        d1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        d0.record()
        for _ in range(n_h):
            for i, c in enumerate(caps):
                aset.load_activations(i, c)
            sstep.perturb()
            host_out.copy_(aset.kalman_sums(), non_blocking=True)
            sstep.update(sstep.broadcast_dd(next_dd()))
        d1.record()
        torch.cuda.synchronize()
        e2e_dev = {"value": d0.elapsed_time(d1) / n_h, "unit": "ms", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": host_out.numel() * 8, "steps": n_h,
                   "activations": "fp32 forward-hook captures in HBM, converted into the bf16 buffers on the device"}
        handoff = {"ms_per_step": h_ms, "bytes_per_step": hbytes, "achieved_GBps": hbytes / (h_ms * 1e-3) / 1e9,
                   "bases_handed_over": f"{nb_h} of {len(aset.bases)}",
                   "e2e_device_resident": e2e_dev,
                   "frac": hbytes / (h_ms * 1e-3) / 1e9 / peaks()[0], "launches_per_step": len(caps),
                   "reference_round_trip_ms_per_step": ref_ms,
                   "reference_round_trip": "fp32 capture to pinned host and back (torch copies), timed on the "
                                           "largest capture and scaled by bytes"}
        del caps, pinned, big

    # contrastive scoring loss on the device: the + and - scoring passes' bf16 logits rows
    # for four completions of 512 scored tokens over the Qwen2.5 vocabulary (152064)
    scoring = None
    if not args.no_e2e and world == 1:
        from dsmezo_b200 import scoring as sc
        sgen = torch.Generator(device=device).manual_seed(cfg["seed"] + 2)
        vocab, lens, adv = 152064, [512] * 4, [0.75, -0.25, -0.25, -0.25]
        rows = {k: (torch.randn(sum(lens), vocab, generator=sgen, device=device) * 4).to(torch.bfloat16)
                for k in ("pos", "neg")}
        tg = torch.randint(0, vocab, (sum(lens),), generator=sgen, device=device, dtype=torch.int32)
        for k in rows:
            sc.contrastive_loss(rows[k], lens, adv, tg)
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        n_s = 5
        torch.cuda.synchronize()
        s0.record()
        for _ in range(n_s):
            lp = sc.contrastive_loss(rows["pos"], lens, adv, tg)
            ln = sc.contrastive_loss(rows["neg"], lens, adv, tg)
        s1.record()
        torch.cuda.synchronize()
        s_ms = s0.elapsed_time(s1) / n_s
        sbytes = 2 * rows["pos"].numel() * rows["pos"].element_size()
        scoring = {"ms_per_step": s_ms, "bytes_per_step": sbytes, "achieved_GBps": sbytes / (s_ms * 1e-3) / 1e9,
                   "frac": sbytes / (s_ms * 1e-3) / 1e9 / peaks()[0], "launches_per_step": 4,
                   "workload": "4 completions x 512 scored tokens x 152064 vocabulary, bf16 logits, + and -",
                   "dd": sc.projected_gradient(float(lp), float(ln), 1e-3)}
        del rows

    # first-step calibration of every basis (once per run; after the timed steps, since it
    # rewrites the bases): ours against the reference's torch.svd_lowrank loop over fp32
    # activations (its hooks hand over fp32), timed on one layer's four and scaled by layers
    calib = None
    if not args.no_e2e and world == 1:
        cgen = torch.Generator(device=device).manual_seed(cfg["seed"] + 3)
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        aset.calibrate(generator=cgen)                       # warm-up
        torch.cuda.synchronize()
        c0.record()
        aset.calibrate(generator=cgen)
        c1.record()
        torch.cuda.synchronize()
        c_ms = c0.elapsed_time(c1)
        per_layer = 4                                        # the qkv, o, gate_up and down inputs
        hs = [aset.H(b).float() for b in range(per_layer)]
        torch.svd_lowrank(hs[0], q=aset.basis_width, niter=3)
        torch.cuda.synchronize()
        c0.record()
        for h in hs:
            torch.svd_lowrank(h, q=aset.basis_width, niter=3)
        c1.record()
        torch.cuda.synchronize()
        r_ms = c0.elapsed_time(c1) * (len(aset.bases) / per_layer)
        calib = {"ms": c_ms, "launches": aset.calibration_launch_count(3),
                 "bases": len(aset.bases), "niter": 3,
                 "reference_svd_lowrank_ms": r_ms,
                 "reference": "torch.svd_lowrank(H.float(), q=R, niter=3) per basis on this GPU, timed on one "
                              "layer's 4 activations and scaled by the layer count"}
        del hs

    # a bounded wait that gave up sets the plan's error word and the kernels after it stop
    # early: such a run has no valid timing
    derr = aset.device_error()
    if derr:
        print(json.dumps({"metric": METRIC, "error": f"device error word {derr}: a bounded wait timed out",
                          "rank": rank}), flush=True)
        sys.exit(3)
    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            sstep.close()
            dist.destroy_process_group()
        return
    hbm, tf, src = peaks()
    ab = alg_bytes(aset, cfg)
    dom = max(kern, key=lambda k: kern[k]["total_ms"]) if kern else None
    roof = None
    if dom is not None and dom in ab:
        achieved = ab[dom] / (kern[dom]["avg_ms"] * 1e-3) / 1e9
        tr = TRAFFIC_PER_ALG_BYTE.get(dom)
        roof = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": ab[dom] * tr if tr is not None else None,
                "peak_source": src, "alg_bytes_per_launch": ab[dom]}
    for k, v in kern.items():
        if k in ab:
            v["alg_GBps"] = ab[k] / (v["avg_ms"] * 1e-3) / 1e9
            v["frac_hbm"] = v["alg_GBps"] / hbm
    # whole model: every rank's factors and activations
    f = aset.pos.element_size()
    fs = f if aset.shadow is not None else 0
    act_layer = cfg["tokens"] * (3 * cfg["hidden"] + cfg["inter"]) * aset.H_arena.element_size()
    # per element: read and write the fp32 master, mu and var once, write the shadow; per
    # direction write pos, neg, z and read z back (K > 1)
    per_elem = 24 + fs + K * (2 * f + (4 if K == 1 else 8))
    # activations: each of the 3 power iterations reads H once on the single-pass path (twice
    # on the two-product path: Y = H V, then W = H^T Y)
    passes = 1 if aset.single_pass_power_iter else 2
    step_bytes = sum(sstep.layout.sizes) * per_elem + passes * 3 * act_layer * cfg["layers"]
    # the reference's power iteration reads each activation once per iteration (Y and H^T Y
    # per token chunk, ds_mezo/kernels.py:214-225): its compulsory traffic has 3 passes
    compulsory_bytes = sum(sstep.layout.sizes) * per_elem + 3 * act_layer * cfg["layers"]
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        s, cores = cpu_oracle_sample(cfg, 1, 1, 0)
        cpu = {"value": s * 1e3 * cfg["layers"], "unit": "ms", "cores": cores, "kind": "port",
               "sample": f"oracle (fp32 torch CPU restatement of the reference step) on 1 of {cfg['layers']} "
                         f"layers, one step, scaled x{cfg['layers']}"}
    out = {
        "metric": METRIC, "value": ms, "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": cfg["fdt"] if cfg["fdt"] == "bf16" else "f32", "data": "synthetic (seeded N(0,1) factors and "
        "momentum, lognormal-scaled N(0,1) activations)",
        "config": dict(config_of(cfg, world, sum(b.T * b.D for b in aset.bases) * aset.H_arena.element_size() / 1e9),
                       power_iteration=args.power_iter, perturbation=args.perturb,
                       factor_gather=sstep.factor_gather if world > 1 else None),
        "roofline": roof,
        "step_roofline": {"alg_bytes": step_bytes, "achieved_GBps": step_bytes / (ms * 1e-3) / 1e9,
                          "frac": step_bytes / (ms * 1e-3) / 1e9 / hbm / (world if world > 1 else 1),
                          "compulsory_bytes": compulsory_bytes,
                          "compulsory_frac": compulsory_bytes / (ms * 1e-3) / 1e9 / hbm / (world if world > 1 else 1)},
        "kernels": kern,
        "allgather_ms_per_step": gather_ms,
        "gathers": gathers,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "activation_handoff": handoff,
        "scoring": scoring,
        "calibration": calib,
        "gpu_launches": launches_timed,
        "clocks": clk.summary(),
    }
    print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        sstep.close()
        dist.destroy_process_group()


def ctypes_void_array(n):
    import ctypes
    return ctypes.c_void_p * n


def run_reference(args, cfg, world, rank):
    """Reference arm: the reference algorithm on the host cores. The reference is
    Python/Triton whose only CPU path is the Triton interpreter, and its source is not on
    the GPU box, so the arm runs the oracle (the reference restated in fp32 torch, pinned to
    the reference's own outputs) with every host thread. Each timed step is a whole step of
    the whole configuration (every layer); as many steps are timed as fit in a time budget
    (at most --steps, at least one), and the line reports that count, so value x steps is
    the time the arm actually spent. Setup (the synthetic inputs) is outside the timing."""
    if rank != 0:
        return
    budget_s = float(os.environ.get("DSMEZO_REFERENCE_BUDGET_S", "150"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle import reference_ops as ref
    from step_harness import make_inputs, oracle_state
    torch.set_num_threads(os.cpu_count() or 1)
    K = cfg.get("directions", 1)
    try:
        mods, bases, A, B, V0, H = make_inputs(cfg["layers"], cfg["hidden"], cfg["inter"], cfg["kv"], cfg["rank"],
                                               cfg["tokens"], cfg["seed"], DT[cfg["fdt"]], torch.float32)
    except RuntimeError as e:      # host memory: the fp32 activations of the whole model
        print(json.dumps({"metric": METRIC, "impl": "reference", "unavailable":
                          f"the fp32 oracle state of the whole {cfg['workload']} does not fit in host memory: {e}"}))
        return
    st = oracle_state(mods, A, B, V0, EPS, TOTAL_STEPS, schedule=ref.get_schedule(cfg["schedule"]))
    g = torch.Generator().manual_seed(cfg["seed"])
    rca = cfg["rank"]

    def one_step():
        dirs = []
        for _ in range(K):
            draws = []
            for m in mods:
                draws.append(torch.randn(cfg["rank"], cfg["rank"], generator=g))
                draws.append(torch.randn(m.d_out, rca, generator=g))
            dirs.append(draws)
        t0 = time.perf_counter()
        st.step_count += 1
        if K == 1:
            perts = ref.perturb_phase(st, H, dirs[0], 3)
            ref.update_phase(st, perts, 1.0)
        else:
            perts = ref.perturb_phase_directions(st, H, dirs, 3)
            ref.update_phase_directions(st, perts, [1.0] * K)
        return time.perf_counter() - t0

    times = []
    t_all = time.perf_counter()
    while len(times) < max(1, args.steps):
        times.append(one_step())
        spent = time.perf_counter() - t_all
        if spent + times[-1] > budget_s:
            break
    ms = sum(times) / len(times) * 1e3
    cores = torch.get_num_threads()
    sample = (f"whole steps of the whole configuration ({cfg['layers']} layers, every adapter): {len(times)} timed, "
              f"no warm-up, {cores} host threads (os.cpu_count() = {os.cpu_count()})")
    out = {"metric": METRIC, "value": ms, "unit": "ms", "n_gpus": world, "steps": len(times), "warmup": 0,
           "ms_per_step": ms, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
           "dtype": cfg["fdt"] if cfg["fdt"] == "bf16" else "f32", "impl": "reference",
           "data": "synthetic (seeded N(0,1) factors, lognormal-scaled N(0,1) activations)",
           "config": dict(config_of(cfg, 1), parallelism="host CPU"),
           "cpu_baseline": {"value": ms, "unit": "ms", "cores": cores, "kind": "port", "sample": sample},
           "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "requested_steps": args.steps, "requested_warmup": args.warmup, "budget_s": budget_s}
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
