#!/usr/bin/env python
"""Benchmark: MoE-layer decode tokens/s and MXFP4 matvec HBM GB/s on B200.

Workload: one MoE layer at decode -- 384 routed + 1 shared
MXFP4 expert (hidden 7168, intermediate 2048), bf16 router [384, 7168] ~ N(0, 0.02),
sigmoid top-8, renormalised weights x 2.5 -- on M tokens (default 8) of bf16 x ~ N(0, 1).
Synthetic data with random-init weights of that architecture (seeded). A step is one
layer forward through ``LatentMoE.__call__`` (router + every routed expert + the shared
expert + weighted scatter-add).

    python bench.py [--gpus N --steps K --warmup W --tokens M] [--impl reference]

    python bench.py --config 1 ...      # configs[1]: single-expert MXFP4 matvec GB/s (--tokens 1 or 8)
    python bench.py --config 3 ...      # configs[3]: prefill, T = 4096 tokens per GPU
    python bench.py --config 4 ...      # configs[4]: experts streamed from pinned host memory
    python bench.py --config 5 ...      # a Kimi-K3 layer at decode (896 experts, top-16, latent
                                        # 3584/3072, bf16 shared expert); supplementary, not a
                                        # BASELINE config

Timing: ``value`` replays CUDA graphs (one per token batch, a ring of up to 64 distinct
batches) with inputs resident in HBM, bracketed by CUDA events; consecutive steps use
different token batches so each reads a different set of experts out of a 9 GB pool
(inputs larger than L2). With several GPUs the step holds NCCL collectives: an eager ring
and one graph over a static input buffer are both timed and the faster is reported
(``config.timing`` names it). ``e2e`` times the public API call on pinned host tensors with
the host->device copy of x and the device->host copy of y inside the timed region.
``roofline`` covers the dominant kernel (the block-scaled gate/up grouped matvec), timed
per launch with CUDA events on its launch stream in a second pass. SM clocks and
throttle reasons are sampled during the timed region (NVML every ~2 ms, plus
nvidia-smi). Multi-GPU runs are expert parallel (configs[2] "expert-sharded across
2/4/8 GPUs"): each rank brings its own M tokens (weak scaling) and holds E/N routed
experts plus the shared one; tokens are all-gathered, each rank runs its experts over
every pair routed to them, and a reduce-scatter returns each rank's rows; the time is the
max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, I_, E, TOPK, SCALE = 7168, 2048, 384, 8, 2.5
PROJ_BYTES = I_ * H // 2 + I_ * H // 32                   # 7,798,784 B per MXFP4 projection
EXPERT_BYTES = 3 * PROJ_BYTES                              # 23,396,352 B
ROUTER_BYTES = E * H * 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per GPU (default: 8 for config 2, 4096 for 3, 1 for 4 and 5)")
    ap.add_argument("--experts", type=int, default=None,
                    help="routed experts in the layer (default 384 = BASELINE, 896 for config 5; for "
                         "config 1 the size of the expert ring, default 64; fewer only for small ncu "
                         "captures)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5],
                    help="BASELINE config: 1 = single-expert MXFP4 matvec GB/s, 2 = MoE-layer decode "
                         "(headline), 3 = MoE-layer prefill (--tokens defaults to 4096), 4 = streamed-expert "
                         "decode; 5 = Kimi-K3 layer decode (supplementary)")
    ap.add_argument("--layers", type=int, default=4, help="config 4: consecutive streamed layers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="auto", choices=["auto", "gather", "a2a", "p2p"],
                    help="N > 1: the expert-parallel token exchange (gather: NCCL all_gather + "
                         "reduce_scatter; a2a: the counted NCCL all_to_all; p2p: the decode step's gather "
                         "and reduce-scatter as kernels over NVLink peer memory; auto: p2p at decode, "
                         "gather at prefill)")
    args = ap.parse_args()
    if args.tokens is None:
        args.tokens = {1: 8, 2: 8, 3: 4096, 4: 1, 5: 1}[args.config]
    if args.experts is None:
        args.experts = {1: 64, 5: 896}.get(args.config, E)
    return args


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ distributed

def dist_init(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


# CUDA graphs that hold NCCL calls, and layers that keep such graphs: released before the
# process group is destroyed, on every exit path (a live one makes the teardown wait)
_NCCL_GRAPHS: list = []


def release_nccl_graphs():
    for o in _NCCL_GRAPHS:
        if hasattr(o, "release_graphs"):
            o.release_graphs()
        else:
            o.reset()
    _NCCL_GRAPHS.clear()


def dist_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ----------------------------------------------------------------------- clocks

class ClockSampler:
    """SM clocks and throttle reasons while the timed region runs. One GPU: NVML every
    ~2 ms plus ``nvidia-smi -lms 200``. Several GPUs (one process each): only local rank
    0 samples, NVML for every GPU of the job every ~10 ms, and the other ranks run no
    sampler, so the ranks' launch loops do not compete with NVML calls."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int, world: int = 1):
        import threading

        import torch
        self.proc = None
        self.nv = []                                  # (gpu, sm MHz, max MHz, reasons bitmask)
        self._stop = threading.Event()
        self._thr = None
        self.active = world == 1 or local_rank == 0
        if not self.active:
            return
        gpus = [local_rank] if world == 1 else list(range(min(world, torch.cuda.device_count())))

        def uuid_of(i):
            u = str(torch.cuda.get_device_properties(i).uuid)
            return u if u.startswith("GPU-") else "GPU-" + u

        period = 0.002 if world == 1 else 0.010
        try:
            import pynvml
            pynvml.nvmlInit()
            hs = [(i, pynvml.nvmlDeviceGetHandleByUUID(uuid_of(i))) for i in gpus]

            def poll():
                while not self._stop.is_set():
                    try:
                        for i, h in hs:
                            self.nv.append((i, pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                            pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM),
                                            pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except Exception:
                        return
                    time.sleep(period)
            self._thr = threading.Thread(target=poll, daemon=True)
            self._thr.start()
        except Exception:
            self._thr = None
        if world == 1:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={uuid_of(local_rank)}", f"--query-gpu={self.Q}",
                     "--format=csv,noheader,nounits", "-lms", "200"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except Exception:
                self.proc = None

    # NVML clocks-event reason bits (nvml.h): sw power cap 0x4, hw slowdown 0x8,
    # sw thermal 0x20, hw thermal 0x40
    NV_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def stop(self):
        if not self.active:
            return None
        self._stop.set()
        if self._thr is not None:
            self._thr.join(timeout=2)
        sm, mx, reasons = [], [], set()
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in out.strip().splitlines():
                f = [c.strip() for c in line.split(",")]
                if len(f) < 8:
                    continue
                try:
                    sm.append(float(f[0]))
                    mx.append(float(f[1]))
                except ValueError:
                    continue
                for n, v in zip(names, f[4:8]):
                    if v.lower() == "active":
                        reasons.add(n)
        for n, b in self.NV_BITS.items():
            if any(r & b for _, _, _, r in self.nv):
                reasons.add(n)
        if self.nv:                                   # in-region NVML samples take precedence
            sm = [c for _, c, _, _ in self.nv]
            mx = mx + [m for _, _, m, _ in self.nv]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        gpus = sorted({g for g, _, _, _ in self.nv})
        out = {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx) if mx else None, "samples": len(sm),
               "source": ("nvml" if self.proc is None else "nvml+nvidia-smi") if self.nv else "nvidia-smi",
               "reasons": sorted(reasons)}
        if len(gpus) > 1:
            out["per_gpu_sm_mhz"] = {str(g): statistics.median(c for gg, c, _, _ in self.nv if gg == g)
                                     for g in gpus}
            out["sampled_by"] = "local rank 0 for every GPU of the job"
        return out


# ------------------------------------------------------------- CPU baseline (oracle)

def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:                                       # noqa: BLE001
        return os.cpu_count() or 1


def cpu_baseline(M: int, seed: int, steps: int, budget_s: float = 20.0, layers: int = 1):
    """The reference path restated on the host cores (oracle port): fp32 router in numpy,
    then the reference fused kernel's loop in C (OpenMP over rows, every host core -- the
    launcher's OMP_NUM_THREADS is overridden) for every expert the step routes to, plus the
    shared expert. Weights are a pool of 8 synthetic experts reused by id (the work per
    expert does not depend on the values). Decode steps (M <= 64) run whole, `layers`
    layers each, until ``budget_s`` is spent (at least one); a prefill step is cut after
    ``budget_s`` of expert compute and extrapolated to all U + 1 experts. Returns a dict:
    tokens/s, cores, ISA level, sample description, steps timed, whether they were whole."""
    from oracle import mxfp4_oracle as O
    cores = host_cores()
    try:
        from threadpoolctl import threadpool_limits
        blas = threadpool_limits(cores)
    except Exception:                                       # noqa: BLE001
        blas = None
    rng = np.random.default_rng(seed)
    gate = O.bf16_bits_to_f32(O.f32_to_bf16_bits((rng.standard_normal((E, H)) * 0.02).astype(np.float32)))
    pool = [(O.random_mxfp4(rng, I_, H), O.random_mxfp4(rng, I_, H), O.random_mxfp4(rng, H, I_))
            for _ in range(8)]
    whole = M <= 64
    t_route, t_exp, n_exp, n_steps, U_tot, wall = 0.0, 0.0, 0, 0, 0, 0.0
    for s in range(max(1, steps)):
        x = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.standard_normal((M, H)).astype(np.float32)))
        w0 = time.perf_counter()
        for _ in range(layers):
            t0 = time.perf_counter()
            r = O.route(x, gate, None, TOPK, True, SCALE)
            t_route += time.perf_counter() - t0
            experts = sorted(set(r.expert_indices.reshape(-1).tolist()))
            U_tot += len(experts) + 1
            y = np.zeros_like(x)
            for j, e in enumerate(experts + [-1]):
                tok = np.arange(M) if e < 0 else np.nonzero(r.expert_indices == e)[0]
                (p1, s1), (p3, s3), (p2, s2) = pool[j % len(pool)]
                t0 = time.perf_counter()
                g = O.matvec_fused(x[tok], p1, s1, threads=cores)
                u = O.matvec_fused(x[tok], p3, s3, threads=cores)
                y[tok] += O.matvec_fused(O.silu(g) * u, p2, s2, threads=cores)
                t_exp += time.perf_counter() - t0
                n_exp += 1
                if not whole and t_exp > budget_s:
                    break
            x = (x + y).astype(np.float32)
        wall += time.perf_counter() - w0
        n_steps += 1
        if t_route + t_exp > budget_s:
            break
    if blas is not None:
        blas.restore_original_limits()
    if whole:
        per_step = wall / n_steps
        sample = (f"{n_steps} whole step(s) of M={M} x {layers} layer(s): numpy fp32 router + C port of the "
                  f"reference fused-kernel loop over every routed expert and the shared one ({n_exp} expert "
                  f"FFNs); wall time per step")
    else:
        per_step = t_route / n_steps + (U_tot / n_steps) * (t_exp / n_exp)
        sample = (f"1 step of M={M} cut after {n_exp} of {U_tot} routed+shared expert FFNs: numpy fp32 router "
                  f"+ C port of the reference fused-kernel loop; step time = router + (U+1) x mean expert time")
    return {"tokens_per_s": M / per_step, "s_per_step": per_step, "cores": cores, "isa": O.oracle_isa(),
            "sample": sample, "steps_timed": n_steps, "whole_steps": whole}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path (oracle port) on this box's host cores, on
    the same config and metric as the B200 arm, with every host core (whatever
    OMP_NUM_THREADS the launcher set). Decode configs time whole steps (router + every
    routed expert + the shared one) after one warm-up step, as many as fit in ~100 s and at
    most --steps; prefill times one step cut after a bounded share of its experts and
    extrapolated. Under torchrun rank 0 alone runs it."""
    if rank != 0:
        return
    cfg = args.config
    if cfg == 5:
        print(json.dumps({"impl": "reference", "metric": "k3_layer_decode_tokens_per_s",
                          "unavailable": "config 5 is supplementary (not a BASELINE config); the CPU reference "
                                         "arm is timed on configs 1-4"}))
        return
    t0 = time.perf_counter()
    if cfg == 1:
        line = reference_matvec(args)
        line["wall_s"] = time.perf_counter() - t0
        print(json.dumps(line))
        return
    M = 1 if cfg == 4 else args.tokens
    layers = args.layers if cfg == 4 else 1
    cpu_baseline(M, args.seed + 999, 1, budget_s=5.0, layers=layers)              # warm-up
    res = cpu_baseline(M, args.seed, args.steps, budget_s=100.0, layers=layers)
    tps = res["tokens_per_s"]
    if cfg == 4:
        metric, unit, value, hib = "streamed_decode_s_per_token", "s/token", res["s_per_step"], False
        workload = (f"BASELINE configs[4]: M=1 token through {layers} MoE layers (expert compute only; "
                    "the reference's SSD reads are not timed)")
    else:
        metric = "moe_layer_prefill_tokens_per_s" if cfg == 3 else "moe_layer_decode_tokens_per_s"
        unit, value, hib = "tokens/s", tps, True
        workload = (f"BASELINE configs[{cfg}]: MoE layer {'prefill' if cfg == 3 else 'decode'}, M={M}, "
                    "384+1 MXFP4 experts 7168/2048, top-8")
    kind = (f"port: numpy router + C restatement of the reference's fused-kernel loop, gcc -O3, "
            f"{res['isa']} clone, OpenMP on {res['cores']} threads")
    line = {
        "impl": "reference", "metric": metric, "value": value,
        "unit": unit, "n_gpus": world, "steps": res["steps_timed"], "warmup": 1,
        "ms_per_step": 1000.0 * res["s_per_step"], "higher_is_better": hib,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "tokens": M, "steps_requested": args.steps,
                   "whole_steps": res["whole_steps"]},
        "cpu_baseline": {"value": value, "unit": unit, "cores": res["cores"], "kind": "port",
                         "build": kind, "sample": res["sample"]},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line))


# ------------------------------------------------------- config 4: streamed experts

def run_stream(args, rank, world, local):
    """one token (M=1) through ``--layers`` MoE layers whose 384
    routed experts live in pinned host memory; per layer only the routed experts are
    copied host->HBM on a side stream while the resident shared expert computes. Reports
    s/token end to end and how much of the copy time is hidden behind compute."""
    import torch
    from kimi_k3_mlx_macmini_b200 import synthetic
    from kimi_k3_mlx_macmini_b200.moe import SHARED
    from kimi_k3_mlx_macmini_b200.stream import HostExpertStore, StreamedMoE
    if world != 1 or rank != 0:
        return
    torch.cuda.set_device(local)
    K, W, NL = args.steps, args.warmup, args.layers
    t0 = time.perf_counter()
    layers, stores = [], []
    for li in range(NL):                                     # each layer: its own router and pool
        ll = synthetic.baseline_layer(seed=args.seed + 1 + li, E=args.experts, H=H, I=I_, top_k=TOPK, scale=SCALE)
        stores.append(HostExpertStore(args.experts, ll.expert))
        w = {"gate.weight": ll.gate, "gate.e_score_correction_bias": ll.bias}
        layers.append(StreamedMoE(ll.cfg, li, w, stores[-1], lambda ll=ll: ll.expert(SHARED)))
    build_s = time.perf_counter() - t0
    store = stores[0]

    def token(i):
        x = synthetic.tokens(args.seed * 7919 + i, 1, H)
        for m in layers:
            x = (x.float() + m(x)).to(torch.bfloat16)        # residual stream between layers
        return x

    for i in range(W):
        token(i)
    torch.cuda.synchronize()
    clk = ClockSampler(local, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        token(W + i)
    e1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    s_per_token = e0.elapsed_time(e1) / 1e3 / K
    # copy-only: the same expert sets staged without compute; compute-only: staged first
    sets = []
    for i in range(K):
        x = synthetic.tokens(args.seed * 7919 + W + i, 1, H)
        per = []
        for m in layers:
            ids = sorted(set(m.router.route(x).expert_indices.reshape(-1).tolist()))
            per.append(ids)
            x = (x.float() + m(x)).to(torch.bfloat16)
        sets.append(per)
    torch.cuda.synchronize()
    # copies of one layer at a time, as the token's layers order them (each layer's copy
    # stream is its own, so queuing them back to back would run layers' copies side by
    # side): from an event on the compute stream before the layer's copies are queued to
    # one after it joined the copy stream
    copy_ms = 0.0
    cur = torch.cuda.current_stream()
    for per in sets:
        for m, ids in zip(layers, per):
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(cur)
            m.stage(ids)
            cur.wait_stream(m.copy_stream)
            c1.record(cur)
            torch.cuda.synchronize()
            copy_ms += c0.elapsed_time(c1)
    copy_s = copy_ms / 1e3 / K
    comp_ms = 0.0
    for i, per in enumerate(sets):
        x = synthetic.tokens(args.seed * 7919 + W + i, 1, H)
        for m, ids in zip(layers, per):
            m.stage(ids)
            torch.cuda.synchronize()
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            d0.record()
            y = m(x, stage=False)
            d1.record()
            torch.cuda.synchronize()
            comp_ms += d0.elapsed_time(d1)
            x = (x.float() + y).to(torch.bfloat16)
    comp_s = comp_ms / 1e3 / K
    from kimi_k3_mlx_macmini_b200 import _lib as L
    L.profile_enable(True)
    L.profile_collect()
    token(W)                                                 # one token's launches, counted
    torch.cuda.synchronize()
    prof = L.profile_collect()
    L.profile_enable(False)
    launches = sum(c for _, c in prof.values())
    cpu = None
    if not args.no_cpu_baseline:
        res = cpu_baseline(1, args.seed, 20, budget_s=15.0, layers=NL)
        cpu = {"value": res["s_per_step"], "unit": "s/token", "cores": res["cores"], "kind": "port",
               "build": f"gcc -O3 {res['isa']} clone, OpenMP", "sample": res["sample"] +
               " (expert compute only: the reference's SSD reads are not timed)"}
    overlap = max(0.0, copy_s + comp_s - s_per_token)
    copied = float(np.mean([sum(len(ids) for ids in per) for per in sets])) * store.nbytes_expert()
    line = {
        "metric": "streamed_decode_s_per_token", "value": s_per_token, "unit": "s/token",
        "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": s_per_token * 1e3, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1 weights x e2m1 activation pieces, e8m0 block scales, f32 accumulate (tcgen05 kind::mxf4)",
        "data": "synthetic (seeded random-init weights of the BASELINE layer)",
        "config": {"workload": f"BASELINE configs[4]: M=1 token through {NL} layers, each layer's "
                               f"{args.experts} routed experts in pinned host memory, its top-{TOPK} "
                               "copied host->HBM per token on a side stream, resident shared expert",
                   "layers": NL, "host_store_gb": NL * args.experts * store.nbytes_expert() / 1e9,
                   "store_build_s": build_s},
        "copy_s_per_token": copy_s,
        "compute_s_per_token": comp_s,
        "overlap_s_per_token": overlap,
        "copy_time_hidden_frac": overlap / copy_s if copy_s > 0 else None,
        "compute_hidden_frac": overlap / comp_s if comp_s > 0 else None,
        "h2d_gbs": copied / copy_s / 1e9,
        "e2e": {"value": s_per_token, "unit": "s/token", "h2d_bytes_per_step": copied + 2 * H,
                "d2h_bytes_per_step": NL * TOPK * 8},
        "gpu_launches": int(launches * K),
        "kernel_ms_per_token": {k: v[0] for k, v in prof.items() if v[1]},
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line))


# ------------------------------------------------------------------ B200 arm

def traffic_ratio_from_profiles():
    """DRAM bytes / algorithmic bytes of a gate/up launch, from the committed ncu summary
    of the small case (dram__bytes_read.sum + dram__bytes_write.sum of a 32-expert launch);
    the full launch's traffic is this ratio x its algorithmic bytes (every weight byte is
    read once, so the traffic grows with the bytes streamed)."""
    f = ROOT / "profiles" / "bs_gemv_gateup_config2.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_ratio_small_case:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


def ep_check(moe, full, x, world):
    """Expert-parallel output check on the GPUs, outside the timed region: one batch
    through the expert-parallel layer, and this rank's same tokens through the whole layer
    (all routed experts + the shared one) on this GPU with the 1-GPU kernels. Returns the
    largest relative L2 difference over the ranks."""
    import torch
    y_ep = moe(x).float()
    p2p = getattr(moe, "p2p", None)
    fallback = None
    if p2p is not None and int(dist_max(float(p2p.status.max().item()), world)) != 0:
        # a peer-memory wait gave up on some rank (the status words are agreed over the
        # ranks): every rank drops the peer-memory exchange for the NCCL step and re-runs
        moe.release_graphs()
        moe.exchange = "gather"
        moe.p2p_error = fallback = "a peer-memory wait timed out in the output check"
        y_ep = moe(x).float()
    y_one = full(x).float()
    torch.cuda.synchronize()
    err = float(torch.linalg.vector_norm((y_ep - y_one).double()) / torch.linalg.vector_norm(y_one.double()))
    full._pool = None                                       # free the whole-layer pool again
    torch.cuda.empty_cache()
    out = {"max_rel_l2_over_ranks": dist_max(err, world),
           "against": "the same tokens through the whole layer on one GPU (LatentMoE, 1-GPU kernels)",
           "exchange": moe.exchange_used(x.shape[0]) if hasattr(moe, "exchange_used") else None}
    if p2p is not None:
        out["p2p_status_ok_on_every_rank"] = fallback is None
    return out


def e2e_loop(call, xh, order, K, W, out_shape, world):
    """End to end through the public API, as a serving loop runs it. Every step copies its
    tokens host->device from pinned memory and its output device->host into pinned
    memory, on one copy stream beside the compute stream, with two buffers each way: the
    next step's upload is queued ahead of this step's download, so both copies overlap the
    neighbouring steps' compute without running against each other on the bus. Timed
    with CUDA events on the compute stream (the first timed upload starts after the
    opening event; the compute stream waits for the last download before the closing
    one); max over ranks. Returns ms per step."""
    import torch
    comp = torch.cuda.current_stream()
    cs = torch.cuda.Stream()
    xd = [torch.empty(tuple(xh.shape[1:]), dtype=xh.dtype, device="cuda") for _ in range(2)]
    yh = [torch.empty(out_shape, dtype=torch.float32).pin_memory() for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]

    def upload_on_cs(i):                                # step i's tokens into xd[i % 2]
        b = i % 2
        cs.wait_event(ev_done[b])                       # the step that last read xd[b] is done
        xd[b].copy_(xh[order(i)], non_blocking=True)
        ev_in[b].record(cs)

    def upload(i):
        with torch.cuda.stream(cs):
            upload_on_cs(i)

    def run(i, last):
        b = i % 2
        comp.wait_event(ev_in[b])
        y = call(xd[b])
        ev_done[b].record(comp)
        with torch.cuda.stream(cs):                     # one stream switch a step
            if not last:
                upload_on_cs(i + 1)
            cs.wait_event(ev_done[b])
            y.record_stream(cs)
            yh[b].copy_(y, non_blocking=True)

    upload(0)
    for i in range(W):
        run(i, i == W - 1)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    cs.wait_stream(comp)
    upload(W)
    for i in range(K):
        run(W + i, i == K - 1)
    comp.wait_stream(cs)
    e1.record(comp)
    torch.cuda.synchronize()
    barrier(world)
    return dist_max(e0.elapsed_time(e1) / K, world)


def run_b200(args, rank, world, local):
    import torch
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic

    torch.cuda.set_device(local)
    M, K, W = args.tokens, args.steps, args.warmup
    R = min(K + W, 64)                                      # distinct token batches
    lay = synthetic.baseline_layer(seed=args.seed, E=args.experts, H=H, I=I_, top_k=TOPK, scale=SCALE)
    router = lay.moe()                                      # whole layer (1 GPU) / router (EP)
    if world > 1:
        # expert parallel: this rank holds experts [rank*E/W, (rank+1)*E/W) + the shared one
        from kimi_k3_mlx_macmini_b200.ep import ExpertParallelMoE
        moe = ExpertParallelMoE(lay.cfg, 0, {"gate.weight": lay.gate, "gate.e_score_correction_bias": lay.bias},
                                lay.source, exchange=args.exchange)
        _NCCL_GRAPHS.append(moe)
    else:
        moe = router
        _ = moe.pool

    def batch(rk, i):
        return synthetic.tokens(args.seed * 7919 + rk * 100003 + i, M, H)

    xs = [batch(rank, i) for i in range(R)]
    check = ep_check(moe, router, xs[0], world) if world > 1 else None
    # experts this rank streams per step: the local experts any rank's tokens route to
    E_loc = args.experts // world
    U = []
    for i in range(R):
        ids = torch.cat([router.route(batch(rk, i)).expert_indices.reshape(-1) for rk in range(world)])
        ids = torch.unique(ids)
        U.append(int(((ids >= rank * E_loc) & (ids < (rank + 1) * E_loc)).sum().item()))
    torch.cuda.synchronize()
    step_x = [(W + i) % R for i in range(K)]                # batch of timed step i

    # ---- device-resident timing
    graphs, modes = step_modes(moe, xs, R, world)
    barrier(world)
    ms, timing, clocks = time_modes(modes, step_x, K, W, R, world, local)
    value = world * M / (ms / 1e3)

    # ---- per-kernel timing of the same batches (eager launches, events per kernel; an
    # expert-parallel layer launches its step itself rather than replaying it)
    n_prof = min(K, 50)
    api_graphs = getattr(moe, "graphs", None)
    if api_graphs is not None:
        moe.graphs = False
    L.profile_enable(True)
    L.profile_collect()
    if world > 1:
        moe.collective_timing = True
        moe.collective_ms()
    torch.cuda.synchronize()
    # keep the GPU busy while the host enqueues, so each event pair brackets device time
    torch.cuda._sleep(int(4e7))
    for i in range(n_prof):
        moe(xs[step_x[i]])
    torch.cuda.synchronize()
    prof = L.profile_collect()
    L.profile_enable(False)
    coll = None
    if world > 1:
        coll = {k: v / n_prof for k, v in moe.collective_ms().items()}
        moe.collective_timing = False
    if api_graphs is not None:
        moe.graphs = api_graphs
    gu_ms, gu_n = prof["gateup"]
    dn_ms, dn_n = prof["down"]
    gu_n, dn_n = max(gu_n, 1), max(dn_n, 1)
    U_t = [U[step_x[i]] for i in range(n_prof)]
    gu_bytes = np.mean([(u + 1) * 2 * PROJ_BYTES for u in U_t]) + M * H * 2
    dn_bytes = np.mean([(u + 1) * PROJ_BYTES for u in U_t])
    layer_bytes = np.mean([(u + 1) * EXPERT_BYTES for u in U_t]) + args.experts * H * 2
    peak, peak_kind = measured_peaks()
    gu_gbs = gu_bytes / (gu_ms / gu_n / 1e3) / 1e9
    dn_gbs = dn_bytes / (dn_ms / dn_n / 1e3) / 1e9

    # ---- end to end through the public API with host buffers
    xh = torch.stack([x.cpu() for x in xs]).pin_memory()
    e2e_ms = e2e_loop(moe, xh, lambda i: i % R, K, W, (M, H), world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res = cpu_baseline(M, args.seed, 20, budget_s=15.0)
        cpu = {"value": res["tokens_per_s"], "unit": "tokens/s", "cores": res["cores"], "kind": "port",
               "build": f"gcc -O3 {res['isa']} clone, OpenMP", "sample": res["sample"]}

    for g in graphs:
        g.reset()
    graph_error = getattr(moe, "graph_error", None)
    if world > 1:
        release_nccl_graphs()                               # NCCL graphs go before the process group
    if rank != 0:
        return
    line = {
        "metric": "moe_layer_decode_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1 weights x e2m1 activation pieces, e8m0 block scales, f32 accumulate (tcgen05 kind::mxf4)",
        "data": "synthetic (seeded random-init weights of the BASELINE layer)",
        "config": {"workload": f"BASELINE configs[2]: one MoE layer decode, M={M} tokens per GPU, "
                               f"{args.experts} routed + 1 shared MXFP4 expert (7168/2048), bf16 router, "
                               "top-8, x2.5",
                   "tokens_per_gpu": M,
                   "parallelism": "single GPU" if world == 1 else
                                  f"ep{world}: {args.experts // world} routed experts per rank + replicated shared, "
                                  + ("counted all_to_all dispatch and combine (NCCL)" if moe.uses_a2a(M) else
                                     "all-gather dispatch and reduce-scatter combine as kernels over NVLink "
                                     "peer memory (CUDA IPC)" if moe.exchange_used(M) == "p2p" else
                                     "all_gather dispatch, reduce_scatter combine (NCCL)"),
                   "l2": f"inputs larger than L2: {9.0 / world:.2f} GB of expert weights per GPU, "
                         "a different token batch every step",
                   "timing": timing + ", events around K steps",
                   "api_graph_error": graph_error,
                   "p2p_error": getattr(moe, "p2p_error", None)},
        "ep_check": check,
        "unique_experts_mean": float(np.mean(U_t)),
        "unique_experts_per_batch": U[:8],
        "layer_hbm_gbs": layer_bytes / (ms / 1e3) / 1e9,
        "roofline": {"bound": "hbm", "kernel": "bs_gemv_kernel<gate/up> (block-scaled grouped MXFP4 matvec, tcgen05)",
                     "achieved": gu_gbs, "peak": peak, "unit": "GB/s", "frac": gu_gbs / peak,
                     "peak_kind": peak_kind,
                     "traffic": (None if traffic_ratio_from_profiles() is None
                                 else traffic_ratio_from_profiles() * gu_bytes),
                     "traffic_source": "ncu dram bytes / algorithmic bytes of a 32-expert launch "
                                       "(profiles/bs_gemv_gateup_config2.md) x this launch's algorithmic bytes",
                     "algorithmic_bytes_per_launch": gu_bytes,
                     "launch_ms": gu_ms / gu_n},
        "down_kernel": {"achieved": dn_gbs, "frac": dn_gbs / peak, "launch_ms": dn_ms / dn_n},
        "kernel_ms_per_step": {k: v[0] / n_prof for k, v in prof.items() if v[1]},
        "collective_ms_per_step": coll,
        "e2e": {"value": world * M / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": M * H * 2, "d2h_bytes_per_step": M * H * 4,
                "ms_per_step": e2e_ms,
                "api": ("LatentMoE.__call__ (k3_moe_decode)" if world == 1 else
                        "ExpertParallelMoE.__call__ (counted all-to-all step, launched per call)"
                        if moe.uses_a2a(M) else "ExpertParallelMoE.__call__ (captured step replayed per call)"),
                "copies": "one copy stream, two buffers each way: the next upload ahead of this download, both overlapping the neighbouring steps"},
        "gpu_launches": int(round(sum(c for _, c in prof.values()) / n_prof * K)),
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line))


def step_modes(moe, xs, R, world):
    """Callables per token batch to time. One GPU: one CUDA graph per batch (a ring of R
    graphs). Several GPUs (NCCL collectives in the step): an eager ring and one graph
    over a static input buffer refilled by a device copy before each replay -- replaying
    many graphs that each hold collectives is slower than launching eagerly."""
    import torch
    cap = torch.cuda.Stream()
    with torch.cuda.stream(cap):
        for i in range(min(2, R)):
            moe(xs[i])
    torch.cuda.synchronize()
    graphs, modes = [], []
    if world == 1:
        try:
            for i in range(R):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=cap):
                    moe(xs[i])
                graphs.append(g)
            modes.append((f"CUDA graph per batch ({R} distinct batches replayed as a ring)",
                          [g.replay for g in graphs]))
        except Exception as exc:                            # noqa: BLE001 -- report and time eagerly
            torch.cuda.synchronize()
            graphs = []
            modes.append((f"eager launches ({R} distinct batches as a ring; graph capture failed: "
                          f"{_exc_text(exc)})", [(lambda x=x: moe(x)) for x in xs]))
    else:
        api = ("public API calls (the layer replays its captured step)" if getattr(moe, "graphs", False)
               else "eager launches")
        modes.append((f"{api} ({R} distinct batches as a ring)", [(lambda x=x: moe(x)) for x in xs]))
        if not moe.capturable(xs[0].shape[0]):
            modes[0] = ("eager launches: the counted all-to-all step reads its split sizes on the host "
                        f"({R} distinct batches as a ring)", modes[0][1])
            return graphs, modes
        xin = xs[0].clone()
        try:
            g = torch.cuda.CUDAGraph()
            _NCCL_GRAPHS.append(g)
            with torch.cuda.graph(g, stream=cap):
                moe(xin)
            graphs.append(g)
            modes.append((f"one CUDA graph over a static input ({R} distinct batches copied in as a ring)",
                          [(lambda x=x: (xin.copy_(x, non_blocking=True), g.replay())) for x in xs]))
        except Exception as exc:                            # noqa: BLE001 -- the eager mode stands, reason kept
            torch.cuda.synchronize()
            modes[0] = (modes[0][0] + f"; graph capture failed: {_exc_text(exc)}", modes[0][1])
    return graphs, modes


def _exc_text(exc: BaseException) -> str:
    return f"{type(exc).__name__}: {str(exc).splitlines()[0][:240] if str(exc) else ''}"


def time_modes(modes, steps, K, W, R, world, local):
    """Times K steps of every mode (W warm-up steps each; events bracketed by barriers and
    synchronisation; max over ranks); returns (ms per step, mode name, clocks) of the
    fastest, with every mode's time in the name when there are several."""
    import torch
    best, seen = None, []
    for name, run in modes:
        for i in range(W):
            run[i % R]()
        torch.cuda.synchronize()
        barrier(world)
        clk = ClockSampler(local, world)
        time.sleep(0.3)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record()
        for i in range(K):
            run[steps[i]]()
        ev1.record()
        torch.cuda.synchronize()
        clocks = clk.stop()
        barrier(world)
        ms = dist_max(ev0.elapsed_time(ev1) / K, world)
        seen.append(f"{name.split(' (')[0]} {ms:.4f} ms")
        if best is None or ms < best[0]:
            best = (ms, name, clocks)
    if len(seen) > 1:
        best = (best[0], best[1] + " [timed: " + "; ".join(seen) + "]", best[2])
    return best


def run_prefill(args, rank, world, local):
    """one MoE layer at prefill, T = 4096 tokens per GPU (x bf16,
    top-8 of 384 + shared), the whole layer in one library call (router GEMM, grouped
    block-scaled GEMMs); at N > 1 the experts are sharded (all_gather dispatch and
    reduce_scatter combine, or with --exchange a2a the counted all-to-all)."""
    import torch
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic

    torch.cuda.set_device(local)
    T = args.tokens
    K, W = args.steps, args.warmup
    R = 4                                                   # distinct token batches (> L2 together)
    lay = synthetic.baseline_layer(seed=args.seed, E=args.experts, H=H, I=I_, top_k=TOPK, scale=SCALE)
    if world > 1:
        from kimi_k3_mlx_macmini_b200.ep import ExpertParallelMoE
        moe = ExpertParallelMoE(lay.cfg, 0, {"gate.weight": lay.gate, "gate.e_score_correction_bias": lay.bias},
                                lay.source, exchange=args.exchange)
        _NCCL_GRAPHS.append(moe)
    else:
        moe = lay.moe()
        _ = moe.pool
    xs = [synthetic.tokens(args.seed * 7919 + rank * 100003 + i, T, H) for i in range(R)]
    check = ep_check(moe, lay.moe(), xs[0], world) if world > 1 else None
    graphs, modes = step_modes(moe, xs, R, world)
    barrier(world)
    ms, timing, clocks = time_modes(modes, [(W + i) % R for i in range(K)], K, W, R, world, local)
    value = world * T / (ms / 1e3)

    # per-kernel device time (profiling events, outside the timed region; launched, not replayed)
    n_prof = min(K, 10)
    api_graphs = getattr(moe, "graphs", None)
    if api_graphs is not None:
        moe.graphs = False
    L.profile_enable(True)
    L.profile_collect()
    if world > 1:
        moe.collective_timing = True
        moe.collective_ms()
    for i in range(n_prof):
        moe(xs[i % R])
    torch.cuda.synchronize()
    prof = L.profile_collect()
    L.profile_enable(False)
    coll = None
    if world > 1:
        coll = {k: v / n_prof for k, v in moe.collective_ms().items()}
        moe.collective_timing = False
    if api_graphs is not None:
        moe.graphs = api_graphs
    gu_ms, gu_n = prof["gateup"]
    dn_ms, dn_n = prof["down"]
    gu_n, dn_n = max(gu_n, 1), max(dn_n, 1)
    peak_hbm, peak_kind = measured_peaks()
    E_loc = args.experts // world
    proj = 7168 * 2048 // 2 + 7168 * 2048 // 32                 # bytes of one MXFP4 projection
    w_bytes = (E_loc + 1) * 3 * proj                           # every local expert is hit at T=4096
    gu_bytes = (E_loc + 1) * 2 * proj
    flops = 2.0 * world * T * (TOPK + 1) * 3 * H * I_ / world  # this rank's share (weak scaling)
    gu_flops = flops * 2 / 3
    gu_launch = gu_ms / max(gu_n, 1)
    FP4_DENSE_NOMINAL = 9000.0                                  # TFLOP/s, B200 dense FP4 (datasheet)

    # ---- end to end through the public API with host buffers
    xh = torch.stack([x.cpu() for x in xs]).pin_memory()
    e2e_ms = e2e_loop(moe, xh, lambda i: i % R, min(K, 20), 2, (T, H), world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res = cpu_baseline(T, args.seed, 1, budget_s=20.0)
        cpu = {"value": res["tokens_per_s"], "unit": "tokens/s", "cores": res["cores"], "kind": "port",
               "build": f"gcc -O3 {res['isa']} clone, OpenMP", "sample": res["sample"]}
    for g in graphs:
        g.reset()
    graph_error = getattr(moe, "graph_error", None)
    if world > 1:
        release_nccl_graphs()                               # NCCL graphs go before the process group
    if rank != 0:
        return
    line = {
        "metric": "moe_layer_prefill_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1 weights x 4 e2m1 activation pieces, e8m0 block scales, f32 accumulate (tcgen05 kind::mxf4)",
        "data": "synthetic (seeded random-init weights of the BASELINE layer)",
        "config": {"workload": f"BASELINE configs[3]: one MoE layer prefill, T={T} tokens per GPU, "
                               f"{args.experts} routed + 1 shared MXFP4 expert (7168/2048), bf16 router, top-8, x2.5",
                   "tokens_per_gpu": T,
                   "parallelism": "single GPU" if world == 1 else
                                  f"ep{world}: {E_loc} routed experts per rank + replicated shared, "
                                  + ("counted all_to_all dispatch and combine (NCCL)" if moe.uses_a2a(T) else
                                     "all_gather dispatch, reduce_scatter combine (NCCL)"),
                   "l2": f"inputs larger than L2: {w_bytes / 1e9:.2f} GB of expert weights per GPU and "
                         f"{R} token batches of {T * H * 2 / 1e6:.0f} MB",
                   "timing": timing + ", events around K steps",
                   "api_graph_error": graph_error},
        "ep_check": check,
        "layer_hbm_gbs": w_bytes / (ms / 1e3) / 1e9,
        "layer_tflops_algorithmic": flops / (ms / 1e3) / 1e12,
        "roofline": {"bound": "tensor", "kernel": "prefill_gemm_kernel<gate/up> (block-scaled grouped GEMM, tcgen05)",
                     "achieved": gu_flops / (gu_launch / 1e3) / 1e12, "peak": FP4_DENSE_NOMINAL,
                     "unit": "TFLOP/s", "frac": gu_flops / (gu_launch / 1e3) / 1e12 / FP4_DENSE_NOMINAL,
                     "peak_kind": "nominal (dense FP4 datasheet; no measured FP4 peak on this pool)",
                     "algorithmic_flops_per_launch": gu_flops,
                     "tensor_instruction_flops_per_launch": 4 * gu_flops,
                     "hbm_view": {"algorithmic_bytes_per_launch": gu_bytes,
                                  "achieved_gbs": gu_bytes / (gu_launch / 1e3) / 1e9,
                                  "peak_gbs": peak_hbm, "peak_kind": peak_kind},
                     "traffic": None, "launch_ms": gu_launch},
        "down_kernel": {"launch_ms": dn_ms / max(dn_n, 1),
                        "achieved_tflops": flops / 3 / (dn_ms / max(dn_n, 1) / 1e3) / 1e12},
        "kernel_ms_per_step": {k: v[0] / n_prof for k, v in prof.items() if v[1]},
        "collective_ms_per_step": coll,
        "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 4,
                "ms_per_step": e2e_ms,
                "api": ("LatentMoE.__call__ (k3_moe_prefill)" if world == 1 else
                        "ExpertParallelMoE.__call__ (counted all-to-all step, launched per call)"
                        if moe.uses_a2a(T) else "ExpertParallelMoE.__call__ (captured step replayed per call)"),
                "copies": "one copy stream, two buffers each way: the next upload ahead of this download, both overlapping the neighbouring steps"},
        "gpu_launches": int(round(sum(c for _, c in prof.values()) / n_prof * K)),
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line))


def run_matvec(args, rank, world, local):
    """the full-width single-expert MXFP4 decode matvec (hidden 7168,
    intermediate 2048) at M tokens (--tokens, 1 or 8), pure HBM-bound dequant-matvec
    bandwidth on one GPU. A step is one expert's SwiGLU FFN through the reference's API
    ``LatentMoE.expert_forward`` (``moe.py:90-103``): gate and up projections (one
    block-scaled launch), silu(gate) * up, the down projection -- 23,396,352 B of MXFP4
    weights -- over a ring of --experts distinct experts (default 64: 1.5 GB, larger than
    L2), one CUDA graph per expert. Beside it, the bare ``mxfp4_matvec_fused`` call (``mxfp4_matvec.py:75-96``)
    on one 7168 -> 2048 projection (7,798,784 B) over a ring of the experts' 2 x --experts
    distinct projections."""
    import torch
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic
    from kimi_k3_mlx_macmini_b200.mxfp4 import mxfp4_matvec_fused

    if world > 1:
        if rank == 0:
            print(json.dumps({"metric": "mxfp4_matvec_hbm_gbs", "unavailable": "config 1 runs on one GPU"}))
        return
    torch.cuda.set_device(local)
    M, K, W = args.tokens, args.steps, args.warmup
    NE = args.experts
    if NE < 8:
        raise SystemExit("config 1 needs a ring of at least 8 experts (larger than L2 from 8 on)")
    lay = synthetic.baseline_layer(seed=args.seed, E=NE, H=H, I=I_, top_k=1, shared=False)
    moe = lay.moe()
    _ = moe.pool
    xs = [synthetic.tokens(args.seed * 7919 + i, M, H) for i in range(NE)]
    step_e = [(W + i) % NE for i in range(K)]
    # ---- expert FFN through expert_forward, a CUDA graph per expert
    cap = torch.cuda.Stream()
    with torch.cuda.stream(cap):
        for e in range(2):
            moe.expert_forward(xs[e], e)
    torch.cuda.synchronize()
    graphs = []
    for e in range(NE):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            moe.expert_forward(xs[e], e)
        graphs.append(g)
    ms, timing, clocks = time_modes([(f"CUDA graph per expert ({NE} distinct experts replayed as a ring)",
                                      [g.replay for g in graphs])], step_e, K, W, NE, 1, local)
    peak, peak_kind = measured_peaks()
    ffn_bytes = EXPERT_BYTES + M * H * 2
    gbs = ffn_bytes / (ms / 1e3) / 1e9
    # ---- per-kernel device time of the same steps
    n_prof = min(K, 64)
    L.profile_enable(True)
    L.profile_collect()
    torch.cuda.synchronize()
    torch.cuda._sleep(int(4e7))
    for i in range(n_prof):
        moe.expert_forward(xs[step_e[i]], step_e[i])
    torch.cuda.synchronize()
    prof = L.profile_collect()
    L.profile_enable(False)
    gu_ms, gu_n = prof["gateup"]
    gu_bytes = 2 * PROJ_BYTES + M * H * 2
    gu_gbs = gu_bytes / (gu_ms / gu_n / 1e3) / 1e9
    dn_ms, dn_n = prof["down"]
    # ---- the bare mxfp4_matvec_fused call over a ring of the experts' w1 and w3 projections
    projs = []
    for e in range(NE):
        for which in ("w1", "w3"):
            projs.append(moe.pool.get(e, which))
    NP = len(projs)
    xp = [synthetic.tokens(args.seed * 31 + i, M, H) for i in range(8)]
    outs = torch.empty((M, I_), dtype=torch.float32, device="cuda")
    pgraphs = []
    with torch.cuda.stream(cap):
        mxfp4_matvec_fused(xp[0], *projs[0])
    torch.cuda.synchronize()
    for j in range(NP):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            outs.copy_(mxfp4_matvec_fused(xp[j % 8], *projs[j]))
        pgraphs.append(g)
    K2 = max(K, 64)
    pms, ptiming, _ = time_modes([("CUDA graph per projection", [g.replay for g in pgraphs])],
                                 [(W + i) % NP for i in range(K2)], K2, W, NP, 1, local)
    L.profile_enable(True)
    L.profile_collect()
    torch.cuda.synchronize()
    torch.cuda._sleep(int(4e7))
    for i in range(min(K2, 64)):
        mxfp4_matvec_fused(xp[i % 8], *projs[(W + i) % NP])
    torch.cuda.synchronize()
    pprof = L.profile_collect()
    L.profile_enable(False)
    mv_ms, mv_n = pprof["matvec"]
    # ---- end to end through expert_forward with host buffers
    xh = torch.stack([x.cpu() for x in xs]).pin_memory()
    yh = torch.empty((M, H), dtype=torch.float32).pin_memory()
    xd = torch.empty((M, H), dtype=torch.bfloat16, device="cuda")
    for i in range(W):
        xd.copy_(xh[i % NE], non_blocking=True)
        yh.copy_(moe.expert_forward(xd, i % NE), non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        xd.copy_(xh[step_e[i]], non_blocking=True)
        yh.copy_(moe.expert_forward(xd, step_e[i]), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import mxfp4_oracle as O
        rng = np.random.default_rng(args.seed)
        (p1, s1), (p3, s3), (p2, s2) = (O.random_mxfp4(rng, I_, H), O.random_mxfp4(rng, I_, H),
                                        O.random_mxfp4(rng, H, I_))
        xf = rng.standard_normal((M, H)).astype(np.float32)
        cores = host_cores()
        n, t = 0, 0.0
        while t < 10.0 and n < 50:
            t0 = time.perf_counter()
            g_ = O.matvec_fused(xf, p1, s1, threads=cores)
            u_ = O.matvec_fused(xf, p3, s3, threads=cores)
            O.matvec_fused(O.silu(g_) * u_, p2, s2, threads=cores)
            t += time.perf_counter() - t0
            n += 1
        cpu = {"value": ffn_bytes / (t / n) / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
               "build": f"gcc -O3 {O.oracle_isa()} clone, OpenMP",
               "sample": f"{n} expert FFNs (M={M}) through the C port of the reference fused-kernel loop"}
    for g in graphs + pgraphs:
        g.reset()
    line = {
        "metric": "mxfp4_matvec_hbm_gbs", "value": gbs, "unit": "GB/s",
        "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1 weights x e2m1 activation pieces, e8m0 block scales, f32 accumulate (tcgen05 kind::mxf4)",
        "data": "synthetic (seeded random-init MXFP4 experts of the BASELINE shape)",
        "config": {"workload": f"BASELINE configs[1]: one expert's SwiGLU FFN (7168 -> 2048 -> 7168, MXFP4) "
                               f"at M={M} through LatentMoE.expert_forward",
                   "tokens": M,
                   "l2": f"inputs larger than L2: a ring of {NE} distinct experts ({NE * EXPERT_BYTES / 1e9:.2f} GB)",
                   "timing": timing + ", events around K steps"},
        "frac_of_peak": gbs / peak,
        "roofline": {"bound": "hbm", "kernel": "bs_gemv_kernel<gate/up> (block-scaled MXFP4 matvec, tcgen05)",
                     "achieved": gu_gbs, "peak": peak, "unit": "GB/s", "frac": gu_gbs / peak,
                     "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_launch": gu_bytes, "launch_ms": gu_ms / gu_n},
        "down_kernel": {"launch_ms": dn_ms / max(dn_n, 1),
                        "achieved": PROJ_BYTES / (dn_ms / max(dn_n, 1) / 1e3) / 1e9},
        "matvec_fused_projection": {
            "api": "mxfp4_matvec_fused (k3_mxfp4_matvec), 7168 -> 2048",
            "gbs": PROJ_BYTES / (pms / 1e3) / 1e9, "frac_of_peak": PROJ_BYTES / (pms / 1e3) / 1e9 / peak,
            "ms_per_call": pms, "kernel_launch_ms": mv_ms / max(mv_n, 1),
            "kernel_gbs": PROJ_BYTES / (mv_ms / max(mv_n, 1) / 1e3) / 1e9,
            "timing": ptiming + f", {K2} calls over a ring of {NP} distinct projections"},
        "kernel_ms_per_step": {k: v[0] / n_prof for k, v in prof.items() if v[1]},
        "e2e": {"value": ffn_bytes / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": M * H * 2, "d2h_bytes_per_step": M * H * 4,
                "ms_per_step": e2e_ms, "api": "LatentMoE.expert_forward (k3_moe_experts_decode)"},
        "gpu_launches": int(round(sum(c for _, c in prof.values()) / n_prof * K)),
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line))


def reference_matvec(args):
    """--impl reference for configs[1]: one expert FFN per step through the C port of the
    reference's fused-kernel loop on every host core."""
    from oracle import mxfp4_oracle as O
    M = args.tokens
    rng = np.random.default_rng(args.seed)
    (p1, s1), (p3, s3), (p2, s2) = (O.random_mxfp4(rng, I_, H), O.random_mxfp4(rng, I_, H),
                                    O.random_mxfp4(rng, H, I_))
    xf = rng.standard_normal((M, H)).astype(np.float32)
    cores = host_cores()

    def step():
        g_ = O.matvec_fused(xf, p1, s1, threads=cores)
        u_ = O.matvec_fused(xf, p3, s3, threads=cores)
        O.matvec_fused(O.silu(g_) * u_, p2, s2, threads=cores)

    for _ in range(max(1, min(args.warmup, 3))):
        step()
    n, t = 0, 0.0
    while n < max(1, args.steps) and t < 60.0:
        t0 = time.perf_counter()
        step()
        t += time.perf_counter() - t0
        n += 1
    v = (EXPERT_BYTES + M * H * 2) / (t / n) / 1e9
    return {"impl": "reference", "metric": "mxfp4_matvec_hbm_gbs", "value": v, "unit": "GB/s", "n_gpus": 1,
            "steps": n, "warmup": max(1, min(args.warmup, 3)), "ms_per_step": 1e3 * t / n,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"BASELINE configs[1]: one expert's SwiGLU FFN (7168 -> 2048 -> 7168, MXFP4) "
                                   f"at M={M}", "tokens": M},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": cores, "kind": "port",
                             "build": f"gcc -O3 {O.oracle_isa()} clone, OpenMP",
                             "sample": f"{n} whole expert FFNs"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_k3(args, rank, world, local):
    """A Kimi-K3 MoE layer at decode (``air_llm/models/kimi_k3/moe.py:1-12,110-131``): 896
    routed MXFP4 experts, top-16, in a 3584-wide latent space (experts 3584 -> 3072 ->
    3584) between bf16 latent projections, plus a bf16 shared expert [2 x 3072, 7168];
    situ activation. One GPU; synthetic seeded weights. Supplementary to the BASELINE
    configs (the reference's own model shapes)."""
    import torch
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic

    if world > 1:
        if rank == 0:
            print(json.dumps({"metric": "k3_layer_decode_tokens_per_s", "unavailable": "config 5 runs on one GPU"}))
        return
    torch.cuda.set_device(local)
    M = args.tokens
    K, W = args.steps, args.warmup
    R = min(K + W, 32)
    Hk, Lk, Ik, Ek = 7168, 3584, 3072, args.experts
    lay = synthetic.k3_layer(seed=args.seed, E=Ek)
    moe = lay.moe()
    xs = [synthetic.tokens(args.seed * 7919 + i, M, Hk) for i in range(R)]
    U = [int(torch.unique(moe.route(x).expert_indices).numel()) for x in xs]
    step_x = [(W + i) % R for i in range(K)]
    graphs, modes = step_modes(moe, xs, R, world)
    ms, timing, clocks = time_modes(modes, step_x, K, W, R, world, local)

    n_prof = min(K, 50)
    L.profile_enable(True)
    L.profile_collect()
    torch.cuda.synchronize()
    torch.cuda._sleep(int(4e7))
    for i in range(n_prof):
        moe(xs[step_x[i]])
    torch.cuda.synchronize()
    prof = L.profile_collect()
    L.profile_enable(False)
    proj = Ik * Lk // 2 + Ik * Lk // 32
    dense_bytes = 2 * (Lk * Hk + Hk * Lk + 2 * Ik * Hk + Hk * Ik)       # latent down/up, shared gate/up/down
    router_bytes = Ek * Hk * 2
    u_mean = float(np.mean([U[step_x[i]] for i in range(n_prof)]))
    layer_bytes = u_mean * 3 * proj + dense_bytes + router_bytes
    peak, peak_kind = measured_peaks()
    d_ms, d_n = prof["dense"]
    d_gbs = dense_bytes / (d_ms / n_prof / 1e3) / 1e9           # the step's two dense matvecs together
    for g in graphs:
        g.reset()
    line = {
        "metric": "k3_layer_decode_tokens_per_s", "value": M / (ms / 1e3), "unit": "tokens/s",
        "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "MXFP4 experts (e2m1 x e2m1 pieces, tcgen05 kind::mxf4); bf16 dense weights x fp32 (f32x2 FMA)",
        "data": "synthetic (seeded random-init weights of the Kimi-K3 layer shapes)",
        "config": {"workload": f"Kimi-K3 MoE layer decode, M={M}: {Ek} routed MXFP4 experts top-16 (latent 3584, "
                               "intermediate 3072), bf16 latent projections 7168<->3584, bf16 shared expert "
                               "2x3072x7168, situ, x2.5",
                   "tokens_per_gpu": M, "parallelism": "single GPU",
                   "l2": f"inputs larger than L2: {Ek * 3 * proj / 1e9:.1f} GB expert pool + "
                         f"{dense_bytes / 1e6:.0f} MB dense weights per step, a different token batch every step",
                   "timing": timing + ", events around K steps"},
        "unique_experts_mean": u_mean,
        "layer_hbm_gbs": layer_bytes / (ms / 1e3) / 1e9,
        "roofline": {"bound": "hbm", "kernel": "dense_matvec_kernel (front: latent down + shared gate/up; "
                                                "back: rmsnorm.up + shared down on act(gate, up); "
                                                "prep kernels included)",
                     "achieved": d_gbs, "peak": peak, "unit": "GB/s", "frac": d_gbs / peak,
                     "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_step": dense_bytes, "ms_per_step": d_ms / n_prof},
        "kernel_ms_per_step": {k: v[0] / n_prof for k, v in prof.items() if v[1]},
        # profiled spans per step; a dense span is two kernels (input prep + matvec)
        "gpu_launches": int(round((sum(c for _, c in prof.values()) + d_n) / n_prof * K)),
        "clocks": clocks,
    }
    print(json.dumps(line))


def main():
    args = parse()
    rank, world, local = dist_init(args)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.config == 5:
            run_k3(args, rank, world, local)
        elif args.config == 4:
            run_stream(args, rank, world, local)
        elif args.config == 3:
            run_prefill(args, rank, world, local)
        elif args.config == 1:
            run_matvec(args, rank, world, local)
        else:
            run_b200(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            release_nccl_graphs()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
