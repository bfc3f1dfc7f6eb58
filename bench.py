"""Benchmark of the MoE hot path on B200: the expert-parallel Mixtral-shaped MoE layer (BASELINE
configs[3]) as the headline, the grouped GEMM (configs[0..2]) and the DeepSeek-V3-shaped layer
(configs[4]) beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--no-sweep] [--no-cpu-baseline] [--no-dsv3] [--profile X]

One JSON line on rank 0. A "step" is one MoE layer forward over T=16384 tokens in total
(H=4096, F=14336, E=8, top-2, bf16): route -> dispatch -> gate/up GEMM with SwiGLU -> down GEMM
-> combine. At N>1 (torchrun, one rank per GPU) the tokens are split over the ranks and the
experts are sharded (expert parallelism over NVLink peer memory): the total work is fixed, so
scaling is strong, and `value` is the whole job's tokens/s from the max-over-ranks device time.
The global problem (tokens, router logits, every expert's weights) is generated from seeds that
do not depend on N, so every N computes the same layer; `ep_parity` checks a seeded sample of
its output tokens against the CPU oracle at every N.

Extra keys: `roofline` (the gate/up SwiGLU grouped-GEMM kernel, the layer's dominant kernel,
against the measured bf16 peak), `stages` (per-stage device ms), `e2e` (fused_moe_host with
pinned host tokens and result), `cpu_baseline` (the reference's per-expert F.linear loop running
the whole layer on the host cores), `clocks` for every leg, `grouped_gemm` (cfg2 TFLOP/s, its
roofline and the dense-cuBLAS efficiency, N=1), `dsv3` and `configs`
(the other grouped-GEMM configs, the token sweep and the launch-overhead comparison, N=1).
`--impl reference` times the reference's own algorithm for the same layer on the CPU.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "groupedgemm-opt_b200"))

# Mixtral-shaped MoE layer
MIX_T, MIX_H, MIX_F, MIX_E, MIX_K = 16384, 4096, 14336, 8, 2
MIX_FLOP = 6.0 * MIX_T * MIX_K * MIX_H * MIX_F
METRIC = "moe_layer_tokens_per_s"
UNIT = "tokens/s"
WORKLOAD = "Mixtral MoE layer T16384 H4096 F14336 E8 top2 bf16 (BASELINE configs[3])"
# the grouped GEMM, README shape
T_TOK, E, K, N = 4096, 8, 4096, 14336
GEMM_FLOP = 2.0 * T_TOK * N * K
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}
SEED_TOKENS, SEED_EXPERTS, SEED_SAMPLE = 11, 1000, 21
DSV3_SEED_TOKENS, DSV3_SEED_EXPERTS = 31, 5000


def layer_config(n):
    """The config dict both arms print (identical, so the two lines compare like for like)."""
    return {"workload": WORKLOAD, "model": "mixtral-8x7b-moe-layer", "global_batch": MIX_T,
            "hidden": MIX_H, "ffn": MIX_F, "experts": MIX_E, "top_k": MIX_K,
            "parallelism": f"ep{n}",
            "l2": "inputs larger than L2 (expert weights 2.8 GB / N per GPU), no flush"}


def _peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return FALLBACK_PEAKS, "fallback"


def _peak(key):
    p, src = _peaks()
    return float(p.get(key, FALLBACK_PEAKS[key])), src


def _traffic(kernel_key: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.txt), or None."""
    try:
        with open(os.path.join(HERE, "profiles", "traffic.txt")) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == kernel_key:
                    return float(parts[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        self.file.seek(0)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.file.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist_init():
    """One process per GPU. The first barrier runs right here, so NCCL's communicator is up
    before any warm loop and never idles the GPU in front of a timed region."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        dist.barrier()
    else:
        torch.cuda.set_device(0)
    torch.cuda.synchronize()
    return world, rank, local


def _barrier_sync(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(x, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _gather_floats(vals, world):
    """All ranks' float vectors (same length) -> list per rank."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    if world == 1:
        return [t.tolist()]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def _timed(fn, steps, world, finish=None):
    """Device time of `steps` calls: events on the launching (current) stream, barrier + sync on
    both sides, max over ranks. `finish` (optional) runs after the last call, before the closing
    event, to order work of other streams before it. Returns (total_ms, per-step event times)."""
    import torch
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    _barrier_sync(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(steps):
        starts[i].record()
        fn()
        ends[i].record()
    if finish is not None:
        finish()
    t1.record()
    _barrier_sync(world)
    total = _max_over_ranks(t0.elapsed_time(t1), world)
    return total, [s.elapsed_time(e) for s, e in zip(starts, ends)]


def _warm(fn, world, seconds=1.0):
    """Untimed back-to-back calls for at least `seconds`, so the clocks have settled under load
    and the clock sampler covers the load. Every rank makes the same number of calls: they stop
    together once all of them have run long enough."""
    import torch
    t_end = time.time() + seconds
    n = 0
    while True:
        for _ in range(4):
            fn()
        n += 4
        torch.cuda.synchronize()
        if _min_over_ranks(1.0 if time.time() >= t_end else 0.0, world) >= 1.0:
            return n


def _min_over_ranks(x, world):
    return -_max_over_ranks(-x, world)


def measure(fn, steps, world, local, warm_s=1.0, finish=None):
    """Warm loop >= warm_s under a clock sampler, then `steps` timed calls (`finish` as in
    _timed). Returns (ms per call, per-call event times, clocks)."""
    with ClockSampler(local) as clk:
        _warm(fn, world, warm_s)
        if finish is not None:
            finish()
        total, per = _timed(fn, steps, world, finish)
    return total / steps, per, clk.summary()


def measure_burst(fn, steps, local, idle_s=1.0, reps=3):
    """A kernel timed alone, as the burst peak (`bf16_tflops` of MEASURED_PEAKS.json) was: after
    an idle gap that lets the GPU fall back under its power cap, `steps` back-to-back calls
    (CUDA events on the launching stream); the median over `reps` gaps. Returns (ms per call,
    clocks) -- the clock samples include the idle gaps."""
    import torch
    per = []
    with ClockSampler(local) as clk:
        for _ in range(reps):
            torch.cuda.synchronize()
            time.sleep(idle_s)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(steps):
                fn()
            t1.record()
            torch.cuda.synchronize()
            per.append(t0.elapsed_time(t1) / steps)
    return statistics.median(per), clk.summary()


# ----------------------------------------------------------------------------- problems
def _tokens(T, H, Ex, seed, rank, world):
    """Global tokens and router logits from one seed (independent of N); this rank's slice."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    logits = torch.randn(T, Ex, device="cuda", generator=g)
    tl = T // world
    return x, logits, x[rank * tl:(rank + 1) * tl].contiguous(), \
        logits[rank * tl:(rank + 1) * tl].contiguous()


def _expert_weights(e, H, F, seed_base, device="cuda"):
    """Expert e's (w_gate_up [2F, H], w_down [H, F]) bf16 ~ N(0, 0.02), seeded by its index."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed_base + e)
    wgu = (torch.randn(2 * F, H, device=device, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(H, F, device=device, generator=g) * 0.02).to(torch.bfloat16)
    return wgu, wd


def _local_weights(H, F, Ex, seed_base, rank, world):
    import torch
    el = Ex // world
    wgu = torch.empty(el, 2 * F, H, dtype=torch.bfloat16, device="cuda")
    wd = torch.empty(el, H, F, dtype=torch.bfloat16, device="cuda")
    for i in range(el):
        a, b = _expert_weights(rank * el + i, H, F, seed_base)
        wgu[i].copy_(a)
        wd[i].copy_(b)
        del a, b
    return wgu, wd


def _rows_per_rank(logits_g, k, world):
    """Routed rows each rank's experts receive (global routing; ties do not occur for N(0,1))."""
    import torch
    Ex = logits_g.size(1)
    ids = logits_g.topk(k, dim=1).indices.reshape(-1)
    tpe = torch.bincount(ids, minlength=Ex)
    return tpe.view(world, Ex // world).sum(1).tolist()


def ep_parity(outs, x_g, logits_g, rank, world, H, F, k, seed_base, n_sample):
    """Seeded sample of global tokens: every rank contributes its rows of each output in `outs`
    (name -> [T/N, H] on this rank), rank 0 compares them with the CPU oracle (all experts,
    global routing). Returns {name: {max_rel, cos, tokens, ok}} on rank 0, None elsewhere."""
    import torch
    import torch.distributed as dist
    T = x_g.size(0)
    tl = T // world
    g = torch.Generator().manual_seed(SEED_SAMPLE)
    idx = torch.randperm(T, generator=g)[:n_sample].sort().values
    mine = (idx >= rank * tl) & (idx < (rank + 1) * tl)
    loc = (idx[mine] - rank * tl).cuda()
    got = {}
    for name, out in outs.items():
        buf = torch.zeros(n_sample, H, dtype=torch.float32, device="cuda")
        buf[mine.cuda()] = out[loc].float()
        if world > 1:
            dist.all_reduce(buf)
        got[name] = buf.cpu()
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import grouped_gemm_oracle as oracle

    def weights(e):
        a, b = _expert_weights(e, H, F, seed_base)
        return a.cpu(), b.cpu()

    ref = oracle.moe_tokens(x_g[idx.cuda()].cpu(), logits_g[idx.cuda()].cpu(), weights, k,
                            round_to=torch.bfloat16)
    res = {}
    for name, o in got.items():
        rel = ((o - ref).abs().max() / ref.abs().max().clamp_min(1e-12)).item()
        cos = torch.nn.functional.cosine_similarity(o.flatten().double(),
                                                    ref.flatten().double(), dim=0).item()
        res[name] = {"max_rel": rel, "cos": cos, "tokens": n_sample,
                     "ok": bool(rel <= 1e-2 and cos >= 0.9999 and torch.isfinite(o).all())}
    return res


# ----------------------------------------------------------------------------- headline
def mixtral_layer_leg(world, rank, local, steps, warmup):
    """the layer on N GPUs (N=1: one GPU, no collectives; N>1: expert
    parallelism on the fused peer-memory path, the NCCL all-to-all path timed beside it)."""
    import torch
    import torch.distributed as dist
    from grouped_gemm_opt import (EPBuffers, MoEHostPipeline, StageEvents, _C, fused_moe,
                                  fused_moe_host)
    T, H, F, Ex, k = MIX_T, MIX_H, MIX_F, MIX_E, MIX_K
    tl = T // world
    x_g, l_g, x, logits = _tokens(T, H, Ex, SEED_TOKENS, rank, world)
    wgu, wd = _local_weights(H, F, Ex, SEED_EXPERTS, rank, world)
    rows = _rows_per_rank(l_g, k, world)
    grp = dist.group.WORLD if world > 1 else None
    bufs = EPBuffers(grp, tl, H, k, Ex, torch.bfloat16) if world > 1 else None
    res = {}

    def layer(b=bufs, timer=None):
        return fused_moe(x, logits, wgu, wd, k, ep_group=grp, ep_buffers=b, timer=timer)

    for _ in range(warmup):
        layer()
    # headline: warm loop under the clock sampler, then exactly `steps` timed layers with a
    # CUDA event after every stage (gate/up kernel duration measured live)
    timer = StageEvents()
    with ClockSampler(local) as clk:
        _warm(layer, world, 1.0)
        l0 = _C.kernel_launches()
        out_holder = {}

        def step():
            out_holder["y"] = layer(timer=timer)

        total_ms, _ = _timed(step, steps, world)
        launches = _C.kernel_launches() - l0
    clocks = clk.summary()
    ms = total_ms / steps
    stages = timer.ms()
    names = sorted(stages)
    per_rank = _gather_floats([stages[n] / steps for n in names], world)
    outs = {"p2p" if world > 1 else "single": out_holder["y"]}
    if bufs is not None:
        bufs.check()  # raises if a peer wait expired anywhere in the timed region

    # roofline of the dominant kernel: the gate/up SwiGLU grouped GEMM on each rank's rows
    peak, src = _peak("bf16_tflops_sustained")
    burst, _ = _peak("bf16_tflops")
    gu_idx = names.index("gate_up")
    ach = [2.0 * rows[r] * 2 * F * H / (per_rank[r][gu_idx] / 1e3) / 1e12 for r in range(world)]
    achieved = statistics.mean(ach)
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "frac_of_burst_peak": achieved / burst,
                "peak_source": f"bf16_tflops_sustained (of {src}); the layer's steps run "
                               "back to back at the power cap",
                "kernel": "grouped_gemm_pair_kernel SwiGLU (gate/up; + its short-tail pass), "
                          "device time per layer from CUDA events around the launch",
                "algorithmic_flop_per_launch": [2.0 * r * 2 * F * H for r in rows],
                "achieved_per_rank": ach}
    t1 = _traffic("moe_gate_up_ep1")
    roofline["traffic"] = None if t1 is None else t1 / world
    roofline["traffic_source"] = (
        "ncu DRAM read+write of the gate/up launch at N=1 (profiles/traffic.txt)" if world == 1
        else f"the N=1 capture / {world}: a rank's launch processes 1/N of the rows and holds "
             "1/N of the experts (not captured at this N)")
    # the whole layer's roofline: FLOPs at the sustained peak vs bytes over NVLink
    t_flop = MIX_FLOP / world / (peak * 1e12) * 1e3
    nvl_bytes = 2.0 * tl * k * H * 2 * (world - 1) / world
    t_nvl = nvl_bytes / 770e9 * 1e3
    layer_roof = {"bound": "tensor" if t_flop >= t_nvl else "nvlink",
                  "target_ms": max(t_flop, t_nvl), "achieved_ms": ms,
                  "frac": max(t_flop, t_nvl) / ms,
                  "nvlink_bytes_per_gpu_per_direction": nvl_bytes}
    stage_tbl = {n: {"max_ms": max(pr[i] for pr in per_rank),
                     "min_ms": min(pr[i] for pr in per_rank)} for i, n in enumerate(names)}
    res.update(value=T / (ms / 1e3), ms=ms, clocks=clocks, launches=launches,
               roofline=roofline, layer_roofline=layer_roof, stages=stage_tbl,
               rows_per_rank=rows, tflops=MIX_FLOP / (ms / 1e3) / 1e12)

    if world > 1:  # NCCL all-to-all path, same layer
        ms_n, _, clk_n = measure(lambda: layer(None), steps, world, local)
        outs["nccl"] = layer(None)
        res["nccl"] = {"value": T / (ms_n / 1e3), "ms": ms_n, "clocks": clk_n}

    # end to end through the public host-buffer API: this rank's tokens and logits from pinned
    # host memory, the result back into pinned host memory, every step
    x_h = x.cpu().pin_memory()
    l_h = logits.cpu().pin_memory()
    o_h = torch.empty(tl, H, dtype=torch.bfloat16).pin_memory()
    # (a) the streaming API: every step submits one batch (copy in, layer, copy out); batch
    # i+1's copy in and batch i's copy out overlap the layers; the timed region ends once the
    # last result is in host memory (the device-wide synchronize of _timed)
    pipe = MoEHostPipeline(wgu, wd, k, ep_group=grp, ep_buffers=bufs)
    ms_e, _, clk_e = measure(lambda: pipe.submit(x_h, l_h, o_h), steps, world, local,
                             finish=lambda: torch.cuda.current_stream().wait_stream(pipe.s_out))
    pipe.synchronize()
    outs["e2e_host"] = o_h.cuda()
    # (b) one isolated call's latency path: fused_moe_host, token chunks overlapped on copy
    # streams inside the call, joined back before the next call
    single_fn = lambda: fused_moe_host(x_h, l_h, wgu, wd, k, out=o_h, chunks=4,  # noqa: E731
                                       ep_group=grp, ep_buffers=bufs)
    ms_s, _, clk_s = measure(single_fn, steps, world, local)
    torch.cuda.synchronize()
    outs["e2e_single_call"] = o_h.cuda()
    res["e2e"] = {"value": T / (ms_e / 1e3), "unit": UNIT,
                  "h2d_bytes_per_step": T * H * 2 + T * Ex * 4,
                  "d2h_bytes_per_step": T * H * 2,
                  "api": "MoEHostPipeline.submit per step (pinned host tokens/logits/result; "
                         "copies of one step overlap the layer of the next); bytes summed over "
                         "all ranks",
                  "ms": ms_e, "clocks": clk_e,
                  "single_call": {"value": T / (ms_s / 1e3), "ms": ms_s, "clocks": clk_s,
                                  "api": "fused_moe_host, 4 token chunks, joined per call"}}
    if bufs is not None:
        bufs.check()
    res["ep_parity"] = ep_parity(outs, x_g, l_g, rank, world, H, F, k, SEED_EXPERTS, 32)
    if bufs is not None:
        bufs.close()
    return res


def dsv3_leg(world, rank, local, steps, warmup):
    """DeepSeek-V3-shaped layer (H=7168, F=2048, E=256, top-8) at T=32768
    and the decode-like T=256 (tokens in total). N>1: fused expert-parallel path."""
    import torch
    import torch.distributed as dist
    from grouped_gemm_opt import EPBuffers, StageEvents, fused_moe
    H, F, Ex, k = 7168, 2048, 256, 8
    el = Ex // world
    wgu, wd = _local_weights(H, F, Ex, DSV3_SEED_EXPERTS, rank, world)
    grp = dist.group.WORLD if world > 1 else None
    hbm, _ = _peak("hbm_gbs")
    out = {"workload": "DSv3 MoE layer H7168 F2048 E256 top8 bf16 (BASELINE configs[4])",
           "parallelism": f"ep{world}", "path": "fused peer-memory EP" if world > 1 else
           "one GPU"}
    for T in (32768, 256):
        tl = T // world
        x_g, l_g, x, logits = _tokens(T, H, Ex, DSV3_SEED_TOKENS + T, rank, world)
        bufs = EPBuffers(grp, tl, H, k, Ex, torch.bfloat16) if world > 1 else None
        holder = {}
        timer = {"t": None}

        def fn():
            holder["y"] = fused_moe(x, logits, wgu, wd, k, ep_group=grp, ep_buffers=bufs,
                                    timer=timer["t"])

        for _ in range(warmup):
            fn()
        with ClockSampler(local) as clk_s:
            _warm(fn, world, 1.0)
            timer["t"] = StageEvents()
            total_ms, _ = _timed(fn, steps, world)
        clk = clk_s.summary()
        ms = total_ms / steps
        st = timer["t"].ms()
        names = sorted(st)
        per_rank = _gather_floats([st[n] / steps for n in names], world)
        stages = {n: {"max_ms": max(pr[i] for pr in per_rank),
                      "min_ms": min(pr[i] for pr in per_rank)} for i, n in enumerate(names)}
        if bufs is not None:
            bufs.check()
        wbytes = 3.0 * el * F * H * 2
        par = ep_parity({"layer": holder["y"]}, x_g, l_g, rank, world, H, F, k,
                        DSV3_SEED_EXPERTS, 4)
        if bufs is not None:
            bufs.close()
        out[f"T{T}"] = {"tokens_per_s": T / (ms / 1e3), "ms_per_step": ms,
                        "tflops": 6.0 * T * k * H * F / (ms / 1e3) / 1e12,
                        "weight_gbs_per_gpu": wbytes / (ms / 1e3) / 1e9,
                        "weight_hbm_frac": wbytes / (ms / 1e3) / 1e9 / hbm,
                        "stages_ms_per_layer": stages, "clocks": clk, "ep_parity": par}
        del x_g, l_g, x, logits, holder
        torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- grouped GEMM
def grouped_gemm_leg(local, steps, warmup):
    """BASELINE configs[1] (cfg2 uniform): TFLOP/s of the grouped GEMM, its roofline, the dense
    cuBLAS GEMM of equal FLOPs (the reference's headline comparison, README.md:4-5,
    benchmark.py:86-88, 338-347) and the host-buffer API end to end."""
    import torch
    import grouped_gemm_opt as ggo
    tpe_h = torch.full((E,), T_TOK // E, dtype=torch.int64)
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(T_TOK, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    tpe = tpe_h.cuda()
    fn = lambda: ggo.grouped_gemm_opt(x, w, tpe)  # noqa: E731
    for _ in range(warmup):
        fn()
    st = max(steps, 200)
    ms, per, clk = measure(fn, st, 1, local)
    ggo.check_device_errors(local)
    kern_ms = statistics.mean(per)
    peak, src = _peak("bf16_tflops_sustained")
    burst, _ = _peak("bf16_tflops")
    achieved = GEMM_FLOP / (kern_ms / 1e3) / 1e12
    wd = w[0].contiguous()
    dense = lambda: torch.nn.functional.linear(x, wd)  # noqa: E731
    for _ in range(warmup):
        dense()
    dms, _, dclk = measure(dense, st, 1, local)
    x_h = x.cpu().pin_memory()
    tpe_hp = tpe_h.pin_memory()
    y_h = torch.empty(T_TOK, N, dtype=torch.bfloat16).pin_memory()
    e2e_fn = lambda: ggo.grouped_gemm_opt_host(x_h, w, tpe_hp, out=y_h, chunks=8)  # noqa: E731
    ems, _, eclk = measure(e2e_fn, max(20, steps), 1, local)
    # the kernel timed alone (bursts of 5 calls after idle gaps) against the burst peak, for
    # uniform and skewed routing (north_star's two cfg2 cases), beside dense cuBLAS timed the same
    # way; the sustained figures above are what a long run holds under the 1 kW cap
    bursts = {}
    for name, counts in (("uniform", tpe), ("skewed", _skewed_counts(T_TOK, E).cuda())):
        f = lambda c=counts: ggo.grouped_gemm_opt(x, w, c)  # noqa: E731
        bms, bclk = measure_burst(f, 5, local)
        bursts[name] = {"ms": bms, "tflops": GEMM_FLOP / bms / 1e9,
                        "frac_of_burst_peak": GEMM_FLOP / bms / 1e9 / burst, "clocks": bclk}
    dbms, _ = measure_burst(dense, 5, local)
    bursts["dense_cublas"] = {"ms": dbms, "tflops": GEMM_FLOP / dbms / 1e9}
    bursts["vs_dense"] = dbms / bursts["uniform"]["ms"]
    bursts["what"] = ("5 calls back to back after a 1 s idle gap, median of 3 gaps; against "
                      "bf16_tflops (the burst peak)")
    return {"workload": "cfg2 grouped GEMM E8 T4096 K4096 N14336 bf16, uniform (configs[1])",
            "burst": bursts,
            "value": GEMM_FLOP / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms": ms, "steps": st,
            "clocks": clk,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak,
                         "frac_of_burst_peak": achieved / burst,
                         "peak_source": f"bf16_tflops_sustained (of {src})",
                         "kernel": "grouped_gemm_pair_kernel (+ its short-tail pass)",
                         "traffic": _traffic("grouped_gemm_cfg2")},
            "vs_dense_gemm": {"dense_cublas_tflops": GEMM_FLOP / dms / 1e9, "dense_ms": dms,
                              "efficiency": dms / ms, "dense_clocks": dclk,
                              "what": "F.linear [4096,4096]x[14336,4096]^T (cuBLAS), same "
                                      "FLOPs as one grouped GEMM"},
            "e2e": {"value": GEMM_FLOP / (ems / 1e3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": T_TOK * K * 2 + E * 8,
                    "d2h_bytes_per_step": T_TOK * N * 2, "clocks": eclk,
                    "api": "grouped_gemm_opt_host (8 expert chunks overlapped)"}}


def _skewed_counts(total, experts, skew=3.0):
    """Power-law routing of the reference's benchmark (benchmark.py:59-69)."""
    import torch
    w = torch.pow(torch.arange(1, experts + 1, dtype=torch.float64), -skew)
    w /= w.sum()
    t = (w * total).long()
    t[0] += total - int(t.sum())
    return t


def _zipf_counts(total, experts, alpha=1.2, seed=0):
    import torch
    g = torch.Generator().manual_seed(seed)
    p = 1.0 / torch.arange(1, experts + 1, dtype=torch.float64) ** alpha
    draws = torch.multinomial(p / p.sum(), total, replacement=True, generator=g)
    return torch.bincount(draws, minlength=experts).to(torch.int64)


def _dirichlet_counts(total, experts, alpha=0.5, seed=0):
    import numpy as np
    import torch
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.multinomial(total, rng.dirichlet(np.full(experts, alpha))))


def launch_overhead(local, repeat=100, warmup=20):
    """The reference's launch-overhead harness (benchmarks/benchmark_launch_overhead.py:48-104,
    configs :119-129, plus cfg1): host wall time of the call vs CUDA-event time, with the counts
    on the GPU (nothing here synchronises) and on the CPU (the reference's .cpu() path). A small
    fill kernel is queued before every call, as the reference does. Medians of `repeat`."""
    import torch
    import grouped_gemm_opt as ggo
    cfgs = [(256, 8, 512, 1024), (4096, 8, 4096, 14336), (4096, 64, 4096, 14336),
            (8192, 8, 4096, 14336), (8192, 64, 4096, 14336), (1024, 8, 2048, 1280),
            (1024, 64, 2048, 1280), (16384, 8, 4096, 14336), (16384, 64, 4096, 14336)]
    out = []
    fill = torch.empty(1024, device="cuda")
    for t, ex, k, n in cfgs:
        g = torch.Generator(device="cuda").manual_seed(3)
        x = torch.randn(t, k, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(ex, n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        tpe = _dirichlet_counts(t, ex, 1.0, seed=3).to(torch.int64)
        row = {"tokens": t, "experts": ex, "K": k, "N": n}
        for label, counts in (("gpu_counts", tpe.cuda()), ("cpu_counts", tpe)):
            for _ in range(warmup):
                ggo.grouped_gemm_opt(x, w, counts, sort_by_m=False)
            torch.cuda.synchronize()
            st = [torch.cuda.Event(enable_timing=True) for _ in range(repeat)]
            en = [torch.cuda.Event(enable_timing=True) for _ in range(repeat)]
            host = []
            for i in range(repeat):
                fill.fill_(1.0)
                st[i].record()
                t0 = time.perf_counter()
                ggo.grouped_gemm_opt(x, w, counts, sort_by_m=False)
                t1 = time.perf_counter()
                en[i].record()
                host.append((t1 - t0) * 1e3)
            torch.cuda.synchronize()
            cuda = sorted(a.elapsed_time(b) for a, b in zip(st, en))
            hm = statistics.median(host)
            cm = cuda[repeat // 2]
            row[label] = {"host_ms": hm, "cuda_ms": cm, "overhead_ms": hm - cm}
        out.append(row)
        del x, w
        torch.cuda.empty_cache()
    return out


def config_sweep(local, steps, warmup=3):
    """Secondary numbers at N=1: the other grouped-GEMM configs (TFLOP/s and, for the
    weight-bound ones, HBM GB/s of algorithmic bytes), the reference's token sweep
    (benchmark.py:523-535) with its "vs Dense" efficiency, backward, FP8 and MXFP8 kernels and
    layers, and the launch-overhead comparison. Every case: >= 1 s warm loop, clocks recorded."""
    import torch
    import grouped_gemm_opt as ggo
    from grouped_gemm_opt import _C
    res = {}
    hbm, _ = _peak("hbm_gbs")
    st = max(steps, 20)
    cases = [
        ("cfg1", 8, 256, 512, 1024, torch.tensor([32] * 8)),
        ("cfg2_readme", 8, 4096, 4096, 14336, torch.tensor([512, 480, 520, 500, 510, 490, 530, 554])),
        ("cfg2_skewed", 8, 4096, 4096, 14336, _skewed_counts(4096, 8)),
        ("cfg3_zipf", 64, 8192, 4096, 14336, _zipf_counts(8192, 64)),
        ("cfg3_dirichlet", 64, 8192, 4096, 14336, _dirichlet_counts(8192, 64)),
        ("single_expert_8192cubed", 1, 8192, 8192, 8192, torch.tensor([8192])),
    ]
    for name, ex, t, k, n, tpe in cases:
        g = torch.Generator(device="cuda").manual_seed(7)
        x = torch.randn(t, k, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(ex, n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        td = tpe.to(torch.int64).cuda()
        fn = lambda: ggo.grouped_gemm_opt(x, w, td)  # noqa: E731
        for _ in range(warmup):
            fn()
        ms, _, clk = measure(fn, st * (10 if name == "cfg1" else 1), 1, local)
        flop = 2.0 * t * n * k
        nz = int((tpe > 0).sum())
        byts = t * k * 2 + nz * n * k * 2 + t * n * 2
        res[name] = {"ms": ms, "tflops": flop / ms / 1e9, "hbm_gbs": byts / ms / 1e6,
                     "hbm_frac": byts / ms / 1e6 / hbm, "nonzero_experts": nz,
                     "tokens_per_expert_max": int(tpe.max()), "clocks": clk}
        del x, w
        torch.cuda.empty_cache()

    # the reference's token sweep: E=8, K=4096, N=14336, uniform, T=1024..16384, vs one dense
    # cuBLAS GEMM of the same FLOPs ([T,K] x [K,N])
    sweep = []
    g = torch.Generator(device="cuda").manual_seed(8)
    w = (torch.randn(8, 14336, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w0 = w[0].contiguous()
    for t in (1024, 2048, 4096, 8192, 16384):
        x = torch.randn(t, 4096, device="cuda", generator=g).to(torch.bfloat16)
        td = torch.full((8,), t // 8, dtype=torch.int64, device="cuda")
        fn = lambda: ggo.grouped_gemm_opt(x, w, td)  # noqa: E731
        ms, _, clk = measure(fn, st, 1, local)
        dn = lambda: torch.nn.functional.linear(x, w0)  # noqa: E731
        dms, _, _ = measure(dn, st, 1, local)
        flop = 2.0 * t * 14336 * 4096
        sweep.append({"tokens": t, "ms": ms, "tflops": flop / ms / 1e9,
                      "dense_tflops": flop / dms / 1e9, "vs_dense": dms / ms,
                      "clocks": clk})
        del x
    res["token_sweep_uniform_e8"] = sweep
    del w, w0
    torch.cuda.empty_cache()

    # backward of the cfg2 grouped GEMM, FP8 and MXFP8 forwards of the same problem
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(T_TOK, K, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(T_TOK, N, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    td = torch.full((E,), T_TOK // E, dtype=torch.int64, device="cuda")
    from grouped_gemm_opt import (grouped_gemm_opt_fp8, grouped_gemm_opt_mxfp8, quantize_fp8,
                                  quantize_mxfp8)
    xq, xs = quantize_fp8(x)
    wq, ws = quantize_fp8(w)
    mxq, mxs = quantize_mxfp8(x, td)
    mwq, mws = quantize_mxfp8(w)
    for name, fn in (("cfg2_dgrad", lambda: _C.grouped_gemm_dgrad(dy, w, td, 4, True)),
                     ("cfg2_wgrad", lambda: _C.grouped_gemm_wgrad(x, dy, td, True)),
                     ("cfg2_fp8", lambda: grouped_gemm_opt_fp8(xq, xs, wq, ws, td)),
                     ("cfg2_mxfp8", lambda: grouped_gemm_opt_mxfp8(mxq, mxs, mwq, mws, td))):
        for _ in range(warmup):
            fn()
        ms, _, clk = measure(fn, max(st, 100), 1, local)
        res[name] = {"ms": ms, "tflops": GEMM_FLOP / ms / 1e9, "clocks": clk}
    del x, dy, w, xq, wq, mxq, mwq
    torch.cuda.empty_cache()

    # the Mixtral layer with FP8 and MXFP8 grouped GEMMs on one GPU (bf16 is the headline)
    from grouped_gemm_opt import (fused_moe_fp8, fused_moe_mxfp8, quantize_moe_weights,
                                  quantize_moe_weights_mxfp8)
    T2, H2, F2, E2, k2 = MIX_T, MIX_H, MIX_F, MIX_E, MIX_K
    _, _, x, logits = _tokens(T2, H2, E2, SEED_TOKENS, 0, 1)
    wgu, wdn = _local_weights(H2, F2, E2, SEED_EXPERTS, 0, 1)
    for name, qfn, lfn in (("mixtral_layer_fp8", quantize_moe_weights, fused_moe_fp8),
                           ("mixtral_layer_mxfp8", quantize_moe_weights_mxfp8, fused_moe_mxfp8)):
        qw = qfn(wgu, wdn)
        torch.cuda.empty_cache()
        fn = lambda: lfn(x, logits, qw, k2)  # noqa: E731
        for _ in range(warmup):
            fn()
        ms, _, clk = measure(fn, st, 1, local)
        res[name] = {"ms": ms, "tokens_per_s": T2 / ms * 1e3,
                     "tflops": MIX_FLOP / ms / 1e9, "clocks": clk}
        del qw
        torch.cuda.empty_cache()
    del x, logits, wgu, wdn
    torch.cuda.empty_cache()
    res["launch_overhead"] = launch_overhead(local)
    return res


def cpu_layer_sample(threads, min_s, tokens):
    """The reference's algorithm for the layer on the host cores: route, permute, the two
    grouped GEMMs as the reference's per-expert F.linear loop in bf16 (benchmark.py:91-107),
    SwiGLU, combine (oracle.moe_layer with native=True). Problem of `tokens` tokens with the
    configs[3] shapes, repeated until `min_s` seconds. Returns (tokens/s, seconds, reps)."""
    import torch
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import grouped_gemm_oracle as oracle
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(SEED_TOKENS)
    H, F, Ex, k = MIX_H, MIX_F, MIX_E, MIX_K
    x = torch.randn(tokens, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(tokens, Ex, generator=g)
    wgu = (torch.randn(Ex, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(Ex, H, F, generator=g) * 0.02).to(torch.bfloat16)
    oracle.moe_layer(x[:64], logits[:64], wgu, wd, k, native=True)  # warm-up
    reps = 0
    t0 = time.perf_counter()
    while True:
        oracle.moe_layer(x, logits, wgu, wd, k, native=True)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= min_s:
            break
    return tokens * reps / dt, dt, reps


def run_reference(args):
    """--impl reference: the reference's CPU algorithm for the layer, on this host's cores.
    Every step is the whole configs[3] layer (16384 tokens) unless --ref-tokens caps it."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    tokens = args.ref_tokens or MIX_T
    vals = []
    for i in range(args.warmup + args.steps):
        v, _, _ = cpu_layer_sample(threads, 0.0, tokens)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    del torch
    sample = (f"whole layer ({tokens} tokens) per step" if tokens == MIX_T else
              f"{tokens} of the {MIX_T} tokens per step")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": MIX_T / value * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens and "
        "logits, N(0,0.02) weights)", "config": layer_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample + "; per-expert F.linear loop in bf16 "
                                   "(reference benchmark.py:91-107), route/permute/combine "
                                   "as the layer's CPU restatement"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- profiling
def profile_run(args):
    """Minimal runs for ncu captures (warm-up + steps of one path, prints a done line):
    gemm (cfg2 grouped GEMM), fp8 / mxfp8 / dgrad / wgrad (cfg2 shapes), moe (the one-GPU
    Mixtral layer), gemm1cta (cfg2 on the single-CTA 128x256 kernel), skinny (cfg3 zipf),
    dsv3down (the DSv3 layer's down-projection shape, 64 experts)."""
    import torch
    torch.cuda.set_device(0)
    import grouped_gemm_opt as ggo
    from grouped_gemm_opt import _C
    g = torch.Generator(device="cuda").manual_seed(0)
    if args.profile in ("gemm", "gemm1cta", "fp8", "mxfp8", "dgrad", "wgrad"):
        x = torch.randn(T_TOK, K, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(E, N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        tpe = torch.full((E,), T_TOK // E, dtype=torch.int64, device="cuda")
        if args.profile == "gemm":
            fn = lambda: ggo.grouped_gemm_opt(x, w, tpe)  # noqa: E731
        elif args.profile == "gemm1cta":
            fn = lambda: ggo.grouped_gemm_opt(x, w, tpe, ggo.TileConfig.Co_128x256x64)  # noqa
        elif args.profile == "fp8":
            xq, xs = ggo.quantize_fp8(x)
            wq, ws = ggo.quantize_fp8(w)
            fn = lambda: ggo.grouped_gemm_opt_fp8(xq, xs, wq, ws, tpe)  # noqa: E731
        elif args.profile == "mxfp8":
            xq, xs = ggo.quantize_mxfp8(x, tpe)
            wq, ws = ggo.quantize_mxfp8(w)
            fn = lambda: ggo.grouped_gemm_opt_mxfp8(xq, xs, wq, ws, tpe)  # noqa: E731
        else:
            dy = torch.randn(T_TOK, N, device="cuda", generator=g).to(torch.bfloat16)
            fn = (lambda: _C.grouped_gemm_dgrad(dy, w, tpe, 4, True)) if args.profile == "dgrad" \
                else (lambda: _C.grouped_gemm_wgrad(x, dy, tpe, True))
    elif args.profile == "dsv3down":
        # the DSv3 layer's down projection per expert (K=2048 -> N=7168, ~1024 rows per expert),
        # 64 of its 256 experts (a few GB on the device)
        ex, rows = 64, 65536
        x = torch.randn(rows, 2048, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(ex, 7168, 2048, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        gc = torch.Generator().manual_seed(3)
        tpe = torch.bincount(torch.randint(0, ex, (rows,), generator=gc), minlength=ex).cuda()
        fn = lambda: ggo.grouped_gemm_opt(x, w, tpe)  # noqa: E731
    elif args.profile == "skinny":
        x = torch.randn(8192, 4096, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(64, 14336, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        tpe = _zipf_counts(8192, 64).cuda()
        fn = lambda: ggo.grouped_gemm_opt(x, w, tpe)  # noqa: E731
    else:
        _, _, x, logits = _tokens(MIX_T, MIX_H, MIX_E, SEED_TOKENS, 0, 1)
        wgu, wd = _local_weights(MIX_H, MIX_F, MIX_E, SEED_EXPERTS, 0, 1)
        fn = lambda: ggo.fused_moe(x, logits, wgu, wd, MIX_K)  # noqa: E731
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    print(f"profile {args.profile}: {args.warmup + args.steps} steps done", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the secondary-config sweep")
    ap.add_argument("--no-dsv3", action="store_true")
    ap.add_argument("--no-gemm", action="store_true", help="skip the cfg2 grouped-GEMM leg")
    ap.add_argument("--ref-tokens", type=int, default=0,
                    help="reference arm: tokens per step (default: the whole layer)")
    ap.add_argument("--profile", choices=["gemm", "gemm1cta", "moe", "fp8", "mxfp8", "dgrad",
                                          "wgrad", "skinny", "dsv3down"], default=None,
                    help="minimal run for ncu captures: warm-up + steps of one path, no JSON")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return
    if args.profile:
        profile_run(args)
        return

    import torch
    world, rank, local = _dist_init()
    import grouped_gemm_opt as ggo

    lay = mixtral_layer_leg(world, rank, local, args.steps, args.warmup)
    ggo.check_device_errors(local)
    torch.cuda.empty_cache()
    dsv3 = None if args.no_dsv3 else dsv3_leg(world, rank, local, args.steps, args.warmup)
    torch.cuda.empty_cache()
    gemm = sweep = None
    if world == 1 and not args.no_gemm:
        gemm = grouped_gemm_leg(local, args.steps, args.warmup)
        torch.cuda.empty_cache()
    if world == 1 and not args.no_sweep:
        sweep = config_sweep(local, args.steps)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, dt, reps = cpu_layer_sample(threads, 10.0, MIX_T)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"the whole configs[3] layer on the CPU (per-expert bf16 F.linear "
                         f"loop) x{reps}, {dt:.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": lay["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": lay["ms"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) tokens and logits, N(0,0.02) weights; the same "
                    "global problem at every N)",
            "config": layer_config(world),
            "path": "one GPU, no collectives" if world == 1 else
                    "expert parallel: dispatch and result scatter over NVLink peer memory "
                    "inside the kernels, device-side signalling",
            "roofline": lay["roofline"],
            "layer_roofline": lay["layer_roofline"],
            "tflops": lay["tflops"],
            "stages_ms_per_layer": lay["stages"],
            "rows_per_rank": lay["rows_per_rank"],
            "clocks": lay["clocks"],
            "gpu_launches": lay["launches"],
            "e2e": lay["e2e"],
            "ep_parity": lay["ep_parity"],
            "nccl_path": lay.get("nccl"),
            "cpu_baseline": cpu,
            "dsv3": dsv3,
            "grouped_gemm": gemm,
            "configs": sweep,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
