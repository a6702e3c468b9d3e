"""MoE-block benchmark (tokens/s and roofline fraction) on 1..8 B200s.

`python bench.py --gpus N --steps K --warmup W` prints ONE JSON line.

Workload (the decode sweep): the Qwen 3.5/3.6 MoE
block with hidden 2048, 128 experts, top-8, expert intermediate 768, 4-bit
affine gs64 experts, bf16 router; one step = one block forward at each token
batch T in {1, 8, 64} on fresh inputs (73 tokens per step per GPU). Each
forward is a captured CUDA graph of the library's block call. L2 is flushed
(a 512 MiB write) before every forward; only the forwards are timed, with
CUDA events on the launching stream. N > 1: one process per GPU, each serving
its own decode batches with the experts replicated (the decode sweep's units,
token batches, are independent: no data-path collective), "scaling": "weak",
value = all tokens / max-over-ranks time. At N > 1 the line also carries
"expert_parallel": the largest configurations (C5 prefill 8192 tokens, C4
16384 tokens, C5 decode 256) run expert-parallel over the N ranks with NCCL
all-to-all dispatch and combine, strong scaling, beside the same batch on one
GPU measured in the same run.

`--impl reference` times the CPU restatement of the reference block (the
reference's own MLX CPU path cannot be built here) on the host cores, on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mlx-rs_b200"))

WORKLOAD = "c2"
BATCHES = [1, 8, 64]
METRIC = "MoE-block tokens/s (decode sweep T=1,8,64; D=2048 E=128 K=8 I=768 q4 gs64)"
UNIT = "tokens/s"
L2_FLUSH_BYTES = 512 << 20


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def ncu_traffic(kernel_key: str):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary line:
    `traffic_bytes_per_launch <key> <bytes>` in profiles/*.md."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for fn in sorted(os.listdir(d)):
        if not fn.endswith(".md"):
            continue
        with open(os.path.join(d, fn)) as f:
            for line in f:
                parts = line.strip().strip("`").split()
                if len(parts) == 3 and parts[0] == "traffic_bytes_per_launch" and parts[1] == kernel_key:
                    return int(float(parts[2]))
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    5 ms while the timed region runs (the nvidia-smi clocks query reads the
    same counters, but its 200 ms period is longer than a timed region).
    Read-only: no clock or power setting is touched."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.samples = []
        self.err = None
        self._stop = threading.Event()
        self.t = None

    def start(self):
        try:
            import pynvml as N

            N.nvmlInit()
            self.N = N
            self.h = N.nvmlDeviceGetHandleByUUID(self.uuid)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report it instead of a clock
            self.err = f"nvml unavailable: {e}"[:200]
            return
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        N = self.N
        while not self._stop.is_set():
            try:
                mhz = N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)
                rs = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception as e:
                self.err = str(e)[:200]
                return
            time.sleep(0.005)

    def stop(self):
        if self.t is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": self.err}
        self._stop.set()
        self.t.join(timeout=2)
        sm = [m for m, _ in self.samples]
        reasons = set()
        for _, rs in self.samples:
            for name, const in self.REASONS:
                if rs & getattr(self.N, const, 0):
                    reasons.add(name)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 5 ms"}
        if not sm:
            out["error"] = self.err or "no samples"
        return out


def smi_id(torch, dev) -> str:
    """The GPU's UUID (survives CUDA_VISIBLE_DEVICES remapping)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index)


def kernels_per_forward(cfg, T: int, sms: int = 148) -> int:
    """Library kernels one block forward launches at T tokens (the launch
    choices of csrc/moe_block.cu: router variant, one-CTA or three-kernel
    permute with or without a separate row gather, split-K / fused / plain
    expert GEMMs, combine, shared expert)."""
    D, E, K, I = cfg.hidden_size, cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size
    R = T * K
    if T == 0:
        return 0
    n = 2 if T > 256 else 1                                    # router (tile + route rows above 256 tokens)
    small = R <= 2048
    n += 1 if small else 3                                     # permute
    n += 0 if (small and R <= 16) else 1                       # row gather (in the one-CTA permute up to 16 rows)

    def pick_bn(avg, cap):
        bn = 16 if avg <= 12 else 32 if avg <= 24 else 64 if avg <= 48 else 128 if avg <= 160 else 256
        return min(bn, cap)

    def splits(items, ksteps):
        if items <= 0 or items * 2 > sms:
            return 1
        return max(1, min(sms // items, ksteps // 4, 8))
    bn1 = pick_bn(R / E, 128)
    bn2 = pick_bn(R / E, 128 if D % 256 == 0 else 256)
    used = min(R, E)
    s1 = splits(used * (I // 128), D // 64) if small and bn1 <= 32 else 1
    s2 = splits(used * (D // 256 if D % 256 == 0 else D // 128), I // 64) if small and bn2 <= 32 else 1
    fuse = s1 == 1 and s2 == 1 and D % 256 == 0 and bn1 <= 32 and bn1 == min(bn2, 128)
    n += 1 if fuse else 2                                      # expert GEMMs
    n += 1                                                     # combine
    if cfg.shared_expert_intermediate_size:
        sb = cfg.shared_bits or cfg.bits
        n += 2 + (1 if (T < 256 or sb == 4) else 0)            # shared gate|up, down (+ padded copy)
    return n


def distinct_experts(routing) -> int:
    return int((routing.counts > 0).sum().item())


# ---------------------------------------------------------------- GPU arm ----
def stage_times(torch, C, _lib, blk, x_in, x_static, out, ws, st, flush, reps, dev):
    """Median per-stage times (ms) of one block forward: a graph of the
    forward captured with the library's stage events recorded between its
    kernels (event-record nodes), replayed `reps` times with L2 flushed."""
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    for e in evs:  # materialise the CUDA events before handing their handles over
        e.record(st)
    torch.cuda.synchronize(dev)
    arr = (C.c_void_p * 7)(*[C.c_void_p(e.cuda_event) for e in evs])
    gs = torch.cuda.CUDAGraph()
    _lib.call("mlxr_cu_moe_set_stage_events", arr, 7)
    try:
        with torch.cuda.stream(st), torch.cuda.graph(gs, stream=st):
            blk.forward(x_static, out=out, workspace=ws)
    finally:
        _lib.call("mlxr_cu_moe_set_stage_events", None, 0)
    times = []
    with torch.cuda.stream(st):
        for i in range(reps):
            if x_in[i % len(x_in)] is not x_static:
                x_static.copy_(x_in[i % len(x_in)])
            flush.fill_(i & 0xFF)
            gs.replay()
            torch.cuda.synchronize(dev)
            times.append([evs[j].elapsed_time(evs[j + 1]) for j in range(6)])
    del gs
    med = [statistics.median(col) for col in zip(*times)]
    return dict(router_ms=med[0], permute_ms=med[1], gate_up_ms=med[2], down_ms=med[3], shared_ms=med[4],
                combine_ms=med[5])


def run_gpu(args):
    import torch
    import torch.distributed as dist

    from mlxr_moe import synth
    from mlxr_moe.moe import Routing

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    peaks = measured_peaks()
    spec = synth.CONFIGS[WORKLOAD]
    cfg = spec["cfg"]
    # Everything (weight synthesis, inputs, workspaces, forwards) runs on one
    # stream, so the caching allocator never hands a buffer that pending work
    # on another stream still touches to the block.
    st = torch.cuda.Stream(dev)
    torch.cuda.set_stream(st)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    blk = synth.make_block(cfg, seed=0, zipf=spec["zipf"], device=dev)
    D = cfg.hidden_size
    torch.cuda.synchronize(dev)
    nsets = 4  # distinct input batches cycled through the steps

    # Per batch size: static input/output/workspace buffers and one graph.
    graphs = {}
    with torch.cuda.stream(st):
        for T in BATCHES:
            xs = [synth.make_input(T, D, seed=0, stream_offset=1000 * rank + 10 * T + i, device=dev)
                  for i in range(nsets)]
            x_static = torch.empty_like(xs[0])
            out = torch.empty_like(xs[0])
            ws = torch.empty(blk.workspace_bytes(T), dtype=torch.uint8, device=dev)
            x_static.copy_(xs[0])
            for _ in range(2):  # warm: sets kernel attributes outside capture
                blk.forward(x_static, out=out, workspace=ws)
            torch.cuda.synchronize(dev)
            blk.status(ws)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                blk.forward(x_static, out=out, workspace=ws)
            r = Routing(T, cfg.num_experts_per_tok, cfg.num_experts, dev)
            blk.forward(xs[0], routing=r, workspace=ws)
            torch.cuda.synchronize(dev)
            graphs[T] = dict(x=xs, xs=x_static, out=out, ws=ws, g=g, U=distinct_experts(r))

    # Stage events for the live per-kernel timing (dominant kernel: gate/up GEMM).
    import ctypes as C

    from mlxr_moe import _lib

    def run_steps(nsteps, timed, stage_capture=False):
        ev = []
        with torch.cuda.stream(st):
            for s in range(nsteps):
                for T in BATCHES:
                    G = graphs[T]
                    G["xs"].copy_(G["x"][s % nsets])
                    flush.fill_(s & 0xFF)
                    if timed:
                        a = torch.cuda.Event(enable_timing=True)
                        b = torch.cuda.Event(enable_timing=True)
                        a.record(st)
                    G["g"].replay()
                    if timed:
                        b.record(st)
                        ev.append((T, a, b))
        return ev

    run_steps(args.warmup, timed=False)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(smi_id(torch, dev))
    clocks.start()
    evs = run_steps(args.steps, timed=True)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    per_T = {T: [] for T in BATCHES}
    for T, a, b in evs:
        per_T[T].append(a.elapsed_time(b))
    total_ms = sum(sum(v) for v in per_T.values())
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    tokens_per_step = sum(BATCHES)
    value = world * tokens_per_step * args.steps / (total_ms / 1e3)

    # Live stage timing: a second graph per batch size with the library's
    # stage events recorded between its kernels (event-record nodes).
    stage = {T: stage_times(torch, C, _lib, blk, graphs[T]["x"], graphs[T]["xs"], graphs[T]["out"], graphs[T]["ws"],
                            st, flush, max(5, args.steps), dev) for T in BATCHES}

    # e2e: the same sweep through the public API with pinned host buffers.
    e2e_ms = 0.0
    h2d = d2h = 0
    host_in = {T: [graphs[T]["x"][i].cpu().pin_memory() for i in range(nsets)] for T in BATCHES}
    host_out = {T: torch.empty_like(graphs[T]["out"], device="cpu").pin_memory() for T in BATCHES}
    e2e_evs = []
    with torch.cuda.stream(st):
        for s in range(args.warmup + args.steps):
            for T in BATCHES:
                G = graphs[T]
                flush.fill_(s & 0xFF)
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(st)
                G["xs"].copy_(host_in[T][s % nsets], non_blocking=True)
                G["g"].replay()
                host_out[T].copy_(G["out"], non_blocking=True)
                b.record(st)
                if s >= args.warmup:
                    e2e_evs.append((a, b))
    torch.cuda.synchronize(dev)
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_evs)
    for T in BATCHES:
        h2d += T * D * 2
        d2h += T * D * 2
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * tokens_per_step * args.steps / (e2e_ms / 1e3)

    # Roofline of the dominant kernel and of the whole block. The dominant
    # kernel is the expert GEMM: at decode widths gate|up (+SwiGLU) and the
    # down projection run as ONE fused launch, so its algorithmic bytes are
    # the routed experts' packed weights (all three matrices) plus the
    # activation rows it reads and writes (x in, h out and back in, y out).
    K_, I_ = cfg.num_experts_per_tok, cfg.moe_intermediate_size
    ex_bytes_unit = synth.expert_bytes(cfg)

    def expert_gemm_bytes(T, U):
        return int(U * ex_bytes_unit + T * K_ * (D + I_) * 2 * 2)

    sweep = []
    ex_bytes_total = ex_ms_total = 0.0
    for T in BATCHES:
        G = graphs[T]
        ms = statistics.median(per_T[T])
        U = G["U"]
        blk_bytes = synth.algorithmic_bytes(cfg, T, U)
        ex_bytes_total += expert_gemm_bytes(T, U)
        ex_ms_total += stage[T]["gate_up_ms"] + stage[T]["down_ms"]
        sweep.append(dict(tokens=T, distinct_experts=U, ms=ms, tokens_per_s=T / (ms / 1e3),
                          block_gbs=blk_bytes / (ms / 1e3) / 1e9,
                          block_hbm_frac=blk_bytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                          stages_ms={k: round(v, 5) for k, v in stage[T].items()}))
    achieved = ex_bytes_total / (ex_ms_total / 1e3) / 1e9
    roofline = dict(bound="hbm",
                    kernel="grouped_dequant_gemm: expert GEMMs (gate|up + SwiGLU, down; one fused launch at "
                           "T=8 and T=64, split-K launches at T=1)",
                    achieved=achieved, peak=peaks["hbm_gbs"], unit="GB/s", frac=achieved / peaks["hbm_gbs"],
                    peak_source=peaks["source"] + " hbm_gbs (burst copy)",
                    traffic=ncu_traffic("experts_c2_T64"),
                    traffic_note="ncu DRAM bytes of the fused launch at T=64 (profiles/*.md)",
                    algorithmic_bytes_per_launch={str(T): expert_gemm_bytes(T, graphs[T]["U"]) for T in BATCHES},
                    timing="stage events around the expert GEMM launch(es) inside the captured forward")

    extra = {}
    if rank == 0 and not args.no_extra and world == 1:
        extra = bench_extra(args, dev, st, flush, peaks)
    ep = None
    if world > 1 and not args.no_extra:
        ep = bench_ep(args, dev, st, world, rank)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(blk, graphs, args)

    if world > 1:
        dist.barrier()
    del graphs
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (Philox seed 0): experts N(0,0.02) bf16 -> 4-bit affine gs64, router bf16, x N(0,1)",
            "config": {"workload": "c2 decode sweep: one block forward at T=1, 8, 64 per step",
                       "hidden": D, "experts": cfg.num_experts, "top_k": cfg.num_experts_per_tok,
                       "moe_intermediate": cfg.moe_intermediate_size, "bits": cfg.bits, "group_size": cfg.group_size,
                       "batches": BATCHES, "l2": "flushed before every forward (512 MiB write)",
                       "graphs": "each forward replayed from a captured CUDA graph",
                       "parallelism": f"dp{world}: token batches per rank, experts replicated" if world > 1
                       else "single GPU"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "pinned host x -> device, graph replay, out -> pinned host, per forward"},
            "gpu_launches": sum(kernels_per_forward(cfg, T) for T in BATCHES) * args.steps,
            "clocks": clk,
            "sweep": sweep,
            "extra": extra,
            "expert_parallel": ep,
        }
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


# The Gemma 4 MoE branch (model_kind 1) on a synthetic block of the C2
# sizes (no Gemma 4 checkpoint or BASELINE configuration exists here):
# hidden 2048, 128 experts, top-8, expert intermediate 768, 4-bit gs64.
def _gemma4_cfg():
    from mlxr_moe.moe import MoeConfig
    return MoeConfig(2048, 128, 8, 768, bits=4, model_kind=1, rms_norm_eps=1e-6)


def bench_extra(args, dev, st, flush, peaks):
    """The other BASELINE configurations on this GPU (informational lines)."""
    import ctypes as C

    import torch

    from mlxr_moe import _lib

    from mlxr_moe import synth
    from mlxr_moe.moe import Routing

    GEMMA4_CFG = _gemma4_cfg()
    res = {}

    def baseline(key):
        spec = synth.CONFIGS[key]
        return synth.make_block(spec["cfg"], 0, spec["zipf"], dev), spec["zipf"]

    def gemma4():
        return synth.make_gemma4_branch(GEMMA4_CFG, 0, dev), False

    for name, T, make in (("c1", 32, lambda: baseline("c1")), ("c3", 4096, lambda: baseline("c3")),
                          ("c5_decode", 256, lambda: baseline("c5")), ("c5_prefill", 8192, lambda: baseline("c5")),
                          ("c4", 16384, lambda: baseline("c4")), ("gemma4_decode", 64, gemma4),
                          ("gemma4_prefill", 4096, gemma4)):
        blk, zipf = make()
        cfg = blk.cfg
        x = synth.make_input(T, cfg.hidden_size, stream_offset=7, device=dev)
        out = torch.empty_like(x)
        ws = torch.empty(blk.workspace_bytes(T), dtype=torch.uint8, device=dev)
        r = Routing(T, cfg.num_experts_per_tok, cfg.num_experts, dev)
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(st):
            blk.forward(x, routing=r, out=out, workspace=ws)
            torch.cuda.synchronize(dev)
            blk.status(ws)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                blk.forward(x, out=out, workspace=ws)
            times = []
            for i in range(3 + max(5, args.steps // 2)):
                flush.fill_(i & 0xFF)
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(st)
                g.replay()
                b.record(st)
                torch.cuda.synchronize(dev)
                if i >= 3:
                    times.append(a.elapsed_time(b))
        ms = statistics.median(times)
        stg = stage_times(torch, C, _lib, blk, [x], x, out, ws, st, flush, 5, dev)
        U = distinct_experts(r)
        fl = synth.algorithmic_flops(cfg, T)
        by = synth.algorithmic_bytes(cfg, T, U)
        tfl = fl / (ms / 1e3) / 1e12
        gbs = by / (ms / 1e3) / 1e9
        prefill = T >= 2048
        res[name] = dict(tokens=T, ms=ms, tokens_per_s=T / (ms / 1e3), tflops=tfl, gbs=gbs,
                         bound="tensor" if prefill else "hbm",
                         frac=(tfl / peaks["bf16_tflops"]) if prefill else (gbs / peaks["hbm_gbs"]),
                         distinct_experts=U, zipf=zipf,
                         stages_ms={k: round(v, 5) for k, v in stg.items()})
        if name == "gemma4_decode" and not args.no_cpu:
            res[name]["cpu_baseline"] = gemma4_cpu_baseline(blk, x)
        del g, blk, ws, out, x
        torch.cuda.empty_cache()
    return res


def gemma4_cpu_baseline(branch, x):
    """The oracle's Gemma 4 branch (fused-fp32 contract, OpenMP on every host
    core) on the same 64 decode tokens, median of 2 forwards."""
    import numpy as np
    import torch

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    u16 = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    q3 = lambda q: (q.weight.detach().cpu().numpy().view(np.uint32), u16(q.scales), u16(q.biases))  # noqa: E731
    c = branch.cfg
    cfg = dict(hidden=c.hidden_size, num_experts=c.num_experts, top_k=c.num_experts_per_tok,
               moe_intermediate=c.moe_intermediate_size, group_size=c.group_size, bits=c.bits, eps=c.rms_norm_eps)
    W = {"router": u16(branch.gate), "router_norm": u16(branch.router_norm), "expert_scale": u16(branch.expert_scale),
         "experts_norm": u16(branch.experts_norm), "gate_up": q3(branch.switch_glu.gate_up_proj),
         "down": q3(branch.switch_glu.down_proj)}
    xs = u16(x)
    times = []
    for _ in range(2):
        t0 = time.perf_counter()
        O.gemma4_block(cfg, W, xs)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"tokens_per_s": xs.shape[0] / sec, "cores": O.max_threads(), "kind": "port",
            "sample": f"2 forwards of {xs.shape[0]} tokens, median; oracle fused-fp32, OpenMP {O.max_threads()} threads"}


def bench_ep(args, dev, st, world, rank):
    """Expert parallelism across the `world` ranks: the largest BASELINE
    configurations with their token batch split evenly over the ranks (strong
    scaling: fixed total tokens). Experts are placed by loads measured on a
    calibration batch. The step exchanges pairs and partial rows inside the
    kernels over peer memory (the product path); the same step over NCCL
    all-to-all is timed beside it. Times are max over ranks; the whole batch on
    rank 0 alone (full block, one GPU) gives the one-GPU time in the same run."""
    import torch
    import torch.distributed as dist

    from mlxr_moe import synth
    from mlxr_moe.ep import ExpertParallelMoeBlock, PeerComm, TorchDistExchange, balanced_placement

    ex = TorchDistExchange()
    res = {}
    for name, T_total in (("c5_prefill", 8192), ("c4", 16384), ("c5_decode", 256)):
        spec = synth.CONFIGS[name.split("_")[0]]
        cfg = spec["cfg"]
        D, K = cfg.hidden_size, cfg.num_experts_per_tok
        T = T_total // world
        full = synth.make_block(cfg, 0, spec["zipf"], dev)
        xs = [synth.make_input(T, D, stream_offset=500 + 16 * rank + i, device=dev) for i in range(2)]
        # Placement from measured expert loads: every rank routes a calibration
        # batch (its own tokens), the counts are summed over ranks, and the
        # experts are spread greedily so each rank gets about the same rows.
        calib = synth.make_input(T, D, stream_offset=900 + rank, device=dev)
        idx, _ = full.router(calib)
        loads = torch.bincount(idx.reshape(-1).long(), minlength=cfg.num_experts).to(torch.float64)
        dist.all_reduce(loads)
        place = balanced_placement(loads.cpu().tolist(), world)
        blk = ExpertParallelMoeBlock.from_block(full, rank, world, place)
        bounds = dict(max_recv_pairs=world * T, max_recv_rows=world * T * K)
        n_steps = max(5, args.steps // 2)
        comm = PeerComm(rank, world, cap=T, hidden=D, k=K)
        exp_rows = max(1, T_total * K // world)

        def timed(fn):
            with torch.cuda.stream(st):
                for i in range(3):
                    fn(xs[i % 2])
                torch.cuda.synchronize(dev)
                blk.status()
                dist.barrier()
                times = []
                for i in range(n_steps):
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record(st)
                    fn(xs[i % 2])
                    b.record(st)
                    b.synchronize()
                    times.append(a.elapsed_time(b))
            torch.cuda.synchronize(dev)
            blk.status()
            t = torch.tensor([statistics.median(times)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        # Peer-memory exchange (the product path), then the NCCL exchange for reference.
        ms = timed(lambda xx: blk.forward_p2p(xx, comm, expected_rows=exp_rows))
        ms_nccl = timed(lambda xx: blk.forward(xx, ex, **bounds))
        torch.cuda.synchronize(dev)
        dist.barrier()
        comm.close()
        one = None
        if rank == 0:  # the whole batch on this GPU alone, for the speed-up
            x1 = synth.make_input(T_total, D, stream_offset=600, device=dev)
            out1 = torch.empty_like(x1)
            ws1 = torch.empty(full.workspace_bytes(T_total), dtype=torch.uint8, device=dev)
            with torch.cuda.stream(st):
                t1 = []
                for i in range(3 + n_steps):
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record(st)
                    full.forward(x1, out=out1, workspace=ws1)
                    b.record(st)
                    b.synchronize()
                    if i >= 3:
                        t1.append(a.elapsed_time(b))
            one = statistics.median(t1)
            del x1, out1, ws1
        dist.barrier()
        fl = synth.algorithmic_flops(cfg, T_total)
        res[name] = dict(tokens=T_total, tokens_per_rank=T, ms=ms, tokens_per_s=T_total / (ms / 1e3),
                         tflops_total=fl / (ms / 1e3) / 1e12, one_gpu_ms=one,
                         speedup_vs_one_gpu=(one / ms) if one else None, zipf=spec["zipf"],
                         exchange="peer memory: dispatch/combine kernels store into the other ranks' CUDA-IPC "
                                  "buffers over NVLink, flag waits on the GPU, no host synchronisation",
                         nccl_ms=ms_nccl, nccl_speedup_vs_one_gpu=(one / ms_nccl) if one else None,
                         placement="balanced: experts spread greedily by loads measured on a calibration batch",
                         nccl_exchange="NCCL all_to_all_single: counts, pair rows, slot rows, partial rows")
        del blk, full, xs
        torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------- CPU baseline ----
def cpu_baseline(blk, graphs, args):
    """The oracle (CPU restatement of the reference block, fused-fp32 mode,
    OpenMP on every host core) on a bounded sample: the same sweep batches."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle as O
    from gpu_helpers import block_to_oracle

    from conftest import bf16_np

    cfg, W = block_to_oracle(blk)
    cores = O.max_threads()
    times = []
    reps = 5
    for rep in range(reps):
        t0 = time.perf_counter()
        for T in BATCHES:
            O.moe_block(cfg, W, bf16_np(graphs[T]["x"][rep % 4]), "fused")
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"value": sum(BATCHES) / sec, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{reps} sweeps (T=1,8,64) of the block, median; oracle fused-fp32 mode, OpenMP {cores} threads"}


def run_reference(args):
    """--impl reference: the CPU port of the reference block (MLX's own CPU
    path cannot be built here) timed on all host cores; rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import numpy as np

    import oracle as O

    cfgd = dict(hidden=2048, num_experts=128, top_k=8, moe_intermediate=768, group_size=64, bits=4)
    W = {"router": O.normal_bf16(0, 0, (128, 2048), 0.02)}
    W["gate"] = O.quantize(O.normal_bf16(0, 1, (128, 768, 2048), 0.02), 64, 4)
    W["up"] = O.quantize(O.normal_bf16(0, 2, (128, 768, 2048), 0.02), 64, 4)
    W["down"] = O.quantize(O.normal_bf16(0, 3, (128, 2048, 768), 0.02), 64, 4)
    xs = {T: O.normal_bf16(0, 8 + 10 * T, (T, 2048), 1.0) for T in BATCHES}
    cores = O.max_threads()
    for _ in range(args.warmup):
        for T in BATCHES:
            O.moe_block(cfgd, W, xs[T], "fused")
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for T in BATCHES:
            O.moe_block(cfgd, W, xs[T], "fused")
    sec = time.perf_counter() - t0
    value = sum(BATCHES) * args.steps / sec
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * sec / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (Philox seed 0), same configuration as the GPU arm",
        "config": {"workload": "c2 decode sweep: one block forward at T=1, 8, 64 per step",
                   "hidden": 2048, "experts": 128, "top_k": 8, "moe_intermediate": 768, "bits": 4, "group_size": 64,
                   "batches": BATCHES, "host": f"CPU, {cores} threads (rank 0 only; the GPUs are unused)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{args.steps} full sweeps on the oracle (CPU restatement; MLX unbuildable here)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    _ = np


def run_case(args):
    """Block forwards of one configuration, for ncu captures (not a bench number)."""
    import torch

    from mlxr_moe import synth

    name, T = args.case.split(":")
    if name == "gemma4":
        blk = synth.make_gemma4_branch(_gemma4_cfg(), 0)
    else:
        spec = synth.CONFIGS[name]
        blk = synth.make_block(spec["cfg"], 0, spec["zipf"])
    x = synth.make_input(int(T), blk.cfg.hidden_size)
    for _ in range(args.iters):
        blk.forward(x)
    torch.cuda.synchronize()
    blk.status()
    print(f"case {args.case}: {args.iters} forwards ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="skip the other BASELINE configurations")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--case", default=None,
                    help="profiling driver: CONFIG:TOKENS (e.g. c2:64, gemma4:64); runs only block forwards, prints nothing timed")
    ap.add_argument("--iters", type=int, default=3, help="forwards for --case")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
