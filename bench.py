"""MoE-block benchmark (tokens/s and roofline fraction) on 1..8 B200s.

`python bench.py --gpus N --steps K --warmup W` prints ONE JSON line.

Workload (C5, the largest configuration): the Qwen
3.5/3.6 MoE block with hidden 4096, 128 experts, top-8, expert intermediate
1536, 4-bit affine gs64 experts, bf16 router, Zipf(1.1)-skewed routing. One
step = one block forward over an 8192-token prefill batch plus one over a
256-token decode batch (8448 tokens), on fresh inputs (two input sets
alternate). L2 is flushed (a 512 MiB write) before every forward; only the
forwards are timed, with CUDA events on the launching stream.

N = 1: each forward is a captured CUDA graph of the library's block call.
N > 1: the same C5 step, expert-parallel over the N ranks (one process per
GPU): every rank routes 8192/N prefill and 256/N decode tokens, experts are
placed by measured load, and pairs and partial rows cross NVLink inside the
library's kernels (peer memory, no collective library on the data path).
Strong scaling: the total batch is fixed, value = 8448 tokens per step / the
max-over-ranks step time.

The other configurations (the C2 decode sweep with its HBM roofline, C1, C3,
C4 and the Gemma 4 branch) are reported under "extra" at N = 1; at N > 1 the
same C5 step over NCCL all-to-all and the C4 block run expert-parallel under
"expert_parallel".

`--impl reference` times the CPU restatement of the reference block (the
reference's own MLX CPU path cannot be built here) on the host cores, on a
bounded sample of the same C5 step.
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

HEADLINE = "c5"
PREFILL_T, DECODE_T = 8192, 256
STEP_TOKENS = PREFILL_T + DECODE_T
METRIC = ("MoE-block tokens/s (C5: D=4096 E=128 K=8 I=1536 q4 gs64, Zipf(1.1) routing; "
          "one step = 8192-token prefill + 256-token decode forward)")
UNIT = "tokens/s"
L2_FLUSH_BYTES = 512 << 20
DATA = ("synthetic (Philox seed 0): experts N(0,0.02) bf16 -> 4-bit affine gs64 (MLX affine_quantize), "
        "router bf16 N(0,0.02) + fixed Zipf(1.1) logit bias, x N(0,1) bf16")
C2_BATCHES = [1, 8, 64]


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


def _clock_sampler_proc(uuid, stop, ready, out_q, period_s):
    """Runs in its own process (spawned): polls the GPU's SM clock and clock
    event reasons through NVML until `stop` is set, after setting `ready`
    once it polls. Being another process, it takes no time from the
    benchmark's launching thread."""
    samples, err, max_mhz = [], None, None
    try:
        import pynvml as N

        N.nvmlInit()
        h = N.nvmlDeviceGetHandleByUUID(uuid)
        max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
        names = {k: getattr(N, v, 0) for k, v in ClockSampler.REASONS}
        ready.set()
        while not stop.is_set():
            mhz = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
            rs = N.nvmlDeviceGetCurrentClocksEventReasons(h)
            samples.append((mhz, [k for k, bit in names.items() if rs & bit]))
            time.sleep(period_s)
    except Exception as e:  # no NVML: report it instead of a clock
        err = f"nvml unavailable: {e}"[:200]
    ready.set()
    out_q.put((samples, max_mhz, err))


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    5 ms while the timed region runs, in a separate process (the nvidia-smi
    clocks query reads the same counters, but its 200 ms period is longer
    than a timed region). Read-only: no clock or power setting is touched."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.p = None
        self.err = None

    def start(self):
        import multiprocessing as mp

        ctx = mp.get_context("spawn")
        self.stop_ev, self.ready, self.q = ctx.Event(), ctx.Event(), ctx.Queue()
        self.p = ctx.Process(target=_clock_sampler_proc, args=(self.uuid, self.stop_ev, self.ready, self.q, 0.005),
                             daemon=True)
        self.p.start()
        self.ready.wait(timeout=60)  # the sampler polls before the timed region starts
        time.sleep(0.2)

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": "not started"}
        self.stop_ev.set()
        try:
            samples, max_mhz, err = self.q.get(timeout=30)
        except Exception as e:
            samples, max_mhz, err = [], None, f"sampler: {e}"[:200]
        self.p.join(timeout=5)
        sm = [m for m, _ in samples]
        reasons = sorted({r for _, rs in samples for r in rs})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max_mhz, "reasons": reasons,
               "samples": len(sm), "source": "nvml 5 ms, separate process"}
        if not sm:
            out["error"] = err or "no samples"
        return out


def smi_id(torch, dev) -> str:
    """The GPU's UUID (survives CUDA_VISIBLE_DEVICES remapping)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index)


def router_kernels(cfg, T: int, sms: int = 148) -> int:
    """Router launches at T tokens (csrc/moe_block.cu run_router,
    csrc/router_tc.cu router_tc_layout): the fp64 split router up to 64
    tokens; beyond, digit planes + the int8 tensor-core kernel (+ the
    partial-sum finish in its split-K form) + route rows."""
    D, E = cfg.hidden_size, cfg.num_experts
    if T == 0:
        return 0
    if T <= 64 or D >= 32768:
        return 1
    bn = 16 if T <= 256 else 64
    tiles = -(-T // bn) * -(-E // 128)
    split = bn == 16 or tiles * 5 < sms * 4
    return 3 + (1 if split else 0)


def kernels_per_forward(cfg, T: int, sms: int = 148) -> int:
    """Library kernels one block forward launches at T tokens (the launch
    choices of csrc/moe_block.cu: router variant, one-CTA or three-kernel
    permute with or without a separate row gather, split-K / fused / plain
    expert GEMMs, combine, shared expert)."""
    D, E, K, I = cfg.hidden_size, cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size
    R = T * K
    if T == 0:
        return 0
    n = router_kernels(cfg, T, sms)                            # router
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
def ep_kernels_per_forward(cfg, T: int, world: int) -> int:
    """Library kernels one expert-parallel peer-memory step launches on a rank
    with T tokens (the launch choices of the three p2p entry points)."""
    K = cfg.num_experts_per_tok
    n = 1                                                      # ep_bump_epoch (device-resident epoch)
    n += router_kernels(cfg, T)                                # router
    n += 1                                                     # ep_pair_dest
    n += 1 if T * K <= 2048 else 3                             # permute of the pairs by rank
    n += 3                                                     # ep_counts, ep_pair_meta, ep_send
    n += 2                                                     # wait, ep_slot_expert
    n += 1 if world * T * K <= 2048 else 3                     # permute of the received slots
    n += 1 + 2 + 1                                             # row gather, gate|up, down, reduce_send
    n += 2                                                     # wait, combine
    if cfg.shared_expert_intermediate_size:
        n += 1 + 2 + (1 if (T < 256 or (cfg.shared_bits or cfg.bits) == 4) else 0)
    return n


class _Timer:
    """CUDA events around each timed forward on the launching stream."""

    def __init__(self, torch, st):
        self.torch, self.st, self.pairs = torch, st, []

    def begin(self):
        a = self.torch.cuda.Event(enable_timing=True)
        a.record(self.st)
        return a

    def end(self, a, key):
        b = self.torch.cuda.Event(enable_timing=True)
        b.record(self.st)
        self.pairs.append((key, a, b))

    def totals(self):
        out = {}
        for key, a, b in self.pairs:
            out.setdefault(key, []).append(a.elapsed_time(b))
        return out


def run_gpu(args):
    import torch
    import torch.distributed as dist

    from mlxr_moe import synth

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
    # Everything (weight synthesis, inputs, workspaces, forwards) runs on one
    # stream, so the caching allocator never hands a buffer that pending work
    # on another stream still touches to the block.
    st = torch.cuda.Stream(dev)
    torch.cuda.set_stream(st)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    spec = synth.CONFIGS[HEADLINE]
    cfg = spec["cfg"]
    blk = synth.make_block(cfg, seed=0, zipf=spec["zipf"], device=dev)
    torch.cuda.synchronize(dev)
    if world == 1:
        head = headline_one_gpu(args, torch, dev, st, flush, blk, peaks)
    else:
        head = headline_ep(args, torch, dist, dev, st, flush, blk, world, rank)

    extra, ep_extra, cpu = {}, None, None
    if world == 1 and not args.no_cpu:
        cpu = cpu_baseline(blk, head.pop("_inputs"), args)
    head.pop("_inputs", None)
    del blk
    torch.cuda.empty_cache()
    if world == 1 and not args.no_extra:
        extra = bench_extra(args, dev, st, flush, peaks)
    if world > 1 and not args.no_extra:
        ep_extra = bench_ep_extra(args, dev, st, world, rank)
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": DATA,
            "config": {"workload": "c5: one block forward over 8192 prefill tokens + one over 256 decode tokens "
                                   "per step (Zipf(1.1) routing)",
                       "hidden": cfg.hidden_size, "experts": cfg.num_experts, "top_k": cfg.num_experts_per_tok,
                       "moe_intermediate": cfg.moe_intermediate_size, "bits": cfg.bits,
                       "group_size": cfg.group_size, "prefill_tokens": PREFILL_T, "decode_tokens": DECODE_T,
                       "l2": "flushed before every forward (512 MiB write); weights 1.36 GB > L2",
                       "graphs": head["graphs"], "parallelism": head["parallelism"]},
            "roofline": head.get("roofline"),
            "cpu_baseline": cpu,
            "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"],
            "clocks": head["clocks"],
            "forwards": head["forwards"],
            "extra": extra,
            "expert_parallel": ep_extra,
        }
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def e2e_pipelined(args, torch, dev, st, flush, blk, G, nsets):
    """End-to-end rate of the C5 step through Qwen35MoeBlock.forward with
    host buffers (see headline_one_gpu): H2D on one copy stream, the
    forward's graph on `st`, D2H on another copy stream; buffer b of a
    forward kind is refilled only after the graph that read it and the copy
    that drained its output have finished."""
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    host_in = {n: [G[n]["x"][i].cpu().pin_memory() for i in range(nsets)] for n in G}
    host_out = {n: [torch.empty_like(G[n]["out"], device="cpu").pin_memory() for _ in range(nsets)] for n in G}
    B = {}
    for n in G:
        g = G[n]
        bufs = []
        for b in range(nsets):
            xb, ob = torch.empty_like(g["xs"]), torch.empty_like(g["out"])
            xb.copy_(g["x"][b])
            with torch.cuda.stream(st):
                blk.forward(xb, out=ob, workspace=g["ws"])  # warm (same launch shapes as the capture)
            torch.cuda.synchronize(dev)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=st):
                blk.forward(xb, out=ob, workspace=g["ws"])
            ev = {k: torch.cuda.Event() for k in ("in_ready", "done", "out_read")}
            bufs.append(dict(x=xb, out=ob, g=gr, ev=ev, used=False))
        B[n] = bufs
    torch.cuda.synchronize(dev)

    def run(nsteps, s0):
        for s in range(s0, s0 + nsteps):
            for n in ("prefill", "decode"):
                q = B[n][s % nsets]
                ev = q["ev"]
                with torch.cuda.stream(h2d):
                    if q["used"]:
                        h2d.wait_event(ev["done"])  # the graph that read this input has finished
                    q["x"].copy_(host_in[n][s % nsets], non_blocking=True)
                    ev["in_ready"].record(h2d)
                with torch.cuda.stream(st):
                    st.wait_event(ev["in_ready"])
                    if q["used"]:
                        st.wait_event(ev["out_read"])  # this output buffer has been read back
                    flush.fill_(s & 0xFF)
                    q["g"].replay()
                    ev["done"].record(st)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev["done"])
                    host_out[n][s % nsets].copy_(q["out"], non_blocking=True)
                    ev["out_read"].record(d2h)
                q["used"] = True

    run(args.warmup, 0)
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(h2d)
    run(args.steps, args.warmup)
    t1.record(d2h)
    torch.cuda.synchronize(dev)
    e2e_ms = t0.elapsed_time(t1)
    ok = all(torch.equal(host_out[n][(args.warmup + args.steps - 1) % nsets], B[n][(args.warmup + args.steps - 1) % nsets]["out"].cpu())
             for n in G)
    blk.status(G["prefill"]["ws"])
    del B
    D = G["prefill"]["x"][0].shape[-1]
    return {"value": STEP_TOKENS * args.steps / (e2e_ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": STEP_TOKENS * D * 2, "d2h_bytes_per_step": STEP_TOKENS * D * 2,
            "ms_per_step": e2e_ms / args.steps, "outputs_read_back": bool(ok),
            "note": "every forward: pinned host x -> device (copy stream), graph replay of Qwen35MoeBlock.forward "
                    "(mlxr_cu_moe_block_forward), out -> pinned host (second copy stream); copies overlap the "
                    "neighbouring forwards' compute; device time from the first H2D to the last D2H"}


def headline_one_gpu(args, torch, dev, st, flush, blk, peaks):
    """The C5 step on one GPU: two captured graphs (prefill 8192, decode 256)."""
    from mlxr_moe import synth
    from mlxr_moe.moe import Routing
    import ctypes as C

    from mlxr_moe import _lib

    cfg = blk.cfg
    D, K, I = cfg.hidden_size, cfg.num_experts_per_tok, cfg.moe_intermediate_size
    nsets = 2
    G = {}
    with torch.cuda.stream(st):
        for name, T in (("prefill", PREFILL_T), ("decode", DECODE_T)):
            xs = [synth.make_input(T, D, seed=0, stream_offset=(10 if name == "prefill" else 20) + i, device=dev)
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
            r = Routing(T, K, cfg.num_experts, dev)
            blk.forward(xs[0], routing=r, workspace=ws)
            torch.cuda.synchronize(dev)
            blk.status(ws)
            G[name] = dict(T=T, x=xs, xs=x_static, out=out, ws=ws, g=g, U=distinct_experts(r),
                           rows_max=int(r.counts.max().item()))

    def run_steps(nsteps, timer=None):
        with torch.cuda.stream(st):
            for s in range(nsteps):
                for name in ("prefill", "decode"):
                    g = G[name]
                    g["xs"].copy_(g["x"][s % nsets])
                    flush.fill_(s & 0xFF)
                    a = timer.begin() if timer else None
                    g["g"].replay()
                    if timer:
                        timer.end(a, name)

    run_steps(args.warmup)
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(smi_id(torch, dev))
    clocks.start()
    timer = _Timer(torch, st)
    run_steps(args.steps, timer)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    tt = timer.totals()
    total_ms = sum(sum(v) for v in tt.values())
    value = STEP_TOKENS * args.steps / (total_ms / 1e3)

    # Live per-stage timing (stage events recorded between the kernels of a
    # second captured graph of each forward).
    stage = {n: stage_times(torch, C, _lib, blk, G[n]["x"], G[n]["xs"], G[n]["out"], G[n]["ws"], st, flush,
                            max(5, args.steps // 2), dev) for n in G}

    # e2e: the same step through the public API with pinned host buffers,
    # as a serving loop runs it: every forward's input is copied in from
    # pinned host memory and its output read back inside the timed region,
    # on two copy streams that overlap the copies with the neighbouring
    # forwards' compute (double-buffered device inputs and outputs, one
    # captured graph per buffer). Timed from the first host-to-device copy to
    # the last device-to-host copy (events on the device), L2 flushed before
    # every forward as in the device-timed loop.
    e2e = e2e_pipelined(args, torch, dev, st, flush, blk, G, nsets)
    # Roofline of the dominant kernel: the prefill forward's expert GEMMs
    # (grouped_dequant_gemm_kernel, gate|up + SwiGLU then down: two launches),
    # tensor-bound. Algorithmic FLOPs = 2 * 3 * I * D per routed row, rows =
    # 8192 tokens x top-8 (no padding counted).
    R = PREFILL_T * K
    gemm_flops = 2 * 3 * I * D * R
    gemm_ms = stage["prefill"]["gate_up_ms"] + stage["prefill"]["down_ms"]
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12
    tr = ncu_traffic("experts_c5_prefill")
    roofline = dict(bound="tensor", achieved=achieved, peak=peaks["bf16_tflops"], unit="TFLOP/s",
                    frac=achieved / peaks["bf16_tflops"], traffic=tr,
                    kernel="grouped_dequant_gemm_kernel: the C5 prefill forward's expert GEMMs (gate|up + SwiGLU, "
                           "then down), 8192 tokens x top-8 = 65536 routed rows",
                    peak_source=peaks["source"] + " bf16_tflops (cuBLAS burst)",
                    algorithmic_flops_per_forward=gemm_flops,
                    gate_up_ms=stage["prefill"]["gate_up_ms"], down_ms=stage["prefill"]["down_ms"],
                    traffic_note="ncu dram__bytes_read.sum + dram__bytes_write.sum of the two launches of one "
                                 "prefill forward (profiles/*.md)",
                    timing="stage events around the expert GEMM launches inside the captured forward")
    # The decode forward's expert GEMM (one fused launch), HBM-bound.
    dec_bytes = int(G["decode"]["U"] * synth.expert_bytes(cfg) + DECODE_T * K * (D + I) * 2 * 2)
    dec_ms = stage["decode"]["gate_up_ms"] + stage["decode"]["down_ms"]
    roofline["decode_gemm"] = dict(bound="hbm", achieved=dec_bytes / (dec_ms / 1e3) / 1e9, peak=peaks["hbm_gbs"],
                                   unit="GB/s", frac=dec_bytes / (dec_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                                   algorithmic_bytes=dec_bytes, ms=dec_ms)
    forwards = {}
    for n in ("prefill", "decode"):
        T = G[n]["T"]
        ms = statistics.median(tt[n])
        fl = synth.algorithmic_flops(cfg, T)
        by = synth.algorithmic_bytes(cfg, T, G[n]["U"])
        forwards[n] = dict(tokens=T, ms=ms, tokens_per_s=T / (ms / 1e3), tflops=fl / (ms / 1e3) / 1e12,
                           tensor_frac=fl / (ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                           gbs=by / (ms / 1e3) / 1e9, hbm_frac=by / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                           distinct_experts=G[n]["U"], busiest_expert_rows=G[n]["rows_max"],
                           stages_ms={k: round(v, 5) for k, v in stage[n].items()})
    inputs = {"prefill": G["prefill"]["x"][0], "decode": G["decode"]["x"][0]}
    launches = (kernels_per_forward(cfg, PREFILL_T) + kernels_per_forward(cfg, DECODE_T)) * args.steps
    return dict(value=value, ms_per_step=total_ms / args.steps, e2e=e2e, roofline=roofline, clocks=clk,
                forwards=forwards, gpu_launches=launches, graphs="each forward replayed from a captured CUDA graph",
                parallelism="single GPU", _inputs=inputs)


def headline_ep(args, torch, dist, dev, st, flush, blk_full, world, rank):
    """The C5 step expert-parallel over `world` ranks, exchange over peer memory."""
    from mlxr_moe import synth
    from mlxr_moe.ep import ExpertParallelMoeBlock, PeerComm, balanced_placement

    cfg = blk_full.cfg
    D, K = cfg.hidden_size, cfg.num_experts_per_tok
    Tp, Td = PREFILL_T // world, DECODE_T // world
    nsets = 2
    xs = {"prefill": [synth.make_input(PREFILL_T, D, stream_offset=10 + i, device=dev)[rank * Tp:(rank + 1) * Tp]
                      .contiguous() for i in range(nsets)],
          "decode": [synth.make_input(DECODE_T, D, stream_offset=20 + i, device=dev)[rank * Td:(rank + 1) * Td]
                     .contiguous() for i in range(nsets)]}
    # Placement from measured expert loads on a calibration batch (summed over ranks).
    calib = synth.make_input(Tp, D, stream_offset=900 + rank, device=dev)
    idx, _ = blk_full.router(calib)
    loads = torch.bincount(idx.reshape(-1).long(), minlength=cfg.num_experts).to(torch.float64)
    dist.all_reduce(loads)
    place = balanced_placement(loads.cpu().tolist(), world)
    blk = ExpertParallelMoeBlock.from_block(blk_full, rank, world, place)
    comm = PeerComm(rank, world, cap=Tp, hidden=D, k=K)
    exp_rows = {"prefill": max(1, PREFILL_T * K // world), "decode": max(1, DECODE_T * K // world)}
    outs = {n: [torch.empty_like(xs[n][0]) for _ in range(nsets)] for n in xs}
    # Every step uses the comm's device-resident epoch, so that each
    # forward is one captured CUDA graph per (forward, buffer): the host
    # issues one replay per forward, and every rank runs the same steps.
    with torch.cuda.stream(st):
        for n in ("prefill", "decode"):
            for b in range(nsets):  # warm each buffer pair once (sets kernel attributes outside capture)
                blk.forward_p2p(xs[n][b], comm, expected_rows=exp_rows[n], out=outs[n][b], device_epoch=True)
    torch.cuda.synchronize(dev)
    blk.status()
    graphs = {}
    for n in ("prefill", "decode"):
        for b in range(nsets):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=st):
                blk.forward_p2p(xs[n][b], comm, expected_rows=exp_rows[n], out=outs[n][b], device_epoch=True)
            graphs[(n, b)] = gr

    def step(s, timer=None):
        with torch.cuda.stream(st):
            for n in ("prefill", "decode"):
                flush.fill_(s & 0xFF)
                a = timer.begin() if timer else None
                graphs[(n, s % nsets)].replay()
                if timer:
                    timer.end(a, n)

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize(dev)
    blk.status()
    # Only rank 0 samples its GPU's clocks (the line reports rank 0's): one
    # sampling process instead of one per rank, whose NVML polling could
    # delay the other ranks' launches.
    clocks = ClockSampler(smi_id(torch, dev)) if rank == 0 else None
    if clocks:
        clocks.start()
    dist.barrier()
    torch.cuda.synchronize(dev)
    timer = _Timer(torch, st)
    for s in range(args.steps):
        step(s, timer)
    torch.cuda.synchronize(dev)
    dist.barrier()
    torch.cuda.synchronize(dev)
    clk = clocks.stop() if clocks else None
    blk.status()
    tt = timer.totals()
    per = torch.tensor([sum(tt["prefill"]), sum(tt["decode"])], dtype=torch.float64, device=dev)
    med = torch.tensor([statistics.median(tt["prefill"]), statistics.median(tt["decode"]),
                        max(tt["prefill"]), max(tt["decode"])], dtype=torch.float64, device=dev)
    dist.all_reduce(med, op=dist.ReduceOp.MAX)
    tot = per.sum().reshape(1).clone()
    dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    dist.all_reduce(per, op=dist.ReduceOp.MAX)
    total_ms = float(tot.item())
    value = STEP_TOKENS * args.steps / (total_ms / 1e3)
    # e2e with pinned host buffers (this rank's share of the batch), as a
    # serving loop runs it: every forward's input copied in and its output
    # read back inside the timed region, on two copy streams that overlap the
    # copies with the neighbouring forwards (double-buffered inputs and
    # outputs); device time from the first H2D to the last D2H, max over ranks.
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    host_in = {n: [xs[n][i].cpu().pin_memory() for i in range(nsets)] for n in xs}
    host_out = {n: [torch.empty_like(outs[n][0], device="cpu").pin_memory() for _ in range(nsets)] for n in xs}
    bufs = {n: [dict(x=xs[n][b], out=outs[n][b], g=graphs[(n, b)], used=False,
                     ev={k: torch.cuda.Event() for k in ("in_ready", "done", "out_read")}) for b in range(nsets)]
            for n in xs}

    def e2e_steps(s0, nsteps):
        for s in range(s0, s0 + nsteps):
            for n in ("prefill", "decode"):
                q = bufs[n][s % nsets]
                ev = q["ev"]
                with torch.cuda.stream(h2d):
                    if q["used"]:
                        h2d.wait_event(ev["done"])
                    q["x"].copy_(host_in[n][s % nsets], non_blocking=True)
                    ev["in_ready"].record(h2d)
                with torch.cuda.stream(st):
                    st.wait_event(ev["in_ready"])
                    if q["used"]:
                        st.wait_event(ev["out_read"])
                    flush.fill_(s & 0xFF)
                    q["g"].replay()
                    ev["done"].record(st)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev["done"])
                    host_out[n][s % nsets].copy_(q["out"], non_blocking=True)
                    ev["out_read"].record(d2h)
                q["used"] = True

    e2e_steps(0, args.warmup)
    torch.cuda.synchronize(dev)
    blk.status()
    dist.barrier()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(h2d)
    e2e_steps(args.warmup, args.steps)
    t1.record(d2h)
    torch.cuda.synchronize(dev)
    blk.status()
    e = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
    dist.all_reduce(e, op=dist.ReduceOp.MAX)
    e2e = {"value": STEP_TOKENS * args.steps / (float(e.item()) / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": STEP_TOKENS * D * 2, "d2h_bytes_per_step": STEP_TOKENS * D * 2,
           "ms_per_step": float(e.item()) / args.steps,
           "note": "every rank, every forward: its pinned host x share -> device (copy stream), "
                   "ExpertParallelMoeBlock.forward_p2p (mlxr_cu_moe_ep_*_p2p), out -> pinned host (second copy "
                   "stream); copies overlap the neighbouring forwards; max over ranks; bytes summed over ranks"}
    # Phase times of each forward (dispatch, experts, combine): events between
    # the three peer-memory calls on a few extra steps, medians, max over ranks.
    ph = {n: [] for n in xs}
    with torch.cuda.stream(st):
        for s in range(max(3, args.steps // 2)):
            for n in ("prefill", "decode"):
                flush.fill_(s & 0xFF)
                evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
                blk.forward_p2p(xs[n][s % nsets], comm, expected_rows=exp_rows[n], out=outs[n][s % nsets], events=evs,
                                device_epoch=True)
                ph[n].append(evs)
    torch.cuda.synchronize(dev)
    blk.status()
    phase = torch.tensor([[statistics.median(e[j].elapsed_time(e[j + 1]) for e in ph[n]) for j in range(3)]
                          for n in ("prefill", "decode")], dtype=torch.float64, device=dev)
    dist.all_reduce(phase, op=dist.ReduceOp.MAX)
    dist.barrier()
    torch.cuda.synchronize(dev)
    del bufs, graphs
    torch.cuda.synchronize(dev)
    comm.close()
    launches = (ep_kernels_per_forward(cfg, Tp, world) + ep_kernels_per_forward(cfg, Td, world)) * args.steps
    forwards = {n: dict(tokens=T_, tokens_per_rank=Tr, ms=float(per[i].item()) / args.steps,
                        ms_median=float(med[i].item()), ms_max=float(med[2 + i].item()),
                        phases_ms={k: round(float(phase[i, j].item()), 5)
                                   for j, k in enumerate(("dispatch", "experts", "combine"))})
                for i, (n, T_, Tr) in enumerate((("prefill", PREFILL_T, Tp), ("decode", DECODE_T, Td)))}
    return dict(value=value, ms_per_step=total_ms / args.steps, e2e=e2e, roofline=None, clocks=clk,
                forwards=forwards, gpu_launches=launches,
                graphs="each forward one captured CUDA graph (device-resident step epoch)",
                parallelism=f"ep{world}: experts spread over {world} ranks by measured load; tokens split "
                            f"evenly; dispatch/combine over NVLink peer memory inside the kernels")


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

    cache = {}

    def once(key, fn):
        if key not in cache:
            cache.clear()
            torch.cuda.empty_cache()
            cache[key] = fn()
        return cache[key]

    for name, T, make in (("c2_T1", 1, lambda: once("c2", lambda: baseline("c2"))),
                          ("c2_T8", 8, lambda: once("c2", lambda: baseline("c2"))),
                          ("c2_T64", 64, lambda: once("c2", lambda: baseline("c2"))),
                          ("c1", 32, lambda: once("c1", lambda: baseline("c1"))),
                          ("c3", 4096, lambda: once("c3", lambda: baseline("c3"))),
                          ("c4", 16384, lambda: once("c4", lambda: baseline("c4"))),
                          ("gemma4_decode", 64, lambda: once("g4", gemma4)),
                          ("gemma4_prefill", 4096, lambda: once("g4", gemma4))):
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
        if name.startswith("c2_"):
            # expert GEMM bytes: the routed experts' packed weights (all three
            # matrices) plus the x, h and y rows the launches read and write
            K_, I_, D_ = cfg.num_experts_per_tok, cfg.moe_intermediate_size, cfg.hidden_size
            res[name]["expert_gemm_bytes"] = int(U * synth.expert_bytes(cfg) + T * K_ * (D_ + I_) * 2 * 2)
            res[name]["expert_gemm_ms"] = stg["gate_up_ms"] + stg["down_ms"]
        if name == "gemma4_decode" and not args.no_cpu:
            res[name]["cpu_baseline"] = gemma4_cpu_baseline(blk, x)
        del g, ws, out, x, blk
    cache.clear()
    torch.cuda.empty_cache()
    # The decode sweep's expert GEMMs as one HBM roofline (T = 1, 8, 64).
    by = sum(res[f"c2_T{T}"]["expert_gemm_bytes"] for T in C2_BATCHES)
    ms = sum(res[f"c2_T{T}"]["expert_gemm_ms"] for T in C2_BATCHES)
    blk_ms = sum(res[f"c2_T{T}"]["ms"] for T in C2_BATCHES)
    res["c2_sweep"] = dict(tokens_per_s=sum(C2_BATCHES) / (blk_ms / 1e3), block_ms=blk_ms,
                           expert_gemm_gbs=by / (ms / 1e3) / 1e9, expert_gemm_frac=by / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                           expert_gemm_ms=ms, traffic_T64=ncu_traffic("experts_c2_T64"),
                           note="expert GEMM launches (fused gate|up + down at T=8, 64; split-K at T=1), "
                                "stage-event timed, L2 flushed; peak = measured hbm_gbs")
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


def bench_ep_extra(args, dev, st, world, rank):
    """Expert parallelism beside the headline: the C5 step with the exchange
    over NCCL all-to-all (counts, pair rows, slot rows, partial rows), and the
    C4 block (16384 tokens) over peer memory; strong scaling, max over ranks."""
    import torch
    import torch.distributed as dist

    from mlxr_moe import synth
    from mlxr_moe.ep import ExpertParallelMoeBlock, PeerComm, TorchDistExchange, balanced_placement

    ex = TorchDistExchange()
    res = {}
    for name, key, T_total, via in (("c5_prefill_nccl", "c5", PREFILL_T, "nccl"), ("c4", "c4", 16384, "p2p")):
        spec = synth.CONFIGS[key]
        cfg = spec["cfg"]
        D, K = cfg.hidden_size, cfg.num_experts_per_tok
        T = T_total // world
        full = synth.make_block(cfg, 0, spec["zipf"], dev)
        xs = [synth.make_input(T, D, stream_offset=500 + 16 * rank + i, device=dev) for i in range(2)]
        calib = synth.make_input(T, D, stream_offset=900 + rank, device=dev)
        idx, _ = full.router(calib)
        loads = torch.bincount(idx.reshape(-1).long(), minlength=cfg.num_experts).to(torch.float64)
        dist.all_reduce(loads)
        place = balanced_placement(loads.cpu().tolist(), world)
        blk = ExpertParallelMoeBlock.from_block(full, rank, world, place)
        n_steps = max(5, args.steps // 2)
        comm = PeerComm(rank, world, cap=T, hidden=D, k=K) if via == "p2p" else None
        bounds = dict(max_recv_pairs=world * T, max_recv_rows=world * T * K)

        def fn(xx):
            if via == "p2p":
                return blk.forward_p2p(xx, comm, expected_rows=max(1, T_total * K // world))
            return blk.forward(xx, ex, **bounds)

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
        ms = float(t.item())
        dist.barrier()
        if comm is not None:
            comm.close()
        fl = synth.algorithmic_flops(cfg, T_total)
        res[name] = dict(tokens=T_total, tokens_per_rank=T, ms=ms, tokens_per_s=T_total / (ms / 1e3),
                         tflops_total=fl / (ms / 1e3) / 1e12, exchange=via, zipf=spec["zipf"])
        del blk, full, xs
        torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------- CPU baseline ----
def _c5_sample_sizes():
    """The bounded CPU sample of one C5 step: 1/32 of each batch (256 prefill
    and 8 decode tokens), so prefill and decode keep the step's proportions."""
    return PREFILL_T // 32, DECODE_T // 32


def cpu_baseline(blk, inputs, args):
    """The oracle (CPU restatement of the reference block, fused-fp32 mode,
    OpenMP on every host core) on a bounded sample of the C5 step."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle as O
    from gpu_helpers import block_to_oracle

    from conftest import bf16_np

    cfg, W = block_to_oracle(blk)
    cores = O.max_threads()
    sp, sd = _c5_sample_sizes()
    xp = bf16_np(inputs["prefill"][:sp])
    xd = bf16_np(inputs["decode"][:sd])
    times = []
    for rep in range(3):
        t0 = time.perf_counter()
        O.moe_block(cfg, W, xp, "fused")
        O.moe_block(cfg, W, xd, "fused")
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"value": (sp + sd) / sec, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"3 runs of {sp} prefill + {sd} decode tokens of the C5 step (1/32 of each batch), median; "
                      f"oracle fused-fp32 mode, OpenMP {cores} threads"}


def _oracle_c5_block():
    """The C5 block's weights generated on the host by the oracle (same
    Philox streams and quantiser as the GPU arm's synth.make_block)."""
    import numpy as np

    import oracle as O

    D, E, K, I = 4096, 128, 8, 1536
    W = {"router": O.normal_bf16(0, 0, (E, D), 0.02)}
    for name, stream, shape in (("gate", 1, (E, I, D)), ("up", 2, (E, I, D)), ("down", 3, (E, D, I))):
        W[name] = O.quantize(O.normal_bf16(0, stream, shape, 0.02), 64, 4)
    keys = O.bf16_to_f32(O.normal_bf16(0, 9, (E,), 1.0))
    order = np.argsort(keys, kind="stable")
    ranks = np.empty(E, np.int64)
    ranks[order] = np.arange(1, E + 1)
    beta, s = 0.62, 1.1
    W["router_bias"] = (-(beta * 0.02 * np.sqrt(D) * s) * np.log(ranks.astype(np.float64))).astype(np.float32)
    cfg = dict(hidden=D, num_experts=E, top_k=K, moe_intermediate=I, group_size=64, bits=4)
    return cfg, W


def run_reference(args):
    """--impl reference: the CPU port of the reference block (MLX's own CPU
    path cannot be built here) timed on all host cores; rank 0 only. Each step
    is the bounded sample of the C5 step (1/32 of the prefill and decode
    batches, fresh tokens per step)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    cfg, W = _oracle_c5_block()
    sp, sd = _c5_sample_sizes()
    nsets = 2
    xp = [O.normal_bf16(0, 8 + 16 * (10 + i), (PREFILL_T, 4096), 1.0)[:sp] for i in range(nsets)]
    xd = [O.normal_bf16(0, 8 + 16 * (20 + i), (DECODE_T, 4096), 1.0)[:sd] for i in range(nsets)]
    cores = O.max_threads()
    for s in range(args.warmup):
        O.moe_block(cfg, W, xp[s % nsets], "fused")
        O.moe_block(cfg, W, xd[s % nsets], "fused")
    t0 = time.perf_counter()
    for s in range(args.steps):
        O.moe_block(cfg, W, xp[s % nsets], "fused")
        O.moe_block(cfg, W, xd[s % nsets], "fused")
    sec = time.perf_counter() - t0
    value = (sp + sd) * args.steps / sec
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * sec / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": DATA,
        "config": {"workload": "c5: one block forward over 8192 prefill tokens + one over 256 decode tokens "
                               "per step (Zipf(1.1) routing)",
                   "hidden": 4096, "experts": 128, "top_k": 8, "moe_intermediate": 1536, "bits": 4, "group_size": 64,
                   "prefill_tokens": PREFILL_T, "decode_tokens": DECODE_T,
                   "host": f"CPU, {cores} threads (rank 0 only; the GPUs are unused)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"each step {sp} prefill + {sd} decode tokens (1/32 of each batch of the C5 step) "
                                   f"through the oracle (CPU restatement; MLX unbuildable here), fused-fp32"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def _case_ep1(cfg_name: str, T: int, iters: int):
    """Expert-parallel peer-memory steps with a world-1 communicator (the
    rank's own exchange buffer, no other process): every ep_* kernel runs on
    this GPU, for ncu captures."""
    import ctypes as C

    import torch

    from mlxr_moe import _lib, synth
    from mlxr_moe.ep import ExpertParallelMoeBlock

    spec = synth.CONFIGS[cfg_name]
    full = synth.make_block(spec["cfg"], 0, spec["zipf"])
    cfg = full.cfg
    blk = ExpertParallelMoeBlock.from_block(full, 0, 1)

    class _Comm:
        pass

    comm = _Comm()
    comm.comm, comm.cap, comm.epoch = C.c_void_p(), T, 0
    handle = (C.c_uint8 * 64)()
    _lib.call("mlxr_cu_ep_comm_create", 1, 0, T, cfg.hidden_size, cfg.num_experts_per_tok, C.byref(comm.comm), handle)
    x = synth.make_input(T, cfg.hidden_size)
    for _ in range(iters):
        blk.forward_p2p(x, comm)
    torch.cuda.synchronize()
    blk.status()
    _lib.call("mlxr_cu_ep_comm_destroy", comm.comm)


def _case_ops(iters: int):
    """The op family (quantize, dequantize, quantized_matmul, gather_qmm,
    gather_mm) at C2 expert shapes, for ncu captures."""
    import torch

    from mlxr_moe import ops, synth

    w = synth.ops.synth_normal_bf16(0, 1, (16, 768, 2048), 0.02)
    x = synth.make_input(64, 2048)
    idx = torch.arange(64, dtype=torch.int32, device="cuda") % 16
    for _ in range(iters):
        wq, s, b = ops.quantize(w, 64, 4)
        wd = ops.dequantize(wq[0], s[0], b[0], 64, 4)
        ops.quantized_matmul(x, wq[0], s[0], b[0], True, 64, 4)
        ops.gather_qmm(x.reshape(64, 1, 2048), wq, s, b, None, idx, True, 64, 4)
        ops.gather_mm(x.reshape(64, 1, 2048), wd.t().contiguous().reshape(1, 2048, 768), None, None)
    torch.cuda.synchronize()


def run_case(args):
    """Block forwards of one configuration, for ncu captures (not a bench
    number). CONFIG:TOKENS for a block forward; ep1:CONFIG:TOKENS for the
    expert-parallel peer-memory step of one rank; ops for the op family."""
    import torch

    from mlxr_moe import synth

    if args.case == "ops":
        _case_ops(args.iters)
        print(f"case ops: {args.iters} rounds ok")
        return
    if args.case.startswith("ep1:"):
        _, cname, T = args.case.split(":")
        _case_ep1(cname, int(T), args.iters)
        print(f"case {args.case}: {args.iters} steps ok")
        return
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
                    help="profiling driver: CONFIG:TOKENS (e.g. c5:8192, gemma4:64); runs only block forwards, prints nothing timed")
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
