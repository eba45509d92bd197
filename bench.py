"""Benchmark of the verify-pass hot path on B200 (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tsb|reference]

Headline workload (the verify-pass qmm sweep the headline metric is quoted on): one
step = the 4-bit g64 quantized matmul at every M in {1, 8, 16, 32, 64} on each
of the shapes (N, K) = (6144, 5120), (34816, 5120), (5120, 17408): 15 calls.
metric = algorithmic bytes of those calls (codes + scales/biases + x + y) per
second, in TB/s. Inputs: seeded synthetic (x ~ N(0,1) bf16, W ~ N(0, 0.02)
quantized); weights rotate through a pool of copies much larger than L2, so
no call reads another call's weights from L2.

At N > 1 GPUs (one process per GPU, torchrun) every weight is N-sharded by
output rows and each layer's output is reassembled on every GPU inside the
timed region by the qmm kernel itself, which stores its columns into every
rank's output over NVLink (total work fixed: strong scaling).

`--impl reference` times the reference's algorithm on the host CPU (the oracle
port: dequantize + float32 matmul over all host threads; the reference's own
kernels are Metal and cannot run here) on a bounded sample of the same
workload, with the same metric and unit.
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
PKG = os.path.join(ROOT, "mlx-tree-spec_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

SHAPES = ((6144, 5120), (34816, 5120), (5120, 17408))
SWEEP_M = (1, 8, 16, 32, 64)
METRIC = "4-bit qmm HBM TB/s (M<=64 verify sweep)"
WORKLOAD = ("verify-pass qmm sweep: M in {1,8,16,32,64} x (N,K) in "
            "{(6144,5120),(34816,5120),(5120,17408)}, 4-bit g64 MLX format")
UNIT = "TB/s"


def alg_bytes(m, n, k):
    return n * k // 2 + n * (k // 64) * 4 + m * k * 2 + m * n * 2


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ helpers

def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


class WeightPool:
    """Per shape, `copies` distinct device copies of this rank's row shard."""

    def __init__(self, world, rank, copies_for, seed=1000):
        import torch

        import tsb

        self.shards = {}
        for (n, k) in SHAPES:
            ns = n // world
            torch.manual_seed(seed + n + k)
            wf = torch.randn(n, k, device="cuda") * 0.02
            wq, s, b = tsb.quantize(wf[rank * ns:(rank + 1) * ns])
            del wf
            c = copies_for(ns, k)
            self.shards[(n, k)] = [(wq, s, b)] + [(wq.clone(), s.clone(), b.clone()) for _ in range(c - 1)]
        torch.cuda.synchronize()


def copies_needed(ns, k, l2_bytes=126 * 2**20, factor=2.5):
    per = ns * k // 2 + ns * (k // 64) * 4
    return max(5, int(-(-factor * l2_bytes // per)))


# ------------------------------------------------------------------ tsb arm

def make_cache(fmt, kf, vf, n_kv):
    """A config-4 KV cache of the given format from float K/V (B, Hkv, rows, D)."""
    import torch

    import tsb

    if fmt == "bf16":
        return tsb.KVCache(kf.to(torch.bfloat16), vf.to(torch.bfloat16), n_kv)
    if fmt == "ref_q8":
        kq, ks = tsb.quantize_rows(kf)
        vq, vs = tsb.quantize_rows(vf)
        return tsb.Q8KVCache(kq, vq, ks, vs, n_kv)
    kw, ks, kb = tsb.quantize_g64(kf)
    vw, vs, vb = tsb.quantize_g64(vf)
    return tsb.MLXQ8KVCache(kw, vw, ks, kb, vs, vb, n_kv)


def run_profile_attn(args):
    """Config-4 tree attention (B=1, L=32768, T=32, 24q/4kv, D=256, KV format
    --attn-kv): --warmup calls, then one."""
    import numpy as np
    import torch

    import tsb
    from oracle import gen

    torch.cuda.set_device(0)
    tsb.load_library()
    bsz, L, t, hq, hkv, d = 1, 32768, 32, 24, 4, 256
    n_kv = L + t
    g = torch.Generator(device="cuda").manual_seed(3)
    kf = torch.randn(bsz, hkv, n_kv, d, device="cuda", generator=g)
    vf = torch.randn(bsz, hkv, n_kv, d, device="cuda", generator=g)
    q = torch.randn(bsz, hq, t, d, device="cuda", generator=g).to(torch.bfloat16)
    parents = torch.from_numpy(np.stack([gen.tree_parents(np.random.default_rng(i), t) for i in range(bsz)])).cuda()
    cache = make_cache(args.attn_kv, kf, vf, n_kv)
    del kf, vf
    for _ in range(args.warmup + 1):
        tsb.tree_flash(q, cache, d**-0.5, parents=parents)
    torch.cuda.synchronize()
    print(json.dumps({"profile": "attn", "kv": args.attn_kv, "calls": args.warmup + 1}))


def run_profile_prefill(args):
    """Config-3 prefill (M = 4096, 5120x17408: the shape with a split tail):
    --warmup calls, then one."""
    import torch

    import tsb
    from tsb import ops

    torch.cuda.set_device(0)
    tsb.load_library()
    m, n, k = 4096, 5120, 17408
    torch.manual_seed(3)
    wq, s, b = tsb.quantize(torch.randn(n, k, device="cuda") * 0.02)
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    for _ in range(args.warmup + 1):
        ops.quantized_matmul_into(x, wq, s, b, y, n)
    torch.cuda.synchronize()
    print(json.dumps({"profile": "prefill", "shape": [m, n, k], "calls": args.warmup + 1}))


def run_tsb(args):
    import numpy as np
    import torch

    import tsb
    from tsb import dist as tdist
    from tsb import ops

    world, rank, local = dist_setup()
    hbm_peak, bf16_peak, peak_src = load_peaks()
    lib = tsb.load_library()
    pool = WeightPool(world, rank, copies_needed)
    calls = [(m, n, k) for m in SWEEP_M for (n, k) in SHAPES]
    total_bytes = sum(alg_bytes(m, n, k) for (m, n, k) in calls)

    gen = torch.Generator(device="cuda").manual_seed(7)
    xs = {(m, k): torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16)
          for m in SWEEP_M for k in {k for _, k in SHAPES}}
    # N > 1: the output of every call is gathered inside the qmm kernel (peer
    # stores into every rank's y over NVLink); no separate collective
    sharded = tdist.GatheredQMM(world, rank) if world > 1 else None
    if sharded is None:
        ys = {(m, n): torch.empty(m, n, dtype=torch.bfloat16, device="cuda") for (m, n, k) in calls}
    else:
        ys = {(m, n): sharded.out_buffer(m, n) for (m, n, k) in calls}

    def launch(m, n, k, copy, y=None):
        wq, s, b = pool.shards[(n, k)][copy % len(pool.shards[(n, k)])]
        x = xs[(m, k)]
        out = ys[(m, n)] if y is None else y
        if sharded is None:
            return ops.quantized_matmul_into(x, wq, s, b, out, n)
        return sharded.forward_into(x, wq, s, b, out)

    # one step = the 15 calls, each shape cycling through its copies
    def step(offset=0):
        used = {}
        for (m, n, k) in calls:
            c = used.get((n, k), 0)
            used[(n, k)] = c + 1
            launch(m, n, k, c + offset)

    # warm-up (eager; sets kernel attributes, checks every call runs)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    if args.profile == "qmm":
        step(args.warmup)
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"profile": "qmm", "launches_per_step": len(calls), "warmup_steps": args.warmup}))
        return

    # CUDA graph of one step (kernel launches only; collectives use NCCL in-graph)
    g = torch.cuda.CUDAGraph()
    s_cap = torch.cuda.Stream()
    s_cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_cap):
        step(0)  # warm the side stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s_cap):
            step(0)
    torch.cuda.current_stream().wait_stream(s_cap)
    torch.cuda.synchronize()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        g.replay()
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = t0.elapsed_time(t1) / args.steps
    clk = clocks.stop()
    # a CUDA graph that holds NCCL calls must be released before the process
    # group is destroyed, or the exit waits for good
    del g
    torch.cuda.synchronize()
    ms = max_over_ranks(ms, world)
    value = total_bytes / (ms * 1e-3) / 1e12

    # per-call device time (graphs rotating through distinct weight copies)
    per_call = {}
    qmm_kernel_us = 0.0
    for (m, n, k) in calls:
        reps = len(pool.shards[(n, k)])
        gc = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(gc, stream=s_cap):
                for c in range(reps):
                    launch(m, n, k, c)
        torch.cuda.current_stream().wait_stream(s_cap)
        gc.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        loops = 10
        e0.record()
        for _ in range(loops):
            gc.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (loops * reps)
        us = max_over_ranks(us, world)
        per_call[f"M{m}_{n}x{k}"] = {"us": round(us, 3),
                                      "GB/s": round(alg_bytes(m, n, k) / (us * 1e-6) / 1e9, 1)}
        qmm_kernel_us += us
        del gc
    achieved_gbs = total_bytes / (qmm_kernel_us * 1e-6) / 1e9

    # end to end through the public API: pinned host x in, y back to pinned host
    host_x = {key: t.cpu().pin_memory() for key, t in xs.items()}
    host_y = {key: torch.empty(t.shape, dtype=t.dtype).pin_memory() for key, t in ys.items()}
    h2d = sum(m * k * 2 for (m, n, k) in calls)
    d2h = sum(m * n * 2 for (m, n, k) in calls)

    # A serving loop's overlap of the host link with compute: the step's input
    # copies go out on a copy stream, each call waits only for its own input,
    # and each output goes back on a second stream behind its call, so copies
    # and matmuls of different calls overlap (every byte still crosses the
    # link inside the step; measured ~16% faster than one serial stream).
    cs_in, cs_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in calls]
    ev_out = [torch.cuda.Event() for _ in calls]

    def e2e_step():
        cur = torch.cuda.current_stream()
        cs_in.wait_stream(cur)
        xds = []
        with torch.cuda.stream(cs_in):
            for i, (m, n, k) in enumerate(calls):
                xds.append(host_x[(m, k)].to("cuda", non_blocking=True))
                ev_in[i].record(cs_in)
        used = {}
        for i, (m, n, k) in enumerate(calls):
            c = used.get((n, k), 0)
            used[(n, k)] = c + 1
            wq, s, b = pool.shards[(n, k)][c % len(pool.shards[(n, k)])]
            cur.wait_event(ev_in[i])
            xds[i].record_stream(cur)
            if sharded is None:
                y = tsb.quantized_matmul(xds[i], wq, s, b)
            else:
                y = sharded.forward(xds[i], wq, s, b)
            ev_out[i].record(cur)
            cs_out.wait_event(ev_out[i])
            with torch.cuda.stream(cs_out):
                host_y[(m, n)].copy_(y, non_blocking=True)
            if sharded is None:  # (the gathered outputs are persistent per-shape buffers; the step's end orders them)
                y.record_stream(cs_out)
        cs_out.synchronize()
        cur.wait_stream(cs_out)

    for _ in range(2):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max(e0.elapsed_time(e1), (time.perf_counter() - w0) * 1e3) / args.steps
    e2e_ms = max_over_ranks(e2e_ms, world)
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e12

    launches_per_step = len(calls)  # one qmm kernel per call

    secondary = {}
    if args.secondary and world > 1:
        secondary = run_dist_secondary(world, rank, pool, xs, total_bytes, bf16_peak)
    if args.secondary and rank == 0 and world == 1:
        secondary = run_secondary(pool, xs, hbm_peak, bf16_peak)

    cpu = None
    if rank == 0 and world == 1 and args.cpu_baseline:
        cpu = cpu_baseline_sample()

    traffic = read_traffic()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD,
                       "bytes_per_step": total_bytes, "calls_per_step": len(calls),
                       "l2": "inputs larger than L2: rotating weight pool, >= 2.5 x 126 MiB of distinct copies per shape",
                       "parallelism": (f"N-shard x{world}, output gathered inside the qmm kernel (peer stores "
                                       "over NVLink)") if world > 1 else "single GPU",
                       "timing": "CUDA graph of one step, CUDA events"},
            "e2e": {"value": round(e2e_value, 4), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4), "path": "tsb.quantized_matmul, pinned host x/y, eager; input copies on a copy stream, "
                            "output copies on a second stream, per-call events"},
            "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved_gbs / hbm_peak, 4), "traffic": traffic,
                         "kernel": "qmm_ts_kernel", "peak_source": peak_src,
                         "traffic_basis": "dram read+write bytes per step (15 launches) from one ncu capture "
                                          "(profiles/qmm_verify_sweep_traffic.txt); algorithmic bytes per step "
                                          f"{total_bytes}",
                         "basis": "sum of algorithmic bytes / sum of per-call device time over the 15 calls"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "per_call": per_call,
        }
        if secondary:
            line["secondary"] = secondary
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def read_traffic():
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "qmm_verify_sweep_traffic.txt")
    try:
        for ln in open(p):
            if ln.startswith("traffic_bytes_per_step:"):
                return float(ln.split(":")[1])
    except OSError:
        pass
    return None


def time_graph(fn, loops=10):
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(loops):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / loops  # us per replay


def build_decoder(fmt: str, layers: int = 16, seed: int = 1005):
    """The decoder workload: random-init 4-bit decoder, 4 requests x 32 tree nodes
    over an 8K prefix per request (KV ~ N(0,1) in the given format)."""
    import numpy as np
    import torch

    import tsb
    from oracle import gen
    from tsb import decoder as tdec

    cfg = tdec.DecoderConfig(layers=layers)
    weights, final_norm = tdec.random_weights(cfg, seed=seed)
    b, t, prefix = 4, 32, 8192
    cap = prefix + t
    code = {"bf16": tsb.TSB_KV_BF16, "mlx_q8": tsb.TSB_KV_MLX_Q8_G64, "ref_q8": tsb.TSB_KV_REF_Q8_ROW}[fmt]
    g = torch.Generator(device="cuda").manual_seed(seed)
    caches = []
    for _ in range(cfg.layers):
        kf = torch.randn(b, cfg.hkv, cap, cfg.d, device="cuda", generator=g)
        vf = torch.randn(b, cfg.hkv, cap, cfg.d, device="cuda", generator=g)
        caches.append(tdec.make_cache(kf, vf, prefix, code))
        del kf, vf
    rng = np.random.default_rng(seed)
    parents = torch.from_numpy(np.stack([gen.tree_parents(rng, t) for _ in range(b)]).astype(np.int32)).cuda()
    h0 = torch.randn(b * t, cfg.hidden, device="cuda", generator=g).to(torch.bfloat16)
    return tdec.VerifyDecoder(cfg, weights, final_norm), h0, parents, caches, prefix


def time_decoder_step(fmt: str):
    """µs per verify step of config 5 (one CUDA graph per step)."""
    import torch

    dec, h0, parents, caches, prefix = build_decoder(fmt)
    us = time_graph(lambda: dec.step(h0, parents, caches, prefix), loops=5)
    n = dec.cfg.layers
    del dec, caches
    torch.cuda.empty_cache()
    return us, n


def run_profile_decoder(args):
    """Config-5 decoder step (bf16 KV): --warmup steps, then one (for ncu)."""
    import torch

    import tsb

    torch.cuda.set_device(0)
    tsb.load_library()
    dec, h0, parents, caches, prefix = build_decoder("bf16")
    for _ in range(args.warmup + 1):
        dec.step(h0, parents, caches, prefix)
    torch.cuda.synchronize()
    print(json.dumps({"profile": "decoder", "steps": args.warmup + 1}))


def run_secondary(pool, xs, hbm_peak, bf16_peak):
    """M=128 sweep, prefill M=4096, tree attention (config 4): reported beside
    the headline, not part of it."""
    import torch

    import tsb
    from tsb import ops

    out = {}
    # M = 128 (tensor-bound past M ~ 70)
    for (n, k) in SHAPES:
        x = torch.randn(128, k, device="cuda").to(torch.bfloat16)
        y = torch.empty(128, n, dtype=torch.bfloat16, device="cuda")
        copies = pool.shards[(n, k)]

        def f():
            for (wq, s, b) in copies:
                ops.quantized_matmul_into(x, wq, s, b, y, n)

        us = time_graph(f) / len(copies)
        out[f"qmm_M128_{n}x{k}"] = {"us": round(us, 2), "TFLOP/s": round(2 * 128 * n * k / us / 1e6, 1),
                                    "GB/s": round(alg_bytes(128, n, k) / us / 1e3, 1)}
    # prefill M = 4096
    for (n, k) in ((34816, 5120), (5120, 17408)):
        x = torch.randn(4096, k, device="cuda").to(torch.bfloat16)
        y = torch.empty(4096, n, dtype=torch.bfloat16, device="cuda")
        wq, s, b = pool.shards[(n, k)][0]
        us = time_graph(lambda: ops.quantized_matmul_into(x, wq, s, b, y, n), loops=3)
        tf = 2 * 4096 * n * k / us / 1e6
        out[f"prefill_M4096_{n}x{k}"] = {"us": round(us, 1), "TFLOP/s": round(tf, 1),
                                         "frac_of_bf16_peak": round(tf / bf16_peak, 4)}
    # tree attention, config 4: T=32, 24q/4kv, D=256
    from oracle import gen
    import numpy as np

    for (bsz, L, fmt) in ((1, 32768, "bf16"), (4, 8192, "bf16"), (1, 32768, "mlx_q8"), (4, 8192, "mlx_q8"),
                          (1, 32768, "ref_q8")):
        t, hq, hkv, d = 32, 24, 4, 256
        n_kv = L + t
        caches = []
        for i in range(4):  # rotate 4 caches so K/V are not L2-resident
            kf = torch.randn(bsz, hkv, n_kv, d, device="cuda")
            vf = torch.randn(bsz, hkv, n_kv, d, device="cuda")
            caches.append(make_cache(fmt, kf, vf, n_kv))
            del kf, vf
        q = torch.randn(bsz, hq, t, d, device="cuda").to(torch.bfloat16)
        parents = torch.from_numpy(np.stack([gen.tree_parents(np.random.default_rng(i), t) for i in range(bsz)])).cuda()

        def f():
            for c in caches:
                tsb.tree_flash(q, c, d**-0.5, parents=parents)

        us = time_graph(f) / len(caches)
        # the same kernel with the mask disabled (no tree rows: every key visible),
        # the unmasked comparator of the 1.3x target
        zero_bits = torch.zeros(t, dtype=torch.int64, device="cuda")

        def fu():
            for c in caches:
                tsb.tree_flash(q, c, d**-0.5, bits=zero_bits, tail=0)

        us_u = time_graph(fu) / len(caches)
        row = {"bf16": 512, "mlx_q8": 272, "ref_q8": 260}[fmt]
        byts = bsz * n_kv * hkv * row * 2 + 2 * bsz * t * hq * d * 2
        fl = 4.0 * bsz * t * hq * n_kv * d
        out[f"attn_B{bsz}_L{L}_{fmt}"] = {"us": round(us, 2), "GB/s": round(byts / us / 1e3, 1),
                                          "TFLOP/s": round(fl / us / 1e6, 1),
                                          "frac_hbm": round(byts / us / 1e3 / hbm_peak, 4),
                                          "us_unmasked": round(us_u, 2),
                                          "masked_over_unmasked": round(us / us_u, 3)}
        del caches
    # verify-step decoder, config 5: 16 layers over 4 requests x 32 nodes at 8K
    for fmt in ("bf16", "mlx_q8"):
        try:
            us, layers = time_decoder_step(fmt)
            out[f"decoder_step_config5_{fmt}"] = {
                "us": round(us, 1), "layers": layers, "rows": 128, "context": 8192,
                "note": "one CUDA graph per step: per layer 4 qmm (qkv 14336x5120, o 5120x6144, gate_up "
                        "34816x5120, down 5120x17408 at M=128), qkv_prep, tree attention, gate, swiglu, "
                        "2 add_rms_norm"}
        except Exception as e:  # pragma: no cover - reported, not fatal
            out[f"decoder_step_config5_{fmt}"] = {"error": str(e)[:200]}
    # unmasked attention comparator: torch SDPA on the same shape and the same 4 KV
    # heads (enable_gqa), bf16, no mask, K/V rotating through 4 caches like ours
    try:
        bsz, L, t, hq, hkv, d = 1, 32768, 32, 24, 4, 256
        kv = [(torch.randn(bsz, hkv, L + t, d, device="cuda").to(torch.bfloat16),
               torch.randn(bsz, hkv, L + t, d, device="cuda").to(torch.bfloat16)) for _ in range(4)]
        q = torch.randn(bsz, hq, t, d, device="cuda").to(torch.bfloat16)
        sdpa = torch.nn.functional.scaled_dot_product_attention
        us = time_graph(lambda: [sdpa(q, k_, v_, enable_gqa=True) for (k_, v_) in kv]) / len(kv)
        byts = bsz * (L + t) * hkv * 512 * 2 + 2 * bsz * t * hq * d * 2
        out["sdpa_gqa_unmasked_B1_L32768_bf16"] = {"us": round(us, 2), "GB/s": round(byts / us / 1e3, 1),
                                                   "note": "torch scaled_dot_product_attention, enable_gqa, no mask"}
        try:
            from flash_attn import flash_attn_func

            qf = q.transpose(1, 2).contiguous()
            kvf = [(k_.transpose(1, 2).contiguous(), v_.transpose(1, 2).contiguous()) for (k_, v_) in kv]
            us_fa = time_graph(lambda: [flash_attn_func(qf, k_, v_) for (k_, v_) in kvf]) / len(kvf)
            out["flash_attn_unmasked_B1_L32768_bf16"] = {"us": round(us_fa, 2), "GB/s": round(byts / us_fa / 1e3, 1),
                                                         "note": "flash_attn.flash_attn_func (library), GQA, no mask"}
            del kvf
        except Exception as e:  # pragma: no cover - library comparator only
            out["flash_attn_unmasked_B1_L32768_bf16"] = {"error": str(e)[:160]}
        del kv
    except Exception as e:  # pragma: no cover - comparator only
        out["sdpa_gqa_unmasked"] = {"error": str(e)[:160]}
    return out


def run_dist_secondary(world, rank, pool, xs, total_bytes, bf16_peak):
    """At N > 1, on every rank (the same collectives in the same order): the
    sweep in the NCCL form (each rank's shard, then an all-gather and a re-layout
    into the full output) beside the in-kernel gather of the headline, and
    config 3 (prefill, M = 4096) N-sharded: the GEMM storing its tiles into
    every rank's output (one kernel), and beside it the NCCL all-gather forms."""
    import torch

    import tsb
    from tsb import dist as tdist
    from tsb import ops

    out = {}
    sq = tdist.ShardedQMM(world, rank)
    gq = tdist.GatheredQMM(world, rank)
    calls = [(m, n, k) for m in SWEEP_M for (n, k) in SHAPES]
    ys = {(m, n): torch.empty(m, n, dtype=torch.bfloat16, device="cuda") for (m, n, k) in calls}

    def step():
        used = {}
        for (m, n, k) in calls:
            c = used.get((n, k), 0)
            used[(n, k)] = c + 1
            wq, s, b = pool.shards[(n, k)][c % len(pool.shards[(n, k)])]
            sq.forward_into(xs[(m, k)], wq, s, b, ys[(m, n)])

    def timed(fn, reps):
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) * 1e3 / reps, world)  # us

    for _ in range(3):
        step()
    us = timed(step, 10)
    out["sweep_nccl_allgather"] = {"TB/s": round(total_bytes / us / 1e6, 4), "us_per_step": round(us, 1),
                                   "note": "same 15 calls: shard matmul + NCCL all_gather + re-layout, eager"}
    m = 4096
    for (n, k) in ((34816, 5120), (5120, 17408)):
        ns = n // world
        g = torch.Generator(device="cuda").manual_seed(4000 + n + rank)
        wq, s, b = tsb.quantize(torch.randn(ns, k, device="cuda", generator=g) * 0.02)
        gx = torch.Generator(device="cuda").manual_seed(4100 + n)
        x = torch.randn(m, k, device="cuda", generator=gx).to(torch.bfloat16)
        y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        local = torch.empty(m, ns, dtype=torch.bfloat16, device="cuda")
        res = {}
        for chunks in (1, 4):
            def f(chunks=chunks):
                sq.forward_into(x, wq, s, b, y, chunks=chunks)
            f()
            res[chunks] = timed(f, 3)
        # the fused form: the GEMM stores every tile into every rank's output
        yg = gq.out_buffer(m, n)
        gq.forward_into(x, wq, s, b, yg)
        us_fused = timed(lambda: gq.forward_into(x, wq, s, b, yg), 3)
        ops.quantized_matmul_into(x, wq, s, b, local, ns)
        us_local = timed(lambda: ops.quantized_matmul_into(x, wq, s, b, local, ns), 3)
        tf = 2.0 * m * n * k / us_fused / 1e6
        out[f"prefill_M4096_{n}x{k}_N{world}"] = {
            "us": round(us_fused, 1), "TFLOP/s": round(tf, 1),
            "frac_of_bf16_peak_per_gpu": round(tf / world / bf16_peak, 4),
            "us_shard_matmul_alone": round(us_local, 1),
            "us_nccl_one_block": round(res[1], 1), "us_nccl_four_blocks_overlapped": round(res[4], 1),
            "note": "N-sharded, full [M, N] output on every rank; us/TFLOP/s: the GEMM storing each tile into "
                    "every rank's output over NVLink (one kernel); the NCCL all_gather forms beside it"}
        del wq, s, b, x, y, local
    return out


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_sweep_data(rng):
    """Inputs of one verify sweep for the oracle port: x per (M, K), one packed
    weight per shape (random codes; scale 2^-7 and bias -2^-6 per group)."""
    import numpy as np

    from oracle import gen

    xs = {(m, k): gen.x_bf16(rng, m, k) for m in SWEEP_M for k in {k for _, k in SHAPES}}
    ws = {}
    for (n, k) in SHAPES:
        wq = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32)
        s = np.full((n, k // 64), 0x3C00, dtype=np.uint16)  # bf16 0.0078125
        b = np.full((n, k // 64), 0xBC80, dtype=np.uint16)
        ws[(n, k)] = (wq, s, b)
    return xs, ws


SWEEP_CALLS = tuple((m, n, k) for m in SWEEP_M for (n, k) in SHAPES)


def _cpu_sweep(xs, ws, threads, calls=SWEEP_CALLS):
    """Calls of the headline workload on the host (default: the 15 calls of one
    sweep), each dequantizing its weight and multiplying (the reference's
    per-call arithmetic). Returns (algorithmic bytes, seconds)."""
    from oracle import qmm

    tot_b, t0 = 0, time.perf_counter()
    for (m, n, k) in calls:
        qmm.qmm_cpu(xs[(m, k)], *ws[(n, k)], threads)
        tot_b += alg_bytes(m, n, k)
    return tot_b, time.perf_counter() - t0


CPU_SAMPLE = ("oracle port of the reference arithmetic (per call: dequantize the packed weight, f32 matmul), "
              "row blocks over all host threads")
REF_CALLS_PER_STEP = 3  # the reference arm's bounded step: 3 of the 15 calls, every 5 steps the whole sweep


def cpu_baseline_sample():
    """The oracle port on this host's cores: one full sweep (after a small warm call)."""
    import numpy as np

    from oracle import qmm

    threads = os.cpu_count() or 1
    xs, ws = _cpu_sweep_data(np.random.default_rng(0))
    (n0, k0) = SHAPES[0]
    qmm.qmm_cpu(xs[(1, k0)], *(a[:256] for a in ws[(n0, k0)]), threads)  # warm the thread pool
    tot_b, dt = _cpu_sweep(xs, ws, threads)
    return {"value": round(tot_b / dt / 1e12, 6), "unit": UNIT, "cores": threads, "cpu_model": cpu_model(),
            "kind": "port", "sample": CPU_SAMPLE + f"; one full 15-call sweep, {dt:.1f} s"}


# ------------------------------------------------------------------ reference arm

def run_reference(args):
    """The reference's algorithm on the host CPU (oracle port), rank 0 only, on
    the GPU arm's workload: each step is a bounded sample of the 15-call sweep
    (3 calls, rotating, so that every 5 steps cover the whole sweep once)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import numpy as np

    threads = os.cpu_count() or 1
    xs, ws = _cpu_sweep_data(np.random.default_rng(0))
    nc = len(SWEEP_CALLS)

    def step_calls(i):
        return [SWEEP_CALLS[(REF_CALLS_PER_STEP * i + c) % nc] for c in range(REF_CALLS_PER_STEP)]

    for i in range(args.warmup):
        _cpu_sweep(xs, ws, threads, step_calls(i))
    tot_b, dt = 0, 0.0
    for i in range(args.steps):
        b_, t_ = _cpu_sweep(xs, ws, threads, step_calls(i))
        tot_b += b_
        dt += t_
    value = tot_b / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "bytes_per_step": sum(alg_bytes(m, n, k) for m in SWEEP_M for (n, k) in SHAPES),
                   "calls_per_step": len(SWEEP_M) * len(SHAPES),
                   "note": "reference kernels are Metal (MLX/MTPLX), unavailable on this box; "
                           "CPU port of its arithmetic"},
        "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": threads, "cpu_model": cpu_model(),
                         "kind": "port",
                         "sample": CPU_SAMPLE + f"; bounded steps of {REF_CALLS_PER_STEP} of the 15 sweep calls, "
                                                "rotating (every 5 steps cover the sweep)"},
        "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["tsb", "reference"], default="tsb")
    ap.add_argument("--no-secondary", dest="secondary", action="store_false")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--profile", choices=["qmm", "attn", "decoder", "prefill"], default=None,
                    help="profiling driver for ncu: --warmup eager steps, then exactly one eager step "
                         "(qmm: the 15 sweep calls; attn: one config-4 B=1 L=32768 call; prefill: one "
                         "M=4096 5120x17408 call); no timing")
    ap.add_argument("--attn-kv", choices=["bf16", "mlx_q8", "ref_q8"], default="bf16",
                    help="KV format of --profile attn")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.profile == "attn":
        run_profile_attn(args)
    elif args.profile == "decoder":
        run_profile_decoder(args)
    elif args.profile == "prefill":
        run_profile_prefill(args)
    else:
        run_tsb(args)


if __name__ == "__main__":
    main()
