#!/usr/bin/env python3
"""Benchmark of the emberllm token loop on B200 (decode tok/s + HBM GB/s).

Workload (the config the headline metric is quoted on):
Qwen3-0.6B-shape decoder, Q8_0, synthetic N(0, 0.02) weights (seed 0), KV cache
prefilled with `--depth` (128) uniform random tokens (seed 1), then single-stream
greedy decode of `--tokens` (128) tokens. One STEP = those 128 greedy tokens from
position `depth` (the cache is rewound to `depth` for every step).

  value  device-resident decode: the step is ember_forward_greedy (captured CUDA
         graphs, argmax on the device, no host round trip per token), timed with
         CUDA events on the state's stream; tok/s over all ranks.
  e2e    the same tokens through the public C API the reference's callers use:
         ember_forward per token (host->device token/position from pinned memory,
         device->host copy of all vocab logits into pinned memory), host argmax.
  roofline  the kernel kind with the largest share of a decode step, timed live
         (every layer in turn, outside the graph) against its algorithmic bytes.
  cpu_baseline  the reference's own `ember bench` (shipped -O3 -ffast-math flags)
         on this host's cores, best thread count of a sweep, bounded sample.

Multi-GPU: `torchrun --nproc-per-node N bench.py --gpus N`: one independent
replica per GPU, no collective on the data path (weak scaling); the step time is
the max over ranks.

`--impl reference` times the reference's CPU implementation (oracle/_ref, built
from its own sources) on the same workload, rank 0 only.
"""
import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

KIND_NAMES = ["qkv_gemv", "attention", "wo_gemv", "w13_swiglu_gemv", "w2_gemv", "lm_head_gemv"]


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="qwen3-0.6b")
    p.add_argument("--depth", type=int, default=128)
    p.add_argument("--tokens", type=int, default=128)
    p.add_argument("--e2e-steps", type=int, default=2)
    p.add_argument("--cpu-baseline", type=int, default=1)
    p.add_argument("--prefill-tokens", type=int, default=512,
                   help="prompt length of the timed batched prefill (the reference's pp512)")
    p.add_argument("--kv-fp16", action="store_true",
                   help="fp16 KV cache (the reference's --kv-type f16) instead of fp32")
    p.add_argument("--streams", type=int, default=0,
                   help="BASELINE's many-sequence workload instead: 8 x N independent streams "
                        "(N = --streams) split over the GPUs, each a 256-token prompt then "
                        "--tokens greedy steps decoded together")
    p.add_argument("--agg-streams", default="16,64",
                   help="with the headline: also decode 8 x N independent streams split over "
                        "the GPUs for each N listed (BASELINE configs[4]); '' or 0 skips")
    p.add_argument("--agg-per-gpu", type=int, default=64,
                   help="with the streams aggregate: also this many streams on every GPU "
                        "(weak scaling); 0 skips")
    p.add_argument("--agg-tokens", type=int, default=64,
                   help="greedy tokens per stream per timed step of the streams aggregate")
    p.add_argument("--prefill-only", action="store_true",
                   help="time only the batched prefill (NVTX range 'prefill' with --nvtx)")
    p.add_argument("--nvtx", action="store_true",
                   help="mark the timed region (and --kernel-case launches) as NVTX ranges "
                        "'timed' / 'case' for ncu --nvtx-include")
    p.add_argument("--kernel-case", type=int, default=-1,
                   help="profiling case: one decode position at --depth, then one untimed and "
                        "one timed round of kernel kind K (%s) over every layer; prints "
                        "its time and bytes and exits" % ", ".join(
                            "%d %s" % kv for kv in enumerate(KIND_NAMES)))
    return p.parse_args()


# ------------------------------------------------------------------ helpers ---

def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def ncu_traffic(kind_name, config, pos):
    """per-launch DRAM bytes (read + write) of one kernel kind at one decode
    position, from the committed ncu summary profiles/dram_traffic.txt, or None"""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 4 and parts[0] == kind_name and parts[1] == config \
                    and parts[2] == str(pos):
                return float(parts[3])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled during the timed region"""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_binary():
    """the reference CLI built by oracle/Makefile; AVX-512 build where the CPU has it"""
    flags = ""
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        pass
    v4 = os.path.join(ROOT, "oracle", "_ref", "ember_ref_v4")
    v3 = os.path.join(ROOT, "oracle", "_ref", "ember_ref_v3")
    if " avx512f " in flags and " avx512bw " in flags and os.path.exists(v4):
        return v4
    return v3 if os.path.exists(v3) else None


def ref_cli_bench(binary, model, pp, tg, threads, reps=1):
    out = subprocess.run([binary, "bench", model, "--pp", str(pp), "--tg", str(tg), "--threads",
                          str(threads), "--reps", str(reps)], capture_output=True, text=True,
                         timeout=600)
    m = re.search(r"decode\s+\(tg\d+\):\s+([\d.]+)\s+tok/s", out.stdout)
    if out.returncode != 0 or not m:
        raise RuntimeError("reference bench failed: " + out.stdout[-300:] + out.stderr[-300:])
    pm = re.search(r"prefill \(pp\d+\):\s+([\d.]+)\s+tok/s", out.stdout)
    return float(m.group(1)), float(pm.group(1)) if pm else None


def thread_sweep():
    """1, 2, 4, 8, ... up to the host's core count, and the count itself"""
    n = os.cpu_count() or 1
    ts, t = [], 1
    while t < n:
        ts.append(t)
        t *= 2
    return ts + [n]


def reference_model(name, binary):
    """The reference arm's own copy of the synthetic model: the fp32 file from
    the numpy writer (no native library involved), quantized by the reference's
    CLI (`ember quantize`, its own quantizer). Its tensors are byte-identical to
    the file this library's arm loads (tests/test_quant_file.py)."""
    from emberllm_b200 import synth      # pure Python: loads no shared library
    cfg = synth.CONFIGS[name]
    d = synth.cache_dir()
    f32 = synth.ensure_model(name, quant="f32", directory=d)
    out = os.path.join(d, os.path.basename(f32).replace("-f32-", "-refq-%s-" % cfg["quant"]))
    if not os.path.exists(out):
        tmp = out + ".tmp%d" % os.getpid()
        r = subprocess.run([binary, "quantize", f32, tmp, cfg["quant"]], capture_output=True, text=True,
                           timeout=1800)
        if r.returncode != 0:
            raise RuntimeError("reference quantize failed: " + r.stderr[-300:])
        os.replace(tmp, out)
    return out


def sweep_threads(binary, model, depth, tg=16):
    """decode tok/s of the reference at each thread count (short runs)"""
    sweep = {}
    for t in thread_sweep():
        try:
            sweep[t] = round(ref_cli_bench(binary, model, depth, tg, t)[0], 1)
        except (RuntimeError, subprocess.TimeoutExpired):
            pass
    return sweep


def cpu_baseline(depth, ntok, model_name):
    """the reference's `ember bench` on the host cores: best thread count of a
    sweep, then one run of the bench workload (pp depth, tg ntok) at that count"""
    binary = reference_binary()
    if not binary:
        return None
    model = reference_model(model_name, binary)
    sweep = sweep_threads(binary, model, depth)
    if not sweep:
        return None
    best = max(sweep, key=sweep.get)
    tg, pp = ref_cli_bench(binary, model, depth, ntok, best)
    return {"value": round(tg, 2), "unit": "tok/s", "cores": best, "kind": "reference",
            "prefill_tok_s": pp,
            "sample": "reference `ember bench --pp %d --tg %d --reps 1` (%s, shipped -O3 -ffast-math "
                      "flags) on its own quantization of the same synthetic model, %d threads, the "
                      "best of a sweep %s (tok/s by thread count, --tg 16) on %d host cores"
                      % (depth, ntok, os.path.basename(binary), best, sweep, os.cpu_count() or 1)}


# ------------------------------------------------------------------ ranks -----

def dist_setup(args=None, backend=None, timeout_s=300):
    """One process per GPU (torchrun env). NCCL on GPUs; gloo when no GPU is
    visible (the host-side logic's tests). Only the timer's max-reduction and
    barriers cross ranks: the replicas / stream partitions share no data."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        os.environ["EMBER_CUDA_DEVICE"] = str(local)
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=timeout_s))
        return world, rank, local, dist
    return 1, 0, 0, None


def stream_range(total, world, rank):
    """streams [lo, hi) of GPU `rank`: an even split of 8 x N streams"""
    return rank * total // world, (rank + 1) * total // world


class Nvtx:
    """NVTX push/pop ranges (through torch's bindings) when --nvtx is given"""

    def __init__(self, on):
        self.nvtx = None
        if on:
            import torch.cuda.nvtx as nvtx
            self.nvtx = nvtx

    def push(self, name):
        if self.nvtx:
            self.nvtx.range_push(name)

    def pop(self):
        if self.nvtx:
            self.nvtx.range_pop()


def barrier(dist):
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, value):
    if dist is None:
        return value
    import torch
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ arms ------

def time_prefill(args, lib, path, vocab, dist, nvtx):
    """Batched prefill of a --prefill-tokens prompt (the reference's ppN): one
    untimed call (builds the weight packs), then 3 timed calls, CUDA events on
    the state's stream; seconds per prefill, max over ranks."""
    import numpy as np
    from emberllm_b200 import Ember
    npf = args.prefill_tokens
    ep = Ember(path, ctx=npf + 8)
    csp = lib.ember_state_cuda(ep.st)
    pprompt = [int(t) for t in np.random.default_rng(2).integers(0, vocab, npf)]
    ep.prefill(pprompt)
    barrier(dist)
    nvtx.push("prefill")
    lib.ember_cuda_mark(csp, 4)
    for _ in range(3):
        ep.prefill(pprompt)
    lib.ember_cuda_mark(csp, 5)
    nvtx.pop()
    ms = ctypes.c_float()
    assert lib.ember_cuda_elapsed_ms(csp, 4, 5, ctypes.byref(ms)) == 0, lib.ember_cuda_error()
    ep.close()
    return max_over_ranks(dist, ms.value / 1e3 / 3)


def streams_measure(args, world, rank, local, dist, total, ntok, steps, warmup):
    """`total` independent streams split over the GPUs:
    GPU g decodes streams [g*total/G, (g+1)*total/G) as one batch (no
    collective). Each stream: its own 256-token prompt, then `ntok` greedy
    tokens per timed step. Device time (CUDA events on the batch's stream,
    max over ranks) and wall time of the same synchronous calls, which include
    the host copies of the step's tokens in and out (the e2e figure)."""
    import numpy as np
    import torch
    from emberllm_b200 import Ember, EmberBatch, load, synth

    path = synth.ensure_model(args.config)
    lib = load()
    lo, hi = stream_range(total, world, rank)
    S = hi - lo
    plen = 256
    e = Ember(path)
    b = EmberBatch(e, S, ctx=plen + ntok + 8, max_steps=ntok)
    firsts = []
    for i in range(S):
        rng = np.random.default_rng(1000 + lo + i)     # stream lo+i's own prompt
        firsts.append(b.prefill(i, [int(t) for t in rng.integers(0, e.vocab, plen)]))
    pos = [plen] * S
    for _ in range(warmup):
        b.greedy(firsts, pos, min(8, ntok))
    # events on the batch's stream (one CUDA stream when the batch runs as GEMMs;
    # concurrent single-stream states use several, and then only wall time counts)
    gemm = S > 8 or os.environ.get("EMBER_BATCH") == "gemm"
    ev = None
    if gemm and torch.cuda.is_available():
        st = torch.cuda.ExternalStream(lib.ember_cuda_batch_stream(lib.ember_batch_cuda(b.b)))
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True), st)
    clocks = ClockSampler(local)
    clocks.start()
    barrier(dist)
    nvtx = Nvtx(args.nvtx)
    if ev:
        ev[0].record(ev[2])
    t0 = time.perf_counter()
    nvtx.push("streams")
    for _ in range(steps):
        b.greedy(firsts, pos, ntok)     # synchronous: tokens come back to the host
    nvtx.pop()
    t_wall = time.perf_counter() - t0
    t_dev = None
    if ev:
        ev[1].record(ev[2])
        ev[1].synchronize()
        t_dev = ev[0].elapsed_time(ev[1]) / 1e3
    clk = clocks.stop()
    t_wall = max_over_ranks(dist, t_wall)
    t_dev = max_over_ranks(dist, t_dev) if t_dev is not None else None
    b.close()
    e.close()
    return {"S": S, "t_wall": t_wall, "t_dev": t_dev, "clk": clk, "gemm": gemm,
            "tokens": total * ntok * steps}


def streams_summary(m, total, world, ntok, steps):
    value = m["tokens"] / (m["t_dev"] if m["t_dev"] else m["t_wall"])
    e2e = m["tokens"] / m["t_wall"]
    return {"streams": total, "streams_per_gpu": m["S"], "n_gpus": world, "tokens_per_step": ntok,
            "value": round(value, 1), "unit": "tok/s", "per_stream_tok_s": round(value / total, 2),
            "timing": "CUDA events on the batch stream, max over ranks" if m["t_dev"] else "wall clock",
            "path": "batched GEMMs" if m["gemm"] else "concurrent single-stream states",
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": m["S"] * 8,
                    "d2h_bytes_per_step": m["S"] * ntok * 4,
                    "path": "ember_batch_greedy (host tokens in, host tokens out), wall clock"},
            "ms_per_step": round((m["t_dev"] or m["t_wall"]) / steps * 1e3, 3)}


def run_streams(args, world, rank, local, dist):
    """8 x N independent streams, N = --streams: strong
    scaling over the GPUs, no collective."""
    from emberllm_b200 import synth
    if rank == 0:
        synth.ensure_model(args.config)
    barrier(dist)
    total, ntok = 8 * args.streams, args.tokens
    m = streams_measure(args, world, rank, local, dist, total, ntok, args.steps, args.warmup)
    sm = streams_summary(m, total, world, ntok, args.steps)
    return {
        "metric": "aggregate decode tok/s (Qwen3-0.6B Q8_0, 8xN independent streams)",
        "value": sm["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sm["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 dot / fp32 (Q8_0 weights, exact reference arithmetic)",
        "data": "synthetic: N(0,0.02) weights seed 0, per-stream uniform random prompts",
        "config": {"workload": "%d streams (8 x %d), 256-token prompts, %d greedy tokens each, decoded "
                               "together per GPU (%s)" % (total, args.streams, ntok, sm["path"]),
                   "model": args.config, "streams": total, "streams_per_gpu": m["S"], "tokens_per_step": ntok,
                   "parallelism": "streams split over %d GPU(s), one replica each" % world},
        "per_stream_tok_s": sm["per_stream_tok_s"],
        "timing": sm["timing"],
        "e2e": sm["e2e"],
        "clocks": m["clk"],
    }


def run_ours(args, world, rank, local, dist):
    import numpy as np
    from emberllm_b200 import Ember, load, synth

    cfg = synth.CONFIGS[args.config]
    if rank == 0:
        path = synth.ensure_model(args.config)
    barrier(dist)
    path = synth.ensure_model(args.config)
    lib = load()
    for name, res, argt in [
            ("ember_cuda_mark", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
            ("ember_cuda_elapsed_ms", ctypes.c_int,
             [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]),
            ("ember_cuda_time_kernel", ctypes.c_int,
             [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float),
              ctypes.POINTER(ctypes.c_double)])]:
        getattr(lib, name).restype = res
        getattr(lib, name).argtypes = argt

    depth, ntok = args.depth, args.tokens
    nvtx = Nvtx(args.nvtx)
    if args.prefill_only:
        s_pf = time_prefill(args, lib, path, cfg["vocab_size"], dist, nvtx)
        return {"prefill_case": args.config, "tokens": args.prefill_tokens,
                "ms": round(s_pf * 1e3, 3), "prefill_tok_s": round(args.prefill_tokens / s_pf, 1)}
    e = Ember(path, ctx=depth + ntok + 8, kv_fp16=args.kv_fp16)
    cs = lib.ember_state_cuda(e.st)
    # kernels are timed alone at the step's mean position (attention length)
    kpos = depth + ntok // 2
    if args.kernel_case >= 0:
        # one decode position at kpos (sets the attended length), then the kernel kind
        e.forward(0, kpos)
        ms, by = ctypes.c_float(), ctypes.c_double()
        nvtx.push("case")
        rc = lib.ember_cuda_time_kernel(cs, args.kernel_case, 1, ctypes.byref(ms), ctypes.byref(by))
        nvtx.pop()
        assert rc == 0, lib.ember_cuda_error()
        e.close()
        return {"kernel_case": KIND_NAMES[args.kernel_case], "config": args.config, "pos": kpos,
                "us_per_launch": round(ms.value * 1e3, 3), "bytes_per_launch": int(by.value),
                "launches": 2 * (1 if args.kernel_case == 5 else cfg["n_layers"])}
    rng = np.random.default_rng(1)
    prompt = [int(t) for t in rng.integers(0, e.vocab, depth)]

    def elapsed(a, b):
        ms = ctypes.c_float()
        assert lib.ember_cuda_elapsed_ms(cs, a, b, ctypes.byref(ms)) == 0, lib.ember_cuda_error()
        return ms.value / 1e3

    # the decode depth: the cache filled by a prefill of `depth` random tokens
    e.prefill(prompt)
    first = int(np.argmax(np.ctypeslib.as_array(e.forward(prompt[-1], depth - 1), (e.vocab,))))

    for _ in range(args.warmup):
        e.greedy(first, depth, ntok)
    clocks = ClockSampler(local)
    clocks.start()
    barrier(dist)
    nvtx.push("timed")
    lib.ember_cuda_mark(cs, 0)
    for _ in range(args.steps):
        e.greedy(first, depth, ntok)
    lib.ember_cuda_mark(cs, 1)
    nvtx.pop()
    t = elapsed(0, 1)
    clk = clocks.stop()
    t_max = max_over_ranks(dist, t)

    # end to end through the public API: ember_forward per token, host argmax
    barrier(dist)
    lib.ember_cuda_mark(cs, 2)
    for _ in range(args.e2e_steps):
        tok = first
        for i in range(ntok):
            logits = np.ctypeslib.as_array(e.forward(tok, depth + i), (e.vocab,))
            tok = int(np.argmax(logits))
    lib.ember_cuda_mark(cs, 3)
    t_e2e = max_over_ranks(dist, elapsed(2, 3))

    npf = args.prefill_tokens
    prefill_s = time_prefill(args, lib, path, e.vocab, dist, nvtx)

    # roofline of the dominant kernel kind, timed live at kpos (overwrites the state)
    e.forward(0, kpos)
    kinds = []
    L = cfg["n_layers"]
    for kind in range(6):
        ms, by = ctypes.c_float(), ctypes.c_double()
        assert lib.ember_cuda_time_kernel(cs, kind, 20, ctypes.byref(ms), ctypes.byref(by)) == 0, \
            lib.ember_cuda_error()
        per_step = ms.value * (1 if kind == 5 else L)
        kinds.append((per_step, kind, ms.value, by.value))
    kinds.sort(reverse=True)
    _, dk, dms, dbytes = kinds[0]
    peak, peak_kind = measured_peaks()
    achieved = dbytes / (dms / 1e3) / 1e9
    # kernels of one greedy token (the greedy graph's launches, counted when captured)
    launches = lib.ember_cuda_state_launches_per_token(cs)
    assert launches > 0
    e.close()

    total_tokens = world * args.steps * ntok
    value = total_tokens / t_max
    ms_per_step = t_max / args.steps * 1e3
    step_bytes = synth.weight_bytes_per_token(cfg)
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    avg_pos = depth + (ntok - 1) / 2.0
    kes = 2 if args.kv_fp16 else 4
    kv_bytes = 2 * cfg["n_layers"] * kvd * kes * (avg_pos + 1) + 2 * cfg["n_layers"] * kvd * kes
    line = {
        "metric": "decode tok/s (Qwen3-0.6B Q8_0, 1 GPU); HBM GB/s; prefill tok/s",
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 dot / fp32 (Q8_0 weights, exact reference arithmetic)",
        "data": "synthetic: N(0,0.02) weights seed 0, uniform random prompt seed 1",
        "config": _workload_config(args, world),
        "hbm_gbs_step": round((step_bytes + kv_bytes) * value / world / 1e9, 1),
        "bytes_per_token": int(step_bytes + kv_bytes),
        "prefill_tok_s": round(world * npf / prefill_s, 1),
        "prefill_note": "ember_prefill of a %d-token random prompt per GPU (batched: tcgen05 int8 "
                        "GEMMs), host ids in, last-token logits out; mean of 3" % npf,
        "e2e": {"value": round(world * args.e2e_steps * ntok / t_e2e, 2), "unit": "tok/s",
                "h2d_bytes_per_step": ntok * 8, "d2h_bytes_per_step": ntok * (cfg["vocab_size"] * 4 + 4),
                "path": "ember_forward per token (pinned host logits) + host argmax"},
        "gpu_launches": args.steps * ntok * launches,
        "roofline": {"kernel": KIND_NAMES[dk], "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak, "peak_source": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": ncu_traffic(KIND_NAMES[dk], args.config, kpos), "pos": kpos,
                     "bytes_per_launch": int(dbytes), "us_per_launch": round(dms * 1e3, 3)},
        "kernel_shares": {KIND_NAMES[k]: round(ps, 4) for ps, k, _, _ in kinds},
        "clocks": clk,
    }
    # BASELINE configs[4] beside the headline: 8 x 16 and 8 x 64 streams split
    # over the N GPUs (strong scaling), and 64 streams on every GPU (weak scaling);
    # the headline stays single-stream
    aggs = []
    for n_per in [int(v) for v in args.agg_streams.split(",") if v.strip() and int(v) > 0]:
        total = 8 * n_per
        m = streams_measure(args, world, rank, local, dist, total, args.agg_tokens, 2, args.warmup)
        sm = streams_summary(m, total, world, args.agg_tokens, 2)
        sm["scaling"] = "strong"
        aggs.append(sm)
    # and a fixed number of streams per GPU (weak scaling: 64 x N streams in all)
    if args.agg_per_gpu > 0 and args.agg_streams.strip():
        total = args.agg_per_gpu * world
        m = streams_measure(args, world, rank, local, dist, total, args.agg_tokens, 2, args.warmup)
        sm = streams_summary(m, total, world, args.agg_tokens, 2)
        sm["scaling"] = "weak"
        aggs.append(sm)
    if aggs:
        line["streams_aggregate"] = aggs
    if rank == 0 and world == 1 and args.cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(depth, ntok, args.config)
    return line


def run_reference(args, world, rank):
    """The reference's own CPU implementation on this host: its CLI (oracle/_ref,
    built from its sources with its shipped flags) running `ember bench` on its
    own quantization of the synthetic model -- no library of this repository is
    loaded. Same workload as this library's arm: prefill `--depth` tokens, then
    `--tokens` decode steps; the thread count is the best of a sweep."""
    if rank != 0:
        return None
    binary = reference_binary()
    if not binary:
        return {"impl": "reference", "unavailable": "oracle/_ref was not built on this machine"}
    model = reference_model(args.config, binary)
    depth, ntok = args.depth, args.tokens
    sweep = sweep_threads(binary, model, depth)
    best_t = max(sweep, key=sweep.get)
    for _ in range(max(0, args.warmup - 1)):
        ref_cli_bench(binary, model, depth, ntok, best_t)
    steps = [ref_cli_bench(binary, model, depth, ntok, best_t) for _ in range(args.steps)]
    v = statistics.mean(tg for tg, _ in steps)
    pp512 = None
    try:
        pp512 = round(ref_cli_bench(binary, model, args.prefill_tokens, 1, best_t)[1], 1)
    except (RuntimeError, subprocess.TimeoutExpired):
        pass
    return {
        "impl": "reference",
        "metric": "decode tok/s (Qwen3-0.6B Q8_0, 1 GPU); HBM GB/s; prefill tok/s",
        "value": round(v, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ntok / v * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 dot / fp32 (Q8_0 weights, exact reference arithmetic)",
        "data": "synthetic: N(0,0.02) weights seed 0; token ids from the reference bench's own "
                "fixed stream (decode time does not depend on the ids)",
        "config": _workload_config(args, world),
        "prefill_tok_s": pp512,
        "prefill_note": "reference `ember bench --pp %d --tg 1` at %d threads" % (args.prefill_tokens, best_t),
        "cpu_baseline": {"value": round(v, 2), "unit": "tok/s", "cores": best_t, "kind": "reference",
                         "sample": "reference `ember bench --pp %d --tg %d --reps 1` per step (%s, shipped "
                                   "-O3 -ffast-math flags) on its own quantization of the synthetic model, "
                                   "%d threads: the best of the sweep %s (tok/s by thread count, --tg 16) "
                                   "on %d host cores" % (depth, ntok, os.path.basename(binary), best_t,
                                                         sweep, os.cpu_count() or 1)},
        "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _workload_config(args, world):
    """the `config` object both arms report for the single-stream workload"""
    return {"workload": "%s Q8_0 single-stream greedy decode of %d tokens at depth %d"
                        % (args.config, args.tokens, args.depth),
            "model": args.config, "depth": args.depth, "tokens_per_step": args.tokens,
            "kv_cache": "fp16" if args.kv_fp16 else "fp32",
            "parallelism": "replicas, one per GPU" if world > 1 else "1 GPU",
            "l2": "weights 634 MB per token > 126 MB L2 (no flush needed)"}


def main():
    args = parse()
    if args.impl == "reference":
        # CPU only: rank 0 runs, the other ranks exit without work
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local, dist = dist_setup(args)
    try:
        line = (run_streams if args.streams > 0 else run_ours)(args, world, rank, local, dist)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
