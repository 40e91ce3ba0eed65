"""Benchmark: Q4_K / Q6_K integer matvec HBM GB/s on B200, bit-exact.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl vtq|reference] [--config NAME]

A step is one pass of the hot path over one batch: every matvec of the
configuration (default c2: Llama-7B FFN Q4_K, 4096->11008 and 11008->4096,
batch 1). `value` is algorithmic bytes (packed weights + 4*in + 4*out per
matvec) / device time, with the weights resident in HBM. Between steps the
weights rotate over enough distinct copies that the set read per rotation
exceeds the 126 MB L2, so no step is served from L2.

`e2e` is the same metric through the public C ABI (vtq_linear with VTQ_PTR_HOST):
every step copies x from pinned host memory, runs the kernel and reads y back.

N > 1 (torchrun, one rank per GPU): weak scaling -- every rank streams its own
weights for the same per-rank workload; no data-path collective (rows are
independent). Timing is bracketed by barrier + synchronize and the max over
ranks is taken.

--impl reference times the reference's CPU path (the oracle port of
linear_q4_k_integer_parallel / linear_q6_k_integer_parallel: the reference is
Rust and no Rust toolchain exists on this image) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "vitni-tensor_b200"))
sys.path.insert(0, REPO)

METRIC = "Q4_K/Q6_K matvec HBM GB/s (% of peak), bit-exact; decode tok/s at 1-8 B200"
L2_BYTES = 126 * 1024 * 1024
ROTATE_MIN_BYTES = 2 * L2_BYTES


def algo_bytes(dtype, n, r, batch=1):
    import vtq
    return r * vtq.row_bytes(dtype, n) + 4 * n * batch + 4 * r * batch


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(cfg, mode, steps_per_launch):
    """DRAM bytes (read + write) per launch of the dominant kernel: the bytes per
    step of one ncu capture of the same kernel on the same workload
    (profiles/dram_traffic.json, machine-readable, keyed by workload and launch
    mode) times the steps one launch processes. None when no capture exists."""
    try:
        with open(os.path.join(REPO, "profiles", "dram_traffic.json")) as f:
            t = json.load(f).get(f"{cfg}/{mode}")
        return None if t is None else float(t["dram_bytes_per_step"]) * steps_per_launch
    except (OSError, ValueError, KeyError):
        return None


class ClockSampler:
    """NVML clocks / throttle reasons sampled in a thread during the timed region."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle",
               0x2: "applications_clocks_setting", 0x10: "sync_boost",
               0x100: "display_clock_setting"}

    def __init__(self, device_index):
        self.samples, self.reasons = [], 0
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _sample(self):
        self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
        self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(0.002)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def stop(self):
        if not self.ok:
            return None
        self._stop.set()
        self.t.join()
        try:
            self._sample()
        except Exception:
            pass
        names = sorted(v for k, v in self.REASONS.items() if self.reasons & k and v != "gpu_idle")
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args, world, rank):
    """CPU reference arm (oracle port of the reference's parallel bench path)."""
    if rank != 0:
        return
    from vtq import synth
    from oracle import oracle as O
    if args.config == PREFILL_CFG_NAME:
        for _ in range(min(args.warmup, 1)):
            prefill_cpu_sample()
        samples = [prefill_cpu_sample() for _ in range(max(1, min(args.steps, 3)))]
        v = statistics.median(x["value"] for x in samples)
        cpu = dict(samples[0], value=v, sample=f"{len(samples)} steps, each " + samples[0]["sample"])
        print(json.dumps({
            "metric": METRIC, "value": v, "unit": "TOPS", "impl": "reference", "n_gpus": world,
            "steps": len(samples), "warmup": min(args.warmup, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": args.config, "tokens": synth.PREFILL_M, "l2": "host run"},
            "cpu_baseline": cpu,
            "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    cfg = synth.CONFIGS[args.config]
    mats = [(dt, n, r, synth.weight(dt, f"{args.config}.w.{n}x{r}", r, n),
             synth.activation(f"{args.config}.x.{n}", 1, n)) for dt, n, r in cfg]
    threads = os.cpu_count() or 1
    name = {12: "q4_k_integer", 14: "q6_k_integer", 8: None}
    step_bytes = sum(algo_bytes(dt, n, r) for dt, n, r in cfg)

    def step():
        for dt, n, r, w, x in mats:
            if name.get(dt):
                O.linear(name[dt], x, w, 1, n, r, threads)
            else:
                O.linear_dispatch(dt, x, w, n, r, threads=threads)

    for _ in range(max(1, args.warmup)):
        step()
    times = []
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = step_bytes * len(times) / total / 1e9
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / len(times), 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": args.config, "batch": 1, "l2": "host run"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{len(times)} full steps of {args.config} on {threads} "
                                   "threads (oracle restatement of linear_*_integer_parallel)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(cfg_name, threads, budget_s=12.0):
    """Oracle timed on `threads` host cores on a bounded sample of the workload."""
    from vtq import synth
    from oracle import oracle as O
    cfg = synth.CONFIGS[cfg_name]
    mats = [(dt, n, r, synth.weight(dt, f"{cfg_name}.w.{n}x{r}", r, n),
             synth.activation(f"{cfg_name}.x.{n}", 1, n)) for dt, n, r in cfg]
    name = {12: "q4_k_integer", 14: "q6_k_integer"}
    nbytes = 0
    t0 = time.perf_counter()
    t_end = t0 + budget_s
    steps = 0
    while time.perf_counter() < t_end or steps == 0:
        for dt, n, r, w, x in mats:
            if dt in name:
                O.linear(name[dt], x, w, 1, n, r, threads)
            else:
                O.linear_dispatch(dt, x, w, n, r, threads=threads)
            nbytes += algo_bytes(dt, n, r)
        steps += 1
    el = time.perf_counter() - t0
    return {"value": round(nbytes / el / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{steps} full steps of {cfg_name} in {el:.1f} s, {threads} threads "
                      "(oracle restatement of the reference's row-parallel integer linears)"}


DECODE_CFG = "c4_tinyllama_decode"
DEFAULT_CFG = "c2_q4_k_llama7b_ffn"
PREFILL_CFG_NAME = "c5_q4_k_prefill_mistral"


def int8_peak_tops():
    """Dense int8 tensor peak measured here with cuBLASLt (torch._int_mm, 8192^3,
    best of 10 after warm-up); falls back to 2x the measured bf16 peak."""
    import torch
    try:
        n = 8192
        a = torch.randint(-64, 64, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-64, 64, (n, n), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = None
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        del a, b
        return 2 * n ** 3 / (best / 1e3) / 1e12, "cuBLASLt int8 torch._int_mm 8192^3, measured in this run"
    except Exception:
        try:
            with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
                return 2 * float(json.load(f)["bf16_tflops"]), "2x measured bf16 (MEASURED_PEAKS.json)"
        except Exception:
            return 2 * 1590.0, "2x fallback bf16"


def prefill_ops(M, linears):
    return sum(2 * M * n * r for _, n, r in linears)


def run_prefill(args, world, rank, local):
    """The prefill workload: the seven Q4_K linears of one Mistral-7B layer at M = 512
    tokens, batched integer path (tcgen05 kind::i8). A step runs all seven
    through vtq_linear on device pointers. N > 1: output rows sharded over the
    ranks (contiguous ranges), y all-gathered over NCCL inside the timed region."""
    import torch
    import torch.distributed as dist
    import vtq
    from vtq import synth, shard
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    M, lins = synth.PREFILL_M, synth.PREFILL_LINEARS
    ctx = vtq.Context(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    host_w = {nm: synth.weight(vtq.Q4_K, f"c5.{nm}", r, n) for nm, n, r in lins}
    host_x = {n: synth.activation(f"c5.x.{n}", M, n) for n in sorted({n for _, n, _ in lins})}
    ranges = {nm: shard.row_range(r, world, rank) for nm, n, r in lins}
    wbytes = sum((ranges[nm][1] - ranges[nm][0]) * vtq.row_bytes(vtq.Q4_K, n) for nm, n, r in lins)
    copies = max(1, -(-ROTATE_MIN_BYTES // wbytes))
    weights = [{nm: ctx.upload(vtq.Q4_K, host_w[nm], n, r, *ranges[nm]) for nm, n, r in lins}
               for _ in range(copies)]
    xs = {n: torch.from_numpy(x).cuda() for n, x in host_x.items()}
    ys = {nm: torch.empty(M * (ranges[nm][1] - ranges[nm][0]), device="cuda") for nm, n, r in lins}
    full = {nm: torch.empty(world * M * (r // world), device="cuda") for nm, n, r in lins} \
        if world > 1 else None

    def step(c, events=None):
        for i, (nm, n, r) in enumerate(lins):
            if events is not None:
                events[i][0].record(stream)
            ctx.linear_ptr(weights[c][nm], xs[n].data_ptr(), ys[nm].data_ptr(), M)
            if events is not None:
                events[i][1].record(stream)
            if world > 1:
                dist.all_gather_into_tensor(full[nm], ys[nm])

    for c in range(copies):
        step(c)
    torch.cuda.synchronize()
    bit_exact = None
    if rank == 0:
        # Bit check (rank 0 holds the first row shard of every linear): wk and wq
        # against the oracle.
        from oracle import oracle as O
        bit_exact = True
        for nm, n, r in lins[:2]:
            a, b = ranges[nm]
            ref = O.linear("q4_k_integer", host_x[n], host_w[nm][a * vtq.row_bytes(vtq.Q4_K, n):
                                                                b * vtq.row_bytes(vtq.Q4_K, n)],
                           M, n, b - a, os.cpu_count())
            got = ys[nm].cpu().numpy()
            bit_exact &= bool(np.array_equal(got.view(np.uint32), ref.view(np.uint32)))
    steps = max(1, min(args.steps, 200))
    warm = max(3, min(args.warmup, 20))
    for i in range(warm):
        step(i % copies)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        step(i % copies)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ops = prefill_ops(M, lins)
    value = ops * steps / (ms / 1e3) / 1e12
    # Per-launch device time of the linears (quantise + GEMM kernels).
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in lins]
    tot = [0.0] * len(lins)
    reps = 5
    for k in range(reps):
        step(k % copies, evs)
        torch.cuda.synchronize()
        for i, (a, b) in enumerate(evs):
            tot[i] += a.elapsed_time(b)
    local_ops = sum(2 * M * n * (ranges[nm][1] - ranges[nm][0]) for nm, n, r in lins)
    achieved = local_ops * reps / (sum(tot) / 1e3) / 1e12
    peak, peak_src = int8_peak_tops()
    # e2e: host buffers through the C ABI (x copied in, y copied out per linear).
    px = {n: torch.from_numpy(x).pin_memory() for n, x in host_x.items()}
    py = {nm: torch.empty(M * (ranges[nm][1] - ranges[nm][0]), dtype=torch.float32).pin_memory()
          for nm, n, r in lins}
    e2e_steps = max(3, min(20, steps))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for s_ in range(e2e_steps):
        for nm, n, r in lins:
            ctx.linear_ptr(weights[s_ % copies][nm], px[n].data_ptr(), py[nm].data_ptr(), M,
                           host=True)
    f1.record(stream)
    torch.cuda.synchronize()
    ems = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e = ops * e2e_steps / (ems / 1e3) / 1e12 if world == 1 else \
        local_ops * world * e2e_steps / (ems / 1e3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = prefill_cpu_sample()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "TOPS", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": round(ms / steps, 4),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": synth.PREFILL_CFG, "tokens": M,
                       "linears": [f"Q4_K {n}->{r}" for _, n, r in lins],
                       "parallelism": f"rows sharded x{world} + NCCL all-gather" if world > 1
                       else "1 GPU",
                       "l2": f"{copies} rotating weight copies ({copies * wbytes / 1e6:.0f} MB)",
                       "ops_per_step": ops},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1),
                         "unit": "TOPS", "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": peak_src, "kernel": "kq_gemm_kernel + quantize_rows",
                         "ops_per_step_local": local_ops},
            "e2e": {"value": round(e2e, 2), "unit": "TOPS",
                    "h2d_bytes_per_step": sum(4 * M * n for _, n, _ in lins),
                    "d2h_bytes_per_step": sum(4 * M * (ranges[nm][1] - ranges[nm][0])
                                              for nm, n, r in lins)},
            "gpu_launches": steps * len(lins) * 2, "clocks": clk, "cpu_baseline": cpu,
            "bit_exact": bit_exact}),
            flush=True)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and not bit_exact:
        raise SystemExit("bench: prefill output differs from the oracle")


def prefill_cpu_sample(reps=1):
    """Oracle linear_q4_k_integer_parallel on the host cores: wk (4096 -> 1024) at
    M = 512, the bounded sample of the prefill workload."""
    from vtq import synth
    from oracle import oracle as O
    import vtq
    M = synth.PREFILL_M
    nm, n, r = synth.PREFILL_LINEARS[1]
    w = synth.weight(vtq.Q4_K, f"c5.{nm}", r, n)
    x = synth.activation(f"c5.x.{n}", M, n)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    for _ in range(reps):
        O.linear("q4_k_integer", x, w, M, n, r, threads)
    el = time.perf_counter() - t0
    return {"value": round(2 * M * n * r * reps / el / 1e12, 5), "unit": "TOPS", "cores": threads,
            "kind": "port", "sample": f"{reps} x wk (Q4_K {n}->{r}) at M={M} in {el:.1f} s, "
                                      f"{threads} threads (oracle linear_q4_k_integer_parallel)"}


def decode_bytes_per_token(cfg, n_pos):
    """Algorithmic HBM bytes of one decode step averaged over positions 0..n_pos-1:
    every weight once (packed) + norms + the embedding row + KV reads 2*kv_dim*4*(pos+1)
    per layer."""
    from vtq import formats
    d, h, L, V = cfg["dim"], cfg["hidden"], cfg["layers"], cfg["vocab"]
    kv = cfg["kv_heads"] * (d // cfg["heads"])
    q4, q6 = formats.Q4_K, formats.Q6_K
    w = L * (formats.row_bytes(q4, d) * (2 * d + kv + 2 * h) + formats.row_bytes(q6, d) * kv +
             formats.row_bytes(q6, h) * d)
    w += formats.row_bytes(q6, d) * V + formats.row_bytes(q4, d) + 4 * d * (2 * L + 1)
    kv_avg = L * 2 * kv * 4 * (n_pos + 1) / 2
    return w + kv_avg


def run_decode(args, world, rank, local):
    """The decode workload: TinyLlama-shaped Q4_K/Q6_K model, 16 prompt + 64 greedy
    tokens per step of the benchmark; replicas on N GPUs (decode does not shard)."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    line = decode_measure(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and not line["bit_exact"]:
        raise SystemExit("bench: decode tokens differ from the oracle")


def decode_measure(args, world, rank, local, sub=False):
    import torch
    import torch.distributed as dist
    import vtq
    from vtq import gguf, receipt
    from oracle import oracle as O
    cfg = gguf.TINYLLAMA
    blob = gguf.synthetic_llama(cfg)
    prompt = gguf.prompt_tokens(16, cfg["vocab"])
    n_new = 64
    sess = vtq.DecodeSession(blob, local)
    warm = max(1, args.warmup // 10)
    for _ in range(warm):
        toks, _ = sess.run(prompt, n_new)
    reps = max(3, min(args.steps, 20))
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    clocks.start()
    steps_ms, call_ms, per = 0.0, 0.0, []
    launches = 0
    same = True
    for _ in range(reps):
        toks2, _ = sess.run(prompt, n_new)
        a, b = sess.timing()
        steps_ms += a
        call_ms += b
        per.append(a)
        launches += sess.launches()
        same &= list(toks2) == list(toks)
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([steps_ms, call_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        steps_ms, call_ms = float(t[0]), float(t[1])
    n_pos = len(prompt) + n_new
    tok_s = reps * n_pos * world / (steps_ms / 1e3)
    e2e = reps * n_pos * world / (call_ms / 1e3)
    per_tok_bytes = decode_bytes_per_token(cfg, n_pos)
    peak, peak_kind = peaks()
    achieved = per_tok_bytes / (steps_ms / reps / n_pos / 1e3) / 1e9
    floor_tok_s = peak * 1e9 / per_tok_bytes
    rc = receipt.decode_receipt(gguf.MODEL_ID, blob, gguf.arch_string(cfg), prompt, n_new, toks)
    cpu = None
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ref, _ = O.decode_run(blob, prompt, n_new, threads=threads)
    el = time.perf_counter() - t0
    exact = bool(same and list(ref) == list(toks))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = {"value": round(n_pos / el, 3), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"one full decode run ({n_pos} positions) in {el:.1f} s"}
    sess.close()
    return {
        "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world,
        "steps": reps, "warmup": warm,
        "ms_per_step": round(steps_ms / reps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": DECODE_CFG, "model": "random-init TinyLlama-1.1B shapes, "
                   "Q4_K/Q6_K GGUF", "prompt": len(prompt), "new_tokens": n_new,
                   "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
                   "l2": "667 MB of weights per token > L2",
                   "prompt_batched": len(prompt) - 1,
                   "step_kind": sess_kind_name(sess),
                   "timing": "CUDA events around each run: the batched prompt positions "
                             "(all but the last) and the per-token steps"},
        "ms_per_token": round(steps_ms / reps / n_pos, 4),
        "bit_exact": exact,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": peak_kind, "bytes_per_token": per_tok_bytes,
                     "hbm_floor_tok_s": round(floor_tok_s, 1),
                     "frac_of_floor": round(tok_s / world / floor_tok_s, 4),
                     "bytes_note": "every position's weights counted; the batched prompt "
                                   "positions share weight reads"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * len(prompt),
                "d2h_bytes_per_step": 4 * n_new + 4},
        "receipt": {"model_digest": rc["model_digest"], "model_digest_v1": rc["model_digest_v1"]},
        "gpu_launches": launches * world, "clocks": clk, "cpu_baseline": cpu}


def sess_kind_name(sess):
    try:
        return {0: "per-op graph", 1: "fused per-op graph", 2: "persistent kernel"}.get(
            int(sess.step_kind), "?")
    except Exception:
        return "?"


def run_sharded(args, world, rank, local, ctx, stream, cfg):
    """N > 1: every matvec is row-sharded over the ranks and y is reassembled on
    every rank inside the timed region.

    Default (weak scaling): each rank owns a full-size shard -- the configured
    matrix -- of a matrix N times taller (rank 0's shard is the N = 1 matrix,
    rank r's is drawn with its own seed), so per-GPU work stays fixed as N
    grows and the all-gather moves N times the rows. --strong: the configured
    matrix itself is split into N contiguous row ranges (fixed total work).

    Q4_K / Q6_K with --launch step (default): one vtq_linear_list_gather launch
    per rotation of the weight copies (the same launches as N = 1), each
    storing its rows into every rank's y over NVLink and signalling every rank
    once; a launch waits for the previous launch's arrivals, so ranks run at
    most one launch apart, and the timed region ends with a wait for the last
    launch's rows. Other formats: local matvec + NCCL all-gather per matvec."""
    import torch
    import torch.distributed as dist
    import vtq
    from vtq import synth, shard
    strong = args.strong
    host_x = [synth.activation(f"{args.config}.x.{n}", 1, n) for dt, n, r in cfg]
    if strong:
        for (dt, n, r) in cfg:
            if r % world:
                raise SystemExit(f"{args.config}: {r} rows do not split evenly over {world} ranks")
        host_w = [synth.weight(dt, f"{args.config}.w.{n}x{r}", r, n) for dt, n, r in cfg]
        rows_log = [r for dt, n, r in cfg]
        rng = [shard.row_range(r, world, rank) for dt, n, r in cfg]
    else:
        tag = f".rank{rank}" if rank else ""
        host_w = [synth.weight(dt, f"{args.config}.w.{n}x{r}{tag}", r, n) for dt, n, r in cfg]
        rows_log = [r * world for dt, n, r in cfg]
        rng = [(rank * r, (rank + 1) * r) for dt, n, r in cfg]
    wbytes = sum((b - a) * vtq.row_bytes(dt, n) for (dt, n, r), (a, b) in zip(cfg, rng))
    copies = max(1, -(-ROTATE_MIN_BYTES // wbytes))
    if strong:
        weights = [[ctx.upload(dt, host_w[i], n, r, *rng[i]) for i, (dt, n, r) in enumerate(cfg)]
                   for _ in range(copies)]
    else:
        weights = [[ctx.upload(dt, host_w[i], n, r) for i, (dt, n, r) in enumerate(cfg)]
                   for _ in range(copies)]
    xs = [torch.from_numpy(x).cuda() for x in host_x]
    ys = [torch.empty(b - a, device="cuda") for a, b in rng]
    fused = all(dt in (vtq.Q4_K, vtq.Q6_K) for dt, n, r in cfg) and world <= 8 and \
        os.environ.get("VTQ_GATHER", "fused") == "fused"
    use_list = fused and args.launch == "step"
    cap = min(args.per_launch if args.per_launch > 0 else 10, vtq.LIST_MAX // len(cfg))
    per = max(d for d in range(1, cap + 1) if args.steps % d == 0) if use_list else 1
    steps = max(copies, min(args.steps, 2000)) // copies * copies
    offs = [sum(rows_log[:i]) for i in range(len(cfg))]
    if fused:
        gat = vtq.Gather(ctx, sum(rows_log))
        full = [device_view(gat.y_ptr + 4 * offs[i], rows_log[i]) for i in range(len(cfg))]
    else:
        full = [torch.empty(rl, device="cuda") for rl in rows_log]

    def launch(c, nsteps, wait=True):
        """nsteps steps from weight copy c. Fused: returns after enqueueing
        launches that signal every rank once per launch (list) or once per
        step (per-matvec kernels: only the step's last matvec signals, its
        system fence covering the step's earlier stores). wait=True: the
        launch waits for the PREVIOUS launch's arrivals from every rank;
        wait=False starts such a chain."""
        if use_list:
            gat.linear_list([(weights[(c + j) % copies][i], xs[i].data_ptr(),
                              offs[i] + rng[i][0]) for j in range(nsteps) for i in range(len(cfg))],
                            wait_signals=world if wait else 0)
            return
        for j in range(nsteps):
            for i in range(len(cfg)):
                w = weights[(c + j) % copies][i]
                if fused:
                    last = i == len(cfg) - 1
                    gat.linear(w, xs[i].data_ptr(), rng[i][0], rows_log[i], offs[i],
                               wait_signals=world if (last and (wait or j > 0)) else 0,
                               defer=not last)
                else:
                    ctx.linear_ptr(w, xs[i].data_ptr(), ys[i].data_ptr(), 1)
                    dist.all_gather_into_tensor(full[i], ys[i])

    def drain():
        """Consume the one outstanding launch's arrivals (y complete everywhere)."""
        if fused:
            gat.wait(world)

    launch(0, copies if use_list else 1, wait=False)
    if not use_list:
        for c in range(1, copies):
            launch(c, 1)
    drain()
    torch.cuda.synchronize()
    # Parity. Strong: the gathered y equals the oracle's full y bit for bit on
    # every rank. Weak: this rank's rows of the gathered y equal the oracle for
    # its shard, and every rank holds the same gathered y (bit checksum).
    from oracle import oracle as O
    threads = max(1, (os.cpu_count() or 1) // world)
    exact = True
    refs = []
    for i, (dt, n, r) in enumerate(cfg):
        name = {12: "q4_k_integer", 14: "q6_k_integer"}.get(dt)
        ref = O.linear(name, host_x[i], host_w[i], 1, n, r, threads) if name else \
            O.linear_dispatch(dt, host_x[i], host_w[i], n, r, threads=threads)
        refs.append(ref)

    def check():
        ok = True
        for i, (dt, n, r) in enumerate(cfg):
            got = full[i].cpu().numpy()
            mine = got if strong else got[rng[i][0]:rng[i][1]]
            ok &= bool(np.array_equal(mine.view(np.uint32), refs[i].view(np.uint32)))
            bits = torch.tensor([int(got.view(np.uint32).astype(np.uint64).sum() % (1 << 62))],
                                dtype=torch.int64, device="cuda")
            hi, lo = bits.clone(), bits.clone()
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            ok &= int(hi.item()) == int(lo.item())
        return ok

    exact &= check()
    K = args.steps if fused else steps

    def block():
        """K steps that start and end with no arrival outstanding."""
        for k in range(0, K, per):
            launch(k % copies, min(per, K - k), wait=k > 0)
        drain()

    for _ in range(max(1, -(-max(3, args.warmup) // K))):
        block()
    torch.cuda.synchronize()
    graph = None
    if fused:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
            block()
        graph.replay()
        torch.cuda.synchronize()
    run_block = graph.replay if graph is not None else block
    a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a_.record(stream)
    run_block()
    b_.record(stream)
    torch.cuda.synchronize()
    est = torch.tensor([max(a_.elapsed_time(b_), 1e-3)], device="cuda")
    dist.all_reduce(est, op=dist.ReduceOp.MAX)
    replays = max(5, int(-(-args.min_ms // float(est.item()))))
    clocks = ClockSampler(local)
    dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(replays + 1)]
    evs[0].record(stream)
    for r_ in range(replays):
        run_block()
        evs[r_ + 1].record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    dist.barrier()
    exact &= check()  # the timed launches' gathered y
    rep_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(replays)]
    ms = torch.tensor([statistics.median(rep_ms)], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    steps = K
    step_bytes = sum(algo_bytes(dt, n, r) for dt, n, r in cfg) * (1 if strong else world)
    value = step_bytes * steps / (ms / 1e3) / 1e9
    # Local kernel time alone (no collective), for the roofline of the shard.
    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    durs = []
    for k in range(20):
        ev[0].record(stream)
        if use_list:
            ctx.linear_list([(weights[(k + j) % copies][i], xs[i].data_ptr(), ys[i].data_ptr())
                             for j in range(per) for i in range(len(cfg))])
        else:
            for i in range(len(cfg)):
                ctx.linear_ptr(weights[k % copies][i], xs[i].data_ptr(), ys[i].data_ptr(), 1)
        ev[1].record(stream)
        torch.cuda.synchronize()
        durs.append(ev[0].elapsed_time(ev[1]))
    launch_steps = per if use_list else 1
    local_bytes = launch_steps * sum(
        (b - a) * vtq.row_bytes(dt, n) + 4 * n + 4 * (b - a) for (dt, n, r), (a, b) in zip(cfg, rng))
    if not use_list:
        local_bytes /= len(cfg)
    peak, peak_kind = peaks()
    avg_launch = statistics.median(durs) / (1 if use_list else len(cfg))
    achieved = local_bytes / (avg_launch / 1e3) / 1e9
    gather_bytes = sum(4 * rl for rl in rows_log)
    # e2e: pinned host x -> device, local matvecs + gather, full y -> pinned host,
    # lock-step (each step waits for its own arrivals before y is copied out).
    px = [torch.from_numpy(x).pin_memory() for x in host_x]
    py = [torch.empty(rl, dtype=torch.float32).pin_memory() for rl in rows_log]
    e2e_steps = max(20, min(1000, steps // 2))
    dist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for k in range(e2e_steps):
        for i in range(len(cfg)):
            xs[i].copy_(px[i], non_blocking=True)
        if fused:
            launch(k % copies, 1, wait=False)
            drain()
        else:
            launch(k % copies, 1)
        for i in range(len(cfg)):
            py[i].copy_(full[i], non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    ems = torch.tensor([f0.elapsed_time(f1)], device="cuda")
    dist.all_reduce(ems, op=dist.ReduceOp.MAX)
    e2e = {"value": round(step_bytes * e2e_steps / (float(ems.item()) / 1e3) / 1e9, 2),
           "unit": "GB/s", "h2d_bytes_per_step": sum(4 * n for dt, n, r in cfg),
           "d2h_bytes_per_step": sum(4 * rl for rl in rows_log), "steps": e2e_steps}
    flag = torch.tensor([1 if exact else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    exact = bool(flag.item())
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms / steps, 5),
            "steps_match": steps == args.steps,
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": args.config,
                       "matvecs": [f"{vtq.formats.NAMES[dt]} {n}->{r}" for dt, n, r in cfg],
                       "batch": 1,
                       "shards": ("the configured matrices split over the ranks" if strong else
                                  "each rank: a full-size shard of an N-times taller matrix"),
                       "parallelism": f"rows sharded x{world} + " + (
                           f"fused NVLink all-gather in one vtq_linear_list_gather launch per "
                           f"{per} steps (rows stored into every rank's y, one arrival signal "
                           "per launch, waited for one launch later)" if use_list else
                           "fused NVLink all-gather per matvec" if fused else
                           "NCCL all-gather of y"),
                       "l2": f"inputs larger than L2: {copies} rotating weight copies per rank "
                             f"({copies * wbytes / 1e6:.0f} MB)",
                       "timing": (f"CUDA graph of the {steps} steps ending with the wait for the "
                                  f"last launch's rows, replayed {replays} times; median replay"
                                  if fused else
                                  f"{replays} eager blocks of {steps} steps (kernel + all_gather "
                                  "per matvec); median block") +
                                 "; CUDA events, max over ranks"},
            "bit_exact": exact,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": peak_kind,
                         "kernel": "kq_list_kernel (local shard)" if use_list else
                         "kq_matvec_kernel (local shard)",
                         "bytes_per_launch": local_bytes,
                         "avg_launch_us": round(1e3 * avg_launch, 3)},
            "nvlink": {"all_gather_bytes_per_step": gather_bytes},
            "parity": "gathered y bit-identical to the oracle on every rank, before and after "
                      "the timed region",
            "e2e": e2e, "gpu_launches": replays * ((-(-steps // per) + 1) if use_list
                                                   else steps * len(cfg) + 1),
            "clocks": clk, "cpu_baseline": None}), flush=True)
    if fused:
        torch.cuda.synchronize()
        dist.barrier()
        gat.close()
    dist.destroy_process_group()
    if not exact:
        raise SystemExit(f"rank {rank}: sharded result differs from the oracle")


def device_view(ptr, n):
    """A float32 torch view of n floats at device address ptr (no copy)."""
    import torch

    class _A:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                    "version": 3}
    return torch.as_tensor(_A(), device="cuda")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="vtq", choices=["vtq", "reference"])
    ap.add_argument("--config", default=DEFAULT_CFG)
    ap.add_argument("--launch", default="step", choices=["step", "single"],
                    help="k-quant matvecs: one vtq_linear_list launch per step (default) or "
                         "one vtq_linear launch per matvec")
    ap.add_argument("--per-launch", type=int, default=0,
                    help="--launch step: at most this many consecutive steps per "
                         "vtq_linear_list launch (0: 10); the largest divisor of --steps")
    ap.add_argument("--min-ms", type=float, default=250.0,
                    help="device time of the timed region (graph replays of --steps steps)")
    ap.add_argument("--no-sub", action="store_true",
                    help="default config: skip the Q6_K head and decode sub-results")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sharded", action="store_true",
                    help="run the row-sharded path (fused gather) even with one rank")
    ap.add_argument("--strong", action="store_true",
                    help="N > 1: split the configured matrices over the ranks (fixed total work) "
                         "instead of one full-size shard per rank")
    ap.add_argument("--launches-only", action="store_true",
                    help="profiling mode: one weight copy, W + K plain launches per matvec, "
                         "no graph, no timing output (for ncu captures)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world, rank, local = setup_dist()

    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.config == PREFILL_CFG_NAME:
        run_prefill(args, world, rank, local)
        return
    if args.config == DECODE_CFG:
        run_decode(args, world, rank, local)
        return

    import torch
    import torch.distributed as dist
    import vtq
    from vtq import synth

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    ctx = vtq.Context(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)

    cfg = synth.CONFIGS[args.config]
    if world > 1 or args.sharded:
        if not dist.is_initialized():
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29533")
            dist.init_process_group("nccl", rank=0, world_size=1,
                                    device_id=torch.device("cuda", local))
        run_sharded(args, world, rank, local, ctx, stream, cfg)
        return
    line = run_matvec(args, ctx, stream, args.config)
    if not line:
        return
    if args.config == DEFAULT_CFG and not args.no_sub:
        # The rest of the metric in the same run: the Q6_K head matvec and the
        # decode loop, each bit-checked.
        sub = run_matvec(args, ctx, stream, "c3_q6_k_head_4096x32000", sub=True)
        line["sub"] = {"c3_q6_k_head_4096x32000": sub}
        ctx.close()
        torch.cuda.synchronize()
        line["sub"][DECODE_CFG] = decode_measure(args, 1, 0, local, sub=True)
        ok = sub["bit_exact"] and line["sub"][DECODE_CFG]["bit_exact"]
        line["bit_exact_all"] = bool(line["bit_exact"] and ok)
    print(json.dumps(line), flush=True)
    if not line.get("bit_exact_all", line["bit_exact"]):
        raise SystemExit("bench: an output differs from the oracle")


def run_matvec(args, ctx, stream, cfg_name, sub=False):
    """One GPU: every matvec of the configuration per step, weights resident.

    The timed work is a CUDA graph of exactly --steps steps (step i reads
    weight copy i mod copies, so the weights read between two reads of the
    same copy exceed L2), replayed until at least --min-ms of device time has
    passed; `value` uses the median replay. --launch step (default for
    Q4_K/Q6_K): each step is ONE vtq_linear_list launch over the step's
    matvecs; --launch single: one vtq_linear launch per matvec."""
    import torch
    import vtq
    from vtq import synth
    from oracle import oracle as O
    cfg = synth.CONFIGS[cfg_name]
    kquant = all(dt in (vtq.Q4_K, vtq.Q6_K) for dt, n, r in cfg)
    mode = args.launch if kquant else "single"
    step_bytes = sum(algo_bytes(dt, n, r) for dt, n, r in cfg)
    wbytes = sum(r * vtq.row_bytes(dt, n) for dt, n, r in cfg)
    copies = max(1, -(-ROTATE_MIN_BYTES // wbytes))
    if args.launches_only and mode != "step":
        copies = 1
    host_w = [synth.weight(dt, f"{cfg_name}.w.{n}x{r}", r, n) for dt, n, r in cfg]
    host_x = [synth.activation(f"{cfg_name}.x.{n}", 1, n) for dt, n, r in cfg]
    weights = [[ctx.upload(dt, host_w[i], n, r) for i, (dt, n, r) in enumerate(cfg)]
               for _ in range(copies)]
    xs = [torch.from_numpy(x).cuda() for x in host_x]
    ys = [torch.empty(r, device="cuda") for dt, n, r in cfg]
    launches_per_step = 1 if mode == "step" else len(cfg)

    # Steps per list launch: --per-launch, else the largest divisor of K up to
    # 10 (so every launch of the timed graph carries the same work).
    cap = min(args.per_launch if args.per_launch > 0 else 10, vtq.LIST_MAX // len(cfg))
    per = max(d for d in range(1, cap + 1) if args.steps % d == 0) if mode == "step" else 1

    def step(c, events=None, nsteps=1):
        """nsteps consecutive steps from weight copy c on (list mode: one launch)."""
        if events is not None:
            events[0].record(stream)
        if mode == "step":
            ctx.linear_list([(weights[(c + j) % copies][i], xs[i].data_ptr(), ys[i].data_ptr())
                             for j in range(nsteps) for i in range(len(cfg))])
        else:
            for i in range(len(cfg)):
                ctx.linear_ptr(weights[c][i], xs[i].data_ptr(), ys[i].data_ptr(), 1)
        if events is not None:
            events[1].record(stream)

    for c in range(copies):
        step(c)
    torch.cuda.synchronize()
    if args.launches_only:
        for k in range(args.warmup + args.steps - 1):
            step(k % copies, nsteps=per)
        torch.cuda.synchronize()
        print(json.dumps({"launches_only": True, "config": cfg_name,
                          "launches": (args.warmup + args.steps) * launches_per_step}))
        return None

    K = args.steps
    g = torch.cuda.CUDAGraph()
    n_launch = 0
    with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
        for k in range(0, K, per):
            step(k % copies, nsteps=min(per, K - k))
            n_launch += 1 if mode == "step" else len(cfg)
    # Warm-up: W steps (graph replays of K steps, at least one).
    warm_replays = max(1, -(-args.warmup // K))
    for _ in range(warm_replays):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    est = max(a.elapsed_time(b), 1e-3)
    replays = max(5, int(-(-args.min_ms // est)))

    # ---- timed region: device time, events on the launching stream ----
    clocks = ClockSampler(torch.cuda.current_device())
    torch.cuda.synchronize()
    clocks.start()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(replays + 1)]
    evs[0].record(stream)
    for r_ in range(replays):
        g.replay()
        evs[r_ + 1].record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    rep_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(replays)]
    total_ms = evs[0].elapsed_time(evs[-1])
    med = statistics.median(rep_ms)
    value = step_bytes * K / (med / 1e3) / 1e9

    # Bit check of the outputs the timed graph left (every weight copy holds
    # the same bytes, so every step's y is the oracle's y).
    threads = os.cpu_count() or 1
    exact = True
    for i, (dt, n, r) in enumerate(cfg):
        ref = O.linear({12: "q4_k_integer", 14: "q6_k_integer"}[dt], host_x[i], host_w[i],
                       1, n, r, threads) if dt in (12, 14) else \
            O.linear_dispatch(dt, host_x[i], host_w[i], n, r, threads=threads)
        exact &= bool(np.array_equal(ys[i].cpu().numpy().view(np.uint32), ref.view(np.uint32)))

    # Eager per-launch events (no graph, no programmatic overlap), for context.
    pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    durs = []
    for k in range(max(3, 60 // len(cfg))):
        step(k % copies, pair)
        torch.cuda.synchronize()
        durs.append(pair[0].elapsed_time(pair[1]) / launches_per_step)
    per_launch_bytes = step_bytes * K / n_launch
    avg_ms = med / n_launch
    peak, peak_kind = peaks()
    achieved = per_launch_bytes / (avg_ms / 1e3) / 1e9
    traffic = profile_traffic(cfg_name, mode, K / n_launch)

    # ---- e2e through the public C ABI with host buffers ----
    # Each of the `per` steps a call covers has its own page-locked x and y.
    px = [[torch.from_numpy(x).pin_memory() for x in host_x] for _ in range(per)]
    py = [[torch.full((r,), float("nan")).pin_memory() for dt, n, r in cfg] for _ in range(per)]
    host_calls = [ctx.prepare_list([(weights[(c + j) % copies][i], px[j][i].data_ptr(),
                                     py[j][i].data_ptr())
                                    for j in range(per) for i in range(len(cfg))], host=True)
                  for c in range(copies)] if mode == "step" else None

    def host_call(c):
        """`per` steps through the public C ABI with host buffers."""
        if mode == "step":
            host_calls[c]()
        else:
            for i in range(len(cfg)):
                ctx.linear_ptr(weights[c][i], px[0][i].data_ptr(), py[0][i].data_ptr(), 1,
                               host=True)

    for k in range(5):
        host_call((k * per) % copies)
    e2e_calls = max(20, min(2000, int(2 * args.min_ms / max(med / K * per, 1e-3) / 8)))
    e2e_steps = e2e_calls * per
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    f0.record(stream)
    for k in range(e2e_calls):
        host_call((k * per) % copies)
    f1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    # Host-pointer calls return only when y is in host memory: the wall clock
    # around them is the end-to-end time (the events bracket the same span).
    ems = max(f0.elapsed_time(f1), 1e3 * wall)
    e2e_value = step_bytes * e2e_steps / (ems / 1e3) / 1e9
    e2e_exact = all(np.array_equal(py[j][i].numpy().view(np.uint32),
                                   ys[i].cpu().numpy().view(np.uint32))
                    for j in range(per) for i in range(len(cfg)))
    h2d = sum(4 * n for dt, n, r in cfg)
    d2h = sum(4 * r for dt, n, r in cfg) if mode == "step" else \
        sum(4 * r + 256 for dt, n, r in cfg)

    cpu = None
    if not args.no_cpu_baseline:
        cpu = {"all_cores": cpu_baseline(cfg_name, threads, budget_s=8.0 if sub else 12.0),
               "one_core": cpu_baseline(cfg_name, 1, budget_s=4.0 if sub else 8.0)}
        cpu = dict(cpu["all_cores"], one_core=cpu["one_core"])
    launch_desc = (f"one vtq_linear_list launch per {per} step(s) (persistent kernel over "
                   f"those steps' {per * len(cfg)} matvecs)" if mode == "step"
                   else "one vtq_linear launch per matvec")
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": 1,
        "steps": K, "warmup": warm_replays * K, "steps_match": True,
        "ms_per_step": round(med / K, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": cfg_name,
                   "matvecs": [f"{vtq.formats.NAMES[dt]} {n}->{r}" for dt, n, r in cfg],
                   "batch": 1, "parallelism": "1 GPU",
                   "l2": f"inputs larger than L2: {copies} rotating weight copies "
                         f"({copies * wbytes / 1e6:.0f} MB)",
                   "launch": launch_desc,
                   "timing": f"CUDA graph of the {K} steps, replayed {replays} times "
                             f"({total_ms:.0f} ms of device time); value from the median "
                             "replay; CUDA events on the launching stream"},
        "pct_of_peak": round(100 * value / peak, 1),
        "bit_exact": exact,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": traffic, "peak_source": peak_kind,
                     "kernel": "kq_list_kernel" if mode == "step" else
                     ("kq_matvec_kernel" if kquant else "canon_matvec_kernel"),
                     "bytes_per_launch": per_launch_bytes,
                     "avg_launch_us": round(avg_ms * 1e3, 3),
                     "avg_launch_source": "median graph replay / launches in it",
                     "eager_launch_us": round(1e3 * statistics.mean(durs), 3),
                     "replay_ms_min_med_max": [round(min(rep_ms), 4), round(med, 4),
                                               round(max(rep_ms), 4)]},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps, "bit_exact": e2e_exact,
                "call": (f"one vtq_linear_list call with VTQ_PTR_HOST per {per} steps (every "
                         "step its own page-locked x and y; the kernel reads x and writes y "
                         "in place, the call returns when y is in host memory)")
                if mode == "step" else "vtq_linear with VTQ_PTR_HOST per matvec"},
        "gpu_launches": n_launch * replays,
        "clocks": clk,
        "cpu_baseline": cpu,
    }


if __name__ == "__main__":
    main()
