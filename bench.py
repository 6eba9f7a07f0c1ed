"""Benchmark of the B200 sqrt(N) sparse attention: fwd + bwd at the
north-star shape (B=1, H=16, D=128, S=65536, bf16), one sequence per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 it is launched with torch.distributed.run (one rank per GPU); each
rank processes its own sequence (batch sharded across GPUs, no collective on
the data path), the timed region is bracketed by barriers and the time is the
max over ranks.  Rank 0 prints one JSON line.

A "step" is one forward + backward pass over one [1, 16, 65536, 128] bf16
batch (q, k, v and an upstream gradient dO), through the public API
(cron_root_attention + torch.autograd.grad).  Throughput is algorithmic
sparse TFLOP/s: 14 * D * visible pairs per (b, h) (4 forward + 10 backward);
masked work done by a kernel is not counted.

Beside the headline the same JSON line carries:
  * per-kernel CUDA-event times of every kernel of the step (forward and
    relay build through their C-ABI calls, the backward kernels through
    cra_bwd_kernel_times), each against its roofline; ``roofline`` is the
    kernel with the largest share of the step;
  * BASELINE configs 4 and 5 (forward only, strong scaling): c4 = B1 H32
    S262144 D128 fp16 with the heads split across the ranks, c5 = B1 H16
    S524288 D128 bf16 with the one sequence split across the ranks (NCCL
    all-gathers of the global rows and the halo).  Rank 0 first runs each
    whole workload alone (the 1-GPU baseline), then every rank runs its
    share; c5's split output is compared with the 1-GPU output.

``--impl reference`` times the reference's CPU algorithm for the same step
(this repository's restatement of cpu_reference.cra_cpu_fast plus its
autograd backward, oracle/cra_oracle.py) on the host cores.  Each of its
steps is a bounded sample: the forward + backward of one (b, h) head of the
16, heads taken in turn, so 16 steps cover one whole north-star step.
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

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "cron-root-attention_b200"))

METRIC = "fwd & fwd+bwd ms and sparse-attn TFLOP/s, H16 D128 S=64K, at 1/2/4/8 B200"
B, H, S, D = 1, 16, 65536, 128  # overridable with --heads / --seq for small profiling runs
SEED = 2
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def visible_pairs(seq_len: int, top_k: int = 2) -> int:
    """Exact visible (query, key) pairs per (b, h) for the FLOP count: local
    window + strided keys + top_k relay rows per visible block, with
    W = ceil(sqrt(S)) and the relay active for S > 2048."""
    import math
    W = math.isqrt(seq_len - 1) + 1 if seq_len > 1 else 1  # ceil(sqrt(S))
    m = torch.arange(seq_len, dtype=torch.int64)
    ls = (m - W + 1).clamp(min=0)
    local = (m - ls + 1).sum().item()
    strided = ((ls + W - 1) // W).sum().item()
    relay = (top_k * (ls // W)).sum().item() if seq_len > 2048 else 0
    return int(local + strided + relay)


def pairs_per_head() -> int:
    return visible_pairs(S)


def flops():
    p = pairs_per_head() * B * H
    return 4.0 * D * p, 10.0 * D * p  # forward, backward


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while active."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, val in zip(names, parts[4:8]):
                if val.lower() in ("active", "1"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(rank: int, dev):
    g = torch.Generator().manual_seed(SEED + rank)
    host = [torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).pin_memory() for _ in range(4)]
    return host, [t.to(dev) for t in host]


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_sample_steps(n_steps: int, n_warmup: int):
    """Restated reference CPU path (fp32): each step is the forward + backward
    of ONE (b, h) head, heads taken in turn (step i -> head i mod H), all host
    threads.  Returns (seconds per step, steps timed, threads)."""
    from oracle import cra_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    heads = {}

    def head(h):  # q, k, v, dO of head h (own seeded generator), drawn once
        if h not in heads:
            g = torch.Generator().manual_seed(SEED * 1000 + h)
            heads[h] = tuple(torch.randn(1, 1, S, D, generator=g).to(torch.bfloat16).float() for _ in range(4))
        return heads[h]

    for i in range(n_warmup):
        O.forward_backward(*head(i % H), dtype=torch.float32)
    for i in range(min(n_steps, H)):
        head(i)  # inputs drawn outside the timed region
    t0 = time.perf_counter()
    for i in range(n_steps):
        O.forward_backward(*head(i % H), dtype=torch.float32)
    return (time.perf_counter() - t0) / n_steps, n_steps, torch.get_num_threads()


def cpu_baseline_line(per_step_s: float, n: int, threads: int) -> dict:
    f = 14.0 * D * pairs_per_head()  # one head
    return {"value": f / per_step_s / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "cpu_model": cpu_model(), "host_cpus": os.cpu_count(),
            "sample": f"{n} steps, each the fwd+bwd of one of the {H} heads of B1 S{S} D{D} (heads in turn), "
                      f"fp32 restatement of cpu_reference.cra_cpu_fast + autograd backward, "
                      f"{per_step_s:.2f} s per head = {per_step_s * H:.1f} s per whole {H}-head step"}


def run_reference(args, rank, world):
    """The reference's CPU algorithm (restated, oracle/cra_oracle.py) on the
    host cores.  Rank 0 alone works; other ranks exit without work."""
    if rank != 0:
        return
    n = max(1, min(args.steps, 24))  # bounded: about 3 s per step on 16 cores
    per, n, threads = cpu_sample_steps(n, min(args.warmup, 3))
    cb = cpu_baseline_line(per, n, threads)
    line = {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": n, "steps_requested": args.steps, "warmup": min(args.warmup, 3), "ms_per_step": per * 1e3,
            "ms_per_full_step": per * H * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"fwd+bwd B{B} H{H} S{S} D{D}; one step = one head's fwd+bwd (bounded "
                                   f"sample), heads in turn", "seq_len": S, "heads": H, "head_dim": D,
                       "global_batch": B},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of each
# kernel, from one ncu capture of the committed kernels at B1 H8 S65536 D128
# bf16, scaled by H / 8 (every kernel's traffic grows in proportion to the
# heads).  None where no capture of the current kernel exists.
TRAFFIC_H8 = {
    "fwd_kernel": 528.839680e6,
    "relay_build_kernel": 141.839616e6,
    "delta_kernel": 277.032192e6,
    "keyglobal_kernel": 797.732864e6,
    "reduce_kernel": 84.846848e6,
    "keylocal_kernel": 788.465664e6,
    "dq_kernel": 660.156416e6,
    "dq_convert_kernel": None,
}


def kernel_work(name: str, W: int, NG: int, fused: bool = False):
    """(bound, algorithmic work per launch, unit) of each kernel at B x H x S x D.
    Attention kernels: the useful (unmasked) MMA FLOPs they perform -- 2 D per
    visible pair per GEMM; forward 2 GEMMs, dQ pass 3 (S, dP, dQ), key passes
    4 (S, dP, dV, dK) over their own pairs.  HBM kernels: bytes they must
    move."""
    import math
    m = torch.arange(S, dtype=torch.int64)
    ls = (m - W + 1).clamp(min=0)
    local = int((m - ls + 1).sum())
    glob = pairs_per_head() - local
    bh = B * H
    eb = 2
    if name == "fwd_kernel":
        return "tensor", 4.0 * D * pairs_per_head() * bh, "TFLOP/s"
    if name == "dq_kernel":
        return "tensor", 6.0 * D * pairs_per_head() * bh, "TFLOP/s"
    # key passes: 4 GEMMs (S, dP, dV, dK); cra_bwd_fused adds dQ there (5)
    gemms = 5 if (fused and D == 128) else 4
    if name == "keyglobal_kernel":
        return "tensor", 2.0 * gemms * D * glob * bh, "TFLOP/s"
    if name == "keylocal_kernel":
        return "tensor", 2.0 * gemms * D * local * bh, "TFLOP/s"
    if name == "dq_convert_kernel":  # fp32 accumulator read, dQ written
        return "hbm", (4 + eb) * S * D * bh, "GB/s"
    if name == "relay_build_kernel":  # K read once + chosen K / V rows read and written as G
        return "hbm", (S * D * eb + 4 * NG * D * eb) * bh, "GB/s"
    if name == "delta_kernel":  # O, dO read; lse read; lse2, delta written (fp32, padded)
        spad = math.ceil(S / 128) * 128
        zero = 4 * spad * D if (fused and D == 128) else 0  # fused: the dQ accumulator is zeroed
        return "hbm", (2 * S * D * eb + 4 * S + 8 * spad + zero) * bh, "GB/s"
    if name == "reduce_kernel":  # n_split partials of dG_k, dG_v read, dG written (fp32)
        return "hbm", None, "GB/s"
    return "other", None, None


def run_ours(args, rank, world, local_rank):
    import ctypes
    import cron_root_attention as cra
    from cron_root_attention import _lib
    from cron_root_attention.core import _err_word

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    host, (q, k, v, do) = make_inputs(rank, dev)
    stream = torch.cuda.current_stream(dev)
    f_fwd, f_bwd = flops()

    def step(q, k, v, do):
        q.requires_grad_(True)
        k.requires_grad_(True)
        v.requires_grad_(True)
        o = cra.cron_root_attention(q, k, v)
        return o, torch.autograd.grad(o, (q, k, v), do)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return t.item()

    def timed(fn, n):
        barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / n)

    for _ in range(max(args.warmup, 3)):
        step(q, k, v, do)
    torch.cuda.synchronize(dev)

    if args.mode != "all":
        # profiling mode: only the chosen pass, nothing else launched
        fn = (lambda: cra.cron_root_attention(q, k, v)) if args.mode == "fwd" else (lambda: step(q, k, v, do))
        with torch.no_grad() if args.mode == "fwd" else torch.enable_grad():
            ms = timed(fn, args.steps)
        if rank == 0:
            print(json.dumps({"mode": args.mode, "ms": ms, "B": B, "H": H, "S": S, "D": D}), flush=True)
        return

    # --- headline: fwd + bwd, inputs resident in HBM (each input 268 MB > L2)
    with ClockSampler(local_rank) as clk:
        time.sleep(0.6)  # let the sampler start before the timed region
        ms_step = timed(lambda: step(q, k, v, do), args.steps)
    clocks = clk.summary()

    # --- forward alone
    with torch.no_grad():
        ms_fwd = timed(lambda: cra.cron_root_attention(q, k, v), args.steps)

    # --- every kernel of the step, timed alone with CUDA events on this stream
    L = _lib.lib()
    W = L.cra_window(S)
    NG = L.cra_global_rows(S, 1, 2)
    NB = (S + W - 1) // W
    gk = torch.empty(B, H, NG, D, device=dev, dtype=torch.bfloat16)
    gv = torch.empty_like(gk)
    gsrc = torch.empty(B, H, NB, 2, device=dev, dtype=torch.int32)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S, device=dev, dtype=torch.float32)
    st = _lib.strides3
    sp = stream.cuda_stream
    err = _err_word(dev).data_ptr()
    args_relay = (k.data_ptr(), v.data_ptr(), st(k), st(v), B, H, S, D, 1, 1, 2, None, gk.data_ptr(), gv.data_ptr(),
                  gsrc.data_ptr(), sp)
    _lib.check(L.cra_relay_build(*args_relay), "relay")
    args_fwd = (q.data_ptr(), k.data_ptr(), v.data_ptr(), gk.data_ptr(), gv.data_ptr(), st(q), st(k), st(v),
                B, H, H, S, D, 1, 1, 2, ctypes.c_float(D ** -0.5), o.data_ptr(), st(o), lse.data_ptr(), err, sp)
    for _ in range(3):
        L.cra_fwd(*args_fwd)
    kern_ms = {"fwd_kernel": timed(lambda: L.cra_fwd(*args_fwd), args.steps),
               "relay_build_kernel": timed(lambda: L.cra_relay_build(*args_relay), args.steps)}
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws_bytes = L.cra_bwd_workspace_bytes(B, H, H, S, D, 1, 2)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    nmax = 8
    ms_arr = (ctypes.c_float * nmax)()
    names = (ctypes.c_char_p * nmax)()
    nk = ctypes.c_int(0)
    samples = {}
    for it in range(3 + args.steps):
        _lib.check(L.cra_bwd_kernel_times(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(), gk.data_ptr(),
            gv.data_ptr(), gsrc.data_ptr(), st(q), st(k), st(v), st(o), st(do), B, H, H, S, D, 1, 1, 2,
            ctypes.c_float(D ** -0.5), None, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), st(dq), st(dk), st(dv),
            None, ws.data_ptr(), ws_bytes, err, sp, ms_arr, names, nmax, ctypes.byref(nk), 0), "cra_bwd_kernel_times")
        if it >= 3:
            for i in range(nk.value):
                samples.setdefault(names[i].decode(), []).append(ms_arr[i])
    for name, xs in samples.items():
        kern_ms[name] = max_over_ranks(statistics.median(xs))
    n_bwd_kernels = nk.value
    # the alternative backward (cra_bwd_fused: dQ inside the key passes by
    # fp32 atomic adds, no dQ pass), timed the same way for comparison
    fws_bytes = L.cra_bwd_fused_workspace_bytes(B, H, H, S, D, 1, 2)
    del ws
    ws = torch.empty(fws_bytes, device=dev, dtype=torch.uint8)
    fsamples = {}
    for it in range(3 + args.steps):
        _lib.check(L.cra_bwd_kernel_times(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(), gk.data_ptr(),
            gv.data_ptr(), gsrc.data_ptr(), st(q), st(k), st(v), st(o), st(do), B, H, H, S, D, 1, 1, 2,
            ctypes.c_float(D ** -0.5), None, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), st(dq), st(dk), st(dv),
            None, ws.data_ptr(), fws_bytes, err, sp, ms_arr, names, nmax, ctypes.byref(nk), 1), "fused kernel times")
        if it >= 3:
            for i in range(nk.value):
                fsamples.setdefault(names[i].decode(), []).append(ms_arr[i])
    fused_ms = {n: max_over_ranks(statistics.median(xs)) for n, xs in fsamples.items()}
    del ws, dq, dk, dv
    bwd_ms = sum(v for n, v in kern_ms.items() if n not in ("fwd_kernel", "relay_build_kernel"))

    # --- end to end through the public API with host buffers: every step copies
    # q, k, v, dO from pinned memory to the device, runs fwd + bwd, and copies
    # dq, dk, dv back into pinned memory.  The copies are pipelined the way a
    # serving loop would: step i + 1's inputs go up (H2D stream) and step
    # i - 1's gradients come down (D2H stream) while step i computes; PCIe is
    # full duplex.  Device inputs and host outputs are double-buffered; events
    # order each buffer's reuse.
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dev_in = [[torch.empty_like(t) for t in (q, k, v, do)] for _ in range(2)]
    out_host = [[torch.empty_like(host[0]).pin_memory() for _ in range(3)] for _ in range(2)]
    in_free = [None, None]    # event: compute finished reading dev_in[s]
    out_free = [None, None]   # event: D2H finished writing out_host[s]

    def e2e_run(n):
        h2d.wait_stream(stream)  # the first upload starts inside the timed region
        for i in range(n):
            s = i & 1
            with torch.cuda.stream(h2d):
                if in_free[s] is not None:
                    h2d.wait_event(in_free[s])
                for dst, src in zip(dev_in[s], host):
                    dst.copy_(src, non_blocking=True)
                up = torch.cuda.Event()
                up.record(h2d)
            stream.wait_event(up)
            _, grads = step(*(t.detach() for t in dev_in[s]))
            done = torch.cuda.Event()
            done.record(stream)
            in_free[s] = done
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                if out_free[s] is not None:
                    d2h.wait_event(out_free[s])
                for hbuf, g in zip(out_host[s], grads):
                    g.record_stream(d2h)
                    hbuf.copy_(g, non_blocking=True)
                down = torch.cuda.Event()
                down.record(d2h)
                out_free[s] = down
        stream.wait_stream(h2d)
        stream.wait_stream(d2h)

    e2e_run(2)
    n_e2e = max(2, min(args.steps, 8))
    ms_e2e = timed(lambda: e2e_run(n_e2e), 1) / n_e2e
    nbytes = host[0].numel() * host[0].element_size()
    del dev_in, out_host, host, gk, gv, gsrc, o, lse

    assert cra.check_device_errors(dev) == 0, "a kernel gave up on a bounded wait"

    extra = {}
    if not args.no_strong:
        del q, k, v, do
        torch.cuda.empty_cache()
        for cfg in ("c4", "c5"):
            extra.update(strong_config(cfg, args, rank, world, local_rank))
        assert cra.check_device_errors(dev) == 0, "a kernel gave up on a bounded wait"

    if rank != 0:
        return
    peaks, peak_src = load_peaks()
    kernels = {}
    for name, ms in kern_ms.items():
        bound, work, unit = kernel_work(name, W, NG)
        ent = {"ms": ms, "share_of_step": ms / ms_step}
        if work is not None:
            if bound == "tensor":
                ach, peak = work / (ms * 1e-3) / 1e12, float(peaks["bf16_tflops"])
            else:
                ach, peak = work / (ms * 1e-3) / 1e9, float(peaks["hbm_gbs"])
            ent.update({"bound": bound, "achieved": ach, "peak": peak, "unit": unit, "frac": ach / peak})
        t8 = TRAFFIC_H8.get(name)
        ent["traffic"] = t8 * (H / 8) if (t8 is not None and (S, D) == (65536, 128)) else None
        kernels[name] = ent
    top = max((n for n in kernels if "frac" in kernels[n]), key=lambda n: kernels[n]["ms"])
    kt = kernels[top]
    roofline = {"kernel": top, "bound": kt["bound"], "achieved": kt["achieved"], "peak": kt["peak"],
                "unit": kt["unit"], "frac": kt["frac"], "traffic": kt["traffic"],
                "peak_source": f"{peak_src} " + ("bf16 dense (burst)" if kt["bound"] == "tensor" else "HBM copy"),
                "kernel_ms": kt["ms"]}
    line = {
        "metric": METRIC,
        "value": world * (f_fwd + f_bwd) / (ms_step * 1e-3) / 1e12,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": ms_step,
        "fwd_ms": ms_fwd,
        "fwd_tflops": world * f_fwd / (ms_fwd * 1e-3) / 1e12,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"fwd+bwd B{B} H{H} S{S} D{D} bf16 per GPU (north-star shape), seed {SEED}+rank",
                   "global_batch": B * world, "seq_len": S, "heads": H, "head_dim": D,
                   "parallelism": f"batch-sharded x{world}, no data-path collective",
                   "l2": "inputs larger than L2 (each of q, k, v, dO is 268 MB; L2 126 MB)",
                   "flops_per_step": f"fwd {f_fwd / 1e9:.3f} GFLOP + bwd {f_bwd / 1e9:.3f} GFLOP per GPU"},
        "roofline": roofline,
        "kernels": kernels,
        "bwd_alternatives": {
            "three_pass": {"entry": "cra_bwd (used by the API)", "kernels_ms": bwd_ms,
                           "dq": "separate dQ pass, fixed summation order"},
            "fused": {"entry": "cra_bwd_fused", "kernels_ms": sum(fused_ms.values()), "per_kernel_ms": fused_ms,
                      "dq": "added by the key passes with fp32 atomics (order varies between calls)"}},
        "e2e": {"value": world * (f_fwd + f_bwd) / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": ms_e2e, "h2d_bytes_per_step": 4 * nbytes, "d2h_bytes_per_step": 3 * nbytes,
                "steps": n_e2e, "copies": "pipelined across steps on separate H2D / D2H streams",
                "limit": "host copies: 1.07 GB up + 0.81 GB down per step per GPU over PCIe; at N > 1 every "
                         "GPU's copies share the host's memory path"},
        # our kernels per timed step: relay build + forward, then the backward's
        # kernels as cra_bwd_kernel_times reported them
        "gpu_launches": (2 + n_bwd_kernels) * args.steps,
        "clocks": clocks,
    }
    line.update(extra)
    if world == 1:
        per, n, threads = cpu_sample_steps(1, 0)
        line["cpu_baseline"] = cpu_baseline_line(per, n, threads)
    print(json.dumps(line), flush=True)


STRONG = {  # BASELINE configs 4 and 5: (B, H, S, D, dtype, seed, sigma)
    "c4": (1, 32, 262144, 128, torch.float16, 3, 0.5),
    "c5": (1, 16, 524288, 128, torch.bfloat16, 4, 1.0),
}


def strong_config(cfg: str, args, rank: int, world: int, local_rank: int) -> dict:
    """Forward of BASELINE config 4 (heads split across ranks) or 5 (one
    sequence split across ranks), strong scaling.  Inputs are drawn on the
    device from a seeded generator (the same values on every rank).  Rank 0
    first times the whole workload alone on its GPU (the 1-GPU baseline);
    then every rank runs its share, timed between barriers, max over ranks.
    c5 at N > 1 also gathers head 0 of the split output and compares it with
    the 1-GPU output (same kernel, different query-tile boundaries)."""
    import cron_root_attention as cra
    from cron_root_attention.parallel import seq_parallel_forward, seq_shard, shard_units
    dev = torch.device("cuda", local_rank)
    Bc, Hc, Sc, Dc, dt, seed, sig = STRONG[cfg]
    g = torch.Generator(device=dev).manual_seed(seed)
    q, k, v = (torch.randn(Bc, Hc, Sc, Dc, generator=g, device=dev).mul_(sig).to(dt) for _ in range(3))
    steps = max(3, min(args.steps, 20))

    def run_timed(fn, n, ranks_all: bool):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / n
        if world > 1 and ranks_all:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = t.item()
        return ms

    out = {}
    with torch.no_grad():
        # 1-GPU baseline: rank 0, whole workload
        ms1, ref0 = None, None
        if rank == 0:
            whole = lambda: cra.cron_root_attention(q, k, v)
            for _ in range(3):
                whole()
            ms1 = run_timed(whole, steps, False) if world == 1 else None
            if world > 1:  # time it alone while the other ranks wait at the barrier below
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(steps):
                    whole()
                e1.record()
                torch.cuda.synchronize(dev)
                ms1 = e0.elapsed_time(e1) / steps
            if cfg == "c5" and world > 1:
                ref0 = whole()[:, 0].float()
        if world > 1:
            # the split run
            if cfg == "c4":
                (b, h0, h1), = shard_units(Bc, Hc, world, rank)
                qs, ks, vs = (t[:, h0:h1].contiguous() for t in (q, k, v))
                fn = lambda: cra.cron_root_attention(qs, ks, vs)
            else:
                s0, s1 = seq_shard(Sc, world, rank)
                qs, ks, vs = (t[:, :, s0:s1].contiguous() for t in (q, k, v))
                fn = lambda: seq_parallel_forward(qs, ks, vs, Sc)
            del q, k, v
            for _ in range(3):
                fn()
            with ClockSampler(local_rank) as clk:
                time.sleep(0.3)
                msN = run_timed(fn, steps, True)
            if cfg == "c5":
                o = fn()[:, 0].float().contiguous()
                s0s1 = [seq_shard(Sc, world, r) for r in range(world)]
                mx = max(e - b for b, e in s0s1)
                buf = torch.zeros(Bc, mx, Dc, device=dev)
                buf[:, :o.shape[1]] = o
                parts = [torch.empty_like(buf) for _ in range(world)]
                torch.distributed.all_gather(parts, buf)
                if rank == 0:
                    split = torch.cat([p[:, :e - b] for p, (b, e) in zip(parts, s0s1)], dim=1)
                    diff = (split - ref0).abs()
                    bar = 2e-3 + 2.0 ** -7 * (ref0.abs() + 1.0)  # one bf16 ulp of the output scale
                    out["c5_vs_1gpu"] = {"head": 0, "max_abs": diff.max().item(), "mean_abs": diff.mean().item(),
                                         "parity_ok": bool((diff <= bar).all().item())}
        else:
            msN = ms1
            clk = None
    if rank == 0:
        f = 4.0 * Dc * visible_pairs(Sc) * Bc * Hc
        out.update({f"{cfg}_ms": msN, f"{cfg}_ms_1gpu": ms1, f"{cfg}_speedup_vs_1": ms1 / msN,
                    f"{cfg}_tflops": f / (msN * 1e-3) / 1e12,
                    f"{cfg}_config": {"B": Bc, "H": Hc, "S": Sc, "D": Dc, "dtype": str(dt).replace("torch.", ""),
                                      "pass": "forward", "scaling": "strong",
                                      "parallelism": ("heads" if cfg == "c4" else "sequence") + f" split x{world}",
                                      "data": "synthetic, seeded on the device"}})
        if clk is not None:
            out[f"{cfg}_clocks"] = clk.summary()
    return out


# Times the reference's own GPU path (cron_root_attention_v14 with its Triton
# kernels, unmodified, from baseline/_ref) at the north-star shape on one GPU:
# forward alone and forward + backward through its public API.  Runs in a
# child process, since the reference's package has the same name as this
# repository's.
_REF_TRITON_CHILD = r"""
import json, statistics, sys, time
import torch
ref = sys.argv[1]
B, H, S, D, steps, warmup = (int(a) for a in sys.argv[2:8])
sys.path.insert(0, ref)
import cron_root_attention as R
assert R.__file__.startswith(ref), R.__file__
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev).manual_seed(2)
q, k, v, do = (torch.randn(B, H, S, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(4))
def fwd():
    with torch.no_grad():
        return R.cron_root_attention(q, k, v)
def step():
    qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
    R.cron_root_attention(qq, kk, vv).backward(do)
def timed(fn):
    t0 = time.time()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    first_s = time.time() - t0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, first_s
fwd_ms, fwd_first = timed(fwd)
step_ms, step_first = timed(step)
if len(sys.argv) > 8:  # heads 0 and 1 of the output and the gradients, for the comparison
    qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
    o = R.cron_root_attention(qq, kk, vv)
    o.backward(do)
    torch.save({n: t[:, :2].detach().cpu() for n, t in (("o", o), ("dq", qq.grad), ("dk", kk.grad), ("dv", vv.grad))},
               sys.argv[8])
# forward alone at BASELINE configs 2 and 4 (one GPU)
fwd_cfg = {}
for name, (b_, h_, s_, d_, sd, sig) in {"c2": (1, 12, 16384, 64, 1, 0.5), "c4": (1, 32, 262144, 128, 3, 0.5)}.items():
    g = torch.Generator(device=dev).manual_seed(sd)
    q, k, v = ((torch.randn(b_, h_, s_, d_, device=dev, generator=g) * sig).to(torch.float16) for _ in range(3))
    fwd_cfg[name] = timed(fwd)[0]
    del q, k, v
print(json.dumps({"fwd_ms": fwd_ms, "fwdbwd_ms": step_ms, "warmup_s": [fwd_first, step_first], "fwd_cfg": fwd_cfg}))
"""


def run_reference_triton(args):
    ref = os.path.join(ROOT, "baseline", "_ref")
    line = {"impl": "reference_triton", "metric": METRIC, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": f"north star fwd and fwd+bwd, B{B} H{H} S{S} D{D} bf16", "B": B, "H": H, "S": S,
                       "D": D, "data": "synthetic, seeded on the device (seed 2)"}}
    if not os.path.isdir(os.path.join(ref, "cron_root_attention")):
        line["unavailable"] = "baseline/_ref holds no install of the reference"
        print(json.dumps(line), flush=True)
        return
    import tempfile
    dump = os.path.join(tempfile.mkdtemp(), "ref_out.pt")
    try:
        r = subprocess.run([sys.executable, "-c", _REF_TRITON_CHILD, ref, str(B), str(H), str(S), str(D),
                            str(args.steps), str(max(args.warmup, 3)), dump],
                           capture_output=True, text=True, timeout=1500)
    except subprocess.TimeoutExpired:
        line["unavailable"] = "the reference's Triton path did not finish in 1500 s"
        print(json.dumps(line), flush=True)
        return
    out = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not out:
        line["unavailable"] = "the reference's Triton path failed: " + (r.stderr.strip().splitlines() or ["?"])[-1][:300]
        print(json.dumps(line), flush=True)
        return
    res = json.loads(out[-1])
    fwd_f, bwd_f = flops()
    line.update({"fwd_ms": res["fwd_ms"], "fwd_tflops": fwd_f / (res["fwd_ms"] * 1e-3) / 1e12,
                 "ms_per_step": res["fwdbwd_ms"], "value": (fwd_f + bwd_f) / (res["fwdbwd_ms"] * 1e-3) / 1e12,
                 "unit": "TFLOP/s", "higher_is_better": True, "warmup_s": res["warmup_s"]})
    # this library on the same inputs: heads 0 and 1 of o, dq, dk, dv against the reference's
    if os.path.exists(dump):
        import cron_root_attention as cra
        refo = torch.load(dump)
        dev = torch.device("cuda", 0)
        g = torch.Generator(device=dev).manual_seed(2)
        q, k, v, do = (torch.randn(B, H, S, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(4))
        qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
        o = cra.cron_root_attention(qq, kk, vv)
        o.backward(do)
        cmp = {}
        for n, t in (("o", o), ("dq", qq.grad), ("dk", kk.grad), ("dv", vv.grad)):
            a, b = t[:, :2].detach().float().cpu(), refo[n].float()
            cmp[n] = {"max_abs": (a - b).abs().max().item(), "mean_abs": (a - b).abs().mean().item(),
                      "rel_l2": ((a - b).norm() / b.norm()).item()}
        line["vs_reference_gpu_heads01"] = cmp
        # forward at configs 2 and 4, this library beside the reference, same inputs
        other = {}
        for name, (b_, h_, s_, d_, sd, sig) in {"c2": (1, 12, 16384, 64, 1, 0.5),
                                               "c4": (1, 32, 262144, 128, 3, 0.5)}.items():
            g = torch.Generator(device=dev).manual_seed(sd)
            q, k, v = ((torch.randn(b_, h_, s_, d_, device=dev, generator=g) * sig).to(torch.float16)
                       for _ in range(3))
            with torch.no_grad():
                for _ in range(3):
                    cra.cron_root_attention(q, k, v)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(args.steps):
                    cra.cron_root_attention(q, k, v)
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / args.steps
            f = 4.0 * d_ * visible_pairs(s_) * b_ * h_
            rms = res.get("fwd_cfg", {}).get(name)
            other[name] = {"shape": f"B{b_} H{h_} S{s_} D{d_} fp16", "ours_fwd_ms": ms,
                           "ours_fwd_tflops": f / (ms * 1e-3) / 1e12, "reference_fwd_ms": rms,
                           "reference_fwd_tflops": f / (rms * 1e-3) / 1e12 if rms else None}
            del q, k, v
        line["fwd_configs"] = other
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference_triton"],
                    help="reference: the reference's CPU algorithm; reference_triton: the reference's own "
                         "Triton GPU path, installed unmodified in baseline/_ref (rank 0, one GPU)")
    ap.add_argument("--mode", default="all", choices=["all", "fwd", "fwdbwd"],
                    help="fwd / fwdbwd: time only that pass (for profiling runs)")
    ap.add_argument("--no-strong", action="store_true", help="skip the config 4 / 5 strong-scaling legs")
    ap.add_argument("--heads", type=int, default=H)
    ap.add_argument("--seq", type=int, default=S)
    args = ap.parse_args()
    globals()["H"], globals()["S"] = args.heads, args.seq
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        backend = "nccl" if args.impl == "ours" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group(backend=backend)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.impl == "reference_triton":
            if rank == 0:
                run_reference_triton(args)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
