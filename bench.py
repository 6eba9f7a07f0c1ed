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

``--impl reference`` times the reference's CPU algorithm for the same step
(this repository's restatement of cpu_reference.cra_cpu_fast plus its
autograd backward, oracle/cra_oracle.py) on the host cores, on a bounded
sample (one of the 16 heads per step), and reports the same metric.
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


def cpu_baseline(steps: int = 1):
    """Restated reference CPU path (fp32) on one head: forward + backward."""
    from oracle import cra_oracle as O
    g = torch.Generator().manual_seed(SEED)
    q, k, v, do = (torch.randn(1, 1, S, D, generator=g).to(torch.bfloat16).float() for _ in range(4))
    threads = torch.get_num_threads()
    t0 = time.perf_counter()
    for _ in range(steps):
        O.forward_backward(q, k, v, do, dtype=torch.float32)
    dt = (time.perf_counter() - t0) / steps
    f = 14.0 * D * pairs_per_head()  # one head
    return {"value": f / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"1 of {H} heads per step (B1 S{S} D{D}), fp32 restatement of cpu_reference.cra_cpu_fast "
                      f"+ autograd backward, {dt:.2f} s per head"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        pass  # the CPU path has no warm-up state worth timing; a sample per step below
    cb = cpu_baseline(steps=max(1, min(args.steps, 3)))
    ms = 14.0 * D * pairs_per_head() * H / (cb["value"] * 1e12) * 1e3  # full step = 16 heads
    line = {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"fwd+bwd B{B} H{H} S{S} D{D} (CPU sample: one head per step)",
                       "seq_len": S, "heads": H, "head_dim": D, "global_batch": B},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


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

    # --- dominant kernel, timed alone through the C ABI on this stream:
    # the attention forward kernel (cra_fwd launches exactly one kernel)
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
    _lib.check(L.cra_relay_build(k.data_ptr(), v.data_ptr(), st(k), st(v), B, H, S, D, 1, 1, 2, None,
                                 gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), sp), "relay")
    args_fwd = (q.data_ptr(), k.data_ptr(), v.data_ptr(), gk.data_ptr(), gv.data_ptr(), st(q), st(k), st(v),
                B, H, H, S, D, 1, 1, 2, ctypes.c_float(D ** -0.5), o.data_ptr(), st(o), lse.data_ptr(),
                _err_word(dev).data_ptr(), sp)
    for _ in range(3):
        L.cra_fwd(*args_fwd)
    ms_kernel = timed(lambda: L.cra_fwd(*args_fwd), args.steps)
    ms_relay = timed(lambda: L.cra_relay_build(k.data_ptr(), v.data_ptr(), st(k), st(v), B, H, S, D, 1, 1, 2,
                                               None, gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), sp),
                     args.steps)

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

    assert cra.check_device_errors(dev) == 0, "a kernel gave up on a bounded wait"

    if rank != 0:
        return
    peaks, peak_src = load_peaks()
    achieved = f_fwd / (ms_kernel * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    # DRAM bytes per forward launch: ncu dram__bytes_read.sum + write.sum of one
    # launch at H = 8 (profiles/kernels_northstar_h8.md: 405.9 + 117.1 MB),
    # scaled by H / 8 (the traffic grows in proportion to the heads)
    traffic = (405.935360e6 + 119.967488e6) * (H / 8) if (S, D) == (65536, 128) else None
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
        "roofline": {"kernel": "fwd_kernel<128,bf16>", "bound": "tensor", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_src} bf16 dense (burst)", "kernel_ms": ms_kernel,
                     "relay_build_ms": ms_relay,
                     # K read once (norms) + the chosen K / V rows read and written as G
                     "relay_build_gbs": (B * H * S * D * 2 + 4 * B * H * NG * D * 2) / (ms_relay * 1e-3) / 1e9},
        "e2e": {"value": world * (f_fwd + f_bwd) / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": ms_e2e, "h2d_bytes_per_step": 4 * nbytes, "d2h_bytes_per_step": 3 * nbytes,
                "steps": n_e2e, "copies": "pipelined across steps on separate H2D / D2H streams"},
        "gpu_launches": 7 * args.steps,
        "clocks": clocks,
    }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline()
    print(json.dumps(line), flush=True)


def run_config(args, rank, world, local_rank):
    """BASELINE configs 4 and 5 (forward only, multi-GPU):
    c4: B1 H32 D128 S262144 fp16, heads split evenly across ranks, no collective
        (strong scaling: the total work is fixed);
    c5: B1 H16 D128 S524288 bf16, one sequence split by W-blocks across ranks,
        global rows and halo exchanged with NCCL all-gathers (strong scaling)."""
    import cron_root_attention as cra
    from cron_root_attention.parallel import seq_parallel_forward, seq_shard, shard_units
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.config == "c4":
        Bc, Hc, Sc, Dc, dt, seed, sig = 1, 32, 262144, 128, torch.float16, 3, 0.5
    else:
        Bc, Hc, Sc, Dc, dt, seed, sig = 1, 16, 524288, 128, torch.bfloat16, 4, 1.0
    g = torch.Generator().manual_seed(seed)
    if args.config == "c4":
        (b, h0, h1), = shard_units(Bc, Hc, world, rank)
        # each rank draws only its own heads' rows: the same values as slicing the full tensors
        q, k, v = (torch.randn(Bc, Hc, Sc, Dc, generator=g)[:, h0:h1].mul_(sig).to(dt).to(dev) for _ in range(3))
        fn = lambda: cra.cron_root_attention(q, k, v)
    else:
        s0, s1 = seq_shard(Sc, world, rank)
        q, k, v = (torch.randn(Bc, Hc, Sc, Dc, generator=g)[:, :, s0:s1].mul_(sig).to(dt).to(dev) for _ in range(3))
        fn = lambda: seq_parallel_forward(q, k, v, Sc)
    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clk:
            time.sleep(0.6)
            e0.record()
            for _ in range(args.steps):
                fn()
            e1.record()
            torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = t.item()
    f_fwd = 4.0 * Dc * visible_pairs(Sc) * Bc * Hc
    if rank == 0:
        print(json.dumps({"metric": METRIC, "config": {"workload": args.config, "B": Bc, "H": Hc, "S": Sc, "D": Dc,
                                                      "dtype": str(dt).replace("torch.", ""),
                                                      "parallelism": ("heads" if args.config == "c4" else "sequence")
                                                      + f" split x{world}"},
                          "value": f_fwd / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "n_gpus": world,
                          "steps": args.steps, "scaling": "strong", "clocks": clk.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="all", choices=["all", "fwd", "fwdbwd"],
                    help="fwd / fwdbwd: time only that pass (for profiling runs)")
    ap.add_argument("--config", default="northstar", choices=["northstar", "c4", "c5"],
                    help="c4 / c5: BASELINE configs 4 and 5 (forward, strong scaling over --gpus)")
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
        elif args.config != "northstar":
            run_config(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
