#!/usr/bin/env python3
"""Benchmark of the quantized Dense forward path on B200.

Metric: quant Dense weight GB/s (GEMV, % HBM) and TFLOP/s (batched, % tensor)
at 1/2/4/8 B200. The configuration quoted "across 1/2/4/8 GPUs" is BASELINE config 5's
column-sharded Dense 16384 -> 65536, FP4 (E2M1, 2 codes/byte, reference layout), W ~ N(0, 0.02),
x ~ N(0, 1), seed 4: 512 MiB of packed weights, more than the 126 MB L2 (no flush needed).

  value    weight GB/s of the whole job at batch 1: one step = one forward of the sharded layer
           over all N GPUs (welvet_b200_sharded_dense_execute_device, fused gather: each rank's
           GEMV stores its columns into every rank's output over NVLink, then a flag exchange),
           every rank holding the whole output when the step ends. N = 1 runs the same call on
           one GPU. Strong scaling (the layer is the same at every N).
  batched  the same layer at batch 256, TFLOP/s (tcgen05 GEMM + fused gather)
  e2e      the metric through the C ABI with host buffers (pinned): welvet_dense_execute at
           N = 1 (the reference's own entry point), welvet_b200_sharded_dense_execute at N > 1;
           x in and the whole output out over the bus every step
  sharded  per N: fused, nccl (local forward + ncclAllGather + permute) and compute-only (the
           shard as a one-GPU layer, no gather) at batch 1 and 256
  volume   BASELINE config 5's volume (2x2x2 cells of 4 Dense 4096x4096 FP4 + ReLU, batch 64):
           one GPU runs the whole chain; N GPUs the cell-per-GPU pipeline
  configs  (N = 1) configs 1-4 at their sizes: C1 us, C2 FP4 / Int8 / E4M3 GB/s (grouped,
           single launches, chain, host buffers; FP4 also on sigma = 2 weights, whose codes are
           not all zero), C3 SwiGLU at M = 1 / 16 / 128 / 512, C4 RMSNorm + MHA + SwiGLU
  reference_cuda  (N = 1) the reference's own CUDA Dense session (oracle/_ref: its kernels
           rebuilt for sm_100a) on C1, C2 and C3's Gate projection, host buffers, per call
  cpu_baseline    the oracle port (reference decode + sequential fp64 dot) on the box's host
           cores, on a bounded row sample of the headline layer

--impl reference times the reference semantics on the host cores (the oracle port of
kernels.cu:130-161 with the reference decode): the reference ships no CPU matvec, and this
is the CPU implementation of the path.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C5_IN, C5_OUT = 16384, 65536
FP4, E4M3, E5M2, INT8 = 16, 4, 5, 9
SIGMA = 0.02
C5_BYTES = C5_OUT * C5_IN // 2  # FP4: 0.5 B / weight
L2_BYTES = 126 * 1000 * 1000
METRIC = "quant Dense weight GB/s (GEMV, % HBM) and TFLOP/s (batched, % tensor) at 1/2/4/8 B200"


def config_for(world: int) -> dict:
    return {"workload": "C5 column-sharded Dense 16384->65536 FP4 (W~N(0,0.02), x~N(0,1), seed 4), batch 1: "
                        "one forward per step, output all-gathered on every rank",
            "global_batch": 1, "seq_len": 1, "parallelism": f"column-sharded x{world} (fused NVLink gather)",
            "l2": "inputs larger than L2 (512 MiB of packed weights per step)",
            "weight_bytes_per_step": C5_BYTES}


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_value(name: str, key: str):
    """A number from a committed ncu summary under profiles/ (a `key: value` line)."""
    try:
        for ln in open(os.path.join(ROOT, "profiles", name)):
            if ln.startswith(key + ":"):
                return float(ln.split(":")[1].split()[0])
    except Exception:
        pass
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, polled through NVML (the data
    nvidia-smi's clocks.sm / clocks_event_reasons.* report) every ~0.5 ms while the timed
    legs run. Read-only."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int):
        self.index = index
        self.sm = []
        self.mask = 0
        self.max_mhz = None
        self.err = None
        self._stop = threading.Event()
        self.active = threading.Event()

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.index]) if vis and vis.split(",")[self.index].isdigit() else self.index
            self.h = N.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
        except Exception as e:  # no NVML: reported as unsampled
            self.err = str(e)
        return self

    def _poll(self):
        N = self.N
        while not self._stop.is_set():
            if not self.active.is_set():
                self.active.wait(0.05)
                continue
            try:
                self.sm.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
                self.mask |= N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception as e:
                self.err = str(e)
                return
            time.sleep(0.0005)

    def __exit__(self, *a):
        self._stop.set()
        self.active.set()
        if hasattr(self, "t"):
            self.t.join(timeout=2)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "error": self.err}
        reasons = sorted(n for n, bit in self.REASONS.items() if self.mask & bit)
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.sm), "source": "NVML (nvmlDeviceGetClockInfo / GetCurrentClocksEventReasons)"}


# --------------------------------------------------------------------------------- CPU legs

def oracle_rows_sample(seconds: float):
    """The oracle port on all host threads over a row sample of the headline layer (rows
    split over the threads): (GB/s of packed weights, threads, sample text)."""
    import oracle as O
    threads = os.cpu_count() or 1
    rows = 1024
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((rows, C5_IN)) * SIGMA).astype(np.float32)
    raw, sc = O.pack(FP4, w)
    x = rng.standard_normal((1, C5_IN)).astype(np.float32)
    O.dense_forward(FP4, raw, sc, x, C5_IN, rows, -1, None, threads)  # warm
    n = 0
    t0 = time.perf_counter()
    while True:
        O.dense_forward(FP4, raw, sc, x, C5_IN, rows, -1, None, threads)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    gbs = n * rows * C5_IN / 2 / dt / 1e9
    return gbs, threads, (f"{n} forwards of a {rows}-row sample (1/{C5_OUT // rows} of the layer) of the "
                          f"16384->65536 FP4 layer, B=1 ({dt:.1f} s): reference decode + sequential fp64 dot "
                          f"(oracle/oracle.c), rows split over {threads} threads")


def cpu_baseline(seconds: float):
    gbs, threads, sample = oracle_rows_sample(seconds)
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}


def run_reference(args):
    """--impl reference: the reference semantics on the host cores, same metric and config."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    import oracle as O
    threads = os.cpu_count() or 1
    rows = 256
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((rows, C5_IN)) * SIGMA).astype(np.float32)
    raw, sc = O.pack(FP4, w)
    x = rng.standard_normal((1, C5_IN)).astype(np.float32)
    # a step is a bounded sample of one forward of the layer: `rows` of its 65536 rows
    for _ in range(args.warmup):
        O.dense_forward(FP4, raw, sc, x, C5_IN, rows, -1, None, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.dense_forward(FP4, raw, sc, x, C5_IN, rows, -1, None, threads)
    dt = time.perf_counter() - t0
    val = args.steps * rows * C5_IN / 2 / dt / 1e9
    sample = (f"per step {rows} of the layer's {C5_OUT} rows (B=1): reference decode + sequential fp64 dot "
              f"(oracle/oracle.c; the reference ships no host matvec), rows split over {threads} threads")
    line = {"metric": METRIC, "value": val, "unit": "GB/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3 * (C5_OUT / rows),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp4 codes, fp64 accumulate",
            "data": "synthetic", "config": config_for(world),
            "cpu_baseline": {"value": val, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------------- GPU legs

class Ctx:
    """Per-process state of a GPU run: torch, the library, ranks, timing helpers."""

    def __init__(self, args):
        import torch
        self.torch = torch
        self.args = args
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180))
            self.dist = dist
        import welvet.cuda_b200 as W
        from welvet.cuda_b200 import volume as V
        W.cuda_init()
        self.W, self.V = W, V
        self.comm = V.Comm.from_torch(self.local) if self.world > 1 else V.Comm(0, 1, self.local, V.Comm.new_job_id())
        self.stream = torch.cuda.current_stream()
        self.launches = 0  # our kernel launches inside the headline's timed region
        self.graphs = []   # captured graphs, released before the communicator
        self.flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], device="cuda", dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, fn, steps: int, warmup: int) -> float:
        """ms per step over `steps` back-to-back steps after `warmup`, CUDA events on the launching
        stream, barrier + synchronize on both sides, max over ranks."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        self.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            fn()
        e1.record(self.stream)
        self.barrier()
        return self.max_over_ranks(e0.elapsed_time(e1)) / steps

    def timed_calls(self, calls, steps: int, warmup: int) -> float:
        """ms per step for a rotation of forwards (`calls`, one step each, in the order they must
        run): after one eager pass the rotation is captured as one CUDA graph (replayed whole)
        and as one graph per call (the last steps % len(calls)); `warmup` steps, then exactly
        `steps` timed, barrier + synchronize on both sides, CUDA events on the launching stream,
        max over ranks."""
        torch = self.torch
        for f in calls:
            f()
        torch.cuda.synchronize()
        whole = torch.cuda.CUDAGraph()
        with torch.cuda.graph(whole):
            for f in calls:
                f()
        singles = []
        for f in calls:
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                f()
            singles.append(gph)
        self.graphs.extend([whole, *singles])

        def run(n):
            q, r = divmod(n, len(calls))
            for _ in range(q):
                whole.replay()
            for i in range(r):
                singles[i].replay()
        return self._timed_run(run, steps, warmup)

    def _timed_run(self, run, steps: int, warmup: int) -> float:
        torch = self.torch
        run(warmup)
        self.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        run(steps)
        e1.record(self.stream)
        self.barrier()
        return self.max_over_ranks(e0.elapsed_time(e1)) / steps

    def graphed(self, fn, n: int = 1):
        """`fn` captured in n CUDA graphs of one call each, replayed in turn (a sharded call
        alternates between two output buffers, so it is captured twice). One eager call first."""
        import itertools
        torch = self.torch
        fn()
        torch.cuda.synchronize()
        graphs = []
        for _ in range(n):
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                fn()
            graphs.append(gph)
        self.graphs.extend(graphs)
        it = itertools.cycle(graphs)
        return lambda: next(it).replay()

    def timed_each(self, fn, reps: int) -> float:
        """Median µs of single calls, L2 flushed (a 256 MiB write) before each (one GPU)."""
        torch = self.torch
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            self.flush.zero_()
            torch.cuda._sleep(200000)  # the GPU stays busy while the host enqueues the call
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)


def sharded_copies(shard_bytes: int) -> int:
    """Weight copies a rank rotates through so that consecutive steps read more than twice the
    126 MB L2 (one copy when the shard alone is that large)."""
    return max(1, -(-2 * L2_BYTES // max(1, shard_bytes)))


def sharded_legs(c: Ctx, batch: int, steps: int, warmup: int, W_rows, b: int, e: int):
    """Fused, nccl and compute-only forwards of the headline layer at `batch` tokens. Each leg
    rotates over `copies` mounts of this rank's rows (sharded_copies); every sharded object is
    called twice per rotation (its two output buffers)."""
    torch, W, V = c.torch, c.W, c.V
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn((batch, C5_IN), device="cuda", generator=g)
    copies = sharded_copies((e - b) * C5_IN // 2)
    res = {"copies": copies}
    fused = [V.ShardedDense(c.comm, W_rows, C5_IN, C5_OUT, batch, FP4, W.LINEAR, None, V.FUSED) for _ in range(copies)]
    res["fused_ms"] = c.timed_calls([(lambda o=o: o.execute_device_ptrs(x)) for _ in range(2) for o in fused],
                                    steps, warmup)
    for o in fused:
        o.check_error()
    nccl = [V.ShardedDense(c.comm, W_rows, C5_IN, C5_OUT, batch, FP4, W.LINEAR, None, V.NCCL) for _ in range(copies)]
    res["nccl_ms"] = c.timed_calls([(lambda o=o: o.execute_device_ptrs(x)) for _ in range(2) for o in nccl],
                                   steps, warmup)
    for o in nccl:
        o.check_error()
    local = [W.DenseSession(W_rows, batch, FP4) for _ in range(copies)] if e > b else []
    if local:
        pre = torch.empty((batch, e - b), device="cuda")
        res["compute_ms"] = c.timed_calls([(lambda o=o: o.execute_device(x, pre, pre)) for o in local], steps, warmup)
        for o in local:
            o.check_error()
    else:
        res["compute_ms"] = c.timed(lambda: None, steps, warmup)
    return res, fused + nccl, local, x


def run_ours(args):
    c = Ctx(args)
    torch, W, V = c.torch, c.W, c.V
    pk, pk_kind = peaks()
    world, rank = c.world, c.rank
    # ---- C5's volume: one GPU runs the chain, N GPUs the cell-per-GPU pipeline. First, on a
    # fresh communicator: at N = 2 the pipeline read 8.2 ms per forward when timed after the
    # sharded legs, against 1.0 ms timed on its own (cause not isolated).
    volume = run_volume(c, args)
    c.graphs.clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    b, e = V.shard_rows(C5_OUT, world, rank)
    g = torch.Generator(device="cuda").manual_seed(4 * 1000 + rank)
    W_rows = torch.randn((e - b, C5_IN), device="cuda", generator=g) * SIGMA

    with ClockSampler(c.local) as clk:
        # ---- headline: batch 1 (the GEMV), whole job
        clk.active.set()
        s1, fused1, local1, x1 = sharded_legs(c, 1, args.steps, args.warmup, W_rows, b, e)
        # ---- batch 256 (the tcgen05 GEMM)
        s256, fused256, local256, x256 = sharded_legs(c, 256, max(3, min(args.steps, 20)), 3, W_rows, b, e)
        clk.active.clear()
    del W_rows
    torch.cuda.empty_cache()
    ms = s1["fused_ms"]
    value = C5_BYTES / (ms / 1e3) / 1e9
    # per step: k_prep_x + k_gemv_tc (the prepared plan of a layer of >= 8192 rows), plus
    # k_flag_exchange when N > 1
    c.launches = args.steps * (3 if world > 1 else 2)
    flops256 = 2.0 * 256 * C5_OUT * C5_IN

    # roofline of the headline's dominant kernel: this rank's GEMV, timed alone (compute-only
    # leg: the shard as a one-GPU layer, the same kernel and launch plan as the fused call's)
    shard_bytes = (e - b) * C5_IN // 2
    achieved = shard_bytes / (s1["compute_ms"] / 1e3) / 1e9
    traffic_full = profile_value("gemv_tc_fp4_65536x16384_b1.md", "dram_bytes_per_launch")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"],
                "traffic": None if traffic_full is None else traffic_full * (e - b) / C5_OUT,
                "peak_source": f"{pk_kind} hbm_gbs (MEASURED_PEAKS.json, burst copy)",
                "kernel": "k_gemv_tc<FP4,B=1> over this rank's rows (welvet/cuda_b200/csrc/gemv_tc.cu)",
                "algorithmic_bytes_per_launch": shard_bytes,
                "step_frac": value / world / pk["hbm_gbs"],
                "traffic_source": "profiles/gemv_tc_fp4_65536x16384_b1.md (full layer, scaled to this rank's rows)"}
    sharded = {
        "b1": {"fused_ms": s1["fused_ms"], "nccl_ms": s1["nccl_ms"], "compute_ms": s1["compute_ms"],
               "fused_GBps": C5_BYTES / (s1["fused_ms"] / 1e3) / 1e9,
               "nccl_GBps": C5_BYTES / (s1["nccl_ms"] / 1e3) / 1e9,
               "gather_share_fused": max(0.0, 1.0 - s1["compute_ms"] / s1["fused_ms"]),
               "gather_share_nccl": max(0.0, 1.0 - s1["compute_ms"] / s1["nccl_ms"]),
               "gather_bytes": C5_OUT * 4},
        "b256": {"fused_ms": s256["fused_ms"], "nccl_ms": s256["nccl_ms"], "compute_ms": s256["compute_ms"],
                 "fused_TFLOPs": flops256 / (s256["fused_ms"] / 1e3) / 1e12,
                 "nccl_TFLOPs": flops256 / (s256["nccl_ms"] / 1e3) / 1e12,
                 "gather_share_fused": max(0.0, 1.0 - s256["compute_ms"] / s256["fused_ms"]),
                 "gather_share_nccl": max(0.0, 1.0 - s256["compute_ms"] / s256["nccl_ms"]),
                 "gather_bytes": 256 * C5_OUT * 4},
        "what": "ms per forward, max over ranks: fused = the product call (GEMV/GEMM epilogues store into every "
                "rank's output over NVLink + flag exchange); nccl = local forward + ncclAllGather + permute; "
                "compute = this rank's shard as a one-GPU layer, no gather; gather_share = 1 - compute / total"}
    batched = {"value": flops256 / (s256["fused_ms"] / 1e3) / 1e12, "unit": "TFLOP/s",
               "ms_per_forward": s256["fused_ms"],
               "config": "C5 column-sharded Dense 16384->65536 FP4, batch 256 (x~N(0,1): two f16 planes), fused gather",
               "frac": flops256 / (s256["fused_ms"] / 1e3) / 1e12 / (world * pk["bf16_tflops"]),
               "peak": world * pk["bf16_tflops"], "peak_source": f"{pk_kind} bf16_tflops (burst) x {world} GPUs",
               "kernels": "k_split_x + k_gemm_tm<FP4> (+ tail / split-K reduce) + k_flag_exchange"}

    # ---- e2e: the same metric through the C ABI with host buffers
    e2e_steps = max(3, min(args.steps, 20))
    xh = torch.randn((1, C5_IN)).pin_memory()
    yh = torch.zeros((1, C5_OUT)).pin_memory()
    ph = torch.zeros((1, C5_OUT)).pin_memory()
    if world == 1:
        c_exec = W.lib().welvet_dense_execute
        h = local1[0]._h
        px, pp, py = ctypes.c_void_p(xh.data_ptr()), ctypes.c_void_p(ph.data_ptr()), ctypes.c_void_p(yh.data_ptr())

        def e2e_step():
            st = c_exec(h, px, pp, py)
            if st.code != 0:
                raise W.WelvetError(st.code, st.message.decode(errors="replace"))
        api = "welvet_dense_execute via ctypes (pinned host buffers, synchronous per call)"
    else:
        c_exec = W.lib().welvet_b200_sharded_dense_execute
        h = fused1[0]._h
        px, py = ctypes.c_void_p(xh.data_ptr()), ctypes.c_void_p(yh.data_ptr())

        def e2e_step():
            st = c_exec(h, px, None, py)
            if st.code != 0:
                raise W.WelvetError(st.code, st.message.decode(errors="replace"))
        api = "welvet_b200_sharded_dense_execute via ctypes (pinned host buffers, synchronous, every rank)"
    for _ in range(3):
        e2e_step()
    c.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    t_e2e = c.max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": C5_BYTES * e2e_steps / t_e2e / 1e9, "unit": "GB/s", "h2d_bytes_per_step": C5_IN * 4 * world,
           "d2h_bytes_per_step": C5_OUT * 4 * world, "steps": e2e_steps, "api": api}
    c.graphs.clear()
    torch.cuda.synchronize()
    for s in (*fused1, *fused256, *local1, *local256):
        s.release()
    torch.cuda.empty_cache()

    # ---- the same shard with sigma-2 weights (at sigma 0.02 every FP4 code of the layer is
    # zero): the compute leg again, batch 1, the same rotation of copies
    g2 = torch.Generator(device="cuda").manual_seed(4 * 1000 + 500 + rank)
    W2 = torch.randn((e - b, C5_IN), device="cuda", generator=g2) * 2.0
    loc2 = [W.DenseSession(W2, 1, FP4) for _ in range(sharded_copies((e - b) * C5_IN // 2))] if e > b else []
    del W2
    pre2 = torch.empty((1, max(1, e - b)), device="cuda")
    ms_s2 = (c.timed_calls([(lambda o=o: o.execute_device(x1, pre2, pre2)) for o in loc2], args.steps, args.warmup)
             if loc2 else c.timed(lambda: None, args.steps, args.warmup))
    for o in loc2:
        o.check_error()
    c.graphs.clear()
    torch.cuda.synchronize()
    for o in loc2:
        o.release()
    torch.cuda.empty_cache()
    sigma2 = {"compute_ms": ms_s2, "GBps": shard_bytes / (ms_s2 / 1e3) / 1e9,
              "frac": shard_bytes / (ms_s2 / 1e3) / 1e9 / pk["hbm_gbs"],
              "what": "this rank's shard of the headline layer with W ~ N(0, 2) (non-zero FP4 codes), batch 1, "
                      "compute leg (max over ranks)"}

    configs, ref_cuda, cpu = None, None, None
    if world == 1 and not args.no_configs:
        configs = run_configs(c, args, pk)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        ref_cuda = reference_cuda(args)
        cpu = cpu_baseline(args.cpu_seconds)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "fp4 codes, fp32 tensor-core sums, fp64 across chunks", "data": "synthetic",
                "config": config_for(world),
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "batched": batched, "sharded": sharded, "sigma2_companion": sigma2,
                "volume": volume, "configs": configs, "reference_cuda": ref_cuda,
                "gpu_launches": c.launches, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    c.comm.release()
    if c.dist is not None:
        c.dist.barrier()
        c.dist.destroy_process_group()
    return 0


def run_volume(c: Ctx, args):
    """C5 volume: 8 cells x 4 Dense 4096x4096 FP4 + ReLU, batch 64."""
    torch, W, V = c.torch, c.W, c.V
    cells, lpc, width, batch = 8, 4, 4096, 64
    hb, he = V.stage_plan(cells, lpc, c.world)[c.rank]
    vol = V.Volume(2, 2, 2, lpc)
    g = torch.Generator(device="cuda").manual_seed(4 * 1000 + 17)
    for h in range(cells * lpc):  # every rank draws all weights in hop order, binds its own
        w = torch.randn((width, width), device="cuda", generator=g) * SIGMA
        if hb <= h < he:
            vol.bind_dense(vol.coord(h), w, W.RELU, FP4)
        del w
    x = torch.randn((batch, width), device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    y = torch.empty((batch, width), device="cuda")
    steps = max(3, min(c.args.steps, 20))
    if c.world == 1:
        # the 32-hop chain replayed from a CUDA graph (96 launches per forward)
        ms = c.timed_calls([lambda: vol.forward_device(x, y, stream=torch.cuda.current_stream())], steps, 3)
        micro = batch
    else:
        micro = max(8, batch // c.world)
        ms = c.timed(lambda: c.comm.pipeline_forward(vol, (hb, he), x, width, micro, y, c.stream), steps, 3)
    vol.release()
    flops = 2.0 * batch * cells * lpc * width * width
    wbytes = cells * lpc * width * width // 2
    return {"ms_per_forward": ms, "TFLOPs": flops / (ms / 1e3) / 1e12, "weight_GBps": wbytes / (ms / 1e3) / 1e9,
            "micro_batch": micro, "placement": "whole chain on one GPU" if c.world == 1 else
            f"cell-per-GPU pipeline over {c.world} GPUs (NCCL point-to-point)"}


def run_configs(c: Ctx, args, pk):
    """Configs 1-4 on one GPU (sub-records of the line)."""
    torch, W = c.torch, c.W
    out = {}
    hbm = pk["hbm_gbs"]
    tens = pk["bf16_tflops"]

    def wt(shape, seed, sigma):
        return torch.randn(shape, device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed)) * sigma

    # C1: Dense 256 -> 128 E4M3 (scale 1), bias, batch 1: latency (parity case)
    w = wt((128, 256), 0, 0.05)
    bias = np.random.default_rng(0).standard_normal(128) * 0.01
    s = W.DenseSession(w, 1, E4M3, W.LINEAR, bias)
    x = torch.rand((1, 256), device="cuda") * 2 - 1
    y = torch.empty((1, 128), device="cuda")
    us = c.timed_each(lambda: s.execute_device(x, y, y), 20)
    xh, yh = x.cpu().numpy(), np.zeros((1, 128), np.float32)
    s.execute(xh, yh, yh)
    t0 = time.perf_counter()
    for _ in range(50):
        s.execute(xh, yh, yh)
    out["C1"] = {"us_device": us, "us_host_buffers": (time.perf_counter() - t0) / 50 * 1e6,
                 "what": "one forward, L2 flushed before each; host buffers through welvet_dense_execute"}
    s.release()

    # C2: Dense 4096 -> 4096 batch 1; FP4 (sigma 0.02 and 2.0), Int8, E4M3: 64 layers per step
    out["C2"] = {}
    for name, dt, sigma in (("fp4", FP4, SIGMA), ("fp4_sigma2", FP4, 2.0), ("int8", INT8, SIGMA),
                            ("e4m3", E4M3, SIGMA)):
        out["C2"][name] = c2_legs(c, dt, sigma, hbm)

    # C3: SwiGLU 4096 / 14336 E4M3, M in {1, 16, 128, 512}
    d, hid = 4096, 14336
    cell = W.SwigluCell(wt((hid, d), 21, SIGMA), wt((hid, d), 22, SIGMA), wt((d, hid), 23, SIGMA), E4M3)
    out["C3"] = {}
    for m in (1, 16, 128, 512):
        xm = torch.randn((m, d), device="cuda").to(torch.bfloat16).float()
        ym = torch.empty((m, d), device="cuda")
        hm = torch.empty((m, hid), device="cuda")
        us = c.timed_each(lambda: cell.execute_device(xm, ym, hm), 10)
        wbytes = 3 * d * hid
        fl = 2.0 * m * 3 * d * hid
        rec = {"us": us, "weight_GBps": wbytes / us / 1e3, "TFLOPs": fl / us / 1e6}
        rec["frac_hbm"] = rec["weight_GBps"] / hbm
        rec["frac_tensor"] = rec["TFLOPs"] / tens
        out["C3"][f"M{m}"] = rec
    cell.release()

    # C4: RMSNorm + MHA (2048, 16 x 128, causal, RoPE) E4M3 + SwiGLU 2048 / 5632 FP4, 4 x 512 tokens
    out["C4"] = c4_legs(c, tens)
    torch.cuda.empty_cache()
    return out


def c2_legs(c: Ctx, dt: int, sigma: float, hbm: float):
    torch, W = c.torch, c.W
    n, rows, cols = 64, 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(1)
    sess = []
    for _ in range(n):
        w = torch.randn((rows, cols), device="cuda", generator=g) * sigma
        sess.append(W.DenseSession(w, 1, dt))
        del w
    x = torch.randn((1, cols), device="cuda", generator=g)
    outs = [(torch.empty((1, rows), device="cuda"), torch.empty((1, rows), device="cuda")) for _ in range(n)]
    acts = [torch.empty((1, rows), device="cuda") for _ in range(2)]
    pre = torch.empty((1, rows), device="cuda")
    wbytes = rows * cols * (0.5 if dt == FP4 else 1.0) + (4 if dt == INT8 else 0)

    def grouped():
        W.dense_execute_group(sess, [x] * n, [o[0] for o in outs], [o[1] for o in outs])

    def singles():
        for i, s in enumerate(sess):
            s.execute_device(x, outs[i][0], outs[i][1])

    def chain():
        xi = x
        for i, s in enumerate(sess):
            s.execute_device(xi, pre, acts[i & 1])
            xi = acts[i & 1]

    rec = {}
    for name, fn in (("grouped", grouped), ("single_launches", singles), ("chain", chain)):
        ms = c.timed(c.graphed(fn), 10, 3)  # one graph launch per step (64 forwards)
        rec[name + "_GBps"] = n * wbytes / (ms / 1e3) / 1e9
    c.graphs.clear()
    rec["grouped_frac"] = rec["grouped_GBps"] / hbm
    rec["single_frac"] = rec["single_launches_GBps"] / hbm
    # host buffers, one synchronous welvet_dense_execute per layer
    xh = torch.randn((1, cols)).pin_memory()
    yh = torch.zeros((1, rows)).pin_memory()
    c_exec = W.lib().welvet_dense_execute
    px, py = ctypes.c_void_p(xh.data_ptr()), ctypes.c_void_p(yh.data_ptr())
    for s in sess:  # a session records its host-buffer graph on its second call
        c_exec(s._h, px, py, py)
        c_exec(s._h, px, py, py)
    t0 = time.perf_counter()
    for s in sess:
        st = c_exec(s._h, px, py, py)
        if st.code != 0:
            raise W.WelvetError(st.code, st.message.decode(errors="replace"))
    dt_s = time.perf_counter() - t0
    rec["host_buffers_GBps"] = n * wbytes / dt_s / 1e9
    rec["host_buffers_us_per_call"] = dt_s / n * 1e6
    for s in sess:
        s.release()
    return rec


def c4_legs(c: Ctx, tens: float):
    torch, W = c.torch, c.W
    B, S, d, heads, hd, inter = 4, 512, 2048, 16, 128, 5632
    T = B * S

    def wt(shape, seed, sigma=SIGMA):
        return torch.randn(shape, device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed)) * sigma

    x = torch.randn((T, d), device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))
    gamma = np.ones(d, np.float32)
    vol = c.V.Volume(1, 1, 1, 1)
    vol.bind_rmsnorm((0, 0, 0, 0), gamma, 1e-6, W.FLOAT32)
    xn = torch.empty_like(x)
    us_norm = c.timed_each(lambda: vol.forward_device(x, xn), 10)
    vol.release()
    qkvo = [wt((d, d), 31 + i) for i in range(4)]
    mha = W.MhaCell(*qkvo, d_model=d, num_heads=heads, num_kv_heads=heads, head_dim=hd, max_seq_len=S, mask=1, pos=0,
                    dtype=E4M3)
    y = torch.empty_like(x)
    attn = torch.empty((T, d), device="cuda")
    us_mha = c.timed_each(lambda: mha.execute_device(xn, B, S, y, attn), 5)
    mha.release()
    # RMSNorm -> Q projection as one volume: the norm as the GEMM's prologue (default) and as
    # its own kernel (WELVET_B200_NORM_PROLOGUE=0); the output copy out of the volume is common
    vol = c.V.Volume(1, 1, 1, 2)
    vol.bind_rmsnorm((0, 0, 0, 0), gamma, 1e-6, W.FLOAT32)
    vol.bind_dense((0, 0, 0, 1), qkvo[0], -1, E4M3)
    vy = torch.empty_like(x)
    us_norm_q = c.timed_each(lambda: vol.forward_device(x, vy), 10)
    os.environ["WELVET_B200_NORM_PROLOGUE"] = "0"
    try:
        us_norm_q_sep = c.timed_each(lambda: vol.forward_device(x, vy), 10)
    finally:
        del os.environ["WELVET_B200_NORM_PROLOGUE"]
    vol.release()
    proj = [W.DenseSession(w, T, E4M3) for w in qkvo]
    del qkvo
    py = torch.empty((T, d), device="cuda")

    def projections():
        for p in proj:
            p.execute_device(xn, py, py)
    us_proj = c.timed_each(projections, 5)
    for p in proj:
        p.release()
    rec = {"us_rmsnorm": us_norm, "us_mha_cell": us_mha, "us_qkvo_projections": us_proj,
           "us_norm_q_prologue": us_norm_q, "us_norm_q_separate": us_norm_q_sep,
           "us_attention_and_rope": max(0.0, us_mha - us_proj),
           "proj_TFLOPs": 2.0 * T * 4 * d * d / us_proj / 1e6}
    for tag, sigma in (("swiglu_fp4", SIGMA), ("swiglu_fp4_sigma2", 2.0)):
        cell = W.SwigluCell(wt((inter, d), 41, sigma), wt((inter, d), 42, sigma), wt((d, inter), 43, sigma), FP4)
        h = torch.empty((T, inter), device="cuda")
        us = c.timed_each(lambda: cell.execute_device(y, py, h), 5)
        rec["us_" + tag] = us
        rec[tag + "_TFLOPs"] = 2.0 * T * 3 * d * inter / us / 1e6
        rec[tag + "_frac"] = rec[tag + "_TFLOPs"] / tens
        cell.release()
    rec["us_cell_total"] = us_norm + us_mha + rec["us_swiglu_fp4"]
    return rec


def reference_cuda(args):
    """The reference's own CUDA Dense session (oracle/_ref, its kernels rebuilt for sm_100a):
    host buffers, synchronous per call, same shapes and seeds as configs 1-3 (C3: its Gate
    projection). A baseline beside ours, never the measured product."""
    import oracle as O
    if not O.ref_available():
        return {"unavailable": "oracle/_ref not built"}
    R = O.ref()
    f = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    msg = ctypes.create_string_buffer(256)
    res = {"what": "reference welvet_dense_execute-equivalent session (resident fp64 mirror, "
                   "dense_matvec_f64_batch + dense_bias_act), host buffers, per call"}

    def one(tag, rows, cols, M, dt, sigma, seed, reps, bias=None):
        rng = np.random.default_rng(seed)
        if rows * cols > (1 << 28):  # C5b: drawn in float32 and scaled in place (4 GiB, not 12)
            w = rng.standard_normal((rows, cols), dtype=np.float32)
            w *= np.float32(sigma)
        else:
            w = (rng.standard_normal((rows, cols)) * sigma).astype(np.float32)
        x = rng.standard_normal((M, cols)).astype(np.float32)
        sess = ctypes.c_void_p()
        b = None if bias is None else np.ascontiguousarray(bias, np.float64)
        bp = None if b is None else b.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
        if R.ref_dense_mount(M, cols, rows, -1, dt, f(w), bp, 0 if b is None else b.size, ctypes.byref(sess), msg,
                             256) != 0:
            res[tag] = {"error": msg.value.decode(errors="replace")}
            return
        pre = np.zeros((M, rows), np.float32)
        post = np.zeros((M, rows), np.float32)
        R.ref_dense_execute(sess, f(x), f(pre), f(post), msg, 256)
        t0 = time.perf_counter()
        for _ in range(reps):
            R.ref_dense_execute(sess, f(x), f(pre), f(post), msg, 256)
        t = (time.perf_counter() - t0) / reps
        R.ref_dense_release(sess)
        wb = rows * cols * (0.5 if dt == FP4 else 1.0)
        res[tag] = {"us_per_call": t * 1e6, "weight_GBps": wb / t / 1e9, "TFLOPs": 2.0 * M * rows * cols / t / 1e12}

    one("C1", 128, 256, 1, E4M3, 0.05, 0, 50, np.random.default_rng(0).standard_normal(128) * 0.01)
    one("C2_fp4", 4096, 4096, 1, FP4, SIGMA, 1, 20)
    one("C2_int8", 4096, 4096, 1, INT8, SIGMA, 1, 20)
    one("C3_gate_M1", 14336, 4096, 1, E4M3, SIGMA, 2, 10)
    one("C3_gate_M512", 14336, 4096, 512, E4M3, SIGMA, 2, 2)
    # C4: one of the four QKVO projections (2048 x 2048 E4M3) at 4 x 512 tokens through the
    # session; the SwiGLU 2048 / 5632 FP4 through the reference's one-shot swiglu::forward
    # (mount, Gate, Up, product, Down); its MHA (Q/K/V, the attention, O) on a sample, batch 1 x
    # seq 128: the reference's attention kernel is one thread (mha_attention_forward_f64<<<1, 1>>>)
    one("C4_q_projection", 2048, 2048, 2048, E4M3, SIGMA, 3, 2)

    def oneshot(tag, fn, reps, flops):
        if fn() != 0:
            res[tag] = {"error": msg.value.decode(errors="replace")}
            return
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        t = (time.perf_counter() - t0) / reps
        res[tag] = {"us_per_call": t * 1e6, "TFLOPs": flops / t / 1e12}

    rng = np.random.default_rng(3)
    d, inter, T = 2048, 5632, 2048
    G, U = [(rng.standard_normal((inter, d)) * SIGMA).astype(np.float32) for _ in range(2)]
    D = (rng.standard_normal((d, inter)) * SIGMA).astype(np.float32)
    xs = rng.standard_normal((T, d)).astype(np.float32)
    hp = np.zeros((T, inter), np.float32)
    yp = np.zeros((T, d), np.float32)
    oneshot("C4_swiglu_fp4", lambda: R.ref_swiglu_forward(4, 512, d, inter, FP4, f(G), f(U), f(D), f(xs), f(hp), f(yp),
                                                          msg, 256), 1, 2.0 * T * 3 * d * inter)
    del G, U, D, hp
    Q, K, Vw, Ow = [(rng.standard_normal((d, d)) * SIGMA).astype(np.float32) for _ in range(4)]
    S = 128
    xm = rng.standard_normal((S, d)).astype(np.float32)
    ap = np.zeros((S, d), np.float32)
    mp = np.zeros((S, d), np.float32)
    oneshot("C4_mha_sample_b1_s128", lambda: R.ref_mha_forward(1, S, d, 16, 16, 128, S, 1, 0, E4M3, f(Q), f(K), f(Vw),
                                                               f(Ow), f(xm), f(ap), f(mp), msg, 256),
            1, 2.0 * S * 4 * d * d)
    del Q, K, Vw, Ow
    # C5: one layer of the volume (4096 x 4096 FP4 at 64 tokens; the volume is 32 such calls in
    # sequence) and the 16384 -> 65536 FP4 layer at batch 1 on one GPU
    one("C5a_layer_M64", 4096, 4096, 64, FP4, SIGMA, 4, 3)
    if "us_per_call" in res.get("C5a_layer_M64", {}):
        res["C5a_volume_ms_32_layers"] = 32 * res["C5a_layer_M64"]["us_per_call"] / 1e3
    one("C5b_B1", 65536, 16384, 1, FP4, SIGMA, 4, 3)
    return res


# --------------------------------------------------------------------------------- single cases

def run_case(args):
    """--case: one kernel's workload alone on one GPU, for timing and ncu captures (prints one
    JSON line with the case's own numbers, not the benchmark line). Weights ~N(0, 0.02)
    generated on the device; x ~N(0, 1) (rounded to bf16 with --x bf16); L2 flushed before
    each rep.
      gemv   one Dense layer rows x cols, --tokens 1..8 (tensor GEMV)
      group  --layers independent layers rows x cols, B=1, grouped launches
      gemm   one Dense layer rows x cols, --tokens > 8 (tcgen05 path)
      swiglu one SwiGLU cell, d = cols, hidden = rows, --tokens (Gate/Up pair GEMM, Down GEMM)
      mha    config 4's MHA cell (4 x 512 tokens, d 2048, 16 heads x 128, causal, RoPE, ring of
             512; E4M3 projections): the projections and the fp64 attention core"""
    import torch
    import welvet.cuda_b200 as W
    W.cuda_init()
    g = torch.Generator(device="cuda").manual_seed(1)
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

    def each(fn):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.reps):
            flush.zero_()
            torch.cuda._sleep(200000)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    if args.case == "mha":
        B, S, d, heads, hd = 4, 512, 2048, 16, 128
        ws = [torch.randn((d, d), device="cuda", generator=g) * SIGMA for _ in range(4)]
        cell = W.MhaCell(*ws, d_model=d, num_heads=heads, num_kv_heads=heads, head_dim=hd, max_seq_len=S, mask=1,
                         pos=0, dtype=E4M3)
        del ws
        x = torch.randn((B * S, d), device="cuda", generator=g)
        y = torch.empty_like(x)
        attn = torch.empty_like(x)
        us = each(lambda: cell.execute_device(x, B, S, y, attn))
        print(json.dumps({"case": "mha", "batch": B, "seq": S, "d": d, "heads": heads, "head_dim": hd,
                          "reps": args.reps, "us_median": round(us, 2)}), flush=True)
        cell.release()
        return 0
    if args.case == "swiglu":
        d, hid, m = args.cols, args.rows, args.tokens
        ws = [torch.randn(sh, device="cuda", generator=g) * SIGMA for sh in ((hid, d), (hid, d), (d, hid))]
        cell = W.SwigluCell(ws[0], ws[1], ws[2], args.dtype)
        del ws
        x = torch.randn((m, d), device="cuda", generator=g)
        if args.x == "bf16":
            x = x.to(torch.bfloat16).float()
        y = torch.zeros((m, d), device="cuda")
        h = torch.zeros((m, hid), device="cuda")
        us = each(lambda: cell.execute_device(x, y, h))
        wbytes = 3 * d * hid * (0.5 if args.dtype == FP4 else 1.0)
        print(json.dumps({"case": "swiglu", "dtype": args.dtype, "d": d, "hidden": hid, "tokens": m, "x": args.x,
                          "reps": args.reps, "us_median": round(us, 2), "weight_GBps": round(wbytes / us / 1e3, 1),
                          "TFLOPs": round(2.0 * m * 3 * d * hid / us / 1e6, 2)}), flush=True)
        cell.release()
        return 0
    n_layers = args.layers if args.case == "group" else 1
    tokens = 1 if args.case == "group" else args.tokens
    sess = []
    for _ in range(n_layers):
        w = torch.randn((args.rows, args.cols), device="cuda", generator=g) * SIGMA
        sess.append(W.DenseSession(w, tokens, args.dtype))
        del w
    x = torch.randn((tokens, args.cols), device="cuda", generator=g)
    if args.x == "bf16":
        x = x.to(torch.bfloat16).float()
    outs = [(torch.zeros((tokens, args.rows), device="cuda"), torch.zeros((tokens, args.rows), device="cuda"))
            for _ in range(n_layers)]

    def fwd():
        if args.case == "group":
            W.dense_execute_group(sess, [x] * n_layers, [o[0] for o in outs], [o[1] for o in outs])
        else:
            sess[0].execute_device(x, outs[0][0], outs[0][1])

    us = each(fwd)
    wbytes = args.rows * args.cols * n_layers * (0.5 if args.dtype == FP4 else 1.0)
    line = {"case": args.case, "dtype": args.dtype, "rows": args.rows, "cols": args.cols, "layers": n_layers,
            "tokens": tokens, "x": args.x, "reps": args.reps, "us_median": round(us, 2),
            "weight_GBps": round(wbytes / us / 1e3, 1),
            "TFLOPs": round(2.0 * tokens * args.rows * args.cols * n_layers / us / 1e6, 2)}
    print(json.dumps(line), flush=True)
    for s in sess:
        s.release()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the host-core and reference-CUDA legs")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs 1-4 sub-records (N = 1)")
    ap.add_argument("--case", choices=["gemv", "group", "gemm", "swiglu", "mha"],
                    help="time one workload alone (see run_case)")
    ap.add_argument("--dtype", type=int, default=FP4, help="--case: 16 FP4, 4 E4M3, 5 E5M2, 9 Int8")
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--x", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
