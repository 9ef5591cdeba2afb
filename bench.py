#!/usr/bin/env python3
"""Benchmark of the quantized Dense forward path on B200.

Metric: quant Dense weight GB/s (GEMV, % HBM). Workload at N=1: BASELINE
config 2 -- Dense GEMV 4096->4096, batch 1, FP4 (E2M1, 2 codes/byte, reference layout),
W ~ N(0, 0.02), x ~ N(0, 1), seed 1. One step = 64 independent forwards, one per
distinct 4096x4096 FP4 weight set (the reference's --bench loop also repeats independent
executes), so each step streams 512 MiB of packed weights -- more than the 126 MB L2, no
flush needed. The same 64 layers run as a dependent chain are reported under "chain". Weights are random
(synthetic; the reference ships no checkpoints).

  value    weight GB/s with x/weights resident in HBM: the 64 forwards go out through
           welvet_b200_dense_execute_group_device, i.e. the tensor-core GEMV kernel over
           32 layers per launch (blockIdx.z = layer), two launches per step
  e2e      the same metric through the reference-facing C ABI welvet_dense_execute, host
           buffers (pinned), x in and pre/post out over the bus inside the timed region, one
           synchronous call per layer
  branches the same 64 forwards as 64 single-layer launches on 8 graph branches
  chain    the same 64 layers as a dependent chain (layer i's post is layer i+1's x)
  batched  the other half of the metric, TFLOP/s of the batched tcgen05 path: BASELINE
           config 3's SwiGLU cell (d 4096, hidden 14336, FP8 E4M3, W ~ N(0, 0.02)) at
           M = 512 tokens of N(0, 1) activations rounded to bf16, seed 2
N > 1 (torchrun): every rank runs its own chain (independent layers, weak scaling, no
collective on the data path); value = all ranks' bytes / max-over-ranks time.

--impl reference times the reference semantics on the host cores (the oracle port of
kernels.cu:130-161 with the reference decode), the only CPU implementation of this path.
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

IN = OUT = 4096
LAYERS = 64
DTYPE_FP4 = 16
SIGMA = 0.02
SEED = 1
WEIGHT_BYTES_PER_LAYER = OUT * IN // 2  # FP4: 0.5 B / weight


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def traffic_from_profile():
    """DRAM bytes of one grouped GEMV launch (32 layers) from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemv_tc_grouped_fp4_4096x4096_b1_32layers.md")
    try:
        for ln in open(p):
            if ln.startswith("dram_bytes_per_launch:"):
                return int(ln.split(":")[1].strip())
    except Exception:
        pass
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, polled through NVML (the data
    nvidia-smi's clocks.sm / clocks_event_reasons.* report) every ~0.5 ms while the timed
    region runs -- short timed regions still get samples. Read-only."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int):
        self.index = index
        self.sm = []
        self.mask = 0
        self.max_mhz = None
        self.err = None
        self._stop = threading.Event()

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
            try:
                self.sm.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
                self.mask |= N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception as e:
                self.err = str(e)
                return
            time.sleep(0.0005)

    def __exit__(self, *a):
        self._stop.set()
        if hasattr(self, "t"):
            self.t.join(timeout=2)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "error": self.err}
        reasons = sorted(n for n, bit in self.REASONS.items() if self.mask & bit)
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.sm), "source": "NVML (nvmlDeviceGetClockInfo / GetCurrentClocksEventReasons)"}


def cpu_baseline(seconds: float = 10.0):
    """The oracle port of the reference semantics on all host threads, on a bounded sample:
    whole 4096x4096 FP4 layers of the same workload until ~`seconds` of CPU time."""
    import oracle as O
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(SEED)
    w = (rng.standard_normal((OUT, IN)) * SIGMA).astype(np.float32)
    raw, sc = O.pack(DTYPE_FP4, w)
    x = rng.standard_normal((1, IN)).astype(np.float32)
    O.dense_forward(DTYPE_FP4, raw, sc, x, IN, OUT, -1, None, threads)  # warm
    n = 0
    t0 = time.perf_counter()
    while True:
        O.dense_forward(DTYPE_FP4, raw, sc, x, IN, OUT, -1, None, threads)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": n * WEIGHT_BYTES_PER_LAYER / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} forwards of one 4096x4096 FP4 layer, B=1 ({dt:.1f} s): reference decode + "
                      f"sequential fp64 dot (oracle/oracle.c), rows split over {threads} threads"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle as O
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(SEED)
    w = (rng.standard_normal((OUT, IN)) * SIGMA).astype(np.float32)
    raw, sc = O.pack(DTYPE_FP4, w)
    x = rng.standard_normal((1, IN)).astype(np.float32)
    for _ in range(args.warmup):
        O.dense_forward(DTYPE_FP4, raw, sc, x, IN, OUT, -1, None, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.dense_forward(DTYPE_FP4, raw, sc, x, IN, OUT, -1, None, threads)
    dt = time.perf_counter() - t0
    val = args.steps * WEIGHT_BYTES_PER_LAYER / dt / 1e9
    line = {"metric": "quant Dense weight GB/s (GEMV)", "value": val, "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp4 codes, fp64 accumulate",
            "data": "synthetic",
            "config": {"workload": "C2 Dense GEMV 4096->4096 B=1 FP4 (one layer per step on the host)",
                       "global_batch": 1, "parallelism": "host threads"},
            "cpu_baseline": {"value": val, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": "one 4096x4096 FP4 layer forward per step: reference decode + sequential "
                                       "fp64 dot (oracle/oracle.c; the reference ships no host matvec)"},
            "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    import welvet.cuda_b200 as W
    W.cuda_init()

    # ---- mount LAYERS distinct layers (weights generated on the device, per rank seed)
    g = torch.Generator(device="cuda").manual_seed(SEED * 1000 + rank)
    sessions = []
    for _ in range(LAYERS):
        wdev = torch.randn((OUT, IN), device="cuda", generator=g) * SIGMA
        sessions.append(W.DenseSession(wdev, 1, DTYPE_FP4))
        del wdev
    torch.cuda.synchronize()
    x0 = torch.randn((1, IN), device="cuda", generator=g)
    acts = [torch.zeros((1, OUT), device="cuda") for _ in range(2)]
    pre = torch.zeros((1, OUT), device="cuda")
    stream = torch.cuda.current_stream()
    NSTREAMS = 8
    streams = [torch.cuda.Stream() for _ in range(NSTREAMS)]
    outs = [(torch.zeros((1, OUT), device="cuda"), torch.zeros((1, OUT), device="cuda")) for _ in range(NSTREAMS)]

    xs_group = [x0] * LAYERS
    outs_group = [(torch.zeros((1, OUT), device="cuda"), torch.zeros((1, OUT), device="cuda")) for _ in range(LAYERS)]

    def step_group():
        # the 64 independent forwards as grouped launches (32 layers per launch)
        W.dense_execute_group(sessions, xs_group, [o[0] for o in outs_group], [o[1] for o in outs_group])

    def step_independent():
        # 64 independent forwards (the reference's --bench loop repeats independent executes),
        # one per distinct weight set, spread over 8 stream branches that the graph runs
        # concurrently; consecutive launches on one branch overlap through PDL.
        cur = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(cur)
        for s in streams:
            s.wait_event(fork)
        for i, sess in enumerate(sessions):
            j = i % NSTREAMS
            sess.execute_device(x0, outs[j][0], outs[j][1], streams[j])
        for s in streams:
            cur.wait_stream(s)

    def step_chain():
        st = torch.cuda.current_stream()  # the capture stream while a graph is recorded
        x = x0
        for i, s in enumerate(sessions):
            y = acts[i & 1]
            s.execute_device(x, pre, y, st)
            x = y

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def capture(fn):
        # A step's launches are captured once in a CUDA graph (PDL edges between consecutive
        # GEMVs of one stream are kept) and replayed per step.
        fn()
        torch.cuda.synchronize()
        if args.no_graph:
            return fn
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graphs.append(graph)
        return graph.replay

    graphs = []
    run = capture(step_group)
    run_branches = capture(step_independent)
    run_chain = capture(step_chain)
    for _ in range(args.warmup):
        run()
        run_branches()
        run_chain()
    barrier()
    stream = torch.cuda.current_stream()

    def timed(fn, steps):
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        barrier()
        a0.record(stream)
        for _ in range(steps):
            fn()
        a1.record(stream)
        barrier()
        return max_over_ranks(a0.elapsed_time(a1))

    # clocks are sampled over all three device-timed legs
    with ClockSampler(local) as clk:
        ms = timed(run, args.steps)
        ms_br = timed(run_branches, args.steps)
        # the same 64 layers as a dependent chain (layer i's post is layer i+1's x)
        ms_chain = timed(run_chain, args.steps)
    group_per_launch = 32
    launches_per_step = (LAYERS + group_per_launch - 1) // group_per_launch
    prep_per_step = launches_per_step  # one k_prep_x per 32 layers ahead of the GEMV launches
    launches = args.steps * launches_per_step
    bytes_per_step = LAYERS * WEIGHT_BYTES_PER_LAYER
    value = world * bytes_per_step * args.steps / (ms / 1e3) / 1e9
    per_launch_s = (ms / 1e3) / launches
    branches_val = world * bytes_per_step * args.steps / (ms_br / 1e3) / 1e9
    chain_val = world * bytes_per_step * args.steps / (ms_chain / 1e3) / 1e9

    # ---- e2e through the reference-facing ABI (host buffers, pinned)
    xh = torch.randn((1, IN)).pin_memory()
    bufs = [torch.zeros((1, OUT)).pin_memory() for _ in range(2)]
    preh = torch.zeros((1, OUT)).pin_memory()
    e2e_steps = max(1, min(args.steps, 20))
    # The C ABI itself, as a cgo / FFI caller of the reference binds it: arguments prepared
    # once, the status checked on every call.
    c_execute = W.lib().welvet_dense_execute
    handles = [s._h for s in sessions]
    p_x, p_pre = ctypes.c_void_p(xh.data_ptr()), ctypes.c_void_p(preh.data_ptr())
    p_post = [ctypes.c_void_p(b.data_ptr()) for b in bufs]

    def e2e_step():
        # welvet_dense_execute on each of the 64 layers: x in from host memory, forward, pre
        # and post out to host memory, synchronize -- the reference's resident-session
        # contract and --bench loop.
        for i, h in enumerate(handles):
            st = c_execute(h, p_x, p_pre, p_post[i & 1])
            if st.code != 0:
                raise W.WelvetError(st.code, st.message.decode(errors="replace"))

    for _ in range(2):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    t_e2e = max_over_ranks(time.perf_counter() - t0)
    e2e_val = world * bytes_per_step * e2e_steps / t_e2e / 1e9

    # ---- batched path: C3 SwiGLU cell at M = 512 (tcgen05 GEMMs for gate, up and down)
    batched = run_batched(args, torch, W, rank, barrier, max_over_ranks, stream) if not args.no_batched else None

    pk, pk_kind = peaks()
    bytes_per_launch = group_per_launch * WEIGHT_BYTES_PER_LAYER
    achieved = bytes_per_launch / per_launch_s / 1e9
    tr = traffic_from_profile()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": tr,
                "peak_source": f"{pk_kind} hbm_gbs (MEASURED_PEAKS.json)" if pk_kind == "measured" else "fallback",
                "kernel": "k_gemv_tc<FP4,B=1> over 32 layers per launch (welvet/cuda_b200/csrc/gemv_tc.cu)",
                "algorithmic_bytes_per_launch": bytes_per_launch}
    if batched is not None:
        batched["frac"] = batched["value"] / pk["bf16_tflops"]
        batched["peak"] = pk["bf16_tflops"]
        batched["peak_source"] = f"{pk_kind} bf16_tflops (burst, MEASURED_PEAKS.json)"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)

    if rank == 0:
        line = {"metric": "quant Dense weight GB/s (GEMV)", "value": value, "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp4 codes, fp32/fp64 accumulate",
                "data": "synthetic",
                "config": {"workload": "C2 Dense GEMV 4096->4096 B=1 FP4 (W~N(0,0.02), seed 1): 64 independent "
                                       "forwards of 64 distinct weight sets per step, grouped 32 layers per launch",
                           "global_batch": world, "seq_len": 1, "parallelism": f"replicas x{world}",
                           "l2": "inputs larger than L2 (512 MiB of packed weights per step)",
                           "bytes_per_step_per_gpu": bytes_per_step},
                "roofline": roofline,
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_val, "unit": "GB/s", "h2d_bytes_per_step": LAYERS * IN * 4,
                        "d2h_bytes_per_step": LAYERS * OUT * 4 * 2, "steps": e2e_steps,
                        "api": "welvet_dense_execute via ctypes (host pinned buffers, synchronous per layer)"},
                "branches": {"value": branches_val, "unit": "GB/s", "ms_per_step": ms_br / args.steps,
                             "what": "the same 64 forwards as 64 single-layer launches on 8 CUDA-graph branches"},
                "chain": {"value": chain_val, "unit": "GB/s", "ms_per_step": ms_chain / args.steps,
                          "what": "the same 64 layers as a dependent chain, layer i's post feeding layer i+1"},
                "batched": batched,
                "gpu_launches": launches + args.steps * prep_per_step,
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    del graphs
    for s in sessions:
        s.release()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_batched(args, torch, W, rank, barrier, max_over_ranks, stream):
    """C3 SwiGLU cell (4096 -> 14336 -> 4096, FP8 E4M3) at M = 512 tokens: TFLOP/s of the
    tcgen05 GEMM path (2 * M * 3 * 4096 * 14336 flops per forward). Weights are 176 MB, more
    than L2; the cell's forward is captured in a CUDA graph."""
    d, hid, m = 4096, 14336, 512
    g = torch.Generator(device="cuda").manual_seed(2 * 1000 + rank)
    ws = [torch.randn(s, device="cuda", generator=g) * SIGMA for s in ((hid, d), (hid, d), (d, hid))]
    cell = W.SwigluCell(ws[0], ws[1], ws[2], 4)
    del ws
    x = torch.randn((m, d), device="cuda", generator=g).to(torch.bfloat16).float()
    y = torch.zeros((m, d), device="cuda")
    h = torch.zeros((m, hid), device="cuda")
    cell.execute_device(x, y, h)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cell.execute_device(x, y, h)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    steps = max(5, min(args.steps, 50))
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    barrier()
    a0.record(stream)
    for _ in range(steps):
        graph.replay()
    a1.record(stream)
    barrier()
    ms = max_over_ranks(a0.elapsed_time(a1)) / steps
    flops = 2.0 * m * 3 * d * hid
    del graph
    cell.release()
    return {"value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_forward": ms, "steps": steps,
            "config": "C3 SwiGLU cell d=4096 hidden=14336 FP8 E4M3 W~N(0,0.02), M=512 tokens, x~N(0,1) "
                      "rounded to bf16, seed 2",
            "kernels": "k_split_x + k_gemm_tm<FP8 E4M3> over the interleaved Gate/Up pair (SiLU(g)*u in the "
                       "epilogue) + k_split_x + k_gemm_tm<FP8 E4M3> (Down)",
            "l2": "176 MB of FP8 weights per forward (more than L2)"}


def run_case_multi(args):
    """--case sharded | pipeline: BASELINE config 5 on 1..N GPUs (torchrun; one process per GPU).
      sharded   Dense rows x cols FP4 (default 65536 x 16384) split by output rows over the
                ranks, --tokens 1 or 256; each rank's slice then NCCL all-gather
      pipeline  volume 2x2x2 with 4 Dense 4096x4096 FP4 + ReLU layers per cell, batch 64:
                cells placed over the ranks in hop order, --micro rows per micro-batch,
                activations sent rank to rank
    Prints one JSON line (rank 0): time per forward (max over ranks) and aggregate rates."""
    import datetime
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    import torch.distributed as dist
    dist.init_process_group("nccl" if world > 1 else "gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            **({} if world > 1 else {"init_method": "tcp://127.0.0.1:29731"}))
    import welvet.cuda_b200 as W
    from welvet.cuda_b200 import volume as V
    W.cuda_init()
    g = torch.Generator(device="cuda").manual_seed(4 * 1000 + rank)
    stream = torch.cuda.current_stream()
    out = {"case": args.case, "n_gpus": world}
    if args.case == "sharded":
        rows, cols, tokens = args.rows, args.cols, args.tokens
        a, b = V.ColumnShardedDense.shard_rows(rows, world, rank)
        w = torch.randn((b - a, cols), device="cuda", generator=g) * SIGMA
        sess = W.DenseSession(w, tokens, DTYPE_FP4)
        del w
        x = torch.randn((tokens, cols), device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
        pre = torch.empty((tokens, b - a), device="cuda")
        post = torch.empty((tokens, b - a), device="cuda")

        def local_fn(xd):
            sess.execute_device(xd, pre, post, stream)
            return pre

        sd = V.ColumnShardedDense(local_fn, rows)
        step = lambda: sd.forward(x)
        compute = lambda: local_fn(x)
        flops = 2.0 * tokens * rows * cols
        wbytes = rows * cols * 0.5
    else:
        lpc, cells, width, batch = 4, 8, 4096, 64
        vol = V.Volume(2, 2, 2, lpc)
        b, e = V.stage_plan(cells, lpc, world)[rank]
        for h in range(b, e):
            w = torch.randn((width, width), device="cuda", generator=g) * SIGMA
            vol.bind_dense(vol.coord(h), w, 0, DTYPE_FP4)
            del w
        x = torch.randn((batch, width), device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))

        def runner(xin):
            o = torch.empty_like(xin)
            vol.forward_device(xin, o, b, e, stream=stream)
            return o

        pv = V.PipelinedVolume(runner, width, [width] * world)
        step = lambda: pv.forward(x, micro=args.micro)
        compute = None
        flops = 2.0 * batch * cells * lpc * width * width
        wbytes = cells * lpc * width * width * 0.5

    def timed(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX) if world > 1 else None
        return float(t.item())

    ms = timed(step, args.reps)
    out.update({"ms_per_forward": ms, "TFLOPs": flops / (ms / 1e3) / 1e12, "weight_GBps": wbytes / (ms / 1e3) / 1e9,
                "tokens": args.tokens if args.case == "sharded" else 64,
                "micro": args.micro if args.case == "pipeline" else None})
    if compute is not None:
        out["compute_ms"] = timed(compute, args.reps)
        gathered = torch.empty((world * args.tokens, (args.rows // world)), device="cuda")
        src = torch.empty((args.tokens, args.rows // world), device="cuda")
        out["gather_ms"] = timed(lambda: dist.all_gather_into_tensor(gathered, src) if world > 1 else None, args.reps)
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_case_swiglu(args, torch, W, g):
    d, hid, m = args.cols, args.rows, args.tokens
    ws = [torch.randn(sh, device="cuda", generator=g) * SIGMA for sh in ((hid, d), (hid, d), (d, hid))]
    cell = W.SwigluCell(ws[0], ws[1], ws[2], args.dtype)
    del ws
    x = torch.randn((m, d), device="cuda", generator=g)
    if args.x == "bf16":
        x = x.to(torch.bfloat16).float()
    y = torch.zeros((m, d), device="cuda")
    h = torch.zeros((m, hid), device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    cell.execute_device(x, y, h)
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.reps):
        flush.zero_()
        torch.cuda._sleep(200000)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        cell.execute_device(x, y, h)
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    us = statistics.median(ts)
    wbytes = 3 * d * hid * (0.5 if args.dtype == DTYPE_FP4 else 1.0)
    print(json.dumps({"case": "swiglu", "dtype": args.dtype, "d": d, "hidden": hid, "tokens": m, "x": args.x,
                      "reps": args.reps, "us_median": round(us, 2), "weight_GBps": round(wbytes / us / 1e3, 1),
                      "TFLOPs": round(2.0 * m * 3 * d * hid / us / 1e6, 2)}), flush=True)
    cell.release()
    return 0


def run_case(args):
    """--case: one kernel's workload alone, for timing and ncu captures (prints one JSON line
    with the case's own numbers, not the benchmark line). Weights ~N(0, 0.02) generated on
    the device; x ~N(0, 1) (rounded to bf16 with --x bf16); L2 flushed before each rep.
      gemv   one Dense layer rows x cols, --tokens 1..4, single launches
      group  --layers independent layers rows x cols, B=1, grouped launches
      gemm   one Dense layer rows x cols, --tokens > 8 (tcgen05 path)
      swiglu one SwiGLU cell, d = cols, hidden = rows, --tokens (Gate/Up pair GEMM, Down GEMM)"""
    import torch
    import welvet.cuda_b200 as W
    W.cuda_init()
    g = torch.Generator(device="cuda").manual_seed(SEED)
    if args.case == "swiglu":
        return run_case_swiglu(args, torch, W, g)
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
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

    def fwd():
        if args.case == "group":
            W.dense_execute_group(sess, [x] * n_layers, [o[0] for o in outs], [o[1] for o in outs])
        else:
            sess[0].execute_device(x, outs[0][0], outs[0][1])

    fwd()
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.reps):
        flush.zero_()
        torch.cuda._sleep(200000)  # the GPU stays busy while the host enqueues the forward
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fwd()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    us = statistics.median(ts)
    wbytes = args.rows * args.cols * n_layers * (0.5 if args.dtype == DTYPE_FP4 else 1.0)
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
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch the step's kernels one by one")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched (SwiGLU M=512) measurement")
    ap.add_argument("--case", choices=["gemv", "group", "gemm", "swiglu", "sharded", "pipeline"],
                    help="time one workload alone (see run_case / run_case_multi)")
    ap.add_argument("--micro", type=int, default=16, help="--case pipeline: rows per micro-batch")
    ap.add_argument("--dtype", type=int, default=DTYPE_FP4, help="--case: 16 FP4, 4 E4M3, 5 E5M2, 9 Int8")
    ap.add_argument("--rows", type=int, default=OUT)
    ap.add_argument("--cols", type=int, default=IN)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--x", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    if args.case in ("sharded", "pipeline"):
        return run_case_multi(args)
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
