"""CPU: placement and multi-GPU orchestration of the volume path, run as gloo ranks.

The per-rank compute is a host stand-in built on the oracle (test infrastructure only);
the code under test is the orchestration in welvet/cuda_b200/volume.py -- stage placement,
micro-batch pipelining with point-to-point sends, and the column-sharded Dense all-gather --
which the GPU ranks run unchanged over NCCL."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT


def _volume_module():
    # volume.py's orchestration needs no GPU; load it without the ctypes library.
    import importlib.util
    import types
    pkg = types.ModuleType("wbstub")
    for n in ("_L", "_ST", "_dev_ptr", "_f32", "_np_ptr", "_sig", "_stream_ptr", "check"):
        setattr(pkg, n, (lambda *a, **k: None) if n in ("_sig", "check") else None)
    sys.modules["wbstub"] = pkg
    src = open(os.path.join(ROOT, "welvet", "cuda_b200", "volume.py")).read().replace("from . import", "from wbstub import")
    mod = types.ModuleType("volume_under_test")
    exec(compile(src, "volume.py", "exec"), mod.__dict__)
    return mod


def test_stage_plan():
    V = _volume_module()
    assert V.stage_plan(8, 4, 8) == [(4 * r, 4 * r + 4) for r in range(8)]  # one cell per GPU
    assert V.stage_plan(8, 4, 2) == [(0, 16), (16, 32)]
    assert V.stage_plan(8, 4, 1) == [(0, 32)]
    assert V.stage_plan(3, 2, 4) == [(0, 2), (2, 4), (4, 6), (6, 6)]  # more GPUs than cells
    assert V.microbatches(64, 16) == [(0, 16), (16, 32), (32, 48), (48, 64)]
    assert V.microbatches(5, 2) == [(0, 2), (2, 4), (4, 5)]
    with pytest.raises(ValueError):
        V.stage_plan(0, 1, 1)


def _chain_ref(layers, x):
    """Reference chain: each layer's post feeds the next (src/runtime/forward.cpp:98-156)."""
    import oracle as O
    for (raw, sc, in_, out, act) in layers:
        x = O.dense_forward(O.FP4, raw, sc, x, in_, out, act)[1]
    return x


def _layers(seed, n, width):
    import oracle as O
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        w = (rng.standard_normal((width, width)) * 0.5).astype(np.float32)
        raw, sc = O.pack(O.FP4, w)
        out.append((raw, sc, width, width, 0))
    return out


def _run_pipeline(rank, world, port, q):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V = _volume_module()
        layers = _layers(3, 4, 48)
        plan = V.stage_plan(2, 2, world)  # 2 cells of 2 layers
        b, e = plan[rank]

        def runner(x):
            return torch.from_numpy(_chain_ref(layers[b:e], x.numpy()))

        pv = V.PipelinedVolume(runner, 48, [48] * world)
        x = torch.from_numpy(np.random.default_rng(9).standard_normal((10, 48)).astype(np.float32))
        y = pv.forward(x, micro=3)
        ref = _chain_ref(layers, x.numpy())
        q.put((rank, bool(np.array_equal(y.numpy(), ref))))
    finally:
        dist.destroy_process_group()


def _run_sharded(rank, world, port, q):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O
        V = _volume_module()
        rng = np.random.default_rng(4)
        out, in_, rows = 64, 40, 3
        w = (rng.standard_normal((out, in_)) * 2).astype(np.float32)
        a, b = V.ColumnShardedDense.shard_rows(out, world, rank)
        raw, sc = O.pack(O.FP4, w[a:b])

        def local(x):
            return torch.from_numpy(O.dense_forward(O.FP4, raw, sc, x.numpy(), in_, b - a)[1])

        sd = V.ColumnShardedDense(local, out)
        x = torch.from_numpy(rng.standard_normal((rows, in_)).astype(np.float32))
        y = sd.forward(x)
        rawf, scf = O.pack(O.FP4, w)
        ref = O.dense_forward(O.FP4, rawf, scf, x.numpy(), in_, out)[1]
        q.put((rank, bool(np.array_equal(y.numpy(), ref))))
    finally:
        dist.destroy_process_group()


def _spawn(fn, world, port):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = sorted(q.get(timeout=10) for _ in range(world))
    return res


def test_pipelined_volume_gloo_two_ranks():
    res = _spawn(_run_pipeline, 2, 29531)
    assert res == [(0, True), (1, True)]


def test_column_sharded_dense_gloo_two_ranks():
    res = _spawn(_run_sharded, 2, 29532)
    assert res == [(0, True), (1, True)]
