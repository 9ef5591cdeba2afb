"""CPU: placement and the multi-GPU dataflow of the volume path, run as gloo ranks.

The plans under test are the library's own (welvet_b200_shard_rows, welvet_b200_stage_plan,
host arithmetic in libwelvet_b200.so, callable without a GPU). The gloo ranks replay the
dataflow the C++ runtime runs over NCCL and peer memory on GPU ranks (welvet/cuda_b200/csrc/
sharded.cu): the pipeline's receive / run hops / send / broadcast per micro-batch, and the
column-sharded layer's two gathers -- every rank's columns stored into every rank's
[batch][out] buffer (fused), and the rank-major all-gather of padded shards and its permute
(nccl). Per-rank compute is the oracle (test infrastructure only)."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT


def _volume_module():
    sys.path.insert(0, ROOT)
    from welvet.cuda_b200 import volume as V
    return V


def test_stage_plan():
    V = _volume_module()
    assert V.stage_plan(8, 4, 8) == [(4 * r, 4 * r + 4) for r in range(8)]  # one cell per GPU
    assert V.stage_plan(8, 4, 2) == [(0, 16), (16, 32)]
    assert V.stage_plan(8, 4, 1) == [(0, 32)]
    assert V.stage_plan(3, 2, 4) == [(0, 2), (2, 4), (4, 6), (6, 6)]  # more GPUs than cells
    assert V.stage_plan(8, 4, 3) == [(0, 8), (8, 20), (20, 32)]
    assert V.microbatches(64, 16) == [(0, 16), (16, 32), (32, 48), (48, 64)]
    assert V.microbatches(5, 2) == [(0, 2), (2, 4), (4, 5)]
    import welvet.cuda_b200 as W
    with pytest.raises(W.WelvetError):
        V.stage_plan(0, 1, 1)


@pytest.mark.parametrize("rows", [1, 127, 128, 1000, 4096, 65536, 65537])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_cover_whole_blocks(rows, world):
    """Every output row belongs to exactly one rank, in rank order, and every boundary is a
    multiple of 128 (a GEMM tile never straddles two ranks)."""
    V = _volume_module()
    ranges = [V.shard_rows(rows, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == rows
    for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
        assert e0 == b1
    for b, e in ranges:
        assert b <= e and b % 128 == 0 and (e % 128 == 0 or e == rows)
    sizes = [e - b for b, e in ranges]
    assert max(sizes) - min(sizes) <= 128 or rows < 128 * world


def test_shard_rows_rejects_bad_arguments():
    import welvet.cuda_b200 as W
    V = _volume_module()
    for args in ((0, 2, 0), (10, 0, 0), (10, 2, 2), (10, 2, -1)):
        with pytest.raises(W.WelvetError) as e:
            V.shard_rows(*args)
        assert e.value.code == W.INVALID


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
    """The pipeline of volume_pipeline_forward: per micro-batch, receive from rank - 1 (rank 0
    reads x), run this rank's hops, send to rank + 1 (the last rank keeps its output); then the
    last rank broadcasts the whole output."""
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V = _volume_module()
        layers = _layers(3, 4, 48)
        b, e = V.stage_plan(2, 2, world)[rank]  # 2 cells of 2 layers
        x = np.random.default_rng(9).standard_normal((10, 48)).astype(np.float32)
        out = torch.zeros((10, 48))
        for (a0, a1) in V.microbatches(10, 3):
            if rank == 0:
                xin = x[a0:a1]
            else:
                t = torch.zeros((a1 - a0, 48))
                dist.recv(t, src=rank - 1)
                xin = t.numpy()
            y = _chain_ref(layers[b:e], xin) if b < e else xin
            if rank < world - 1:
                dist.send(torch.from_numpy(np.ascontiguousarray(y)), dst=rank + 1)
            else:
                out[a0:a1] = torch.from_numpy(y)
        dist.broadcast(out, src=world - 1)
        ref = _chain_ref(layers, x)
        q.put((rank, bool(np.array_equal(out.numpy(), ref))))
    finally:
        dist.destroy_process_group()


def _run_sharded(rank, world, port, q):
    """Both gathers of sharded.cu: (fused) each rank's columns land at [b][begin:end] of every
    rank's output; (nccl) shards padded to the largest, gathered rank-major, then permuted."""
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O
        V = _volume_module()
        rng = np.random.default_rng(4)
        out, in_, batch = 300, 40, 3  # 3 blocks of 128 rows over 2 ranks: shards of 128 and 172
        w = (rng.standard_normal((out, in_)) * 2).astype(np.float32)
        x = rng.standard_normal((batch, in_)).astype(np.float32)
        ranges = [V.shard_rows(out, world, r) for r in range(world)]
        b, e = ranges[rank]
        raw, sc = O.pack(O.FP4, w[b:e])
        mine = O.dense_forward(O.FP4, raw, sc, x, in_, e - b)[1] if e > b else np.zeros((batch, 0), np.float32)
        # fused: every rank writes its columns into every rank's buffer
        fused = torch.zeros((batch, out))
        for r, (rb, re) in enumerate(ranges):
            blk = torch.from_numpy(np.ascontiguousarray(mine)) if r == rank else torch.zeros((batch, re - rb))
            dist.broadcast(blk, src=r)  # rank r's columns reach every rank's buffer
            fused[:, rb:re] = blk
        # nccl: padded shards, rank-major gather, permute
        smax = max(re - rb for rb, re in ranges)
        pad = torch.zeros((batch, smax))
        pad[:, :e - b] = torch.from_numpy(mine)
        gathered = [torch.zeros((batch, smax)) for _ in range(world)]
        dist.all_gather(gathered, pad)
        nccl = torch.zeros((batch, out))
        for (rb, re), g in zip(ranges, gathered):
            nccl[:, rb:re] = g[:, :re - rb]
        rawf, scf = O.pack(O.FP4, w)
        ref = O.dense_forward(O.FP4, rawf, scf, x, in_, out)[1]
        q.put((rank, bool(np.array_equal(fused.numpy(), ref) and np.array_equal(nccl.numpy(), ref))))
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
