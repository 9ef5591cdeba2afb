"""GPU, two ranks over NCCL: the volume pipeline (a cell range per GPU, activations sent
between consecutive ranks) and the column-sharded Dense (rows split over the GPUs, slices
all-gathered), each against a single-GPU run or the fp64 oracle. Skipped with fewer than 2
GPUs; runs as child processes, one per GPU (127.0.0.1 rendezvous)."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

WIDTH, ROWS, MICRO, SEED = 256, 8, 3, 41


def _two_gpus():
    try:
        import torch
        return torch.cuda.device_count() >= 2
    except Exception:
        return False


def _weights():
    rng = np.random.default_rng(SEED)
    return [(rng.standard_normal((WIDTH, WIDTH)) * 0.4).astype(np.float32) for _ in range(4)], \
        rng.standard_normal((ROWS, WIDTH)).astype(np.float32)


def _pipeline_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WELVET_B200_EXACT="0")
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import welvet.cuda_b200 as W
        from welvet.cuda_b200 import volume as V
        W.cuda_init()
        ws, x = _weights()
        vol = V.Volume(2, 1, 1, 2)  # 4 hops, 2 cells of 2 layers
        b, e = V.stage_plan(2, 2, world)[rank]
        for h in range(b, e):
            vol.bind_dense(vol.coord(h), ws[h], 0, W.FP4)

        def runner(xin):
            out = torch.empty_like(xin)
            vol.forward_device(xin, out, b, e, stream=torch.cuda.current_stream())
            return out

        pv = V.PipelinedVolume(runner, WIDTH, [WIDTH] * world)
        y = pv.forward(torch.from_numpy(x).cuda(), micro=MICRO)
        torch.cuda.synchronize()
        ok = True
        if rank == 0:
            # the whole chain on one GPU, micro-batch by micro-batch (same kernels per launch)
            full = V.Volume(2, 1, 1, 2)
            for h in range(4):
                full.bind_dense(full.coord(h), ws[h], 0, W.FP4)
            parts = []
            for (a0, a1) in V.microbatches(ROWS, MICRO):
                xi = torch.from_numpy(x[a0:a1]).cuda()
                oi = torch.empty_like(xi)
                full.forward_device(xi, oi)
                parts.append(oi)
            ref = torch.cat(parts)
            torch.cuda.synchronize()
            ok = bool(torch.equal(ref, y))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def _sharded_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WELVET_B200_EXACT="0")
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import welvet.cuda_b200 as W
        from welvet.cuda_b200 import volume as V
        import oracle as O
        from test_dense_gpu import check_dense
        W.cuda_init()
        rng = np.random.default_rng(SEED + 1)
        out, in_ = 1024, 768
        w = (rng.standard_normal((out, in_)) * 2.0).astype(np.float32)
        results = []
        for tokens in (1, 24):  # tensor GEMV and tcgen05 GEMM per rank
            x = rng.standard_normal((tokens, in_)).astype(np.float32)
            a, b = V.ColumnShardedDense.shard_rows(out, world, rank)
            sess = W.DenseSession(w[a:b], tokens, W.FP4)

            def local(xd):
                pre = torch.empty((tokens, b - a), device="cuda")
                post = torch.empty((tokens, b - a), device="cuda")
                sess.execute_device(xd, pre, post, torch.cuda.current_stream())
                return pre

            y = V.ColumnShardedDense(local, out).forward(torch.from_numpy(x).cuda())
            torch.cuda.synchronize()
            raw, sc = O.pack(W.FP4, w)
            ref = O.dense_forward(W.FP4, raw, sc, x, in_, out)
            yh = y.cpu().numpy()
            check_dense(yh, yh, (ref[0], ref[0], ref[2], ref[3]), -1, f"sharded tokens={tokens}")
            results.append(True)
            sess.release()
        q.put((rank, all(results)))
    finally:
        dist.destroy_process_group()


def _spawn(fn, port):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return sorted(q.get(timeout=30) for _ in range(2))


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_pipelined_volume_nccl():
    assert _spawn(_pipeline_rank, 29611) == [(0, True), (1, True)]


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_column_sharded_dense_nccl():
    assert _spawn(_sharded_rank, 29612) == [(0, True), (1, True)]
