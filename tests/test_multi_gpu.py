"""GPU, one process per GPU through the library's C++ multi-GPU runtime (welvet_b200_comm_*,
welvet_b200_sharded_dense_*, welvet_b200_volume_pipeline_forward_device):

* the column-sharded Dense in both gather modes -- fused (each rank's kernels store its columns
  into every rank's output over NVLink peer memory, then a flag exchange) and nccl (local
  forward, ncclAllGather, permute) -- against the fp64 oracle, on the tensor GEMV (1 token)
  and the tcgen05 GEMM (24 and 256 tokens), with a ragged last shard and a bias / activation;
* the cell-per-GPU volume pipeline, bit-identical to the one-GPU forward of the same
  micro-batches;
* a rank that does not come to an output exchange: the others' bounded wait runs out and
  check_error reports status 4 (no GPU fault: the wait is a flag nothing sets, given 0.5 s).

Ranks run as child processes (spawn), the job id handed over a gloo group on 127.0.0.1;
NVLS is off (NCCL_NVLS_ENABLE=0) and nothing here uses multicast. The world sizes that need
more GPUs than the box has are skipped; the 1-rank cases run on any B200.
"""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

SEED = 41


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WELVET_B200_EXACT="0", NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    import welvet.cuda_b200 as W
    from welvet.cuda_b200 import volume as V
    W.cuda_init()
    return torch, dist, W, V, V.Comm.from_torch(rank)


def _sharded_rank(rank, world, port, q):
    torch, dist, W, V, comm = _init(rank, world, port)
    try:
        import oracle as O
        from test_dense_gpu import check_dense
        rng = np.random.default_rng(SEED + world)
        out, in_ = 128 * (2 * world) + 72, 768  # ragged last shard
        w = (rng.standard_normal((out, in_)) * 2.0).astype(np.float32)
        bias = rng.standard_normal(out - 100) * 0.5  # covers the first rows only
        b, e = V.shard_rows(out, world, rank)
        raw, sc = O.pack(W.FP4, w)
        ok = True
        for mode in (V.FUSED, V.NCCL):
            for tokens, act, bi in ((1, W.LINEAR, None), (24, W.LINEAR, None), (24, W.RELU, bias),
                                    (256, W.LINEAR, None), (3, W.RELU, bias)):
                x = rng.standard_normal((tokens, in_)).astype(np.float32)
                s = V.ShardedDense(comm, torch.from_numpy(w[b:e]).cuda(), in_, out, tokens, W.FP4, act, bi, mode)
                assert s.rows == (b, e)
                xd = torch.from_numpy(x).cuda()
                for call in range(3):  # both output buffers, and one reused
                    post, pre = s.execute_device(xd)
                    s.check_error()
                    ref = O.dense_forward(W.FP4, raw, sc, x, in_, out, act, bi)
                    ph, qh = pre.cpu().numpy(), post.cpu().numpy()
                    if bi is None and act == W.LINEAR:
                        check_dense(ph, qh, ref, act, f"sharded mode={mode} tokens={tokens} call={call}")
                    else:
                        # post is gathered; pre holds this rank's columns (checked there)
                        pre_full = np.array(ref[0], copy=True)
                        pre_full[:, b:e] = ph[:, b:e]
                        check_dense(pre_full, qh, ref, act, f"sharded mode={mode} tokens={tokens} act={act}")
                        assert not np.any(ph[:, :b]) and not np.any(ph[:, e:]), "pre outside this rank's columns"
                # the host-buffer call (x in, pre / post out, synchronous): the same floats as
                # the last device call (whose buffer stays valid until the call after next)
                ph, qh = s.execute(x)
                assert np.array_equal(qh, post.cpu().numpy()), f"host-buffer call, mode={mode} tokens={tokens}"
                s.release()
        q.put((rank, ok))
    finally:
        comm.release()
        dist.destroy_process_group()


def _pipeline_rank(rank, world, port, q):
    torch, dist, W, V, comm = _init(rank, world, port)
    try:
        width, rows, micro, cells, lpc = 256, 10, 3, 2 * world, 2
        rng = np.random.default_rng(SEED)
        ws = [(rng.standard_normal((width, width)) * 0.4).astype(np.float32) for _ in range(cells * lpc)]
        x = rng.standard_normal((rows, width)).astype(np.float32)
        vol = V.Volume(cells, 1, 1, lpc)
        b, e = V.stage_plan(cells, lpc, world)[rank]
        for h in range(b, e):
            vol.bind_dense(vol.coord(h), ws[h], W.RELU, W.FP4)
        y = torch.empty((rows, width), device="cuda")
        comm.pipeline_forward(vol, (b, e), torch.from_numpy(x).cuda() if rank == 0 else None, width, micro, y)
        torch.cuda.synchronize()
        # the whole chain on this GPU, micro-batch by micro-batch (the same kernels per launch)
        full = V.Volume(cells, 1, 1, lpc)
        for h in range(cells * lpc):
            full.bind_dense(full.coord(h), ws[h], W.RELU, W.FP4)
        parts = []
        for (a0, a1) in V.microbatches(rows, micro):
            xi = torch.from_numpy(x[a0:a1]).cuda()
            oi = torch.empty_like(xi)
            full.forward_device(xi, oi)
            parts.append(oi)
        ref = torch.cat(parts)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(ref, y))))
        vol.release()
        full.release()
    finally:
        comm.release()
        dist.destroy_process_group()


def _absent_rank(rank, world, port, q):
    """Rank world-1 mounts but skips the forward; the others' flag wait must run out."""
    os.environ["WELVET_B200_SHARD_WAIT_MS"] = "500"
    torch, dist, W, V, comm = _init(rank, world, port)
    try:
        out, in_ = 128 * world, 256
        w = np.ones((out, in_), np.float32) * 0.5
        b, e = V.shard_rows(out, world, rank)
        s = V.ShardedDense(comm, w[b:e], in_, out, 1, W.FP4)
        code = 0
        if rank != world - 1:
            x = torch.ones((1, in_), device="cuda")
            s.execute_device(x)
            try:
                s.check_error()
            except W.WelvetError as err:
                code = err.code
        dist.barrier()  # every rank is between calls before any releases its buffers
        s.release()
        q.put((rank, code if rank != world - 1 else W.INTERNAL))
    finally:
        comm.release()
        dist.destroy_process_group()


def _spawn(fn, world, port):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return sorted(q.get(timeout=30) for _ in range(world))


WORLDS = [1, 2, 4, 8]


@pytest.mark.parametrize("world", WORLDS)
def test_column_sharded_dense(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    assert _spawn(_sharded_rank, world, 29610 + world) == [(r, True) for r in range(world)]


@pytest.mark.parametrize("world", WORLDS)
def test_pipelined_volume(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    assert _spawn(_pipeline_rank, world, 29630 + world) == [(r, True) for r in range(world)]


def test_absent_rank_times_out_with_status_4():
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import welvet.cuda_b200 as W
    assert _spawn(_absent_rank, 2, 29650) == [(0, W.INTERNAL), (1, W.INTERNAL)]
