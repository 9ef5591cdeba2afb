"""Volume (Grid) forward and its multi-GPU placement.

`Volume` binds the device-resident volume runtime of libwelvet_b200.so (reference
architecture::Grid + runtime::forward::volume_dense, include/welvet/architecture.hpp:100-141,
src/runtime/forward.cpp:98-156).

Multi-GPU (one process per GPU, torch.distributed for the plumbing):

* `stage_plan` / `PipelinedVolume` -- the volume's cells are placed one per GPU (contiguous
  runs of cells in hop order when there are fewer GPUs than cells). The hop order is a
  sequential chain, so the GPUs form a pipeline; the batch is cut into micro-batches (rows
  are independent through Dense/ReLU cells, so results do not change) and activations move
  between consecutive ranks with point-to-point sends.
* `ColumnShardedDense` -- a Dense layer too large for one GPU: rank r holds rows
  [r*out/N, (r+1)*out/N), computes its slice of y, and the slices are all-gathered.

The orchestration only needs a stage runner (`run(rows, x) -> y` on the rank's device); the
product passes the volume runtime, and the CPU tests pass a host stand-in over gloo.
"""
from __future__ import annotations

from ctypes import POINTER, byref, c_double, c_float, c_int32, c_size_t, c_void_p

from . import _L, _ST, _dev_ptr, _f32, _np_ptr, _sig, _stream_ptr, check

_sig("welvet_b200_volume_create", _ST, c_int32, c_int32, c_int32, c_int32, POINTER(c_void_p))
_sig("welvet_b200_volume_bind_dense", _ST, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
     c_int32, c_void_p, c_void_p, c_size_t, c_int32)
_sig("welvet_b200_volume_bind_dense_native", _ST, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
     c_int32, c_int32, c_void_p, c_size_t, c_float, c_void_p, c_size_t)
_sig("welvet_b200_volume_bind_swiglu", _ST, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
     c_void_p, c_void_p, c_void_p, c_int32)
_sig("welvet_b200_volume_bind_mha", _ST, c_void_p, *([c_int32] * 13), c_void_p, c_void_p, c_void_p, c_void_p, c_int32)
_sig("welvet_b200_volume_bind_rmsnorm", _ST, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_double,
     c_int32, c_void_p)
_sig("welvet_b200_volume_set_remote_link", _ST, c_void_p, *([c_int32] * 8))
_sig("welvet_b200_volume_set_disabled", _ST, c_void_p, *([c_int32] * 5))
_sig("welvet_b200_volume_hops", c_int32, c_void_p)
_sig("welvet_b200_volume_forward_device", _ST, c_void_p, c_int32, c_void_p, c_int32, c_int32, c_int32, c_void_p,
     POINTER(c_int32), c_void_p)
_sig("welvet_b200_volume_forward_f32", _ST, c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_size_t,
     POINTER(c_int32))
_sig("welvet_b200_volume_cell_outputs", _ST, c_void_p, c_int32, c_int32, c_int32, c_int32, POINTER(c_void_p),
     POINTER(c_int32), POINTER(c_void_p), POINTER(c_int32))
_sig("welvet_b200_volume_release", None, c_void_p)


def _wptr(t):
    """(pointer, on_device) for a weight array: torch CUDA tensor or host numpy array."""
    if hasattr(t, "is_cuda"):
        return c_void_p(_dev_ptr(t)), 1, t
    a = _f32(t)
    return _np_ptr(a), 0, a


class Volume:
    """A depth x rows x cols x layers_per_cell grid of cells run in hop order on one GPU."""

    def __init__(self, depth: int, rows: int, cols: int, layers_per_cell: int):
        self._h = c_void_p()
        check(_L.welvet_b200_volume_create(depth, rows, cols, layers_per_cell, byref(self._h)))
        self.dims = (max(depth, 1), max(rows, 1), max(cols, 1), max(layers_per_cell, 1))

    def index(self, z, y, x, l) -> int:
        D, R, C, L = self.dims
        return ((z * R + y) * C + x) * L + l

    def coord(self, idx: int):
        D, R, C, L = self.dims
        l = idx % L
        r = idx // L
        x = r % C
        r //= C
        return r // R, r % R, x, l

    @property
    def hops(self) -> int:
        return int(_L.welvet_b200_volume_hops(self._h))

    def bind_dense(self, coord, W, act: int, dtype: int, bias=None):
        import numpy as np
        p, dev, keep = _wptr(W)
        out, in_ = W.shape
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float64)
        check(_L.welvet_b200_volume_bind_dense(self._h, *coord, in_, out, act, dtype, p, _np_ptr(b),
                                               0 if b is None else b.size, dev))

    def bind_dense_native(self, coord, native, scale: float, in_: int, out: int, act: int, dtype: int, bias=None):
        import numpy as np
        raw = np.ascontiguousarray(native, dtype=np.uint8)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float64)
        check(_L.welvet_b200_volume_bind_dense_native(self._h, *coord, in_, out, act, dtype, _np_ptr(raw), raw.size,
                                                      scale, _np_ptr(b), 0 if b is None else b.size))

    def bind_swiglu(self, coord, G, U, D, dtype: int):
        (pg, dev, kg), (pu, _, ku), (pd, _, kd) = _wptr(G), _wptr(U), _wptr(D)
        inter, in_ = G.shape
        check(_L.welvet_b200_volume_bind_swiglu(self._h, *coord, in_, inter, dtype, pg, pu, pd, dev))

    def bind_mha(self, coord, Q, K, V, O, d_model, num_heads, num_kv_heads=0, head_dim=0, max_seq_len=0, mask=1,
                 pos=0, seq=1, dtype=1):
        ps = [_wptr(t) for t in (Q, K, V, O)]
        check(_L.welvet_b200_volume_bind_mha(self._h, *coord, d_model, num_heads, num_kv_heads, head_dim,
                                             max_seq_len, mask, pos, seq, dtype, *[p[0] for p in ps], ps[0][1]))

    def bind_rmsnorm(self, coord, gamma, eps: float, dtype: int):
        g = _f32(gamma)
        check(_L.welvet_b200_volume_bind_rmsnorm(self._h, *coord, g.size, eps, dtype, _np_ptr(g)))

    def set_remote_link(self, coord, target):
        check(_L.welvet_b200_volume_set_remote_link(self._h, *coord, *target))

    def set_disabled(self, coord, disabled: bool = True):
        check(_L.welvet_b200_volume_set_disabled(self._h, *coord, 1 if disabled else 0))

    def forward_device(self, x, out=None, hop_begin: int = 0, hop_end: int = -1, stream=None) -> int:
        """x: CUDA tensor [rows][in]; returns the output width (out may be None)."""
        ow = c_int32()
        check(_L.welvet_b200_volume_forward_device(self._h, x.shape[0], c_void_p(_dev_ptr(x)), x.shape[1], hop_begin,
                                                   hop_end, None if out is None else c_void_p(_dev_ptr(out)),
                                                   byref(ow), _stream_ptr(stream)))
        return ow.value

    def forward_f32(self, x, out_width_cap: int):
        """Host x [rows][in] -> host output [rows][out width]; out_width_cap bounds the width."""
        import numpy as np
        x = _f32(x)
        rows = x.shape[0]
        out = np.zeros(rows * out_width_cap, np.float32)  # filled as [rows][out width], densely
        ow = c_int32()
        check(_L.welvet_b200_volume_forward_f32(self._h, rows, _np_ptr(x), x.shape[1], _np_ptr(out), out.size,
                                                byref(ow)))
        return out[:rows * ow.value].reshape(rows, ow.value).copy()

    def cell_outputs(self, coord):
        pre, post = c_void_p(), c_void_p()
        pw, ow = c_int32(), c_int32()
        check(_L.welvet_b200_volume_cell_outputs(self._h, *coord, byref(pre), byref(pw), byref(post), byref(ow)))
        return pre.value, pw.value, post.value, ow.value

    def release(self):
        if self._h:
            _L.welvet_b200_volume_release(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


# ---------------------------------------------------------------------------------- placement

def stage_plan(cells: int, layers_per_cell: int, world: int) -> list[tuple[int, int]]:
    """Hop ranges [begin, end) per rank: whole cells, one per GPU when world == cells,
    otherwise contiguous runs of cells split as evenly as possible (earlier ranks take the
    extra cell). Ranks beyond the cell count get an empty range."""
    if world < 1 or cells < 1:
        raise ValueError("stage_plan: need cells >= 1 and world >= 1")
    out = []
    for r in range(world):
        c0 = cells * r // world if world <= cells else min(r, cells)
        c1 = cells * (r + 1) // world if world <= cells else min(r + 1, cells)
        out.append((c0 * layers_per_cell, c1 * layers_per_cell))
    return out


def microbatches(rows: int, size: int) -> list[tuple[int, int]]:
    if size <= 0:
        raise ValueError("micro-batch size must be positive")
    return [(r, min(r + size, rows)) for r in range(0, rows, size)]


class PipelinedVolume:
    """Cell-per-GPU pipeline over torch.distributed.

    `runner(x) -> y` runs this rank's hop range on a [mb][in] tensor of its device and
    returns a [mb][out] tensor. Rank 0 feeds the input, rank world-1 produces the output,
    which `forward` returns on every rank after a broadcast from the last rank (so that the
    caller sees the result where it called). Sends are issued as each micro-batch finishes
    (isend), so rank r works on micro-batch i+1 while rank r+1 works on micro-batch i.
    """

    def __init__(self, runner, in_width: int, out_widths: list[int], group=None):
        import torch.distributed as dist
        self.dist = dist
        self.runner = runner
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.group = group
        self.in_width = in_width
        self.out_widths = out_widths  # output width of every rank's stage

    def forward(self, x, micro: int):
        import torch
        dist = self.dist
        rank, world = self.rank, self.world
        rows = x.shape[0]
        dev = x.device
        width_in = self.in_width if rank == 0 else self.out_widths[rank - 1]
        outs = []
        pending = []
        for (a, b) in microbatches(rows, micro):
            if rank == 0:
                xin = x[a:b].contiguous()
            else:
                xin = torch.empty((b - a, width_in), dtype=torch.float32, device=dev)
                dist.recv(xin, src=rank - 1, group=self.group)
            y = self.runner(xin)
            if rank < world - 1:
                pending.append(dist.isend(y.contiguous(), dst=rank + 1, group=self.group))
            else:
                outs.append(y)
        for p in pending:
            p.wait()
        ow = self.out_widths[-1]
        if rank == world - 1:
            result = torch.cat(outs, dim=0).contiguous()
        else:
            result = torch.empty((rows, ow), dtype=torch.float32, device=dev)
        if world > 1:
            dist.broadcast(result, src=world - 1, group=self.group)
        return result


class ColumnShardedDense:
    """A Dense layer out x in split by output rows over the ranks of a group.

    `local(x) -> y_slice` computes this rank's [rows][out/N] slice (the product passes a
    DenseSession mounted on the rank's rows); `forward` all-gathers the slices into
    [rows][out] on every rank (NCCL over NVLink on B200 ranks)."""

    def __init__(self, local, out: int, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.local = local
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if out % self.world != 0:
            raise ValueError("ColumnShardedDense: out must be divisible by the number of ranks")
        self.out = out
        self.shard = out // self.world

    @staticmethod
    def shard_rows(out: int, world: int, rank: int) -> tuple[int, int]:
        s = out // world
        return rank * s, (rank + 1) * s

    def forward(self, x):
        import torch
        y = self.local(x).contiguous()  # [rows][shard]
        if self.world == 1:
            return y
        rows = y.shape[0]
        # [world*rows][shard]: rank slices concatenated along dim 0 (the layout every backend accepts)
        gathered = torch.empty((self.world * rows, self.shard), dtype=y.dtype, device=y.device)
        self.dist.all_gather_into_tensor(gathered, y, group=self.group)
        if rows == 1:
            return gathered.view(1, self.out)
        return gathered.view(self.world, rows, self.shard).permute(1, 0, 2).reshape(rows, self.out)
