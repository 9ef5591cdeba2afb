"""Volume (Grid) forward and its multi-GPU placement.

`Volume` binds the device-resident volume runtime of libwelvet_b200.so (reference
architecture::Grid + runtime::forward::volume_dense, include/welvet/architecture.hpp:100-141,
src/runtime/forward.cpp:98-156).

Multi-GPU (one process per GPU): the library's C++ runtime does the work (NCCL loaded by the
library, CUDA IPC peer memory over NVLink); Python only hands the 128-byte job id from rank 0
to the others.

* `Comm` -- the ranks of one job on the GPUs of one box.
* `stage_plan` / `Comm.pipeline_forward` -- the volume's cells placed one per GPU (contiguous
  runs of cells in hop order when there are fewer GPUs than cells). The hop order is a
  sequential chain, so the GPUs form a pipeline: the batch is cut into micro-batches (rows
  are independent through the cells, so results do not change) and activations move between
  consecutive ranks with NCCL point-to-point transfers.
* `shard_rows` / `ShardedDense` -- a Dense layer too large for one GPU: rank r holds whole
  128-row blocks of its output rows; its kernels store its columns of the output straight into
  every rank's output buffer (mode FUSED) or all-gather after the local forward (mode NCCL).
"""
from __future__ import annotations

import ctypes
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


# ---------------------------------------------------------------------------------- multi-GPU

_sig("welvet_b200_nccl_available", c_int32)
_sig("welvet_b200_comm_unique_id", _ST, c_void_p)
_sig("welvet_b200_comm_create", _ST, c_void_p, c_int32, c_int32, c_int32, POINTER(c_void_p))
_sig("welvet_b200_comm_release", None, c_void_p)
_sig("welvet_b200_shard_rows", _ST, c_int32, c_int32, c_int32, POINTER(c_int32), POINTER(c_int32))
_sig("welvet_b200_stage_plan", _ST, c_int32, c_int32, c_int32, c_int32, POINTER(c_int32), POINTER(c_int32))
_sig("welvet_b200_sharded_dense_mount", _ST, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p,
     c_int32, c_void_p, c_size_t, c_int32, POINTER(c_void_p))
_sig("welvet_b200_sharded_dense_execute_device", _ST, c_void_p, c_void_p, c_void_p, POINTER(c_void_p),
     POINTER(c_void_p))
_sig("welvet_b200_sharded_dense_execute", _ST, c_void_p, c_void_p, c_void_p, c_void_p)
_sig("welvet_b200_sharded_dense_check_error", _ST, c_void_p, c_void_p)
_sig("welvet_b200_sharded_dense_rows", _ST, c_void_p, POINTER(c_int32), POINTER(c_int32))
_sig("welvet_b200_sharded_dense_release", None, c_void_p)
_sig("welvet_b200_volume_pipeline_forward_device", _ST, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p,
     c_int32, c_int32, c_void_p, c_int32, c_void_p)

FUSED, NCCL = 0, 1


def nccl_available() -> bool:
    return bool(_L.welvet_b200_nccl_available())


def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Output rows [begin, end) rank `rank` holds of a column-sharded layer (whole 128-row
    blocks dealt in rank order)."""
    b, e = c_int32(), c_int32()
    check(_L.welvet_b200_shard_rows(rows, world, rank, byref(b), byref(e)))
    return b.value, e.value


def stage_plan(cells: int, layers_per_cell: int, world: int) -> list[tuple[int, int]]:
    """Hop ranges [begin, end) per rank of the cell-per-GPU pipeline: whole cells, one per GPU
    when world == cells, otherwise contiguous runs of cells split as evenly as possible
    (earlier ranks take fewer). Ranks beyond the cell count get an empty range."""
    out = []
    for r in range(world):
        b, e = c_int32(), c_int32()
        check(_L.welvet_b200_stage_plan(cells, layers_per_cell, world, r, byref(b), byref(e)))
        out.append((b.value, e.value))
    return out


def microbatches(rows: int, size: int) -> list[tuple[int, int]]:
    if size <= 0:
        raise ValueError("micro-batch size must be positive")
    return [(r, min(r + size, rows)) for r in range(0, rows, size)]


class _DevView:
    """A library-owned device buffer seen as a torch tensor (no copy)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_tensor(ptr: int, shape):
    import torch
    return torch.as_tensor(_DevView(ptr, shape), device="cuda")


class Comm:
    """This process as rank `rank` of `world` on CUDA device `device` (collective)."""

    def __init__(self, rank: int, world: int, device: int, job_id: bytes):
        if len(job_id) != 128:
            raise ValueError("job id must be 128 bytes")
        self._h = c_void_p()
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(job_id)
        check(_L.welvet_b200_comm_create(buf, world, rank, device, byref(self._h)))
        self.rank, self.world, self.device = rank, world, device

    @staticmethod
    def new_job_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        check(_L.welvet_b200_comm_unique_id(buf))
        return bytes(buf)

    @classmethod
    def from_torch(cls, device: int, group=None) -> "Comm":
        """The ranks of a torch.distributed group (any backend): rank 0 makes the job id and
        the group hands it to the others; the communicator itself is the library's."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.new_job_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(rank, world, device, obj[0])

    def pipeline_forward(self, volume: "Volume", hop_range, x, stage_in_width: int, micro: int, out,
                         stream=None) -> None:
        """Collective: the cell-per-GPU pipeline forward (see the module docstring). x (rank 0)
        is a CUDA tensor [rows][width]; out [rows][out width] receives the volume's output on
        every rank."""
        b, e = hop_range
        rows = out.shape[0]
        check(_L.welvet_b200_volume_pipeline_forward_device(
            volume._h, self._h, b, e, rows, None if x is None else c_void_p(_dev_ptr(x)), stage_in_width, micro,
            c_void_p(_dev_ptr(out)), out.shape[1], _stream_ptr(stream)))

    def release(self):
        if self._h:
            _L.welvet_b200_comm_release(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class ShardedDense:
    """A Dense layer in -> out split by output rows over the ranks of `comm` (collective).
    W_rows: this rank's rows (shard_rows), a CUDA tensor or host array [end - begin][in];
    bias: the whole layer's (host, applies to rows o < len(bias))."""

    def __init__(self, comm: Comm, W_rows, in_: int, out: int, batch: int, dtype: int, act: int = -1, bias=None,
                 mode: int = FUSED):
        import numpy as np
        self._h = c_void_p()
        p, dev, self._keep = _wptr(W_rows)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float64)
        check(_L.welvet_b200_sharded_dense_mount(comm._h, batch, in_, out, act, dtype, p, dev, _np_ptr(b),
                                                 0 if b is None else b.size, mode, byref(self._h)))
        self._keep = None
        self.comm, self.batch, self.in_, self.out = comm, batch, in_, out

    @property
    def rows(self) -> tuple[int, int]:
        b, e = c_int32(), c_int32()
        check(_L.welvet_b200_sharded_dense_rows(self._h, byref(b), byref(e)))
        return b.value, e.value

    def execute_device_ptrs(self, x, stream=None) -> tuple[int, int]:
        """Collective, asynchronous: (post, pre) device addresses of the whole output
        [batch][out] on this rank (valid until the call after next)."""
        post, pre = c_void_p(), c_void_p()
        check(_L.welvet_b200_sharded_dense_execute_device(self._h, c_void_p(_dev_ptr(x)), _stream_ptr(stream),
                                                          byref(post), byref(pre)))
        return post.value, pre.value

    def execute_device(self, x, stream=None):
        """Collective: (post, pre) as torch tensors viewing the library's buffers."""
        post, pre = self.execute_device_ptrs(x, stream)
        shape = (self.batch, self.out)
        return device_tensor(post, shape), device_tensor(pre, shape)

    def execute(self, x):
        """Collective, synchronous, host buffers: (pre, post) numpy [batch][out]."""
        import numpy as np
        x = _f32(x)
        pre = np.zeros((self.batch, self.out), np.float32)
        post = np.zeros((self.batch, self.out), np.float32)
        check(_L.welvet_b200_sharded_dense_execute(self._h, _np_ptr(x), _np_ptr(pre), _np_ptr(post)))
        return pre, post

    def check_error(self, stream=None) -> None:
        check(_L.welvet_b200_sharded_dense_check_error(self._h, _stream_ptr(stream)))

    def release(self):
        if self._h:
            _L.welvet_b200_sharded_dense_release(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass
