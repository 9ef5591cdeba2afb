"""WMN1 model descriptor writer for the tests (test infrastructure).

Writes the byte layout the reference's welvet_model_mount reads
(src/interop/model_session.cpp:317-396): magic "WMN1", root (0 Stack, 1 Parallel, 2 Grid),
child count, four grid dims; the children in the child_wire.hpp:21-192 layouts; empty training
controls for the root and each child (model_wire.hpp:195-263); the store section
(model_session.cpp:135-153, stores in the order cam_sync.cpp:8-40 collects them); for a Grid
root each cell's enabled flag and remote link. Little-endian, no padding.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = 0x314E4D57
FLOAT32 = 1


def _f32(a) -> bytes:
    return np.ascontiguousarray(a, dtype="<f4").tobytes()


def dense_child(in_, out, act, dtype, W, bias=None) -> bytes:
    b = b"" if bias is None else np.ascontiguousarray(bias, dtype="<f8").tobytes()
    n = 0 if bias is None else len(bias)
    return struct.pack("<5i", 1, in_, out, act, dtype) + _f32(W) + struct.pack("<I", n) + b


def rmsnorm_child(dim, dtype, eps, gamma) -> bytes:
    return struct.pack("<3i", 2, dim, dtype) + struct.pack("<d", eps) + _f32(gamma)


def swiglu_child(in_, inter, dtype, G, U, D) -> bytes:
    return struct.pack("<4i", 4, in_, inter, dtype) + _f32(G) + _f32(U) + _f32(D)


def mha_child(seq, d_model, heads, kv, head_dim, msl, mask, pos, dtype, Q, K, V, O) -> bytes:
    return (struct.pack("<10i", 7, seq, d_model, heads, kv, head_dim, msl, mask, pos, dtype) + _f32(Q) + _f32(K)
            + _f32(V) + _f32(O))


def none_child() -> bytes:
    return struct.pack("<i", 0)


def controls() -> bytes:
    """No training modes, no branch rates, zero coefficients, no sync configuration."""
    return struct.pack("<ii", 0, 0) + struct.pack("<3d", 0.0, 0.0, 0.0) + struct.pack("<i", 0)


def store_f32(rows, cols, values, bias=()) -> tuple:
    return (FLOAT32, rows, cols, 1.0, np.ascontiguousarray(values, dtype=np.float32).ravel(), b"", bias)


def store_native(dtype, rows, cols, native, scale, bias=()) -> tuple:
    return (dtype, rows, cols, float(scale), np.zeros(0, np.float32), bytes(native), bias)


def _store(s) -> bytes:
    dt, rows, cols, scale, f32, native, bias = s
    bias = np.ascontiguousarray(bias, dtype="<f8")
    return (struct.pack("<3i", dt, rows, cols) + struct.pack("<f", scale) + struct.pack("<i", len(f32)) + _f32(f32)
            + struct.pack("<i", len(native)) + bytes(native) + struct.pack("<i", bias.size) + bias.tobytes())


def descriptor(root, children, stores, dims=None, cells=None) -> bytes:
    """cells (Grid root): one (enabled, remote, tz, ty, tx, tl) per child in hop order."""
    n = len(children)
    dims = dims or (1, 1, 1, n)
    out = struct.pack("<I", MAGIC) + struct.pack("<6i", root, n, *dims)
    out += b"".join(children)
    out += controls() + controls() * n
    out += struct.pack("<i", len(stores)) + b"".join(_store(s) for s in stores)
    if root == 2:
        out += b"".join(struct.pack("<6i", *c) for c in cells)
    return out


def tensor(x) -> bytes:
    x = np.ascontiguousarray(x, dtype="<f4")
    return struct.pack("<i", x.ndim) + struct.pack(f"<{x.ndim}i", *x.shape) + x.tobytes()


def read_tensor(b: bytes) -> np.ndarray:
    rank = struct.unpack_from("<i", b, 0)[0]
    dims = struct.unpack_from(f"<{rank}i", b, 4)
    return np.frombuffer(b, dtype="<f4", offset=4 + 4 * rank).reshape(dims).copy()
