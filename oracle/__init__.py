"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for welvet.cuda's quantized Dense path.

`liboracle.so` (built from oracle.c by oracle/Makefile) is a plain-C restatement of the
reference's codecs (src/core/float_codecs.cpp:57-200), FormatNone packing and decode
(src/weights/native_codec.cpp:174-262, :513-568, :1043-1078) and the fp64 Dense kernels
(src/cuda/kernels.cu:22-46, :130-161, :296-305). `libwelvet_ref.so` (oracle/_ref) is the
reference itself compiled from its sources; it pins the restatement and, on a GPU box, runs
the reference's own CUDA Dense path as a baseline.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline / reference arm may import
this package. The product library never loads it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int64, c_size_t, c_uint8, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libwelvet_ref.so")

# DType ids (include/welvet/dtype.hpp:9-44) and Activation ids (include/welvet/activate.hpp:8-17)
FLOAT32, FP8E4M3, FP8E5M2, INT8, FP4 = 1, 4, 5, 9, 16
QUANT_DTYPES = (FP8E4M3, FP8E5M2, FP4, INT8)
ACT_LINEAR, ACT_RELU, ACT_SILU, ACT_GELU, ACT_TANH, ACT_SIGMOID, ACT_LEAKY, ACT_RELU2 = -1, 0, 1, 2, 3, 4, 5, 6

_f32p = POINTER(c_float)
_f64p = POINTER(c_double)
_u8p = POINTER(c_uint8)


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference tree is present)."""
    subprocess.run(["make", "-C", HERE, "-j8", "-s"], check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t) if a is not None else None


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        for n in ("or_e4m3_encode", "or_e5m2_encode", "or_fp4_encode"):
            getattr(L, n).restype = c_uint8
            getattr(L, n).argtypes = [c_float]
        for n in ("or_e4m3_decode", "or_e5m2_decode", "or_fp4_decode"):
            getattr(L, n).restype = c_float
            getattr(L, n).argtypes = [c_uint8]
        L.or_native_bytes.restype = c_int64
        L.or_native_bytes.argtypes = [c_int, c_int64]
        L.or_pack.restype = c_int
        L.or_pack.argtypes = [c_int, _f32p, c_int64, _u8p, _f32p]
        L.or_decode_f64.restype = c_int
        L.or_decode_f64.argtypes = [c_int, _u8p, c_float, c_int64, c_int64, _f64p]
        L.or_activate.restype = c_double
        L.or_activate.argtypes = [c_int, c_double]
        L.or_dense_forward_f64w.restype = None
        L.or_dense_forward_f64w.argtypes = [c_int, c_int, c_int, c_int, _f64p, _f64p, c_int, _f32p,
                                            _f32p, _f32p, _f64p, _f64p, c_int]
        L.or_dense_forward_native.restype = None
        L.or_dense_forward_native.argtypes = [c_int, _u8p, c_float, c_int, c_int, c_int, c_int, _f64p,
                                              c_int, _f32p, _f32p, _f32p, _f64p, _f64p, c_int]
        L.or_swiglu_product.restype = None
        L.or_swiglu_product.argtypes = [_f32p, _f32p, _f32p, c_int64]
        L.or_encode_digest.restype = c_uint64
        L.or_encode_digest.argtypes = [c_int, c_uint64, c_uint64, c_int]
        L.or_activate_deriv.restype = c_double
        L.or_activate_deriv.argtypes = [c_int, c_double]
        L.or_dense_backward.restype = c_int
        L.or_dense_backward.argtypes = [c_int, _u8p, c_float, c_int, c_int, c_int, c_int, c_int, _f32p, _f32p,
                                        _f32p, _f32p, _f32p, _f32p]
        L.or_apply_sgd.restype = c_int
        L.or_apply_sgd.argtypes = [c_int, _u8p, c_float, c_int64, _f64p, c_double]
        L.or_mse.restype = c_double
        L.or_mse.argtypes = [_f32p, _f32p, c_int64, _f32p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own codec / store / Dense session, compiled from its sources."""
    global _ref
    if _ref is None:
        R = ctypes.CDLL(REF_SO)
        for n in ("ref_e4m3_encode", "ref_e5m2_encode", "ref_fp4_encode"):
            getattr(R, n).restype = c_uint8
            getattr(R, n).argtypes = [c_float]
        for n in ("ref_e4m3_decode", "ref_e5m2_decode", "ref_fp4_decode"):
            getattr(R, n).restype = c_float
            getattr(R, n).argtypes = [c_uint8]
        R.ref_encode_digest.restype = c_uint64
        R.ref_encode_digest.argtypes = [c_int, c_uint64, c_uint64, c_int]
        R.ref_store_make.restype = c_int
        R.ref_store_make.argtypes = [c_int, c_int, c_int, _f32p, _u8p, c_size_t, POINTER(c_size_t), _f32p,
                                     c_char_p, c_int]
        R.ref_store_decode.restype = c_int
        R.ref_store_decode.argtypes = [c_int, c_int, c_int, _u8p, c_size_t, c_float, _f64p, c_char_p, c_int]
        R.ref_dense_mount.restype = c_int
        R.ref_dense_mount.argtypes = [c_int, c_int, c_int, c_int, c_int, _f32p, _f64p, c_size_t,
                                      POINTER(c_void_p), c_char_p, c_int]
        R.ref_dense_execute.restype = c_int
        R.ref_dense_execute.argtypes = [c_void_p, _f32p, _f32p, _f32p, c_char_p, c_int]
        R.ref_dense_release.restype = None
        R.ref_dense_release.argtypes = [c_void_p]
        R.ref_swiglu_forward.restype = c_int
        R.ref_swiglu_forward.argtypes = [c_int, c_int, c_int, c_int, c_int, _f32p, _f32p, _f32p, _f32p,
                                         _f32p, _f32p, c_char_p, c_int]
        R.ref_mha_forward.restype = c_int
        R.ref_mha_forward.argtypes = [c_int] * 10 + [_f32p] * 7 + [c_char_p, c_int]
        R.ref_store_apply_sgd.restype = c_int
        R.ref_store_apply_sgd.argtypes = [c_int, c_int, c_int, _u8p, c_size_t, c_float, _f64p, c_double, c_char_p,
                                          c_int]
        R.ref_dense_normalbp.restype = c_int
        R.ref_dense_normalbp.argtypes = [c_int, c_int, c_int, c_int, c_int, _f32p, _f64p, c_size_t, _f32p, _f32p,
                                         c_int, c_double, _f32p, _f32p, _f32p, _f32p, _f32p, POINTER(c_double),
                                         c_char_p, c_int]
        _ref = R
    return _ref


# ------------------------------------------------------------------ numpy helpers

def pack(dtype: int, w: np.ndarray) -> tuple[np.ndarray, float]:
    """FormatNone pack of a float32 matrix -> (native bytes, scale) (oracle restatement)."""
    w = np.ascontiguousarray(w, dtype=np.float32).ravel()
    n = w.size
    out = np.zeros(lib().or_native_bytes(dtype, n), dtype=np.uint8)
    sc = np.zeros(1, dtype=np.float32)
    rc = lib().or_pack(dtype, _ptr(w, _f32p), n, _ptr(out, _u8p), _ptr(sc, _f32p))
    if rc != 0:
        raise ValueError(f"oracle pack: dtype {dtype} not on the quantized path")
    return out, float(sc[0])


def decode(dtype: int, raw: np.ndarray, scale: float, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.zeros(n, dtype=np.float64)
    rc = lib().or_decode_f64(dtype, _ptr(raw, _u8p), scale, 0, n, _ptr(out, _f64p))
    if rc != 0:
        raise ValueError("oracle decode: bad dtype")
    return out


def dense_forward(dtype: int, raw: np.ndarray, scale: float, x: np.ndarray, in_: int, out: int,
                  act: int = ACT_LINEAR, bias: np.ndarray | None = None, threads: int = 0):
    """Reference Dense forward semantics (decode row, sequential fp64 sum, bias/act).

    Returns (pre f32 [B,out], post f32 [B,out], y64 f64 [B,out], sabs f64 [B,out]) where y64
    is the unrounded f64 sum and sabs = sum_k |W[o,k] x[b,k]| (for error bounds)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    batch = x.size // in_
    raw = np.ascontiguousarray(raw).view(np.uint8)
    pre = np.zeros((batch, out), np.float32)
    post = np.zeros((batch, out), np.float32)
    y64 = np.zeros((batch, out), np.float64)
    sabs = np.zeros((batch, out), np.float64)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float64)
    if threads <= 0:
        threads = os.cpu_count() or 1
    lib().or_dense_forward_native(dtype, _ptr(raw, _u8p), scale, batch, in_, out, act,
                                  _ptr(b, _f64p), 0 if b is None else b.size, _ptr(x, _f32p),
                                  _ptr(pre, _f32p), _ptr(post, _f32p), _ptr(y64, _f64p),
                                  _ptr(sabs, _f64p), threads)
    return pre, post, y64, sabs


def swiglu_product(gate_pre: np.ndarray, up_post: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate_pre, dtype=np.float32)
    u = np.ascontiguousarray(up_post, dtype=np.float32)
    h = np.zeros_like(g)
    lib().or_swiglu_product(_ptr(g, _f32p), _ptr(u, _f32p), _ptr(h, _f32p), g.size)
    return h


def encode_digest(codec: int, start: int, count: int, threads: int = 0) -> int:
    return int(lib().or_encode_digest(codec, start, count, threads or (os.cpu_count() or 1)))


def ref_pack(dtype: int, w: np.ndarray, rows: int, cols: int) -> tuple[np.ndarray, float]:
    """The reference's WeightStore::make on the same float32 matrix."""
    w = np.ascontiguousarray(w, dtype=np.float32).ravel()
    cap = max(16, w.size * 4 + 16)
    out = np.zeros(cap, np.uint8)
    ln = c_size_t(0)
    sc = np.zeros(1, np.float32)
    msg = ctypes.create_string_buffer(256)
    rc = ref().ref_store_make(rows, cols, dtype, _ptr(w, _f32p), _ptr(out, _u8p), cap, ctypes.byref(ln),
                              _ptr(sc, _f32p), msg, 256)
    if rc != 0:
        raise RuntimeError(f"reference store make: {rc} {msg.value.decode()}")
    return out[: ln.value].copy(), float(sc[0])


def ref_decode(dtype: int, raw: np.ndarray, scale: float, rows: int, cols: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.zeros((rows, cols), np.float64)
    msg = ctypes.create_string_buffer(256)
    rc = ref().ref_store_decode(rows, cols, dtype, _ptr(raw, _u8p), raw.size, scale, _ptr(out, _f64p), msg, 256)
    if rc != 0:
        raise RuntimeError(f"reference decode: {rc} {msg.value.decode()}")
    return out


def ref_encode_digest(codec: int, start: int, count: int, threads: int = 0) -> int:
    return int(ref().ref_encode_digest(codec, start, count, threads or (os.cpu_count() or 1)))


def dense_backward(dtype: int, raw: np.ndarray, scale: float, gy: np.ndarray, x: np.ndarray, pre: np.ndarray,
                   in_: int, out: int, act: int, linear: bool = False):
    """Reference Dense NormalBP backward (kernels.cu:83-128): (d_pre, gx [B,in], dW [out,in])."""
    gy = np.ascontiguousarray(gy, np.float32).reshape(-1, out)
    batch = gy.shape[0]
    x = np.ascontiguousarray(x, np.float32).reshape(batch, in_)
    pre = np.ascontiguousarray(pre, np.float32).reshape(batch, out)
    raw = np.ascontiguousarray(raw).view(np.uint8)
    d_pre = np.zeros((batch, out), np.float32)
    gx = np.zeros((batch, in_), np.float32)
    dW = np.zeros((out, in_), np.float32)
    rc = lib().or_dense_backward(dtype, _ptr(raw, _u8p), scale, batch, in_, out, act, 1 if linear else 0,
                                 _ptr(gy, _f32p), _ptr(x, _f32p), _ptr(pre, _f32p), _ptr(d_pre, _f32p),
                                 _ptr(gx, _f32p), _ptr(dW, _f32p))
    if rc != 0:
        raise ValueError("oracle dense_backward: bad dtype")
    return d_pre, gx, dW


def apply_sgd(dtype: int, raw: np.ndarray, scale: float, dW: np.ndarray, lr: float) -> np.ndarray:
    """WeightStore::apply_sgd (native_codec.cpp:1080-1133) on a copy of the payload."""
    out = np.array(raw, dtype=np.uint8, copy=True)
    d = np.ascontiguousarray(dW, np.float64).ravel()
    if lib().or_apply_sgd(dtype, _ptr(out, _u8p), scale, d.size, _ptr(d, _f64p), lr) != 0:
        raise ValueError("oracle apply_sgd: bad dtype")
    return out


def mse(pred: np.ndarray, target: np.ndarray):
    """training.cpp:44-69: (loss, grad)."""
    p = np.ascontiguousarray(pred, np.float32).ravel()
    t = np.ascontiguousarray(target, np.float32).ravel()
    g = np.zeros_like(p)
    loss = lib().or_mse(_ptr(p, _f32p), _ptr(t, _f32p), p.size, _ptr(g, _f32p))
    return float(loss), g.reshape(np.shape(pred))


def store_of(dtype: int, w: np.ndarray) -> tuple[np.ndarray, float]:
    """A store's payload as bytes: Float32 keeps the float master, other dtypes pack."""
    if dtype == FLOAT32:
        return np.ascontiguousarray(w, np.float32).ravel().view(np.uint8).copy(), 1.0
    return pack(dtype, w)


def decode_f32(dtype: int, raw: np.ndarray, scale: float, n: int) -> np.ndarray:
    """WeightStore::export_f32 (store.cpp:42-70): weight_at per element, as float32."""
    if dtype == FLOAT32:
        return np.ascontiguousarray(raw).view(np.float32)[:n].copy()
    return decode(dtype, raw, scale, n).astype(np.float32)


def dense_normalbp(dtype: int, W: np.ndarray, x: np.ndarray, grad_or_target: np.ndarray, act: int,
                   bias=None, use_target: bool = False, lr: float = 0.0):
    """The steps of welvet_dense_normalbp_f32 (src/interop/c_abi.cpp:119-184) over the oracle:
    pack, forward, MSE (use_target) or the given gradient, backward, SGD when lr != 0, export.
    Returns (pre, post, dX, dW, W_after, loss)."""
    out, in_ = W.shape
    raw, scale = store_of(dtype, W)
    pre, post, _, _ = dense_forward(dtype, raw, scale, x, in_, out, act, bias)
    g = np.ascontiguousarray(grad_or_target, np.float32).reshape(post.shape)
    loss = 0.0
    if use_target:
        loss, g = mse(post, g)
    _, gx, dW = dense_backward(dtype, raw, scale, g, x, pre, in_, out, act)
    if lr != 0.0:
        raw = apply_sgd(dtype, raw, scale, dW, lr)
    W_after = decode_f32(dtype, raw, scale, out * in_).reshape(out, in_)
    return pre, post, gx, dW, W_after, loss


def ref_store_apply_sgd(dtype: int, raw: np.ndarray, scale: float, rows: int, cols: int, dW: np.ndarray,
                        lr: float) -> np.ndarray:
    """The reference's WeightStore::apply_sgd (native_codec.cpp:1080-1133) on a copy."""
    out = np.array(raw, dtype=np.uint8, copy=True)
    d = np.ascontiguousarray(dW, np.float64).ravel()
    msg = ctypes.create_string_buffer(256)
    rc = ref().ref_store_apply_sgd(rows, cols, dtype, _ptr(out, _u8p), out.size, scale, _ptr(d, _f64p), lr, msg, 256)
    if rc != 0:
        raise RuntimeError(f"reference apply_sgd: {rc} {msg.value.decode()}")
    return out


def ref_dense_normalbp(dtype: int, W: np.ndarray, x: np.ndarray, grad_or_target: np.ndarray, act: int,
                       bias=None, use_target: bool = False, lr: float = 0.0):
    """The reference's own Dense training step on its CUDA kernels (needs a GPU): the same
    return tuple as dense_normalbp."""
    out, in_ = W.shape
    W = np.ascontiguousarray(W, np.float32)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, in_)
    batch = x.shape[0]
    g = np.ascontiguousarray(grad_or_target, np.float32).reshape(batch, out)
    b = None if bias is None else np.ascontiguousarray(bias, np.float64)
    pre = np.zeros((batch, out), np.float32)
    post = np.zeros((batch, out), np.float32)
    dX = np.zeros((batch, in_), np.float32)
    dW = np.zeros((out, in_), np.float32)
    W_after = np.zeros((out, in_), np.float32)
    loss = c_double(0.0)
    msg = ctypes.create_string_buffer(256)
    rc = ref().ref_dense_normalbp(batch, in_, out, act, dtype, _ptr(W, _f32p), _ptr(b, _f64p),
                                  0 if b is None else b.size, _ptr(x, _f32p), _ptr(g, _f32p), int(bool(use_target)),
                                  lr, _ptr(pre, _f32p), _ptr(post, _f32p), _ptr(dX, _f32p), _ptr(dW, _f32p),
                                  _ptr(W_after, _f32p), ctypes.byref(loss), msg, 256)
    if rc != 0:
        raise RuntimeError(f"reference dense normalbp: {rc} {msg.value.decode()}")
    return pre, post, dX, dW, W_after, loss.value
