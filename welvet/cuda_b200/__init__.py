"""welvet.cuda_b200 -- Python host binding of libwelvet_b200.so (the sm_100a library).

The functions here mirror the reference's C ABI (include/welvet_c.h) one for one, with the
same argument meaning and the same status codes, raising `WelvetError` for a non-zero
status. Device-pointer variants accept torch CUDA tensors. There is no CPU path: importing
this module without the built library raises ImportError.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, byref, c_char, c_double, c_float, c_int32, c_int64, c_size_t, c_uint8, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# WELVET_B200_LIB names another build of the library to load instead of the in-tree one.
LIB_PATH = os.environ.get("WELVET_B200_LIB") or os.path.join(HERE, "libwelvet_b200.so")

# DType ids (reference include/welvet/dtype.hpp:9-44) served on the GPU.
FLOAT32, FP8E4M3, FP8E5M2, INT8, FP4 = 1, 4, 5, 9, 16
DTYPES = {"float32": FLOAT32, "fp8e4m3": FP8E4M3, "fp8e5m2": FP8E5M2, "int8": INT8, "fp4": FP4}
# Activation ids (reference include/welvet/activate.hpp:8-17).
LINEAR, RELU, SILU, GELU, TANH, SIGMOID, LEAKY_RELU, RELU2 = -1, 0, 1, 2, 3, 4, 5, 6
# Status codes (reference include/welvet_c.h:26-29).
OK, INVALID, UNSUPPORTED, GAP, INTERNAL = 0, 1, 2, 3, 4


class welvet_status(ctypes.Structure):
    _fields_ = [("code", c_int32), ("message", c_char * 256)]


class WelvetError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"welvet status {code}: {message}")
        self.code = code
        self.message = message


def build() -> None:
    """Compile libwelvet_b200.so for sm_100a (nvcc; no GPU needed)."""
    subprocess.run(["make", "-C", os.path.join(HERE, "csrc"), "-j8", "-s"], check=True)


if not os.path.exists(LIB_PATH):
    raise ImportError(f"welvet.cuda_b200: {LIB_PATH} is not built (run welvet.cuda_b200.build() / make -C "
                      f"welvet/cuda_b200/csrc); there is no CPU fallback")

_L = ctypes.CDLL(LIB_PATH)

_f32p, _f64p, _u8p = POINTER(c_float), POINTER(c_double), POINTER(c_uint8)
_ST = welvet_status


def _sig(name, res, *args):
    fn = getattr(_L, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


_sig("welvet_version", ctypes.c_char_p)
_sig("welvet_runtime_identity", ctypes.c_char_p)
_sig("welvet_b200_build_id", ctypes.c_char_p)
_sig("welvet_cuda_init", _ST)
_sig("welvet_cuda_available", c_int32)
_sig("welvet_gaps_count", c_int32)
_sig("welvet_gaps_done", c_int32)
_sig("welvet_dense_forward_f32", _ST, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
     c_size_t, c_void_p, c_void_p, c_void_p)
_sig("welvet_dense_normalbp_f32", _ST, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
     c_size_t, c_void_p, c_void_p, c_int32, c_double, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
     POINTER(c_double))
_sig("welvet_dense_mount", _ST, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_size_t,
     POINTER(c_void_p))
_sig("welvet_b200_dense_mount_device", _ST, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
     c_size_t, POINTER(c_void_p))
_sig("welvet_b200_dense_mount_native", _ST, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_size_t,
     c_float, c_void_p, c_size_t, POINTER(c_void_p))
_sig("welvet_dense_execute", _ST, c_void_p, c_void_p, c_void_p, c_void_p)
_sig("welvet_b200_dense_execute_device", _ST, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p)
_sig("welvet_b200_dense_execute_device_noalloc", _ST, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p)
_sig("welvet_b200_dense_check_error", _ST, c_void_p, c_void_p)
_sig("welvet_b200_dense_execute_group_device", _ST, POINTER(c_void_p), c_int32, POINTER(c_void_p),
     POINTER(c_void_p), POINTER(c_void_p), c_void_p)
_sig("welvet_dense_release", None, c_void_p)
_sig("welvet_b200_dense_store", _ST, c_void_p, POINTER(c_int32), POINTER(c_int32), POINTER(c_int32),
     POINTER(c_float), c_void_p, c_size_t, POINTER(c_size_t))
_sig("welvet_rmsnorm_forward_f32", _ST, c_int32, c_int32, c_int32, c_double, c_int32, c_int32, c_void_p, c_void_p,
     c_void_p, c_void_p)
_sig("welvet_swiglu_forward_f32", _ST, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
     c_void_p, c_void_p, c_void_p, c_void_p)
_sig("welvet_mha_forward_f32", _ST, *([c_int32] * 11), *([c_void_p] * 7))
_sig("welvet_b200_codec_encode", _ST, c_int32, c_void_p, c_int64, c_void_p, c_void_p, c_void_p)
_sig("welvet_b200_codec_decode", _ST, c_int32, c_void_p, c_int64, c_float, c_void_p, c_void_p)
_sig("welvet_b200_codec_digest", _ST, c_int32, c_uint64, c_uint64, POINTER(c_uint64))
_sig("welvet_b200_codec_selftest_decode", _ST, c_int32, c_void_p)
_sig("welvet_b200_swiglu_mount", _ST, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32,
     POINTER(c_void_p))
_sig("welvet_b200_swiglu_execute_device", _ST, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p)
_sig("welvet_b200_swiglu_release", None, c_void_p)
_sig("welvet_b200_mha_mount", _ST, *([c_int32] * 8), *([c_void_p] * 4), c_int32, POINTER(c_void_p))
_sig("welvet_b200_mha_execute_device", _ST, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p)
_sig("welvet_b200_mha_release", None, c_void_p)


def lib() -> ctypes.CDLL:
    return _L


def check(st: welvet_status) -> None:
    if st.code != OK:
        raise WelvetError(st.code, st.message.decode(errors="replace"))


_F32 = np.dtype(np.float32)


def _np_ptr(a):
    """Address of an array's data. A ctypes view of a writable buffer is several times cheaper
    than ndarray.ctypes or the array interface on a per-call path; read-only arrays take the
    slower route."""
    if a is None:
        return None
    try:
        return ctypes.addressof(c_char.from_buffer(a))
    except (TypeError, ValueError):
        return a.ctypes.data


def _f32(a) -> np.ndarray:
    if type(a) is np.ndarray and a.dtype is _F32 and a.flags.c_contiguous:
        return a
    return np.ascontiguousarray(a, dtype=np.float32)


def _out_f32(a, n: int, shape, what: str) -> np.ndarray:
    """A caller-supplied output array (written in place by the library) or a new one."""
    if a is None:
        return np.zeros(shape, np.float32)
    if not (type(a) is np.ndarray and a.dtype is _F32 and a.flags.c_contiguous and a.flags.writeable):
        raise ValueError(f"{what}: expected a writable C-contiguous float32 array")
    if a.size != n:
        raise ValueError(f"{what}: expected {n} elements, got {a.size}")
    return a


def _dev_ptr(t) -> int:
    """Device pointer of a torch CUDA tensor (contiguous)."""
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("expected a contiguous CUDA tensor")
    return t.data_ptr()


def _stream_ptr(stream) -> c_void_p:
    if stream is None:
        import torch
        return c_void_p(torch.cuda.current_stream().cuda_stream)
    return c_void_p(getattr(stream, "cuda_stream", stream))


def version() -> str:
    return _L.welvet_version().decode()


def runtime_identity() -> str:
    return _L.welvet_runtime_identity().decode()


def cuda_init() -> None:
    check(_L.welvet_cuda_init())


def cuda_available() -> bool:
    return bool(_L.welvet_cuda_available())


# ------------------------------------------------------------------ Dense

def dense_forward_f32(W: np.ndarray, x: np.ndarray, dtype: int, act: int = LINEAR, bias=None):
    """welvet_dense_forward_f32: W [out, in] float32, x [batch, in] -> (pre, post) [batch, out]."""
    W = _f32(W)
    out, in_ = W.shape
    x = _f32(x).reshape(-1, in_)
    batch = x.shape[0]
    pre = np.zeros((batch, out), np.float32)
    post = np.zeros((batch, out), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float64)
    check(_L.welvet_dense_forward_f32(batch, in_, out, act, dtype, 0, _np_ptr(W), _np_ptr(b),
                                      0 if b is None else b.size, _np_ptr(x), _np_ptr(pre), _np_ptr(post)))
    return pre, post


def dense_normalbp_f32(W: np.ndarray, x: np.ndarray, grad_or_target: np.ndarray, dtype: int, act: int = LINEAR,
                       bias=None, use_target: bool = False, lr: float = 0.0):
    """welvet_dense_normalbp_f32 (reference src/interop/c_abi.cpp:119-184): one training step.

    W [out, in], x [batch, in], grad_or_target [batch, out] (the output gradient, or the MSE
    target when use_target). Returns (pre, post, dX, dW, W_after, loss)."""
    W = _f32(W)
    out, in_ = W.shape
    x = _f32(x).reshape(-1, in_)
    batch = x.shape[0]
    g = _f32(grad_or_target).reshape(batch, out)
    pre = np.zeros((batch, out), np.float32)
    post = np.zeros((batch, out), np.float32)
    dX = np.zeros((batch, in_), np.float32)
    dW = np.zeros((out, in_), np.float32)
    W_after = np.zeros((out, in_), np.float32)
    loss = c_double(0.0)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float64)
    check(_L.welvet_dense_normalbp_f32(batch, in_, out, act, dtype, 0, _np_ptr(W), _np_ptr(b),
                                       0 if b is None else b.size, _np_ptr(x), _np_ptr(g), int(bool(use_target)),
                                       float(lr), _np_ptr(pre), _np_ptr(post), _np_ptr(dX), _np_ptr(dW),
                                       _np_ptr(W_after), ctypes.byref(loss)))
    return pre, post, dX, dW, W_after, loss.value


class DenseSession:
    """welvet_dense_mount / execute / release (+ device-pointer extensions)."""

    def __init__(self, W, batch: int, dtype: int, act: int = LINEAR, bias=None, *, native=None, scale: float = 1.0,
                 shape=None):
        self._h = c_void_p()
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float64)
        blen = 0 if b is None else b.size
        if native is not None:
            out, in_ = shape
            raw = np.ascontiguousarray(native, dtype=np.uint8)
            check(_L.welvet_b200_dense_mount_native(batch, in_, out, act, dtype, _np_ptr(raw), raw.size, scale,
                                                    _np_ptr(b), blen, byref(self._h)))
        elif hasattr(W, "is_cuda"):
            out, in_ = W.shape
            check(_L.welvet_b200_dense_mount_device(batch, in_, out, act, dtype, c_void_p(_dev_ptr(W)), _np_ptr(b),
                                                    blen, byref(self._h)))
        else:
            W = _f32(W)
            out, in_ = W.shape
            check(_L.welvet_dense_mount(batch, in_, out, act, dtype, _np_ptr(W), _np_ptr(b), blen, byref(self._h)))
        self.batch, self.in_, self.out, self.dtype = batch, in_, out, dtype

    def execute(self, x: np.ndarray, pre: np.ndarray | None = None, post: np.ndarray | None = None):
        """welvet_dense_execute: x holds batch x in floats; pre / post (batch x out floats, written
        in place; allocated when None) receive the pre-activation and the output."""
        x = _f32(x)
        if x.size != self.batch * self.in_:
            raise ValueError(f"execute: x has {x.size} elements, the session takes {self.batch} x {self.in_}")
        n = self.batch * self.out
        pre = _out_f32(pre, n, (self.batch, self.out), "pre")
        post = _out_f32(post, n, (self.batch, self.out), "post")
        st = _L.welvet_dense_execute(self._h, _np_ptr(x), _np_ptr(pre), _np_ptr(post))
        if st.code != OK:
            raise WelvetError(st.code, st.message.decode(errors="replace"))
        return pre, post

    def execute_device(self, x, pre, post, stream=None) -> None:
        check(_L.welvet_b200_dense_execute_device(self._h, c_void_p(_dev_ptr(x)), c_void_p(_dev_ptr(pre)),
                                                  c_void_p(_dev_ptr(post)), _stream_ptr(stream)))

    def execute_device_noalloc(self, x, pre, post, stream=None) -> None:
        """execute_device for callers that cannot allocate device memory during a forward
        (allocation-free serving loops, frameworks owning all device memory):
        batched sessions only, scratch in the library's static 32 MiB device array; calls
        that overlap on one GPU race on that array."""
        check(_L.welvet_b200_dense_execute_device_noalloc(self._h, c_void_p(_dev_ptr(x)), c_void_p(_dev_ptr(pre)),
                                                          c_void_p(_dev_ptr(post)), _stream_ptr(stream)))

    def check_error(self, stream=None) -> None:
        """Synchronizes `stream` and raises (code 4) if a tensor-core pipeline wait of an earlier
        asynchronous call on this session timed out."""
        check(_L.welvet_b200_dense_check_error(self._h, _stream_ptr(stream)))

    def store(self):
        """(dtype, rows, cols, scale, native bytes in the reference layout)."""
        dt, r, c, sc, ln = c_int32(), c_int32(), c_int32(), c_float(), c_size_t()
        check(_L.welvet_b200_dense_store(self._h, byref(dt), byref(r), byref(c), byref(sc), None, 0, byref(ln)))
        buf = np.zeros(ln.value, np.uint8)
        check(_L.welvet_b200_dense_store(self._h, byref(dt), byref(r), byref(c), byref(sc), _np_ptr(buf), buf.size,
                                         byref(ln)))
        return dt.value, r.value, c.value, sc.value, buf

    def release(self) -> None:
        if self._h:
            _L.welvet_dense_release(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def dense_execute_group(sessions, xs, pres, posts, stream=None) -> None:
    """n independent forwards (device tensors) in grouped launches where the sessions share
    dtype, shape and a batch of 1..4 (welvet_b200_dense_execute_group_device)."""
    n = len(sessions)
    if not (len(xs) == len(pres) == len(posts) == n):
        raise ValueError("dense_execute_group: one x, pre and post per session")
    arr = c_void_p * n
    hs = arr(*[s._h.value for s in sessions])
    xp = arr(*[_dev_ptr(t) for t in xs])
    pp = arr(*[_dev_ptr(t) for t in pres])
    qp = arr(*[_dev_ptr(t) for t in posts])
    check(_L.welvet_b200_dense_execute_group_device(hs, n, xp, pp, qp, _stream_ptr(stream)))


# ------------------------------------------------------------------ cells

def rmsnorm_forward_f32(gamma, x, batch: int, seq: int, dim: int, eps: float = 1e-6, dtype: int = FLOAT32):
    g = _f32(gamma)
    x = _f32(x)
    pre = np.zeros(batch * seq * dim, np.float32)
    post = np.zeros_like(pre)
    check(_L.welvet_rmsnorm_forward_f32(batch, seq, dim, eps, dtype, 0, _np_ptr(g), _np_ptr(x), _np_ptr(pre),
                                        _np_ptr(post)))
    return pre, post


def swiglu_forward_f32(G, U, D, x, batch: int, seq: int, dtype: int):
    G, U, D, x = _f32(G), _f32(U), _f32(D), _f32(x)
    inter, in_ = G.shape
    pre = np.zeros(batch * seq * inter, np.float32)
    post = np.zeros(batch * seq * in_, np.float32)
    check(_L.welvet_swiglu_forward_f32(batch, seq, in_, inter, dtype, 0, _np_ptr(G), _np_ptr(U), _np_ptr(D),
                                       _np_ptr(x), _np_ptr(pre), _np_ptr(post)))
    return pre, post


def mha_forward_f32(Q, K, V, O, x, batch: int, seq: int, d_model: int, num_heads: int, num_kv_heads: int = 0,
                    head_dim: int = 0, max_seq_len: int = 0, mask: int = 1, pos: int = 0, dtype: int = FLOAT32):
    Q, K, V, O, x = _f32(Q), _f32(K), _f32(V), _f32(O), _f32(x)
    hd = head_dim if head_dim > 0 else d_model // num_heads
    q_dim = num_heads * hd
    pre = np.zeros(batch * seq * q_dim, np.float32)
    post = np.zeros(batch * seq * d_model, np.float32)
    check(_L.welvet_mha_forward_f32(batch, seq, d_model, num_heads, num_kv_heads, head_dim, max_seq_len, mask, pos,
                                    dtype, 0, _np_ptr(Q), _np_ptr(K), _np_ptr(V), _np_ptr(O), _np_ptr(x),
                                    _np_ptr(pre), _np_ptr(post)))
    return pre, post


class SwigluCell:
    """Persistent SwiGLU cell (welvet_b200_swiglu_*): weights as torch CUDA tensors or numpy."""

    def __init__(self, G, U, D, dtype: int):
        self._h = c_void_p()
        on_dev = hasattr(G, "is_cuda")
        if on_dev:
            ptrs = [c_void_p(_dev_ptr(t)) for t in (G, U, D)]
            self._keep = None
        else:
            self._keep = [_f32(t) for t in (G, U, D)]
            ptrs = [_np_ptr(t) for t in self._keep]
        inter, in_ = G.shape
        check(_L.welvet_b200_swiglu_mount(in_, inter, dtype, *ptrs, 1 if on_dev else 0, byref(self._h)))
        self._keep = None
        self.in_, self.inter = in_, inter

    def execute_device(self, x, y, h=None, stream=None) -> None:
        rows = x.shape[0]
        check(_L.welvet_b200_swiglu_execute_device(self._h, rows, c_void_p(_dev_ptr(x)),
                                                   None if h is None else c_void_p(_dev_ptr(h)),
                                                   c_void_p(_dev_ptr(y)), _stream_ptr(stream)))

    def release(self):
        if self._h:
            _L.welvet_b200_swiglu_release(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class MhaCell:
    """Persistent MHA cell (welvet_b200_mha_*)."""

    def __init__(self, Q, K, V, O, d_model: int, num_heads: int, num_kv_heads: int = 0, head_dim: int = 0,
                 max_seq_len: int = 0, mask: int = 1, pos: int = 0, dtype: int = FLOAT32):
        self._h = c_void_p()
        on_dev = hasattr(Q, "is_cuda")
        if on_dev:
            ptrs = [c_void_p(_dev_ptr(t)) for t in (Q, K, V, O)]
        else:
            keep = [_f32(t) for t in (Q, K, V, O)]
            ptrs = [_np_ptr(t) for t in keep]
        check(_L.welvet_b200_mha_mount(d_model, num_heads, num_kv_heads, head_dim, max_seq_len, mask, pos, dtype,
                                       *ptrs, 1 if on_dev else 0, byref(self._h)))

    def execute_device(self, x, batch: int, seq: int, y, attn=None, stream=None) -> None:
        check(_L.welvet_b200_mha_execute_device(self._h, batch, seq, c_void_p(_dev_ptr(x)),
                                                None if attn is None else c_void_p(_dev_ptr(attn)),
                                                c_void_p(_dev_ptr(y)), _stream_ptr(stream)))

    def release(self):
        if self._h:
            _L.welvet_b200_mha_release(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


# ------------------------------------------------------------------ model sessions


class welvet_cuda_blob(ctypes.Structure):
    _fields_ = [("data", ctypes.POINTER(c_uint8)), ("size", c_size_t)]


_sig("welvet_model_mount", _ST, c_void_p, c_size_t, POINTER(c_void_p))
_sig("welvet_model_forward", _ST, c_void_p, c_void_p, c_size_t, POINTER(welvet_cuda_blob))
_sig("welvet_model_release", None, c_void_p)
_sig("welvet_cuda_blob_free", None, POINTER(welvet_cuda_blob))


def tensor_record(x) -> bytes:
    """The reference's tensor record: int32 rank, int32 dims, float32 data (little-endian)."""
    x = np.ascontiguousarray(x, dtype="<f4")
    return np.array([x.ndim, *x.shape], dtype="<i4").tobytes() + x.tobytes()


def parse_tensor_record(b: bytes) -> np.ndarray:
    rank = int(np.frombuffer(b, dtype="<i4", count=1)[0])
    dims = np.frombuffer(b, dtype="<i4", count=rank, offset=4)
    return np.frombuffer(b, dtype="<f4", offset=4 * (1 + rank)).reshape(tuple(int(d) for d in dims)).copy()


class ModelSession:
    """welvet_model_mount / welvet_model_forward / welvet_model_release: a stored WMN1 model
    (Stack or Grid root of Dense, RMSNorm, SwiGLU and MHA children) resident on the GPU."""

    def __init__(self, descriptor: bytes):
        self._h = c_void_p()
        buf = ctypes.create_string_buffer(bytes(descriptor), len(descriptor))
        check(_L.welvet_model_mount(ctypes.addressof(buf), len(descriptor), byref(self._h)))

    def forward(self, x) -> np.ndarray:
        rec = tensor_record(x)
        buf = ctypes.create_string_buffer(rec, len(rec))
        blob = welvet_cuda_blob()
        check(_L.welvet_model_forward(self._h, ctypes.addressof(buf), len(rec), byref(blob)))
        try:
            return parse_tensor_record(ctypes.string_at(blob.data, blob.size))
        finally:
            _L.welvet_cuda_blob_free(byref(blob))

    def release(self) -> None:
        if self._h:
            _L.welvet_model_release(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


# ------------------------------------------------------------------ codecs

def codec_digest(codec: int, start: int, count: int) -> int:
    d = c_uint64()
    check(_L.welvet_b200_codec_digest(codec, start, count, byref(d)))
    return int(d.value)


def codec_selftest_decode(dtype: int) -> np.ndarray:
    out = np.zeros(512 if dtype == FP4 else 256, np.float32)
    check(_L.welvet_b200_codec_selftest_decode(dtype, _np_ptr(out)))
    return out


def codec_encode(dtype: int, w, native, scale, stream=None) -> None:
    """Device encode: w float32 CUDA tensor -> native uint8 CUDA tensor, scale float32[1] CUDA tensor."""
    check(_L.welvet_b200_codec_encode(dtype, c_void_p(_dev_ptr(w)), w.numel(), c_void_p(_dev_ptr(native)),
                                      c_void_p(_dev_ptr(scale)), _stream_ptr(stream)))


def codec_decode(dtype: int, native, n: int, scale: float, out, stream=None) -> None:
    check(_L.welvet_b200_codec_decode(dtype, c_void_p(_dev_ptr(native)), n, scale, c_void_p(_dev_ptr(out)),
                                      _stream_ptr(stream)))
