"""The reference's C++ layer API over libwelvet_b200: dense::forward_f32, swiglu::forward and
mha::forward with the reference's types (include/welvet/*.hpp of this repository).

CPU: tests/cxx/api_caller.cpp, written against the reference's signatures, compiles against
include/ and links against the library (every symbol it calls is exported). GPU: the same
caller, called through ctypes, matches the library's C ABI one-shot forwards bit for bit and
the fp64 oracle within the Dense tolerance; a weight change with invalidate_gpu() and a batch
change remount lazily, as in the reference (src/layers/dense/dense.cpp:78-80)."""
import ctypes
import os
import subprocess
import tempfile

import numpy as np
import pytest

from conftest import ROOT

LIBDIR = os.path.join(ROOT, "welvet", "cuda_b200")
SRC = os.path.join(ROOT, "tests", "cxx", "api_caller.cpp")


def _build(out_dir: str) -> str:
    so = os.path.join(out_dir, "libapi_caller.so")
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-I", os.path.join(ROOT, "include"), SRC,
                    "-L", LIBDIR, "-lwelvet_b200", f"-Wl,-rpath,{LIBDIR}", "-Wl,--no-undefined", "-o", so],
                   check=True, capture_output=True, text=True)
    return so


def test_caller_compiles_and_links_against_the_library():
    with tempfile.TemporaryDirectory() as d:
        so = _build(d)
        assert os.path.exists(so)
        ctypes.CDLL(so)  # loads without a GPU: nothing runs at load time


@pytest.fixture(scope="module")
def caller():
    d = tempfile.mkdtemp()
    lib = ctypes.CDLL(_build(d))
    return lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [16, 4, 9])
def test_dense_forward_f32_matches_c_abi_and_oracle(wb, oracle, caller, dt):
    from test_dense_gpu import check_dense
    rng = np.random.default_rng(60 + dt)
    out, in_ = 1024, 1536
    W1 = (rng.standard_normal((out, in_)) * 2).astype(np.float32)
    W2 = (rng.standard_normal((out, in_)) * 2).astype(np.float32)
    bias = rng.standard_normal(out - 9)
    x1 = rng.standard_normal((1, in_)).astype(np.float32)
    x2 = rng.standard_normal((24, in_)).astype(np.float32)
    pre1, post1 = np.zeros((1, out), np.float32), np.zeros((1, out), np.float32)
    pre2, post2 = np.zeros((24, out), np.float32), np.zeros((24, out), np.float32)
    msg = ctypes.create_string_buffer(256)
    rc = caller.run_dense(in_, out, wb.RELU, dt, _p(W1), _p(W2), _p(bias), bias.size, 1, _p(x1), 24, _p(x2),
                          _p(pre1), _p(post1), _p(pre2), _p(post2), msg)
    assert rc == 0, msg.value
    for W, x, pre, post in ((W1, x1, pre1, post1), (W2, x2, pre2, post2)):
        raw, sc = oracle.pack(dt, W)
        check_dense(pre, post, oracle.dense_forward(dt, raw, sc, x, in_, out, wb.RELU, bias), wb.RELU, f"C++ dt={dt}")
        p_c, q_c = wb.dense_forward_f32(W, x, dt, wb.RELU, bias)
        assert np.array_equal(pre, p_c.reshape(pre.shape)) and np.array_equal(post, q_c.reshape(post.shape))


@pytest.mark.gpu
@pytest.mark.parametrize("batch,seq", [(1, 1), (2, 12)])
def test_swiglu_forward_matches_c_abi(wb, caller, batch, seq):
    rng = np.random.default_rng(70 + batch)
    d, inter, dt = 256, 640, 4
    G, U, D = [(rng.standard_normal(s) * 0.5).astype(np.float32) for s in ((inter, d), (inter, d), (d, inter))]
    x = rng.standard_normal((batch * seq, d)).astype(np.float32)
    pre = np.zeros((batch * seq, inter), np.float32)
    post = np.zeros((batch * seq, d), np.float32)
    msg = ctypes.create_string_buffer(256)
    rc = caller.run_swiglu(batch, seq, d, inter, dt, _p(G), _p(U), _p(D), _p(x), _p(pre), _p(post), msg)
    assert rc == 0, msg.value
    p_c, q_c = wb.swiglu_forward_f32(G, U, D, x, batch, seq, dt)
    assert np.array_equal(pre, p_c.reshape(pre.shape)) and np.array_equal(post, q_c.reshape(post.shape))


@pytest.mark.gpu
def test_mha_forward_matches_c_abi(wb, caller):
    rng = np.random.default_rng(80)
    batch, seq, d, nh, nkv, hd, msl, dt = 2, 16, 64, 4, 2, 16, 16, 16
    Q = (rng.standard_normal((nh * hd, d)) * 0.3).astype(np.float32)
    K, V = [(rng.standard_normal((nkv * hd, d)) * 0.3).astype(np.float32) for _ in range(2)]
    O = (rng.standard_normal((d, nh * hd)) * 0.3).astype(np.float32)
    x = rng.standard_normal((batch * seq, d)).astype(np.float32)
    pre = np.zeros((batch * seq, nh * hd), np.float32)
    post = np.zeros((batch * seq, d), np.float32)
    msg = ctypes.create_string_buffer(256)
    rc = caller.run_mha(batch, seq, d, nh, nkv, hd, msl, dt, _p(Q), _p(K), _p(V), _p(O), _p(x), _p(pre), _p(post), msg)
    assert rc == 0, msg.value
    p_c, q_c = wb.mha_forward_f32(Q, K, V, O, x, batch, seq, d, nh, nkv, hd, msl, 1, 0, dt)
    assert np.array_equal(pre, p_c.reshape(pre.shape)) and np.array_equal(post, q_c.reshape(post.shape))
