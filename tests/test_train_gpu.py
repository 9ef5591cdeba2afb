"""Dense training step on the GPU (welvet_dense_normalbp_f32 and the C++ API's backward_f32 /
linear_grad_in / grad_w_only / apply_grad_sgd / WeightStore::export_f32) against the oracle and
against the reference's own CUDA training step (oracle/_ref: new_layer, forward_f32,
backward_f32, apply_grad_sgd, export_f32 on its kernels, src/interop/c_abi.cpp:119-184).

Bar: on layers that take the fp64 forward (at most 2^20 weights) pre, post, dX, dW and W_after
equal the reference's bit for bit for every activation whose derivative is arithmetic (linear,
ReLU, LeakyReLU, ReLU2); SiLU / GELU / Tanh / Sigmoid go through CUDA's double exp / tanh in
both builds and are held to 1 ulp of float in d_pre's consumers (rtol 2e-7). The MSE loss is a
fixed-order tree sum here and a sequential sum in the reference: rtol 1e-12. Larger layers run
the tensor-core forward, whose pre differs from the fp64 sum by the forward's own tolerance;
there dX / dW are checked against the oracle fed with the GPU's own pre."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DTYPES = [1, 4, 5, 9, 16]
EXACT_ACTS = [-1, 0, 5, 6]
TRANSCENDENTAL_ACTS = [1, 2, 3, 4]


def _case(seed, batch, out, in_, spread=1.0):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((out, in_)) * spread).astype(np.float32)
    x = rng.standard_normal((batch, in_)).astype(np.float32)
    g = rng.standard_normal((batch, out)).astype(np.float32)
    bias = rng.standard_normal(out - 3)
    return W, x, g, bias


def _assert_same(ours, want, exact, names=("pre", "post", "dX", "dW", "W_after")):
    for name, a, b in zip(names, ours, want):
        if exact:
            np.testing.assert_array_equal(a, b, err_msg=name)
        else:
            np.testing.assert_allclose(a, b, rtol=2e-7, atol=1e-30, err_msg=name)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("act", EXACT_ACTS + TRANSCENDENTAL_ACTS)
@pytest.mark.parametrize("use_target,lr", [(False, 0.0), (True, 0.05), (False, -0.3)])
def test_normalbp_matches_reference_cuda_step(wb, oracle, dt, act, use_target, lr):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    W, x, g, bias = _case(dt * 100 + act * 7 + int(use_target), 3, 29, 41)
    ours = wb.dense_normalbp_f32(W, x, g, dt, act, bias, use_target, lr)
    ref = oracle.ref_dense_normalbp(dt, W, x, g, act, bias, use_target, lr)
    _assert_same(ours[:5], ref[:5], act in EXACT_ACTS)
    if use_target:
        assert ours[5] == pytest.approx(ref[5], rel=1e-12)
    else:
        assert ours[5] == 0.0 and ref[5] == 0.0


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", [(1, 7, 5), (17, 96, 160), (4, 1024, 1024)])
def test_normalbp_matches_oracle(wb, oracle, dt, shape):
    """Batch 1, a ragged mid size and the largest fp64-forward size, against the CPU oracle."""
    batch, out, in_ = shape
    W, x, g, bias = _case(7 + dt + batch, batch, out, in_, 2.0)
    for use_target, lr in ((True, 0.01), (False, 0.0)):
        ours = wb.dense_normalbp_f32(W, x, g, dt, 0, bias, use_target, lr)
        want = oracle.dense_normalbp(dt, W, x, g, 0, bias, use_target, lr)
        _assert_same(ours[:5], want[:5], True)
        assert ours[5] == pytest.approx(want[5], rel=1e-12)


@pytest.mark.parametrize("dt", [16, 4, 9])
def test_normalbp_tensor_forward_sizes(wb, oracle, dt):
    """A layer above 2^20 weights (tensor-core forward): dX / dW / W_after from the GPU's own
    pre are the oracle's bit for bit; pre itself is within the forward tolerance."""
    batch, out, in_ = 5, 1536, 2048
    W, x, g, bias = _case(300 + dt, batch, out, in_)
    pre, post, dX, dW, W_after, _ = wb.dense_normalbp_f32(W, x, g, dt, -1, bias, False, 0.02)
    raw, scale = oracle.store_of(dt, W)
    from test_dense_gpu import check_dense
    check_dense(pre, post, oracle.dense_forward(dt, raw, scale, x, in_, out, -1, bias), -1, "train fwd")
    _, gx_o, dW_o = oracle.dense_backward(dt, raw, scale, g, x, pre, in_, out, -1)
    np.testing.assert_array_equal(dX, gx_o)
    np.testing.assert_array_equal(dW, dW_o)
    raw2 = oracle.apply_sgd(dt, raw, scale, dW_o, 0.02)
    np.testing.assert_array_equal(W_after, oracle.decode_f32(dt, raw2, scale, out * in_).reshape(out, in_))


def test_normalbp_sgd_moves_weights_and_lowers_loss(wb):
    """Repeated steps with W_after fed back: the MSE falls (Float32 master, small lr)."""
    rng = np.random.default_rng(11)
    batch, out, in_ = 8, 16, 32
    W_true = rng.standard_normal((out, in_)).astype(np.float32)
    x = rng.standard_normal((batch, in_)).astype(np.float32)
    target = x @ W_true.T
    W = np.zeros_like(W_true)
    losses = []
    for _ in range(30):
        _, _, _, _, W, loss = wb.dense_normalbp_f32(W, x, target, 1, -1, None, True, 0.05)
        losses.append(loss)
    assert losses[-1] < 0.2 * losses[0]


@pytest.fixture(scope="module")
def caller():
    from test_cxx_api import _build
    import tempfile
    return ctypes.CDLL(_build(tempfile.mkdtemp()))


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("act", [0, 3])
def test_cxx_training_api_matches_c_abi(wb, oracle, caller, dt, act):
    """backward_f32 / apply_grad_sgd / export_f32 through the C++ API equal the C ABI's step;
    linear_grad_in equals the backward with Linear; grad_w_only equals backward_f32's dW; the
    forward after the SGD uses the updated store."""
    batch, out, in_ = 6, 48, 80
    W, x, g, _ = _case(500 + dt + act, batch, out, in_)
    lr = 0.125
    outs = {k: np.zeros(s, np.float32) for k, s in
            (("pre", (batch, out)), ("post", (batch, out)), ("dX", (batch, in_)), ("dW", (out, in_)),
             ("W_after", (out, in_)), ("gx_lin", (batch, in_)), ("dw_only", (out, in_)),
             ("post_after", (batch, out)))}
    msg = ctypes.create_string_buffer(256)
    caller.run_dense_train.restype = ctypes.c_int
    caller.run_dense_train.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 2 + \
        [ctypes.c_double] + [ctypes.c_void_p] * 8 + [ctypes.c_char_p]
    rc = caller.run_dense_train(in_, out, act, dt, _p(W), batch, _p(x), _p(g), lr, *[_p(outs[k]) for k in
                                ("pre", "post", "dX", "dW", "W_after", "gx_lin", "dw_only", "post_after")], msg)
    assert rc == 0, msg.value
    abi = wb.dense_normalbp_f32(W, x, g, dt, act, None, False, lr)
    for name, a in zip(("pre", "post", "dX", "dW", "W_after"), abi[:5]):
        np.testing.assert_array_equal(outs[name], a, err_msg=name)
    # linear_grad_in / grad_w_only ran on the updated layer: compare with the oracle there.
    raw, scale = oracle.store_of(dt, W)
    raw2 = oracle.apply_sgd(dt, raw, scale, outs["dW"], lr)
    _, gx_lin, _ = oracle.dense_backward(dt, raw2, scale, g, x, np.zeros((batch, out), np.float32), in_, out, act,
                                         linear=True)
    np.testing.assert_array_equal(outs["gx_lin"], gx_lin)
    _, _, dw_only = oracle.dense_backward(dt, raw2, scale, g, x, outs["pre"], in_, out, act)
    np.testing.assert_array_equal(outs["dw_only"], dw_only)
    _, post2, _, _ = oracle.dense_forward(dt, raw2, scale, x, in_, out, act)
    np.testing.assert_array_equal(outs["post_after"], post2)
