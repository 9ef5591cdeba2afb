"""Dense training step (welvet_dense_normalbp_f32) on the CPU side: the oracle's SGD against
the reference's own WeightStore::apply_sgd (oracle/_ref), its backward and MSE against direct
numpy statements of the reference's formulas, and the C ABI's argument checks (which run
before any device work, so they need no GPU).

Reference: src/interop/c_abi.cpp:119-184 (the step), src/cuda/kernels.cu:48-128 (act', W^T,
outer), src/weights/native_codec.cpp:1080-1133 (SGD), src/runtime/training.cpp:44-69 (MSE)."""
import ctypes

import numpy as np
import pytest

DTYPES = [1, 4, 5, 9, 16]


def _w(rng, out, in_, spread=1.0):
    return (rng.standard_normal((out, in_)) * spread).astype(np.float32)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("lr", [0.05, 1e-3, -0.7])
def test_oracle_sgd_matches_reference_store(oracle, dt, lr):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(dt * 31 + int(abs(lr) * 1000))
    out, in_ = 37, 53  # odd element count: the FP4 tail nibble
    W = _w(rng, out, in_, 2.0)
    raw, scale = oracle.store_of(dt, W)
    dW = (rng.standard_normal((out, in_)) * 3).astype(np.float32)
    ours = oracle.apply_sgd(dt, raw, scale, dW, lr)
    ref = oracle.ref_store_apply_sgd(dt, raw, scale, out, in_, dW, lr)
    np.testing.assert_array_equal(ours, ref)


@pytest.mark.parametrize("dt", [9])
def test_oracle_sgd_int8_scale_zero_reads_as_one(oracle, dt):
    """weight_at / set_weight_at treat a zero scale as 1 (native_codec.cpp:513-568)."""
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(5)
    raw = rng.integers(0, 256, 64, dtype=np.uint8)
    dW = rng.standard_normal(64).astype(np.float32) * 40
    np.testing.assert_array_equal(oracle.apply_sgd(dt, raw, 0.0, dW, 0.1),
                                  oracle.ref_store_apply_sgd(dt, raw, 0.0, 8, 8, dW, 0.1))


def _act_deriv(act, x):
    x = x.astype(np.float64)
    if act == -1:
        return np.ones_like(x)
    if act == 0:
        return (x > 0).astype(np.float64)
    if act == 6:
        return np.where(x > 0, 2 * x, 0.0)
    if act == 5:
        return np.where(x > 0, 1.0, 0.01)
    if act == 1:
        s = 1 / (1 + np.exp(-x))
        return s * (1 + x * (1 - s))
    if act == 2:
        k = 0.7978845608028654
        th = np.tanh(k * (x + 0.044715 * x ** 3))
        return 0.5 * (1 + th) + 0.5 * x * (1 - th * th) * k * (1 + 3 * 0.044715 * x * x)
    if act == 3:
        return 1 - np.tanh(x) ** 2
    if act == 4:
        s = 1 / (1 + np.exp(-x))
        return s * (1 - s)
    raise ValueError(act)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("act", [-1, 0, 1, 2, 3, 4, 5, 6])
def test_oracle_backward_matches_formula(oracle, dt, act):
    """d_pre = float(gy * act'(pre)); gx = float(sum_o W[o,i] d_pre); dW accumulated over the
    batch as acc = float(double(acc) + d_pre * x) (kernels.cu:83-128)."""
    rng = np.random.default_rng(100 + dt * 8 + act)
    batch, out, in_ = 3, 29, 41
    W = _w(rng, out, in_)
    raw, scale = oracle.store_of(dt, W)
    x = rng.standard_normal((batch, in_)).astype(np.float32)
    pre = rng.standard_normal((batch, out)).astype(np.float32)
    gy = rng.standard_normal((batch, out)).astype(np.float32)
    d_pre, gx, dW = oracle.dense_backward(dt, raw, scale, gy, x, pre, in_, out, act)
    Wd = oracle.decode_f32(dt, raw, scale, out * in_).reshape(out, in_).astype(np.float64)
    want_dpre = (gy.astype(np.float64) * _act_deriv(act, pre)).astype(np.float32)
    np.testing.assert_allclose(d_pre, want_dpre, rtol=1e-12, atol=0)
    want_gx = (d_pre.astype(np.float64) @ Wd).astype(np.float32)
    np.testing.assert_allclose(gx, want_gx, rtol=1e-5, atol=1e-6)
    want_dw = np.zeros((out, in_), np.float32)
    for b in range(batch):
        prod = np.outer(d_pre[b].astype(np.float64), x[b].astype(np.float64))
        want_dw = (want_dw.astype(np.float64) + prod).astype(np.float32)
    np.testing.assert_array_equal(dW, want_dw)


def test_oracle_linear_flag_skips_derivative(oracle):
    rng = np.random.default_rng(9)
    W = _w(rng, 16, 24)
    raw, scale = oracle.store_of(4, W)
    x = rng.standard_normal((2, 24)).astype(np.float32)
    pre = rng.standard_normal((2, 16)).astype(np.float32)
    gy = rng.standard_normal((2, 16)).astype(np.float32)
    d_pre, gx, _ = oracle.dense_backward(4, raw, scale, gy, x, pre, 24, 16, 0, linear=True)
    np.testing.assert_array_equal(d_pre, gy)
    d_lin, gx_lin, _ = oracle.dense_backward(4, raw, scale, gy, x, pre, 24, 16, -1)
    np.testing.assert_array_equal(gx, gx_lin)


def test_oracle_mse_matches_formula(oracle):
    rng = np.random.default_rng(3)
    p = rng.standard_normal((5, 7)).astype(np.float32)
    t = rng.standard_normal((5, 7)).astype(np.float32)
    loss, g = oracle.mse(p, t)
    d = p.astype(np.float64) - t.astype(np.float64)
    assert loss == pytest.approx(float(np.sum(d * d) / d.size), rel=1e-14)
    np.testing.assert_array_equal(g, (2.0 / d.size * d).astype(np.float32))


@pytest.fixture(scope="module")
def L():
    import welvet.cuda_b200 as W
    return W


def test_normalbp_argument_checks(L):
    """The reference's checks and codes (c_abi.cpp:125-138) come before any device work."""
    W = np.zeros((4, 3), np.float32)
    x = np.zeros((2, 3), np.float32)
    g = np.zeros((2, 4), np.float32)
    with pytest.raises(L.WelvetError) as e:
        L.dense_normalbp_f32(W, x, g, 40)
    assert e.value.code == 1 and "bad dtype 40" in str(e.value)
    with pytest.raises(L.WelvetError) as e:
        L.dense_normalbp_f32(W, x, g, -1)
    assert e.value.code == 1
    with pytest.raises(L.WelvetError) as e:
        L.dense_normalbp_f32(W, x, g, 0)  # Float64: off the GPU path
    assert e.value.code == 2
    lib = L.lib()
    st = lib.welvet_dense_normalbp_f32(0, 3, 4, -1, 4, 0, None, None, 0, None, None, 0, 0.0, None, None, None,
                                       None, None, None)
    assert st.code == 1 and st.message == b"invalid argument"
