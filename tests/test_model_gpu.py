"""GPU: welvet_model_mount / welvet_model_forward over WMN1 descriptors
(src/interop/model_session.cpp:317-410).

The descriptors carry the weights as the reference's store section does: native bytes and
scale from the reference codec (the oracle's pack) or float32 values. A model session must
give bit for bit what a volume bound from the same float32 weights gives (the GPU encoders
reproduce those bytes exactly, and the same kernels run), and a Dense-only model what the
fp64 oracle gives within the GEMV bound."""
import numpy as np
import pytest

from test_dense_gpu import check_dense
from wmn1 import (dense_child, descriptor, mha_child, none_child, rmsnorm_child, store_f32, store_native,
                  swiglu_child)

pytestmark = pytest.mark.gpu

FP8E4M3, FP8E5M2, INT8, FP4, F32 = 4, 5, 9, 16, 1


@pytest.fixture(scope="module")
def V(wb):
    from welvet.cuda_b200 import volume
    return volume


def _store(oracle, dt, w, bias=()):
    if dt == F32:
        return store_f32(w.shape[0], w.shape[1], w, bias)
    raw, sc = oracle.pack(dt, w)
    return store_native(dt, w.shape[0], w.shape[1], np.asarray(raw, np.uint8).tobytes(), sc, bias)


def _mat(rng, r, c, s=0.4):
    return (rng.standard_normal((r, c)) * s).astype(np.float32)


def test_stack_matches_volume(wb, oracle, V):
    """Stack root: RMSNorm (float32 gamma) -> Dense FP4 (ReLU, bias) -> SwiGLU Int8 -> MHA E4M3
    (one sequence of 12 tokens, GQA) -> Dense E5M2."""
    rng = np.random.default_rng(3)
    rows, d0, d1, inter, nh, nkv, hd, msl, d2 = 12, 64, 96, 160, 4, 2, 24, 16, 48
    g = (1.0 + 0.1 * rng.standard_normal(d0)).astype(np.float32)
    W1 = _mat(rng, d1, d0)
    b1 = rng.standard_normal(d1 - 5)
    G, U, D = _mat(rng, inter, d1), _mat(rng, inter, d1), _mat(rng, d1, inter)
    Q, K, Vw, O = _mat(rng, nh * hd, d1, 0.2), _mat(rng, nkv * hd, d1, 0.2), _mat(rng, nkv * hd, d1, 0.2), \
        _mat(rng, d1, nh * hd, 0.2)
    W2 = _mat(rng, d2, d1)
    children = [rmsnorm_child(d0, F32, 1e-5, g), dense_child(d0, d1, 0, FP4, W1, b1),
                swiglu_child(d1, inter, INT8, G, U, D),
                mha_child(rows, d1, nh, nkv, hd, msl, 1, 0, FP8E4M3, Q, K, Vw, O),
                dense_child(d1, d2, -1, FP8E5M2, W2)]
    stores = [store_f32(1, d0, g), _store(oracle, FP4, W1, b1), _store(oracle, INT8, G), _store(oracle, INT8, U),
              _store(oracle, INT8, D), _store(oracle, FP8E4M3, Q), _store(oracle, FP8E4M3, K),
              _store(oracle, FP8E4M3, Vw), _store(oracle, FP8E4M3, O), _store(oracle, FP8E5M2, W2)]
    m = wb.ModelSession(descriptor(0, children, stores))
    x = rng.standard_normal((rows, d0)).astype(np.float32)
    y = m.forward(x)
    y2 = m.forward(x)
    m.release()
    assert y.shape == (rows, d2)
    vol = V.Volume(1, 1, 1, 5)
    vol.bind_rmsnorm(vol.coord(0), g, 1e-5, F32)
    vol.bind_dense(vol.coord(1), W1, 0, FP4, bias=b1)
    vol.bind_swiglu(vol.coord(2), G, U, D, INT8)
    vol.bind_mha(vol.coord(3), Q, K, Vw, O, d1, nh, nkv, hd, msl, 1, 0, seq=rows, dtype=FP8E4M3)
    vol.bind_dense(vol.coord(4), W2, -1, FP8E5M2)
    ref = vol.forward_f32(x, 256)
    np.testing.assert_array_equal(y, ref)
    np.testing.assert_array_equal(y2, ref)


def test_grid_remote_link_and_disabled_cell(wb, oracle, V):
    """Grid root 1x1x2x2: hop 1 disabled, hop 3 remote-linked to hop 0's output."""
    rng = np.random.default_rng(8)
    W = [_mat(rng, 64, 48), _mat(rng, 80, 64), _mat(rng, 40, 64), _mat(rng, 32, 64)]
    acts, dts = [0, 0, 2, -1], [FP4, FP4, FP8E4M3, INT8]
    children = [dense_child(w.shape[1], w.shape[0], a, dt, w) for w, a, dt in zip(W, acts, dts)]
    stores = [_store(oracle, dt, w) for w, dt in zip(W, dts)]
    cells = [(1, 0, 0, 0, 0, 0), (0, 0, 0, 0, 0, 0), (1, 0, 0, 0, 0, 0), (1, 1, 0, 0, 0, 0)]
    m = wb.ModelSession(descriptor(2, children, stores, dims=(1, 1, 2, 2), cells=cells))
    x = rng.standard_normal((5, 48)).astype(np.float32)
    y = m.forward(x)
    m.release()
    vol = V.Volume(1, 1, 2, 2)
    for h, (w, a, dt) in enumerate(zip(W, acts, dts)):
        vol.bind_dense(vol.coord(h), w, a, dt)
    vol.set_disabled(vol.coord(1))
    vol.set_remote_link(vol.coord(3), vol.coord(0))
    np.testing.assert_array_equal(y, vol.forward_f32(x, 128))
    assert y.shape == (5, 32)


def test_batched_sequences_and_shape_rules(wb, oracle, V):
    """[batch, seq, d] input: MHA takes seq from the shape; a Dense child needs [batch, in]."""
    rng = np.random.default_rng(11)
    d, nh, hd, inter, seq, batch = 64, 4, 16, 96, 4, 3
    g = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    Q, K, Vw = (_mat(rng, nh * hd, d, 0.3) for _ in range(3))
    O = _mat(rng, d, nh * hd, 0.3)
    G, U, D = _mat(rng, inter, d), _mat(rng, inter, d), _mat(rng, d, inter)
    children = [rmsnorm_child(d, FP8E4M3, 1e-6, g), mha_child(seq, d, nh, nh, hd, 16, 1, 0, FP4, Q, K, Vw, O),
                swiglu_child(d, inter, FP8E4M3, G, U, D), none_child()]
    stores = [_store(oracle, FP8E4M3, g[None, :]), _store(oracle, FP4, Q), _store(oracle, FP4, K),
              _store(oracle, FP4, Vw), _store(oracle, FP4, O), _store(oracle, FP8E4M3, G),
              _store(oracle, FP8E4M3, U), _store(oracle, FP8E4M3, D)]
    m = wb.ModelSession(descriptor(0, children, stores))
    x = rng.standard_normal((batch, seq, d)).astype(np.float32)
    y = m.forward(x)
    assert y.shape == (batch, seq, d)
    vol = V.Volume(1, 1, 1, 3)
    vol.bind_rmsnorm(vol.coord(0), g, 1e-6, FP8E4M3)
    vol.bind_mha(vol.coord(1), Q, K, Vw, O, d, nh, nh, hd, 16, 1, 0, seq=seq, dtype=FP4)
    vol.bind_swiglu(vol.coord(2), G, U, D, FP8E4M3)
    np.testing.assert_array_equal(y.reshape(batch * seq, d), vol.forward_f32(x.reshape(batch * seq, d), 128))
    m.release()
    md = wb.ModelSession(descriptor(0, [dense_child(d, 8, -1, FP4, _mat(rng, 8, d))],
                                    [_store(oracle, FP4, _mat(rng, 8, d))]))
    with pytest.raises(wb.WelvetError) as e:
        md.forward(x)
    assert e.value.code == 1 and "[batch,in]" in e.value.message
    md.release()


@pytest.mark.parametrize("dt", [FP4, FP8E4M3, INT8, F32])
def test_dense_model_vs_oracle(wb, oracle, dt):
    """A one-Dense model against the fp64 oracle of the reference kernel (GEMV bound); a
    float32 store against the library's one-shot Float32 Dense (the oracle packs quantized
    dtypes only)."""
    rng = np.random.default_rng(20 + dt)
    out, in_ = 640, 1024
    w = (rng.standard_normal((out, in_)) * 2.0).astype(np.float32)
    bias = rng.standard_normal(out)
    m = wb.ModelSession(descriptor(0, [dense_child(in_, out, 1, dt, w, bias)], [_store(oracle, dt, w, bias)]))
    x = rng.standard_normal((3, in_)).astype(np.float32)
    y = m.forward(x)
    m.release()
    if dt == F32:
        _, post = wb.dense_forward_f32(w, x, F32, 1, bias)
        np.testing.assert_array_equal(y, post)
        return
    raw, sc = oracle.pack(dt, w)
    ref = oracle.dense_forward(dt, raw, sc, x, in_, out, 1, bias)
    check_dense(ref[0], y, ref, 1, f"model dense dt={dt}")
