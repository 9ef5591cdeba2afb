"""GPU: the opt-in (WELVET_B200_GEMV16=1) tensor GEMV for 9..16 tokens (x prepared once per K segment, two row groups per
warp, the launch's token count rounded up to 12 or 16) and the SwiGLU cell's opt-in 5..16-row form
(Gate and Up as two such GEMVs, the reference's product, Down), against the fp64 oracle within
the GEMV bound (2^-18 * sum |W x| + 2 ulp). Shapes cover ragged rows and K, more row sets than
SMs, several K segments per row set (clusters), every quantized dtype, bias / activation,
and a K too long for the GEMV at 16 tokens (which then runs the tcgen05 GEMM)."""
import numpy as np
import pytest

from test_dense_gpu import TOL_REL, _case, check_dense, ulp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [9, 12, 13, 16])
@pytest.mark.parametrize("dt", [16, 4, 5, 9])
@pytest.mark.parametrize("shape", [(300, 1000), (4096, 4096), (1100, 7000)])
def test_gemv_9_to_16_tokens(wb, oracle, dt, shape, batch, monkeypatch):
    monkeypatch.setenv("WELVET_B200_EXACT", "0")
    monkeypatch.setenv("WELVET_B200_GEMV16", "1")
    out, in_ = shape
    w, x, bias, ref = _case(oracle, dt, out, in_, batch, 2.0, out + in_ + batch + dt, 2, True, out - 5)
    pre, post = wb.dense_forward_f32(w, x, dt, 2, bias)
    check_dense(pre, post, ref, 2, f"gemv16 dt={dt} shape={shape} batch={batch}")


def test_gemv16_matches_gemm_fallback_for_long_k(wb, oracle, monkeypatch):
    """At 16 tokens a K of 65536 FP4 is too long for the GEMV's shared memory; the session runs
    the tcgen05 GEMM, still within the bound."""
    monkeypatch.setenv("WELVET_B200_EXACT", "0")
    monkeypatch.setenv("WELVET_B200_GEMV16", "1")
    w, x, bias, ref = _case(oracle, 16, 256, 65536, 16, 2.0, 77, -1, False)
    pre, post = wb.dense_forward_f32(w, x, 16, -1, None)
    err = np.abs(pre.astype(np.float64) - ref[0]) - 2 * ulp(ref[0])
    assert float(np.max(err / np.maximum(ref[3], 1e-300))) <= 2.0 ** -15


def test_gemv16_equals_repeated_8_token_launches_in_tolerance(wb, oracle, monkeypatch):
    """16 tokens in one launch vs the same tokens through the 8-token GEMV in two halves: both
    within the bound of the oracle (the K segments differ, so sums differ in order only)."""
    monkeypatch.setenv("WELVET_B200_EXACT", "0")
    monkeypatch.setenv("WELVET_B200_GEMV16", "1")
    dt, out, in_ = 4, 2048, 3072
    w, x, bias, ref = _case(oracle, dt, out, in_, 16, 2.0, 5, -1, False)
    pre16, _ = wb.dense_forward_f32(w, x, dt, -1, None)
    pa, _ = wb.dense_forward_f32(w, x[:8], dt, -1, None)
    pb, _ = wb.dense_forward_f32(w, x[8:], dt, -1, None)
    for got in (pre16, np.concatenate([pa, pb])):
        check_dense(got, got, ref, -1, "16 vs 2 x 8 tokens")


@pytest.mark.parametrize("rows", [5, 8, 12, 16])
@pytest.mark.parametrize("dt", [16, 4])
def test_swiglu_5_to_16_rows(wb, oracle, dt, rows, monkeypatch):
    monkeypatch.setenv("WELVET_B200_EXACT", "0")
    monkeypatch.setenv("WELVET_B200_GEMV16", "1")
    rng = np.random.default_rng(200 + rows)
    d, inter = 1024, 2816
    G, U, D = [(rng.standard_normal(s) * 0.5).astype(np.float32) for s in ((inter, d), (inter, d), (d, inter))]
    x = rng.standard_normal((rows, d)).astype(np.float32)
    pre, post = wb.swiglu_forward_f32(G, U, D, x, rows, 1, dt)
    rg, sg = oracle.pack(dt, G)
    ru, su = oracle.pack(dt, U)
    rd, sd = oracle.pack(dt, D)
    gp, _, _, gsa = oracle.dense_forward(dt, rg, sg, x, d, inter)
    _, upp, _, usa = oracle.dense_forward(dt, ru, su, x, d, inter)
    h = oracle.swiglu_product(gp, upp)
    hb = 1.1 * TOL_REL * gsa * np.abs(upp) + TOL_REL * usa * np.abs(h / np.where(upp == 0, 1, upp)) + 4 * ulp(h)
    assert np.all(np.abs(pre.reshape(h.shape) - h) <= hb + 1e-30)
    ref = oracle.dense_forward(dt, rd, sd, pre.reshape(h.shape), inter, d)
    check_dense(post, post, ref, -1, f"swiglu rows={rows} dt={dt}")
