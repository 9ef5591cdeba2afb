"""GPU: the device-resident volume forward (src/runtime/forward.cpp:98-156) against the oracle.

Every hop is checked on its own: the oracle's Dense forward (fp64, reference order) is applied
to the GPU's own input of that hop -- read back through a hop range ending there -- so the
tolerance is the single-layer one, independent of depth."""
import numpy as np
import pytest

from test_dense_gpu import check_dense

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def V(wb):
    from welvet.cuda_b200 import volume
    return volume


def _torch():
    import torch
    return torch


def _hop_output(vol, x, hop_end, width):
    torch = _torch()
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((x.shape[0], width), dtype=torch.float32, device="cuda")
    ow = vol.forward_device(xd, out, 0, hop_end)
    torch.cuda.synchronize()
    assert ow == width
    return out.cpu().numpy()


@pytest.mark.parametrize("dt", [4, 5, 9, 16])
def test_dense_chain_each_hop(wb, oracle, V, dt):
    rng = np.random.default_rng(10 + dt)
    widths = [96, 128, 64, 160, 96]
    acts = [0, 2, -1, 5]
    vol = V.Volume(2, 1, 1, 2)
    layers = []
    for h in range(4):
        w = (rng.standard_normal((widths[h + 1], widths[h])) * 0.4).astype(np.float32)
        bias = rng.standard_normal(widths[h + 1] - 3)
        vol.bind_dense(vol.coord(h), w, acts[h], dt, bias=bias)
        raw, sc = oracle.pack(dt, w)
        layers.append((raw, sc, w.shape, bias))
    rows = 5
    x = rng.standard_normal((rows, widths[0])).astype(np.float32)
    cur = x
    for h in range(4):
        got = _hop_output(vol, x, h + 1, widths[h + 1])
        raw, sc, (out, in_), bias = layers[h]
        ref = oracle.dense_forward(dt, raw, sc, cur, in_, out, acts[h], bias)
        check_dense(_pre_of(vol, h, rows, out), got, ref, acts[h], f"dt={dt} hop {h}")
        cur = got
    full = vol.forward_f32(x, 256)
    np.testing.assert_array_equal(full, cur)


def _pre_of(vol, h, rows, width):
    """The cell's recorded pre, read from its device buffer."""
    torch = _torch()
    pre_ptr, pw, _, _ = vol.cell_outputs(vol.coord(h))
    assert pw == width and pre_ptr

    class _View:
        __cuda_array_interface__ = {"shape": (rows, width), "typestr": "<f4", "data": (pre_ptr, False),
                                    "version": 2, "strides": None}

    torch.cuda.synchronize()
    return torch.as_tensor(_View(), device="cuda").cpu().numpy()


def test_remote_link_and_disabled_cells(wb, oracle, V):
    """Hop order 0,1,2,3: cell 2 disabled, cell 3 remote-linked to cell 0's post."""
    rng = np.random.default_rng(21)
    dt = oracle.FP4
    vol = V.Volume(1, 1, 1, 4)
    W = [(rng.standard_normal(s) * 0.5).astype(np.float32) for s in ((64, 48), (80, 64), (33, 80), (40, 64))]
    for h, w in enumerate(W):
        vol.bind_dense(vol.coord(h), w, 0, dt)
    vol.set_disabled(vol.coord(2))
    vol.set_remote_link(vol.coord(3), vol.coord(0))
    x = rng.standard_normal((3, 48)).astype(np.float32)
    y = vol.forward_f32(x, 128)
    assert y.shape == (3, 40)
    r0, s0 = oracle.pack(dt, W[0])
    r3, s3 = oracle.pack(dt, W[3])
    h0 = _hop_output(vol, x, 1, 64)
    ref0 = oracle.dense_forward(dt, r0, s0, x, 48, 64, 0)
    check_dense(_pre_of(vol, 0, 3, 64), h0, ref0, 0, "hop 0")
    ref3 = oracle.dense_forward(dt, r3, s3, h0, 64, 40, 0)
    check_dense(_pre_of(vol, 3, 3, 40), y, ref3, 0, "remote hop")


def test_errors(wb, oracle, V):
    rng = np.random.default_rng(5)
    vol = V.Volume(1, 1, 1, 3)
    w = rng.standard_normal((32, 32)).astype(np.float32)
    x = rng.standard_normal((2, 32)).astype(np.float32)
    vol.bind_dense(vol.coord(0), w, 0, oracle.FP8E4M3)
    with pytest.raises(wb.WelvetError) as e:  # enabled cell with no op
        vol.forward_f32(x, 64)
    assert e.value.code == wb.INVALID and "no op at" in str(e.value)
    vol.set_disabled(vol.coord(1))
    vol.set_disabled(vol.coord(2))
    assert vol.forward_f32(x, 64).shape == (2, 32)
    with pytest.raises(wb.WelvetError) as e:  # width mismatch
        vol.forward_f32(rng.standard_normal((2, 31)).astype(np.float32), 64)
    assert e.value.code == wb.INVALID and "width mismatch" in str(e.value)
    vol.set_disabled(vol.coord(0))
    with pytest.raises(wb.WelvetError) as e:
        vol.forward_f32(x, 64)
    assert "no enabled cells" in str(e.value)
    # remote link to a cell later in hop order has no recorded activation in this forward
    vol.set_disabled(vol.coord(0), False)
    vol.set_disabled(vol.coord(2), False)
    vol.bind_dense(vol.coord(2), w, 0, oracle.FP4)
    vol.set_remote_link(vol.coord(0), vol.coord(2))
    with pytest.raises(wb.WelvetError) as e:
        vol.forward_f32(x, 64)
    assert "no recorded activation" in str(e.value)
    with pytest.raises(wb.WelvetError) as e:
        vol.set_remote_link(vol.coord(0), (0, 0, 0, 7))
    assert e.value.code == wb.INVALID
    with pytest.raises(wb.WelvetError) as e:
        vol.bind_dense((0, 0, 1, 0), w, 0, oracle.FP4)
    assert e.value.code == wb.INVALID
    with pytest.raises(wb.WelvetError) as e:
        vol.bind_dense(vol.coord(1), w, 0, 2)
    assert e.value.code == wb.UNSUPPORTED


def test_mixed_cells_match_one_shot_entry_points(wb, oracle, V):
    """RMSNorm -> SwiGLU -> MHA -> Dense in one volume equals the chain of the library's
    one-shot entry points (each checked against the oracle in test_dense_gpu.py)."""
    rng = np.random.default_rng(33)
    batch, seq, d, inter, nh, hd = 2, 4, 64, 96, 4, 16
    dt = oracle.FP8E4M3
    g = rng.standard_normal(d).astype(np.float32)
    G, U = [(rng.standard_normal((inter, d)) * 0.3).astype(np.float32) for _ in range(2)]
    D = (rng.standard_normal((d, inter)) * 0.3).astype(np.float32)
    Q, K, Vw = [(rng.standard_normal((nh * hd, d)) * 0.3).astype(np.float32) for _ in range(3)]
    O = (rng.standard_normal((d, nh * hd)) * 0.3).astype(np.float32)
    Wd = (rng.standard_normal((48, d)) * 0.3).astype(np.float32)
    vol = V.Volume(1, 2, 2, 1)
    vol.bind_rmsnorm((0, 0, 0, 0), g, 1e-6, wb.FLOAT32)
    vol.bind_swiglu((0, 0, 1, 0), G, U, D, dt)
    vol.bind_mha((0, 1, 0, 0), Q, K, Vw, O, d, nh, nh, hd, 16, 1, 0, seq=seq, dtype=dt)
    vol.bind_dense((0, 1, 1, 0), Wd, 2, dt)
    x = rng.standard_normal((batch * seq, d)).astype(np.float32)
    y = vol.forward_f32(x, 64)
    # each stage against the one-shot entry point applied to the volume's own input of that stage
    stages = [_hop_output(vol, x, h + 1, w) for h, w in enumerate((d, d, d, 48))]
    _, a = wb.rmsnorm_forward_f32(g, x, batch, seq, d, 1e-6, wb.FLOAT32)
    _, b = wb.swiglu_forward_f32(G, U, D, stages[0], batch, seq, dt)
    _, c = wb.mha_forward_f32(Q, K, Vw, O, stages[1], batch, seq, d, nh, nh, hd, 16, 1, 0, dt)
    _, e = wb.dense_forward_f32(Wd, stages[2], dt, 2)
    for name, got, ref in (("rmsnorm", stages[0], a), ("swiglu", stages[1], b), ("mha", stages[2], c),
                           ("dense", stages[3], e)):
        ref = ref.reshape(got.shape)
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6 * np.abs(ref).max(), err_msg=name)
    np.testing.assert_array_equal(y, stages[3])
    y2 = vol.forward_f32(x, 64)
    np.testing.assert_array_equal(y, y2)


def _kernel_names(fn):
    """Names of the CUDA kernels launched while fn runs (torch's CUPTI-based profiler)."""
    from torch.profiler import ProfilerActivity, profile
    torch = _torch()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type.name == "CUDA"]


@pytest.mark.parametrize("kind,d", [("dense", 1024), ("dense", 1002), ("swiglu", 1024), ("mha", 1024)])
def test_rmsnorm_prologue(wb, oracle, V, kind, d, monkeypatch):
    """An RMSNorm cell followed by a projection cell runs inside that cell's tcgen05 GEMM launch
    (the x-split kernel normalises, writes the norm's pre / post and splits post): no k_rmsnorm
    launch, and every recorded output bit-identical to the norm as its own kernel
    (WELVET_B200_NORM_PROLOGUE=0). d = 1002 makes rows that start off 16-byte boundaries and a
    ragged last 4-element chunk. The norm against the fp64 formula (src/cuda/kernels.cu:172-204)
    and the Dense against the oracle on the GPU's normalised rows."""
    torch = _torch()
    rng = np.random.default_rng(77 + d)
    T, dt = 48, oracle.FP8E4M3
    g = rng.standard_normal(d).astype(np.float32)
    x = (rng.standard_normal((T, d)) * 3.0).astype(np.float32)
    vol = V.Volume(1, 1, 1, 2)
    vol.bind_rmsnorm((0, 0, 0, 0), g, 1e-6, wb.FLOAT32)
    if kind == "dense":
        W = (rng.standard_normal((1536, d)) * 0.05).astype(np.float32)
        bias = rng.standard_normal(1536) * 0.1
        vol.bind_dense((0, 0, 0, 1), W, 2, dt, bias)
        width = 1536
    elif kind == "swiglu":
        G, U = [(rng.standard_normal((1536, d)) * 0.05).astype(np.float32) for _ in range(2)]
        D = (rng.standard_normal((d, 1536)) * 0.05).astype(np.float32)
        vol.bind_swiglu((0, 0, 0, 1), G, U, D, dt)
        width = d
    else:
        # 16 heads x 128: Q is 2048 x d, above 2^20 weights, so on the tcgen05 GEMM
        Q, K, Vw = [(rng.standard_normal((2048, d)) * 0.05).astype(np.float32) for _ in range(3)]
        O = (rng.standard_normal((d, 2048)) * 0.05).astype(np.float32)
        vol.bind_mha((0, 0, 0, 1), Q, K, Vw, O, d, 16, 16, 128, 16, 1, 0, seq=16, dtype=dt)
        width = d
    xd = torch.from_numpy(x).cuda()

    def run():
        out = torch.empty((T, width), dtype=torch.float32, device="cuda")
        vol.forward_device(xd, out)
        torch.cuda.synchronize()
        rec = [out.cpu().numpy()]
        for h in range(2):
            pre, pw, post, ow = vol.cell_outputs(vol.coord(h))
            rec.append(V.device_tensor(pre, (T, pw)).cpu().numpy())
            rec.append(V.device_tensor(post, (T, ow)).cpu().numpy())
        return rec

    fused = run()
    names = _kernel_names(lambda: vol.forward_device(xd, torch.empty((T, width), device="cuda")))
    if names:  # the profiler saw kernels: the norm ran inside the GEMM launch
        assert not any("k_rmsnorm" in n for n in names), names
        assert any("k_split_x" in n for n in names), names
    monkeypatch.setenv("WELVET_B200_NORM_PROLOGUE", "0")
    alone = run()
    if names:
        names0 = _kernel_names(lambda: vol.forward_device(xd, torch.empty((T, width), device="cuda")))
        assert any("k_rmsnorm" in n for n in names0), names0
    for a, b, what in zip(fused, alone, ("out", "norm pre", "norm post", "cell pre", "cell post")):
        np.testing.assert_array_equal(a, b, err_msg=what)
    xx = x.astype(np.float64)
    inv = 1.0 / np.sqrt((xx * xx).sum(1, keepdims=True) / d + 1e-6)
    np.testing.assert_allclose(fused[1], (xx * inv).astype(np.float32), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(fused[2], (xx * inv * g.astype(np.float64)).astype(np.float32), rtol=1e-6,
                               atol=1e-7)
    if kind == "dense":
        raw, sc = oracle.pack(dt, W)
        ref = oracle.dense_forward(dt, raw, sc, fused[2], d, 1536, 2, bias)
        check_dense(fused[3], fused[4], ref, 2, f"dense after the norm, d={d}")
    vol.release()
