"""GPU: the allocation-free forward (welvet_b200_dense_execute_device_noalloc).

It is for callers that may not allocate device memory while a forward runs -- a serving loop
that must not stall on cudaMalloc, a framework or plugin host that owns all device memory --
and keeps the batched tensor-core kernel's scratch in a static device array instead. Checked
through the C ABI against the allocating entry point on the same session, two calls in a row
(the second one reuses the array's leftover contents): both run the same kernel with the same
launch plan, so the results must be identical bit for bit; the fp64 oracle checks both.
Runs alone in a fresh process or after the other tests.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_REL = 2.0 ** -16  # the tcgen05 path's bound for 3 x planes, as in test_dense_gpu.py


def test_noalloc_matches_allocating_entry_point(wb, oracle, monkeypatch):
    import torch
    monkeypatch.setenv("WELVET_B200_EXACT", "0")
    monkeypatch.setenv("WELVET_B200_XSPLIT", "3")
    rng = np.random.default_rng(7)
    out, in_, batch = 1024, 1536, 24
    for dt in (16, 4):
        w = (rng.standard_normal((out, in_)) * 2.0).astype(np.float32)
        bias = rng.standard_normal(out) * 0.1
        s = wb.DenseSession(w, batch, dt, wb.RELU, bias)
        raw, sc = oracle.pack(dt, w)
        for call in range(2):
            x = rng.standard_normal((batch, in_)).astype(np.float32)
            xd = torch.from_numpy(x).cuda()
            pre_a = torch.zeros(batch, out, device="cuda")
            post_a = torch.zeros(batch, out, device="cuda")
            pre_b = torch.full((batch, out), float("nan"), device="cuda")
            post_b = torch.full((batch, out), float("nan"), device="cuda")
            s.execute_device(xd, pre_a, post_a)
            s.execute_device_noalloc(xd, pre_b, post_b)
            s.check_error()  # no pipeline wait timed out in either call
            pa, pb = pre_a.cpu().numpy(), pre_b.cpu().numpy()
            assert np.array_equal(pb, pa), f"dt={dt} call={call}: pre differs from the allocating path"
            assert np.array_equal(post_b.cpu().numpy(), post_a.cpu().numpy()), f"dt={dt} call={call}: post"
            pre_o, post_o, y64, sabs = oracle.dense_forward(dt, raw, sc, x, in_, out, wb.RELU, bias)
            bound = TOL_REL * sabs + 2 * np.spacing(np.abs(pre_o)).astype(np.float64)
            assert np.all(np.abs(pb.astype(np.float64) - pre_o) <= bound), f"dt={dt} call={call}"
        s.release()


def test_noalloc_rejects_what_it_cannot_serve(wb, monkeypatch):
    import torch
    s = wb.DenseSession(np.ones((8, 8), np.float32), 1, wb.FP4)  # batch 1: not the batched path
    x = torch.ones(1, 8, device="cuda")
    y = torch.zeros(1, 8, device="cuda")
    with pytest.raises(wb.WelvetError) as e:
        s.execute_device_noalloc(x, y, y)
    assert e.value.code == wb.UNSUPPORTED
    s.release()
    # A call whose scratch exceeds the static array is refused with status 1. With 1024 tokens
    # of 16384 inputs the x planes alone take 32 MiB at one plane, so the call is too large
    # for the 32 MiB array at every plane setting; the setting is pinned all the same.
    monkeypatch.setenv("WELVET_B200_XSPLIT", "3")
    batch, in_, out = 1024, 16384, 256
    w = torch.randn(out, in_, device="cuda") * 0.02
    big = wb.DenseSession(w, batch, wb.FP4)
    del w
    xb = torch.randn(batch, in_, device="cuda")
    yb = torch.zeros(batch, out, device="cuda")
    with pytest.raises(wb.WelvetError) as e:
        big.execute_device_noalloc(xb, yb, yb)
    assert e.value.code == wb.INVALID and "static array" in e.value.message
    big.release()
