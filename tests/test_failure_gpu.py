"""Failure path of the tcgen05 GEMM's bounded waits, without a GPU fault.

Every mbarrier wait in k_gemm_tm is bounded by %globaltimer; on expiry the waiting thread
records a stage code in the launch's error word and the kernel winds down. Here each CTA of
the launch first waits 1 ms on a barrier that nothing arrives on (WELVET_B200_TEST_WAIT_TIMEOUT=1,
read per launch), before it issues any copy, allocates TMEM or touches its cluster peer: the
wait runs out, the error word reads 30, and the host reports status 4 through the session's
check_error. The context stays usable: the next call without the switch is bit-identical to a
fresh session's. (The flag exchange of the column-sharded layer has its own timeout test with an
absent rank, tests/test_multi_gpu.py.)"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", [16, 4])
def test_gemm_wait_timeout_reports_status_4_and_context_survives(wb, monkeypatch, dt):
    import torch
    rng = np.random.default_rng(70 + dt)
    rows, cols, batch = 1024, 2048, 64
    W = (rng.standard_normal((rows, cols)) * 0.5).astype(np.float32)
    x = torch.from_numpy(rng.standard_normal((batch, cols)).astype(np.float32)).cuda()
    s = wb.DenseSession(W, batch, dt)
    pre = torch.empty((batch, rows), device="cuda")
    post = torch.empty((batch, rows), device="cuda")
    s.execute_device(x, pre, post)
    s.check_error()
    want = post.cpu().numpy().copy()

    monkeypatch.setenv("WELVET_B200_TEST_WAIT_TIMEOUT", "1")
    post.fill_(0)
    s.execute_device(x, pre, post)
    with pytest.raises(wb.WelvetError) as e:
        s.check_error()
    assert e.value.code == 4 and "stage code 30" in str(e.value)
    monkeypatch.delenv("WELVET_B200_TEST_WAIT_TIMEOUT")

    s.execute_device(x, pre, post)
    s.check_error()  # the error word was cleared by the report
    np.testing.assert_array_equal(post.cpu().numpy(), want)
    torch.cuda.synchronize()
