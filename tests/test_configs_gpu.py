"""GPU: BASELINE.json's configs 3, 4 and 5 at their own sizes and seeds, through the library's
C ABI, against the fp64 oracle (oracle/: the reference decode and its sequential fp64 dot,
test infrastructure only).

The GPU always runs the whole config (every token, every row); where the oracle would take
minutes on the host it checks sampled tokens or rows, and a stage is checked on the GPU's own
input of that stage (so that the check of layer i does not depend on layers before it).
FP4 weights drawn with sigma = 0.02 all encode to code 0 (the reference FP4 codec has no scale),
so those configs are also run on a companion whose codes are not all zero (sigma 2.0 for one
layer; 0.1 for the 32-layer volume, whose activations would overflow float32 at sigma 2.0
through 32 layers with ReLU).

Tolerances: tensor GEMV and GEMM outputs within 2^-18 * sum_k |W x| + 2 ulp of the oracle
(check_dense); SwiGLU h as test_swiglu_tensor_paths; attention rtol 1e-4 (its fp64 inputs
differ from the oracle's by the projections' rounding).
"""
import numpy as np
import pytest

from test_dense_gpu import TOL_REL, check_dense, ulp

pytestmark = pytest.mark.gpu

E4M3, FP4 = 4, 16


def _randn(shape, seed, sigma):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(shape, device="cuda", generator=g) * sigma


def _h_bound(gsa, usa, upp, h):
    return 1.1 * TOL_REL * gsa * np.abs(upp) + TOL_REL * usa * np.abs(h / np.where(upp == 0, 1, upp)) + 4 * ulp(h)


def _check_swiglu(oracle, dt, packs, x, h_gpu, y_gpu, d, inter, what):
    (rg, sg), (ru, su), (rd, sd) = packs
    gp, _, _, gsa = oracle.dense_forward(dt, rg, sg, x, d, inter)
    _, upp, _, usa = oracle.dense_forward(dt, ru, su, x, d, inter)
    h = oracle.swiglu_product(gp, upp)
    hb = _h_bound(gsa, usa, upp, h)
    bad = ~(np.abs(h_gpu - h) <= hb + 1e-30)
    assert not bad.any(), f"{what}: h outside tolerance at {np.argwhere(bad)[:4]}"
    ref = oracle.dense_forward(dt, rd, sd, h_gpu, inter, d)
    check_dense(y_gpu, y_gpu, ref, -1, f"{what}: Down")


@pytest.fixture(scope="module")
def c3():
    """Config 3's SwiGLU cell: d 4096, hidden 14336, FP8 E4M3, W ~ N(0, 0.02), seed 2."""
    import oracle as O
    import welvet.cuda_b200 as W
    d, hid = 4096, 14336
    ws = [_randn((hid, d), 2000, 0.02), _randn((hid, d), 2001, 0.02), _randn((d, hid), 2002, 0.02)]
    cell = W.SwigluCell(ws[0], ws[1], ws[2], E4M3)
    packs = [O.pack(E4M3, w.cpu().numpy()) for w in ws]
    del ws
    yield cell, packs, d, hid
    cell.release()


@pytest.mark.parametrize("M", [1, 16, 128, 512])
def test_c3_swiglu_config(wb, oracle, c3, M):
    """Config 3 at M = 1 (fused Gate/Up tensor GEMV), 16, 128 and 512 tokens (tcgen05 GEMMs):
    all tokens checked at M <= 16, 16 evenly spaced tokens above."""
    import torch
    cell, packs, d, hid = c3
    x = _randn((M, d), 2 + M, 1.0).to(torch.bfloat16).float()
    y = torch.empty((M, d), device="cuda")
    h = torch.empty((M, hid), device="cuda")
    cell.execute_device(x, y, h)
    torch.cuda.synchronize()
    toks = np.arange(M) if M <= 16 else np.linspace(0, M - 1, 16).astype(np.int64)
    xs = x.cpu().numpy()[toks]
    _check_swiglu(oracle, E4M3, packs, xs, h.cpu().numpy()[toks], y.cpu().numpy()[toks], d, hid, f"C3 M={M}")


def test_c4_transformer_cell_config(wb, oracle, V):
    """Config 4: RMSNorm(2048, gamma 1, eps 1e-6) -> MHA(d 2048, 16 x 128, causal, RoPE 1e4,
    max_seq_len 512, E4M3) -> SwiGLU(2048 / 5632, FP4) on batch 4 x seq 512 tokens of N(0, 1),
    seed 3, as one volume; then the SwiGLU rebound with sigma-2 FP4 weights (the companion).
    Sampled query rows of batches 0 and 3 (the KV ring holds each batch's own 512 rows)."""
    import torch
    from oracle.attention import attention_rows
    B, S, d, nh, hd, inter = 4, 512, 2048, 16, 128, 5632
    T = B * S
    x = _randn((T, d), 3, 1.0)
    vol = V.Volume(1, 1, 1, 3)
    gamma = np.ones(d, np.float32)
    vol.bind_rmsnorm((0, 0, 0, 0), gamma, 1e-6, wb.FLOAT32)
    Q, K, Vw, O = [_randn((d, d), 3100 + i, 0.02) for i in range(4)]
    vol.bind_mha((0, 0, 0, 1), Q, K, Vw, O, d, nh, nh, hd, S, 1, 0, seq=S, dtype=E4M3)
    packs_qkvo = [oracle.pack(E4M3, t.cpu().numpy()) for t in (Q, K, Vw, O)]
    del Q, K, Vw, O
    rows = np.array([0, 1, 255, 511, 1536, 1800, 2047])
    for sigma in (0.02, 2.0):
        G, U, D = _randn((inter, d), 3200, sigma), _randn((inter, d), 3201, sigma), _randn((d, inter), 3202, sigma)
        vol.bind_swiglu((0, 0, 0, 2), G, U, D, FP4)
        packs_sw = [oracle.pack(FP4, t.cpu().numpy()) for t in (G, U, D)]
        del G, U, D
        out = torch.empty((T, d), device="cuda")
        vol.forward_device(x, out)
        torch.cuda.synchronize()
        st = []
        for hop in range(3):
            pre, pw, post, ow = vol.cell_outputs(vol.coord(hop))
            st.append((V.device_tensor(pre, (T, pw)).cpu().numpy(), V.device_tensor(post, (T, ow)).cpu().numpy()))
        # RMSNorm (src/cuda/kernels.cu:172-204): x / rms in fp64, then gamma
        xx = x.cpu().numpy().astype(np.float64)
        inv = 1.0 / np.sqrt((xx * xx).sum(1, keepdims=True) / d + 1e-6)
        np.testing.assert_allclose(st[0][1], (xx * inv).astype(np.float32), rtol=1e-6, atol=1e-7)
        xn = st[0][1]
        if sigma == 0.02:
            # MHA on the GPU's normalised rows: Q of the sampled rows, K / V of their batches
            (rq, sq), (rk, sk), (rv, sv), (ro, so) = packs_qkvo
            q = oracle.dense_forward(E4M3, rq, sq, xn[rows], d, d)[1]
            kk = np.zeros((T, d), np.float32)
            vv = np.zeros((T, d), np.float32)
            for b in sorted({int(r) // S for r in rows}):
                sl = slice(b * S, (b + 1) * S)
                kk[sl] = oracle.dense_forward(E4M3, rk, sk, xn[sl], d, d)[1]
                vv[sl] = oracle.dense_forward(E4M3, rv, sv, xn[sl], d, d)[1]
            att = attention_rows(q, kk, vv, rows, B, S, nh, nh, hd, S, 1, 0)
            got = st[1][0][rows]
            np.testing.assert_allclose(got, att, rtol=1e-4, atol=1e-5 * np.abs(att).max())
            ref = oracle.dense_forward(E4M3, ro, so, got, d, d)
            check_dense(st[1][1][rows], st[1][1][rows], ref, -1, "C4 MHA output projection")
        # SwiGLU on the GPU's MHA output rows
        _check_swiglu(oracle, FP4, packs_sw, st[1][1][rows], st[2][0][rows], st[2][1][rows], d, inter,
                      f"C4 SwiGLU sigma={sigma}")
        if sigma == 0.02:
            assert not np.any(st[2][0]), "sigma-0.02 FP4 codes all decode to 0: h must be 0"
    vol.release()


@pytest.mark.parametrize("sigma", [0.02, 0.1])
def test_c5_volume_config(wb, oracle, V, sigma):
    """Config 5's volume: 2 x 2 x 2 cells x 4 Dense 4096 x 4096 FP4 + ReLU, batch 64, seed 4,
    on one GPU; every layer checked on 8 tokens against the oracle applied to the GPU's own
    input of that layer."""
    import torch
    cells, lpc, width, batch = 8, 4, 4096, 64
    vol = V.Volume(2, 2, 2, lpc)
    packs = []
    for h in range(cells * lpc):
        w = _randn((width, width), 4000 + h, sigma)
        vol.bind_dense(vol.coord(h), w, wb.RELU, FP4)
        packs.append(oracle.pack(FP4, w.cpu().numpy()))
        del w
    x = _randn((batch, width), 4, 1.0)
    y = torch.empty((batch, width), device="cuda")
    vol.forward_device(x, y)
    torch.cuda.synchronize()
    toks = np.arange(0, batch, 8)
    prev = x.cpu().numpy()[toks]
    for h in range(cells * lpc):
        pre, _, post, _ = vol.cell_outputs(vol.coord(h))
        got_pre = V.device_tensor(pre, (batch, width)).cpu().numpy()[toks]
        got_post = V.device_tensor(post, (batch, width)).cpu().numpy()[toks]
        raw, sc = packs[h]
        ref = oracle.dense_forward(FP4, raw, sc, prev, width, width, wb.RELU)
        check_dense(got_pre, got_post, ref, wb.RELU, f"C5 volume hop {h} sigma={sigma}")
        prev = got_post
    assert np.array_equal(y.cpu().numpy()[toks], prev)
    if sigma == 0.02:
        assert not np.any(prev)
    else:
        assert np.isfinite(prev).all() and np.any(prev)
    vol.release()


@pytest.mark.parametrize("sigma", [0.02, 2.0])
def test_c5_sharded_layer_config_one_gpu(wb, oracle, V, sigma):
    """Config 5's column-sharded Dense 16384 -> 65536 FP4 at batch 1 and 256 through the
    sharded entry points on a one-rank communicator (the same call that bench.py times at
    1..8 GPUs); 512 sampled output rows checked on every token."""
    import torch
    rows_out, cols = 65536, 16384
    comm = V.Comm(0, 1, torch.cuda.current_device(), V.Comm.new_job_id())
    w = _randn((rows_out, cols), 4100, sigma)
    sample = np.sort(np.random.default_rng(4).choice(rows_out, 512, replace=False))
    raw, sc = oracle.pack(FP4, w[torch.from_numpy(sample).cuda()].cpu().numpy())
    for batch in (1, 256):
        s = V.ShardedDense(comm, w, cols, rows_out, batch, FP4)
        assert s.rows == (0, rows_out)
        x = _randn((batch, cols), 4 + batch, 1.0)
        post, pre = s.execute_device(x)
        s.check_error()
        got = post.cpu().numpy()[:, sample]
        ref = oracle.dense_forward(FP4, raw, sc, x.cpu().numpy(), cols, len(sample))
        check_dense(got, got, ref, -1, f"C5 sharded layer batch={batch} sigma={sigma}")
        assert torch.equal(pre, post)  # Linear without bias: pre is post
        s.release()
    del w
    comm.release()


@pytest.fixture(scope="module")
def V():
    import welvet.cuda_b200 as W
    from welvet.cuda_b200 import volume
    W.cuda_init()
    return volume
