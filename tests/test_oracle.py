"""CPU: pin the oracle (oracle/oracle.c) against the reference's own codec.

Golden fixtures in tests/golden/ were produced by the reference compiled from its sources
(tests/golden/make_golden.py); where oracle/_ref is present the oracle is also compared
with the reference live.
"""
import json
import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN, pack_cases


def f32bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def b2f(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


def test_decode_tables_match_reference(oracle):
    t = json.load(open(os.path.join(GOLDEN, "codec_tables.json")))
    L = oracle.lib()
    assert [f32bits(L.or_e4m3_decode(b)) for b in range(256)] == t["e4m3"]
    assert [f32bits(L.or_e5m2_decode(b)) for b in range(256)] == t["e5m2"]
    assert [f32bits(L.or_fp4_decode(b)) for b in range(16)] == t["fp4"]


def test_decode_quirks(oracle):
    """Facts about the reference decode the GPU mirror must reproduce."""
    L = oracle.lib()
    for b in range(1, 8):  # E4M3 / E5M2 subnormal codes decode to signed zero
        assert f32bits(L.or_e4m3_decode(b)) == 0 and f32bits(L.or_e4m3_decode(0x80 | b)) == 0x80000000
    for b in range(1, 4):
        assert f32bits(L.or_e5m2_decode(b)) == 0 and f32bits(L.or_e5m2_decode(0x80 | b)) == 0x80000000
    assert L.or_e4m3_decode(0x7F) == 448.0 and L.or_e4m3_decode(0xFF) == -448.0
    assert np.isinf(L.or_e5m2_decode(0x7C)) and np.isnan(L.or_e5m2_decode(0x7D))


def test_encode_kats(oracle):
    kat = json.load(open(os.path.join(GOLDEN, "codec_kat.json")))
    L = oracle.lib()
    bad = []
    for bits, e4, e5, f4 in kat["rows"]:
        x = b2f(bits)
        got = (L.or_e4m3_encode(x), L.or_e5m2_encode(x), L.or_fp4_encode(x))
        if got != (e4, e5, f4):
            bad.append((hex(bits), got, (e4, e5, f4)))
    assert not bad, bad[:10]


def test_codec_edge_cases(oracle):
    """Hand-checked reference probe values (E4M3 half-up and saturation, FP4 ties)."""
    L = oracle.lib()
    assert L.or_e4m3_encode(0.01) == 0x05 and L.or_e4m3_encode(1.0625) == 0x39
    assert L.or_e4m3_encode(240.0) == 0x77
    for v in (250.0, 256.0, 300.0, 500.0, float("inf")):
        assert L.or_e4m3_encode(v) == 0x7E
    assert L.or_e4m3_encode(float("nan")) == 0x00
    assert L.or_e5m2_encode(1.125) == 0x3D and L.or_e5m2_encode(60000.0) == 0x7B
    assert L.or_e5m2_encode(float("nan")) == 0x7E and L.or_e5m2_encode(-0.0) == 0x80
    assert [L.or_fp4_encode(v) for v in (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, 7.0, 100.0)] == \
        [0, 1, 2, 3, 4, 5, 6, 0, 9, 7, 7]
    assert L.or_fp4_encode(float("nan")) == 0 and L.or_fp4_encode(float("inf")) == 0
    assert L.or_fp4_encode(1e30) == 0  # f - v rounds to f for every table value


@pytest.mark.slow
def test_exhaustive_encode_digests(oracle):
    """All 2^32 float32 inputs through each oracle encoder == the reference's digests."""
    d = json.load(open(os.path.join(GOLDEN, "encode_digests.json")))
    n = 1 << d["chunk_bits"]
    for codec, row in enumerate(d["digests"]):
        got = [format(oracle.encode_digest(codec, c * n, n), "016x") for c in range(len(row))]
        mism = [c for c in range(len(row)) if got[c] != row[c]]
        assert not mism, f"codec {codec} chunks {mism[:8]}"


def test_packs_match_reference(oracle, packs):
    for name, dt, rows, cols, scale, w, raw, dec in pack_cases(packs):
        got, sc = oracle.pack(dt, w)
        assert np.array_equal(got, raw), name
        assert np.float32(sc).view(np.uint32) == np.float32(scale).view(np.uint32), name
        d = oracle.decode(dt, raw, scale, rows * cols)
        assert np.array_equal(d.view(np.uint64), dec.ravel().view(np.uint64)) or \
            np.array_equal(np.nan_to_num(d), np.nan_to_num(dec.ravel())), name


def test_dense_oracle_semantics(oracle):
    """The oracle's forward equals a plain fp64 restatement (kernels.cu:130-161)."""
    rng = np.random.default_rng(5)
    out, in_, batch = 17, 45, 3
    w = (rng.standard_normal((out, in_)) * 2).astype(np.float32)
    raw, sc = oracle.pack(oracle.FP8E4M3, w)
    W64 = oracle.decode(oracle.FP8E4M3, raw, sc, out * in_).reshape(out, in_)
    x = rng.standard_normal((batch, in_)).astype(np.float32)
    bias = rng.standard_normal(out - 5)  # shorter than out: rows >= bias_len get no bias
    pre, post, y64, sabs = oracle.dense_forward(oracle.FP8E4M3, raw, sc, x, in_, out, oracle.ACT_GELU, bias)
    for b in range(batch):
        for o in range(out):
            s = 0.0
            for k in range(in_):
                s += W64[o, k] * float(x[b, k])
            assert y64[b, o] == s
            p = np.float32(s)
            v = float(p)
            if o < bias.size:
                v += bias[o]
                p = np.float32(v)
            assert pre[b, o] == p
            g = 0.5 * v * (1.0 + np.tanh(0.7978845608028654 * (v + 0.044715 * v * v * v)))
            assert abs(float(post[b, o]) - g) <= 2e-7 * max(1.0, abs(g))


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="reference build absent")
def test_oracle_vs_reference_live(oracle):
    """Random matrices of every dtype: oracle pack/decode == reference WeightStore."""
    rng = np.random.default_rng(99)
    for dt in oracle.QUANT_DTYPES:
        for rows, cols, sigma in ((5, 31, 0.02), (16, 64, 2.0), (3, 7, 300.0)):
            w = (rng.standard_normal(rows * cols) * sigma).astype(np.float32)
            raw_r, sc_r = oracle.ref_pack(dt, w, rows, cols)
            raw_o, sc_o = oracle.pack(dt, w)
            assert np.array_equal(raw_r, raw_o) and sc_r == sc_o
            dec_r = oracle.ref_decode(dt, raw_r, sc_r, rows, cols)
            assert np.array_equal(dec_r.ravel(), oracle.decode(dt, raw_o, sc_o, rows * cols))


@pytest.mark.parametrize("cfg", [
    dict(batch=2, seq=6, nh=4, nkv=2, hd=8, msl=8, mask=1, pos=0),   # ring wraps across batches
    dict(batch=1, seq=5, nh=3, nkv=3, hd=8, msl=16, mask=2, pos=2),  # bidirectional + ALiBi
    dict(batch=3, seq=4, nh=2, nkv=1, hd=16, msl=4, mask=1, pos=3),  # RoPE + ALiBi, GQA, msl == seq
    dict(batch=3, seq=5, nh=2, nkv=2, hd=4, msl=7, mask=1, pos=0),   # msl not a multiple of seq
])
def test_attention_rows_matches_the_loop_restatement(cfg):
    """oracle.attention.attention_rows (numpy, selected query rows: the config-size checks) gives
    the same floats as the sequential-loop restatement of the reference attention core."""
    from oracle.attention import attention, attention_rows
    rng = np.random.default_rng(12)
    c = cfg
    T = c["batch"] * c["seq"]
    q = rng.standard_normal((T, c["nh"] * c["hd"])).astype(np.float32)
    k = rng.standard_normal((T, c["nkv"] * c["hd"])).astype(np.float32)
    v = rng.standard_normal((T, c["nkv"] * c["hd"])).astype(np.float32)
    args = (c["batch"], c["seq"], c["nh"], c["nkv"], c["hd"], c["msl"], c["mask"], c["pos"])
    full = attention(q, k, v, *args)
    rows = [0, T // 2, T - 1]
    got = attention_rows(q[rows], k, v, rows, *args)
    np.testing.assert_allclose(got, full[rows], rtol=1e-6, atol=1e-7)
