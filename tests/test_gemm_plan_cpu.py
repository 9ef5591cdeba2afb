"""CPU: invariants of the batched tensor-core GEMM's launch plan (welvet_b200_gemm_plan, host
arithmetic only), over shapes, x-plane counts, token-block caps and the tuning switches. Each
invariant is a limit the kernel relies on: TMEM columns, shared memory per CTA, the widths a
tcgen05 MMA takes, TMA box heights, token passes that cover a block, and a work-item count
that matches the schedule."""
import ctypes
import itertools
import os

import pytest

from conftest import ROOT

LIB = os.path.join(ROOT, "welvet", "cuda_b200", "libwelvet_b200.so")
FIELDS = ("pair TB tp1 tp2 tp3 nacc1 nacc2 nacc3 acc_cols acc_buf a_col sx sw x_bytes w_bytes smem nkb splits "
          "kb_per_split tiles_t tiles tail_first tail_s tail_kbps n_items wg").split()
FP4, E4M3, E5M2, INT8 = 16, 4, 5, 9


@pytest.fixture(scope="module")
def lib():
    L = ctypes.CDLL(LIB)
    L.welvet_b200_gemm_plan.restype = ctypes.c_int32
    L.welvet_b200_gemm_plan.argtypes = [ctypes.c_int32] * 6 + [ctypes.POINTER(ctypes.c_int64), ctypes.c_int32]
    return L


def plan(lib, M, cols, rows, xsplit, dt, max_tb=0):
    out = (ctypes.c_int64 * len(FIELDS))()
    n = lib.welvet_b200_gemm_plan(M, cols, rows, xsplit, dt, max_tb, out, len(FIELDS))
    assert n == len(FIELDS)
    return dict(zip(FIELDS, out))


def check(p, M, cols, rows, xsplit, dt):
    pair = bool(p["pair"])
    TB = p["TB"]
    assert 16 <= TB <= 256 and TB % (32 if pair else 16) == 0
    assert TB >= min(M, 16)
    cols_used = 0
    xrows = 0
    for P in range(1, xsplit + 1):
        T, nacc = p[f"tp{P}"], p[f"nacc{P}"]
        assert 16 <= T <= TB and T % (32 if pair else 16) == 0
        npass = -(-TB // T)
        assert npass * T >= TB and npass * T - TB < 16 * npass * (2 if pair else 1)  # passes of equal size
        ntot = P * T
        if pair:
            # one MMA of min(P, 2) * T columns (N a multiple of 32, at most 256); plane 2 of a
            # 3-plane stage a second MMA of T columns onto plane 1's accumulator
            n0 = min(P, 2) * T
            assert n0 <= 256 and n0 % 32 == 0
            acols = n0
            xrows = max(xrows, n0)
            assert T // 2 <= 256 and (T // 2) % 8 == 0  # TMA box of half a pass, whole 128-byte swizzle atoms
        else:
            # up to two MMAs: N0 = min(ntot, 256), N1 = ntot - 256, each a multiple of 16
            assert ntot <= 384 and ntot % 16 == 0
            if ntot > 256:
                assert (ntot - 256) % 16 == 0
            acols = ntot
            xrows = max(xrows, ntot)
            assert T <= 256 and T % 8 == 0  # TMA box height
        assert nacc >= 1 and nacc * acols <= p["acc_cols"]
        cols_used = max(cols_used, nacc * acols)
    assert p["acc_cols"] == cols_used
    buffers = 2 if p["acc_buf"] else 1
    if p["acc_buf"]:
        assert p["acc_buf"] >= p["acc_cols"] and p["a_col"] == 2 * p["acc_buf"]
    else:
        assert p["a_col"] >= p["acc_cols"]
    assert p["a_col"] % 32 == 0 and p["a_col"] + 32 * p["sx"] <= 512  # TMEM: accumulators + A stages
    assert 2 <= p["sx"] <= 8 and 2 <= p["sw"] <= 32
    assert p["x_bytes"] % 1024 == 0 and p["x_bytes"] >= xrows * (64 if pair else 128)
    assert p["wg"] in (1, 2, 4, 8)  # W stages per bulk copy
    assert p["w_bytes"] == 128 * (32 if dt == FP4 else 64) * p["wg"]
    assert p["sx"] * p["x_bytes"] + p["sw"] * p["w_bytes"] + 2048 + 32 * 1024 <= p["smem"] <= 227 * 1024
    assert p["smem"] >= 116 * 1024  # one CTA per SM
    nkb = -(-cols // 64)
    assert p["nkb"] == nkb
    sub = 2 if pair else 1
    assert p["tiles_t"] == -(-M // TB)
    assert p["tiles"] == (-(-rows // 128) // sub) * p["tiles_t"]
    if pair:
        assert (-(-rows // 128)) % 2 == 0
    assert 1 <= p["splits"] <= 8 and p["splits"] * p["kb_per_split"] >= nkb
    assert (p["splits"] - 1) * p["kb_per_split"] < nkb
    if p["tail_first"] >= 0:
        units = 74 if pair else 148
        ntail = p["tiles"] - p["tail_first"]
        assert p["splits"] == 1 and 0 < ntail <= units // 2 and p["tiles"] > units
        assert 2 <= p["tail_s"] <= 8 and p["tail_s"] * p["tail_kbps"] >= nkb
        assert (p["tail_s"] - 1) * p["tail_kbps"] < nkb  # every slice non-empty
        assert p["n_items"] == p["tail_first"] + ntail * p["tail_s"]
    else:
        assert p["n_items"] == p["tiles"] * p["splits"]
    return buffers


SHAPES = [(M, cols, rows) for M, cols, rows in itertools.product(
    (9, 16, 32, 48, 64, 100, 128, 160, 200, 256, 300, 512, 1024, 4096),
    (64, 1000, 4096, 14336),
    (128, 256, 640, 4096, 9600, 9728, 28672))]


@pytest.mark.parametrize("mode", ["default", "pair", "pairall", "dbuf192", "dbuf128", "tb128", "xslots3", "wg4"])
def test_plan_invariants(lib, mode, monkeypatch):
    for k in ("WELVET_B200_GEMM_PAIR", "WELVET_B200_GEMM_DBUF", "WELVET_B200_GEMM_TB", "WELVET_B200_GEMM_XSLOTS",
              "WELVET_B200_GEMM_WG"):
        monkeypatch.delenv(k, raising=False)
    if mode == "pair":
        monkeypatch.setenv("WELVET_B200_GEMM_PAIR", "1")
    elif mode == "pairall":
        monkeypatch.setenv("WELVET_B200_GEMM_PAIR", "all")
    elif mode.startswith("dbuf"):
        monkeypatch.setenv("WELVET_B200_GEMM_DBUF", mode[4:])
    elif mode == "tb128":
        monkeypatch.setenv("WELVET_B200_GEMM_TB", "128")
    elif mode == "xslots3":
        monkeypatch.setenv("WELVET_B200_GEMM_XSLOTS", "3")
    elif mode == "wg4":
        monkeypatch.setenv("WELVET_B200_GEMM_WG", "4")
    seen_pair = seen_dbuf = 0
    for (M, cols, rows), xsplit, dt in itertools.product(SHAPES, (1, 2, 3), (FP4, E4M3, INT8)):
        p = plan(lib, M, cols, rows, xsplit, dt)
        seen_dbuf += check(p, M, cols, rows, xsplit, dt) == 2
        seen_pair += p["pair"]
        if mode == "tb128":
            assert p["TB"] <= 128
        if mode == "xslots3":
            assert p["sx"] <= 3
        assert p["wg"] == (4 if mode == "wg4" else 1)
    if mode in ("pair", "pairall"):
        assert seen_pair > 0
    if mode.startswith("dbuf"):
        assert seen_dbuf > 0


def test_token_block_cap(lib):
    """A caller's cap (fp32 activations: blocks of 128, one pass at two planes) and the plan
    it gives the SwiGLU Down shape: 32 row tiles x 4 token blocks, no split-K."""
    p = plan(lib, 512, 14336, 4096, 2, E4M3, max_tb=128)
    assert p["TB"] == 128 and p["tp2"] == 128 and p["tiles"] == 128 and p["splits"] == 1
    assert p["n_items"] == 128
    check(p, 512, 14336, 4096, 2, E4M3)
    q = plan(lib, 512, 14336, 4096, 2, E4M3)
    assert q["TB"] == 256 and q["tp2"] == 128  # two passes of 128, not 192 + 64


def test_known_plans(lib):
    """Plans the measured numbers were taken with: 16384^2 at 256 bf16-valued tokens (one
    block, 128 tiles, 4 x stages of 32 KB, 8 W slots) and the SwiGLU Gate/Up pair shape (448
    tiles: 444 whole, the last 4 cut into 8 K slices)."""
    p = plan(lib, 256, 16384, 16384, 2, E4M3)
    assert (p["TB"], p["tiles"], p["splits"], p["sx"], p["sw"], p["x_bytes"]) == (256, 128, 1, 4, 8, 32768)
    u = plan(lib, 512, 4096, 28672, 2, E4M3)
    assert (u["tiles"], u["tail_first"], u["tail_s"], u["n_items"]) == (448, 444, 8, 444 + 4 * 8)


def test_rejects_unserved(lib):
    out = (ctypes.c_int64 * len(FIELDS))()
    assert lib.welvet_b200_gemm_plan(256, 64, 128, 2, 1, 0, out, len(FIELDS)) == -1  # Float32: no GEMM
    assert lib.welvet_b200_gemm_plan(0, 64, 128, 2, E4M3, 0, out, len(FIELDS)) == -1
    assert lib.welvet_b200_gemm_plan(256, 64, 128, 4, E4M3, 0, out, len(FIELDS)) == -1
    assert lib.welvet_b200_gemm_plan(256, 64, 128, 2, E4M3, 0, None, 0) == len(FIELDS)
