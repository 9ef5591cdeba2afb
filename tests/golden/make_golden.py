"""Generate tests/golden/ fixtures from the welvet.cuda reference itself.

Run in a container where the reference tree exists (oracle/Makefile builds
oracle/_ref/libwelvet_ref.so from its sources):

    python tests/golden/make_golden.py

Every value written here comes from the reference's own code (src/core/float_codecs.cpp,
src/weights/store.cpp + native_codec.cpp), never from the oracle restatement:

  codec_tables.json   decode of every E4M3 / E5M2 byte and every FP4 code (float32 bits)
  codec_kat.json      encode of edge-case and seeded random float32 bit patterns
  encode_digests.json for each encoder, 256 digests covering all 2^32 float32 patterns
                      (chunk c = patterns [c*2^24, (c+1)*2^24); digest definition in oracle.c)
  packs.npz           seeded weight matrices with the reference's native bytes, scale and
                      decode_row_f64 output, per dtype and shape (incl. odd shapes, zeros)

The random inputs use numpy's PCG64 (np.random.default_rng(seed)); the inputs are stored
in the fixtures, so tests never regenerate them.
"""
from __future__ import annotations

import json
import os
import struct
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
import oracle as O  # noqa: E402

CHUNK_BITS = 24


def f2b(f: float) -> int:
    return struct.unpack("<I", struct.pack("<f", f))[0]


def b2f(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b & 0xFFFFFFFF))[0]


def edge_inputs() -> list[int]:
    vals = [0.0, -0.0, float("inf"), float("-inf"), 1.0, -1.0, 0.01, 0.003, 0.0015, 1.0625, 240.0,
            248.0, 250.0, 256.0, 300.0, 448.0, 464.0, 500.0, 1.125, 60000.0, 57344.0, 61440.0,
            65536.0, 1e-5, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, 7.0, 100.0,
            2.0 ** -6, 2.0 ** -7, 2.0 ** -9, 2.0 ** -10, 2.0 ** -14, 2.0 ** -16, 2.0 ** -17,
            1.4375, 1.46875, 3e38, -3e38, 6.0, 5.9999, 4.9999, 5.0001, 67108864.0, 67108858.0,
            1e30, -1e30, 16777216.0, 2.0 ** 26 + 8]
    bits = [f2b(v) for v in vals]
    bits += [0x7FC00000, 0xFFC00000, 0x7F800001, 0x00000001, 0x80000001, 0x007FFFFF, 0x00800000,
             0x7F7FFFFF, 0xFF7FFFFF]
    # every mantissa-rounding boundary around the FP8 grids, both signs
    for e in range(-20, 20):
        for m in range(8):
            base = (1.0 + m / 8.0) * 2.0 ** e
            for d in (-1, 0, 1):
                b = f2b(base) + d
                bits += [b, b | 0x80000000]
            mid = (1.0 + (m + 0.5) / 8.0) * 2.0 ** e
            for d in (-1, 0, 1):
                b = f2b(mid) + d
                bits += [b, b | 0x80000000]
    # FP4 decision midpoints
    grid = [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    for a, b in zip(grid, grid[1:]):
        m = (a + b) / 2
        for d in (-1, 0, 1):
            x = f2b(m) + d
            bits += [x, x | 0x80000000]
    return sorted(set(b & 0xFFFFFFFF for b in bits))


def main() -> None:
    O.build()
    if not O.ref_available():
        raise SystemExit("reference build missing: oracle/_ref/libwelvet_ref.so")
    R = O.ref()

    # 1. decode tables
    tables = {
        "e4m3": [f2b(R.ref_e4m3_decode(b)) for b in range(256)],
        "e5m2": [f2b(R.ref_e5m2_decode(b)) for b in range(256)],
        "fp4": [f2b(R.ref_fp4_decode(b)) for b in range(16)],
    }
    with open(os.path.join(HERE, "codec_tables.json"), "w") as f:
        json.dump(tables, f, indent=0)

    # 2. encode KATs
    rng = np.random.default_rng(20261201)
    ins = edge_inputs() + [int(v) for v in rng.integers(0, 2 ** 32, size=4000, dtype=np.uint64)]
    kat = []
    for b in ins:
        x = b2f(b)
        kat.append([b, R.ref_e4m3_encode(x), R.ref_e5m2_encode(x), R.ref_fp4_encode(x)])
    with open(os.path.join(HERE, "codec_kat.json"), "w") as f:
        json.dump({"columns": ["f32_bits", "e4m3", "e5m2", "fp4"], "rows": kat}, f)

    # 3. exhaustive encode digests
    t0 = time.time()
    dig = {"chunk_bits": CHUNK_BITS, "codecs": ["e4m3", "e5m2", "fp4"], "digests": []}
    n = 1 << CHUNK_BITS
    for codec in range(3):
        row = [format(O.ref_encode_digest(codec, c * n, n), "016x") for c in range(1 << (32 - CHUNK_BITS))]
        dig["digests"].append(row)
        print(f"codec {codec} digests done at {time.time() - t0:.1f}s", flush=True)
    with open(os.path.join(HERE, "encode_digests.json"), "w") as f:
        json.dump(dig, f, indent=0)

    # 4. seeded packs through the reference WeightStore
    cases = []
    # (name, dtype, rows, cols, sigma, seed)
    cases.append(("c1_e4m3", O.FP8E4M3, 128, 256, 0.05, 0))
    for dt, nm in ((O.FP8E4M3, "e4m3"), (O.FP8E5M2, "e5m2"), (O.FP4, "fp4"), (O.INT8, "int8")):
        cases.append((f"{nm}_64x96_s2", dt, 64, 96, 2.0, 11))
        cases.append((f"{nm}_7x13_s2", dt, 7, 13, 2.0, 12))
        cases.append((f"{nm}_33x130_s002", dt, 33, 130, 0.02, 13))
        cases.append((f"{nm}_1x1_s2", dt, 1, 1, 2.0, 14))
    arrays = {}
    for name, dt, rows, cols, sigma, seed in cases:
        r = np.random.default_rng(seed)
        w = (r.standard_normal(rows * cols) * sigma).astype(np.float32)
        raw, sc = O.ref_pack(dt, w, rows, cols)
        dec = O.ref_decode(dt, raw, sc, rows, cols)
        arrays[f"{name}.w"] = w
        arrays[f"{name}.raw"] = raw
        arrays[f"{name}.meta"] = np.array([dt, rows, cols, f2b(sc)], dtype=np.int64)
        arrays[f"{name}.dec"] = dec
    # special matrices: zeros (Int8 scale 0 -> 1), specials (NaN / Inf / huge)
    specials = np.array([0.0, -0.0, np.nan, np.inf, -np.inf, 1e30, -1e30, 448.0, 500.0, 6.0, -6.0,
                         2.0 ** -10, -(2.0 ** -10), 57344.0, 1e-8, 3.0], dtype=np.float32)
    for dt, nm in ((O.FP8E4M3, "e4m3"), (O.FP8E5M2, "e5m2"), (O.FP4, "fp4"), (O.INT8, "int8")):
        for tag, w in (("zeros_4x8", np.zeros(32, np.float32)), ("specials_2x8", specials),
                       ("finite_specials_2x6", specials[[0, 1, 7, 8, 9, 10, 11, 12, 13, 14, 15, 5]])):
            rows = int(tag.split("_")[-1].split("x")[0])
            cols = w.size // rows
            raw, sc = O.ref_pack(dt, w, rows, cols)
            name = f"{nm}_{tag}"
            arrays[f"{name}.w"] = w
            arrays[f"{name}.raw"] = raw
            arrays[f"{name}.meta"] = np.array([dt, rows, cols, f2b(sc)], dtype=np.int64)
            arrays[f"{name}.dec"] = O.ref_decode(dt, raw, sc, rows, cols)
    np.savez_compressed(os.path.join(HERE, "packs.npz"), **arrays)

    # 5. the reference's exported C-ABI names (include/welvet_c.h), for the link-compatibility test
    import re
    ref_root = os.environ.get("REF", os.path.join(HERE, "..", "..", "..", "reference"))  # checkout beside the repo
    with open(os.path.join(ref_root, "include", "welvet_c.h")) as f:
        names = sorted(set(re.findall(r"\b(welvet_[a-z0-9_]+)\(", f.read())))
    with open(os.path.join(HERE, "reference_symbols.txt"), "w") as f:
        f.write("\n".join(names) + "\n")
    print("golden fixtures written", flush=True)


if __name__ == "__main__":
    main()
