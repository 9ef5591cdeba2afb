"""CPU: the C-ABI library loads and exports every symbol include/*.h declares, and every
symbol of the reference ABI (so a reference-built program links unchanged). No compute
calls: this container has no GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import GOLDEN, ROOT

LIB = os.path.join(ROOT, "welvet", "cuda_b200", "libwelvet_b200.so")


def exported() -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], check=True, capture_output=True, text=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def declared() -> set[str]:
    names = set()
    for h in ("welvet_c.h", "welvet_b200.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        names |= set(re.findall(r"WELVET_API[^;(]*?\b(welvet_[a-z0-9_]+)\s*\(", src, re.S))
    return names


def test_library_built():
    assert os.path.exists(LIB), "build with make -C welvet/cuda_b200/csrc"
    ctypes.CDLL(LIB)


def test_exports_every_declared_symbol():
    d = declared()
    assert len(d) >= 30
    missing = d - exported()
    assert not missing, sorted(missing)


def test_exports_every_reference_symbol():
    ref = set(open(os.path.join(GOLDEN, "reference_symbols.txt")).read().split())
    assert len(ref) == 71
    missing = ref - exported()
    assert not missing, sorted(missing)


def test_out_of_scope_entry_points_return_gap():
    """Reference symbols off the quantized forward path answer status 3, without CUDA."""
    L = ctypes.CDLL(LIB)

    class St(ctypes.Structure):
        _fields_ = [("code", ctypes.c_int32), ("message", ctypes.c_char * 256)]

    for name in ("welvet_layernorm_forward_f32", "welvet_dense_normalbp_f32", "welvet_model_mount"):
        fn = getattr(L, name)
        fn.restype = St
        fn.argtypes = []
        st = fn()
        assert st.code == 3 and st.message.startswith(b"gap?"), name
    L.welvet_gaps_count.restype = ctypes.c_int32
    L.welvet_gaps_done.restype = ctypes.c_int32
    assert L.welvet_gaps_count() + L.welvet_gaps_done() == 71
    L.welvet_version.restype = ctypes.c_char_p
    assert L.welvet_version() == b"0.79"


def test_no_gpu_is_reported_not_faked():
    """Without a GPU the library reports unavailability; it has no host fallback."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    L = ctypes.CDLL(LIB)
    L.welvet_cuda_available.restype = ctypes.c_int32
    assert L.welvet_cuda_available() == 0
