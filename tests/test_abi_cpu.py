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

    for name in ("welvet_layernorm_forward_f32", "welvet_swiglu_normalbp_f32", "welvet_model_train_mse"):
        fn = getattr(L, name)
        fn.restype = St
        fn.argtypes = []
        st = fn()
        assert st.code == 3 and st.message.startswith(b"gap?"), name
    L.welvet_gaps_count.restype = ctypes.c_int32
    L.welvet_gaps_done.restype = ctypes.c_int32
    assert L.welvet_gaps_count() + L.welvet_gaps_done() == 71
    # the gap count is the number of status-3 stubs the library defines
    src = open(os.path.join(ROOT, "welvet", "cuda_b200", "csrc", "c_abi.cpp")).read()
    assert L.welvet_gaps_count() == len(re.findall(r"^WB_GAP\(", src, re.M))
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


def test_model_descriptor_checks_without_cuda():
    """welvet_model_mount reads the WMN1 descriptor before touching the GPU: bad arguments,
    versions and layouts are status 1, model roots and child kinds off this path status 3
    (src/interop/model_session.cpp:317-396; include/welvet/interop/child_wire.hpp)."""
    import struct
    from wmn1 import dense_child, descriptor, store_f32

    L = ctypes.CDLL(LIB)

    class St(ctypes.Structure):
        _fields_ = [("code", ctypes.c_int32), ("message", ctypes.c_char * 256)]

    L.welvet_model_mount.restype = St
    L.welvet_model_mount.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]

    def mount(b):
        h = ctypes.c_void_p()
        st = L.welvet_model_mount(b, len(b), ctypes.byref(h))
        assert not h.value
        return st.code, st.message.decode()

    code, msg = mount(b"")
    assert code == 1 and "invalid mount arguments" in msg
    good = descriptor(0, [dense_child(4, 3, -1, 1, [0.5] * 12)], [store_f32(3, 4, [0.5] * 12)])
    code, msg = mount(b"XXXX" + good[4:])
    assert code == 1 and "descriptor version" in msg
    code, msg = mount(good + b"\0\0\0\0")
    assert code == 1 and "trailing" in msg
    code, msg = mount(good[:-8])
    assert code == 1
    par = bytearray(good)
    par[4:8] = struct.pack("<i", 1)  # Parallel root
    assert mount(bytes(par))[0] == 3
    ln = struct.pack("<i", 3) + struct.pack("<iid", 4, 1, 1e-5) + struct.pack("<4f", 1, 1, 1, 1) * 2
    code, msg = mount(descriptor(0, [ln], []))  # LayerNorm child
    assert code == 3 and "kind 3" in msg
    code, msg = mount(descriptor(0, [dense_child(4, 3, -1, 1, [0.5] * 12)], []))  # no stores
    assert code == 1 and "store count" in msg
