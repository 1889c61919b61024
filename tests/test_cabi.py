"""The C ABI library on a host without a GPU: it loads, exports every entry
point include/neon_cuda.h declares, and the reference-mirroring argument checks
of the Python surface raise the reference's errors before touching a device."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import neon_cuda as N
from conftest import ROOT


def header_functions():
    text = open(os.path.join(ROOT, "include", "neon_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(neon_cuda_\w+)\s*\(", text)))


def test_library_builds_and_loads():
    L = N.load()
    assert L.neon_cuda_version().decode().count(".") == 2


def test_exports_every_declared_symbol():
    L = N.load()
    declared = header_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/neon_cuda.h but not exported"
    assert sorted(N.C_ENTRY_POINTS) == declared
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (neon_cuda_\w+)", out)))
    assert exported == declared, "exported C symbols differ from the header"


def test_python_binding_types_every_argument():
    """ctypes passes an untyped argument as a C int: a pointer or size_t would
    be cut to 32 bits. Every entry point that takes arguments has argtypes."""
    text = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", "neon_cuda.h")).read(), flags=re.S)
    L = N.load()
    for name, params in re.findall(r"\b(neon_cuda_\w+)\s*\(([^)]*)\)", text):
        if params.strip() in ("", "void"):
            continue
        assert getattr(L, name).argtypes is not None, f"{name}: no argtypes in neon_cuda.py"


def test_no_gpu_host_calls_fail_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    L = N.load()
    n = ctypes.c_int(-1)
    assert L.neon_cuda_device_count(ctypes.byref(n)) == 0 and n.value == 0
    h = ctypes.c_void_p()
    raw = np.zeros(18, np.uint8)
    rc = L.neon_cuda_upload(raw.ctypes.data, 2, 1, 32, 0, 0, 1, ctypes.byref(h))
    assert rc != 0 and L.neon_cuda_last_error()


def test_upload_argument_checks_precede_device_use():
    L = N.load()
    h = ctypes.c_void_p()
    raw = np.zeros(64, np.uint8)
    assert L.neon_cuda_upload(raw.ctypes.data, 2, 1, 31, 0, 0, 1, ctypes.byref(h)) == -1
    assert b"multiple of its quant block size" in L.neon_cuda_last_error()
    # types the reference does not dequantise either (Q8_1, Q2_K, Q3_K, IQ4_NL)
    for t in (9, 10, 11, 25):
        assert L.neon_cuda_upload(raw.ctypes.data, t, 1, 256, 0, 0, 1, ctypes.byref(h)) == -2
    # K-quants: 256-value super-blocks; float types: any input dim passes the check
    assert L.neon_cuda_upload(raw.ctypes.data, 12, 1, 96, 0, 0, 1, ctypes.byref(h)) == -1
    assert b"quant block size (256)" in L.neon_cuda_last_error()
    assert L.neon_cuda_upload(raw.ctypes.data, 14, 4, 256, 1, 3, 2, ctypes.byref(h)) == -1  # bad shard
    assert L.neon_cuda_upload(raw.ctypes.data, 1, 2, 45, 2, 0, 2, ctypes.byref(h)) == -2  # ragged column split
    assert L.neon_cuda_upload(None, 2, 1, 32, 0, 0, 1, ctypes.byref(h)) == -1
    assert L.neon_cuda_upload(raw.ctypes.data, 2, 4, 32, 1, 3, 2, ctypes.byref(h)) == -1
    assert L.neon_cuda_matvec(None, None, 0, None, 0, 1, None) == -1


def test_reference_error_messages():
    W = N.TensorInfo("blk.0.attn_q.weight", [4096], N.GGML_Q4_0, np.zeros(18, np.uint8))
    with pytest.raises(RuntimeError, match="expected a 2D weight tensor: blk.0.attn_q.weight"):
        N.proj_all_positions(W, np.zeros(4096, np.float32), 4096, np.zeros(1, np.float32), 1, 1)
    W = N.TensorInfo("blk.0.ffn_up.weight", [100, 2], N.GGML_Q4_0, np.zeros(36, np.uint8))
    with pytest.raises(RuntimeError, match=r"input dim \(100\) isn't a multiple of its quant block size \(32\)"):
        N.proj_all_positions(W, np.zeros(100, np.float32), 100, np.zeros(2, np.float32), 2, 1)


def test_switch_arguments_are_checked():
    """The process-wide switches refuse out-of-range arguments with
    NEON_ERR_INVALID and a message, on the host, and keep their value: the
    decode attention's rows (multiples of 32 from 32 to 16384) and head split
    (a power of two from 1 to 8), the resident kernel's CTAs per SM (0..8)."""
    L = N.load()
    for lo, share in ((16, 128), (32, 0), (48, 128), (32, 100), (32, 16416)):
        assert L.neon_cuda_set_attn_rows(lo, share) == -1, (lo, share)
        assert b"attention rows" in L.neon_cuda_last_error()
    for split in (0, 3, 16, -1):
        assert L.neon_cuda_set_attn_head_split(split) == -1, split
        assert b"head split" in L.neon_cuda_last_error()
    for k in (-1, 9):
        assert L.neon_cuda_set_resident(k) != 0, k
    # accepted values, then the defaults back
    assert L.neon_cuda_set_attn_rows(64, 256) == 0 and L.neon_cuda_set_attn_head_split(2) == 0
    assert L.neon_cuda_set_resident(2) == 0
    N.set_attn_rows()
    N.set_attn_head_split()
    N.set_resident()
