"""On-load quantisation (csrc/neon_quant.cuh), host build of the block code
the device kernel runs, against the quantiser of the reference's exporters:
gguf-py's gguf.quants.quantize (export_gguf, train_nanity_fixed.py:1162-1169;
nanity_convert.py:472-484). Byte for byte, on the committed fixtures that
gguf-py 0.19.0 wrote (tests/golden/make_golden.py --quant) and, where gguf-py
is importable, on fresh F16 / BF16 source rows."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

import synth as S
from conftest import PKG, ROOT, load_golden

QTYPES = (S.GGML_Q8_0, S.GGML_Q4_0, S.GGML_Q4_1, S.GGML_Q5_0, S.GGML_Q5_1, S.GGML_F16, S.GGML_BF16)
ids = lambda t: S.TYPE_NAMES[t]  # noqa: E731


@pytest.fixture(scope="module")
def qh(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("qhost") / "libquanthost.so")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.check_call([nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
                           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(PKG, "csrc"),
                           os.path.join(ROOT, "tests", "cpp", "quant_host.cu"), "-o", so])
    L = C.CDLL(so)
    L.q_host_quantize_rows.argtypes = [C.c_void_p, C.c_int, C.c_longlong, C.c_longlong, C.c_int, C.c_void_p]
    L.q_host_f16_bits.argtypes = [C.c_void_p, C.c_longlong, C.c_void_p]
    return L


def host_quantize(L, src, src_type, dst):
    rows = src.shape[0]
    cols = src.shape[1]
    out = np.zeros((rows, S.row_bytes(dst, cols)), np.uint8)
    assert L.q_host_quantize_rows(np.ascontiguousarray(src).ctypes.data, src_type, rows, cols, dst,
                                  out.ctypes.data) == 0
    return out


@pytest.mark.parametrize("dst", QTYPES, ids=ids)
def test_f32_rows_match_gguf_fixture(qh, dst):
    g = load_golden("quant_gguf.npz")
    got = host_quantize(qh, g["x"], S.GGML_F32, dst)
    want = g[f"q{dst}"]
    for r in range(got.shape[0]):
        assert np.array_equal(got[r], want[r]), (S.TYPE_NAMES[dst], r, np.nonzero(got[r] != want[r])[0][:8])


@pytest.mark.parametrize("src", [S.GGML_F16, S.GGML_BF16], ids=ids)
@pytest.mark.parametrize("dst", [S.GGML_Q8_0, S.GGML_Q4_0, S.GGML_Q5_1], ids=ids)
def test_half_sources_match_gguf(qh, src, dst):
    gguf = pytest.importorskip("gguf")
    from gguf.constants import GGMLQuantizationType as Q
    x = (np.random.default_rng(src + dst).standard_normal((6, 512)) * 0.05).astype(np.float32)
    raw = x.astype(np.float16) if src == S.GGML_F16 else (x.view(np.uint32) >> 16).astype(np.uint16)
    vals = raw.astype(np.float32) if src == S.GGML_F16 else (raw.astype(np.uint32) << 16).view(np.float32)
    want = np.ascontiguousarray(gguf.quants.quantize(vals, Q(dst))).view(np.uint8).reshape(6, -1)
    assert np.array_equal(host_quantize(qh, raw, src, dst), want)


def test_roundtrip_through_the_oracle_decoder(qh):
    """Quantised rows decode (oracle dequantize_row, pinned to the reference)
    to within each type's step of the input."""
    import oracle as O
    x = (np.random.default_rng(3).standard_normal((4, 1024)) * 0.1).astype(np.float32)
    for dst, steps in ((S.GGML_Q8_0, 127), (S.GGML_Q4_0, 8), (S.GGML_Q5_0, 16), (S.GGML_Q4_1, 15), (S.GGML_Q5_1, 31)):
        q = host_quantize(qh, x, S.GGML_F32, dst)
        for r in range(4):
            y = O.dequantize_row(dst, q[r], 1024).reshape(-1, 32)
            amax = np.abs(x[r].reshape(-1, 32)).max(axis=1, keepdims=True)
            span = x[r].reshape(-1, 32).max(axis=1, keepdims=True) - x[r].reshape(-1, 32).min(axis=1, keepdims=True)
            step = (span if dst in (S.GGML_Q4_1, S.GGML_Q5_1) else 2 * amax) / steps
            assert np.all(np.abs(y - x[r].reshape(-1, 32)) <= 0.51 * step + 1e-3 * amax), S.TYPE_NAMES[dst]


def test_f16_conversion_matches_numpy(qh):
    """The quantiser's integer fp32 -> fp16 (the scales it stores, and F16
    output) against numpy's cast: every exponent, ties, subnormals, overflow."""
    rng = np.random.default_rng(9)
    bits = rng.integers(0, 2**32, 2_000_000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    edges = np.array([0.0, -0.0, 1.0, 65504.0, 65519.996, 65520.0, 2.0**-14, 2.0**-24, 2.0**-25, 3 * 2.0**-26,
                      2.0**-25 * 1.0000001, 6.1e-5, -5.96e-8, 1.0 + 2.0**-11, 1.0 + 3 * 2.0**-11, np.inf, -np.inf],
                     np.float32)
    x = np.concatenate([edges, x, (rng.standard_normal(100000) * 1e-3).astype(np.float32)])
    got = np.empty(x.size, np.uint16)
    qh.q_host_f16_bits(x.ctypes.data, x.size, got.ctypes.data)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:10]
