"""The C++ drop-in header (host/neon_proj_cuda.hpp): compiles against the C ABI
with TensorInfo/ProjTarget-shaped types, links libneon_cuda.so, and on a GPU
reproduces the oracle through proj_all_positions[_multi]."""
import os
import subprocess

import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, PKG, ROOT, max_rel_err

SRC = os.path.join(ROOT, "tests", "cpp", "shim_driver.cpp")


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    N.load()  # builds libneon_cuda.so if needed
    exe = str(tmp_path_factory.mktemp("shim") / "shim_driver")
    subprocess.check_call(["g++", "-std=c++17", "-O2", SRC, "-I", os.path.join(ROOT, "include"),
                           "-I", os.path.join(PKG, "host"), "-L", PKG, "-lneon_cuda",
                           f"-Wl,-rpath,{PKG}", "-o", exe])
    return exe


def test_shim_compiles_and_links(driver):
    assert os.access(driver, os.X_OK)


def test_shim_reference_error_before_device_use(driver):
    out = subprocess.run([driver, "badshape"], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert "blk.3.attn_k.weight input dim (100) isn't a multiple of its quant block size (32)" in out.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
def test_shim_single_matches_oracle(driver, tmp_path, typ):
    rows, cols, seq = 96, 1024, 2
    W = S.weights(typ, rows, cols, seed=41)
    X = S.activations(seq, cols, seed=42)
    W.tofile(tmp_path / "W.bin")
    X.tofile(tmp_path / "X.bin")
    subprocess.check_call([driver, "single", str(typ), str(rows), str(cols), str(seq), str(tmp_path / "W.bin"),
                           str(tmp_path / "X.bin"), str(tmp_path / "Y.out")])
    Y = np.fromfile(tmp_path / "Y.out", np.float32).reshape(seq, rows)
    assert max_rel_err(Y, O.proj_all_positions(typ, W, rows, cols, X)) <= MATVEC_RTOL


@pytest.mark.gpu
def test_shim_multi_matches_oracle(driver, tmp_path):
    cols, seq = 512, 1
    specs = [(S.GGML_Q4_0, 256), (S.GGML_Q4_0, 128), (S.GGML_Q4_0, 128)]  # Q/K/V-shaped
    X = S.activations(seq, cols, seed=43)
    X.tofile(tmp_path / "X.bin")
    args, Ws = [], []
    for i, (typ, rows) in enumerate(specs):
        W = S.weights(typ, rows, cols, seed=50 + i)
        W.tofile(tmp_path / f"W{i}.bin")
        Ws.append(W)
        args += [str(typ), str(rows), str(tmp_path / f"W{i}.bin")]
    subprocess.check_call([driver, "multi", str(cols), str(seq), str(tmp_path / "X.bin"),
                           str(tmp_path / "Y.out"), *args])
    Y = np.fromfile(tmp_path / "Y.out", np.float32)
    off = 0
    for (typ, rows), W in zip(specs, Ws):
        ref = O.proj_all_positions(typ, W, rows, cols, X)
        assert max_rel_err(Y[off:off + rows * seq], ref) <= MATVEC_RTOL
        off += rows * seq
