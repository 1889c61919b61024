"""The allocation-free Q4_0 matvec (neon_cuda_matvec_q4_0_noalloc), called
through the C ABI, against the allocating entry point (neon_cuda_matvec).

The entry point serves callers that cannot let a library allocate device
memory -- a server that has reserved all of HBM for its own pools, a framework
caching allocator that holds the free memory, a loop that cannot take
cudaMalloc's device-wide synchronisation. Its activation scratch is a fixed
array compiled into the library instead of library-allocated memory, so its
results must equal those of neon_cuda_matvec on the same inputs. Two calls in
a row share that array, which is what the second call checks.

This file is collected last on purpose: a run that stops at its first failure
has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, max_rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.last]

torch = pytest.importorskip("torch")

LIMIT = 1 << 20  # seq * cols the fixed array holds


@pytest.fixture(scope="module")
def lib():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    N.init(0)
    return N.load()


def test_noalloc_matches_allocating_entry_point_on_two_calls(lib):
    """Two calls in a row through the shared array: each bit-identical to the
    allocating entry point's default multi-position path (the same quantiser
    and matvec kernels), and within the per-row bar of the oracle."""
    rows, cols = 1024, 4096
    W = S.q4_0_weights(rows, cols, seed=61)
    dt = N.DeviceTensor(W, S.GGML_Q4_0, rows, cols)
    N.set_prefill_mma(False)  # the allocating entry point's CUDA-core multi-position kernel, the same as this one's
    try:
        _two_calls(lib, dt, W, rows, cols)
    finally:
        N.set_prefill_mma(True)  # the default


def _two_calls(lib, dt, W, rows, cols):
    for call, seq in enumerate((16, 5)):
        X = S.activations(seq, cols, seed=62 + call)
        dx = torch.from_numpy(X).cuda()
        y_noalloc = torch.full((seq * rows,), float("nan"), device="cuda")
        y_alloc = torch.zeros(seq * rows, device="cuda")
        rc = lib.neon_cuda_matvec_q4_0_noalloc(dt.handle, dx.data_ptr(), cols, y_noalloc.data_ptr(), rows,
                                               seq, None)
        assert rc == 0, lib.neon_cuda_last_error()
        dt.matvec(dx, y_alloc, seq=seq)
        torch.cuda.synchronize()
        got = y_noalloc.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), y_alloc.cpu().numpy().view(np.uint32)), f"call {call + 1}"
        ref = O.proj_all_positions(S.GGML_Q4_0, W, rows, cols, X).reshape(-1)
        err = max_rel_err(got, ref)
        assert err <= MATVEC_RTOL, f"call {call + 1}: max rel err {err} against the oracle"


def test_noalloc_one_position_and_limits(lib):
    rows, cols = 256, 1024
    dt = N.DeviceTensor(S.q4_0_weights(rows, cols, seed=71), S.GGML_Q4_0, rows, cols)
    X = S.activations(1, cols, seed=72)
    dx = torch.from_numpy(X).cuda()
    y0 = torch.zeros(rows, device="cuda")
    y1 = torch.zeros(rows, device="cuda")
    assert lib.neon_cuda_matvec_q4_0_noalloc(dt.handle, dx.data_ptr(), cols, y0.data_ptr(), rows, 1, None) == 0
    dt.matvec(dx, y1)
    torch.cuda.synchronize()
    # one position: the allocating entry point streams (a different kernel), so
    # the two agree within the per-row bar, and both with the oracle
    assert max_rel_err(y0.cpu().numpy(), y1.cpu().numpy()) <= MATVEC_RTOL
    W = S.q4_0_weights(rows, cols, seed=71)
    ref = O.proj_all_positions(S.GGML_Q4_0, W, rows, cols, X).reshape(-1)
    assert max_rel_err(y0.cpu().numpy(), ref) <= MATVEC_RTOL
    # beyond the fixed array: a clear error, nothing launched
    seq = LIMIT // cols + 1
    before = N.launch_count()
    rc = lib.neon_cuda_matvec_q4_0_noalloc(dt.handle, dx.data_ptr(), cols, y0.data_ptr(), rows, seq, None)
    assert rc == -1 and b"exceeds the allocation-free limit" in lib.neon_cuda_last_error()
    assert N.launch_count() == before
    # Q8_0 tensors need no scratch and are refused
    q8 = N.DeviceTensor(S.q8_0_weights(8, 64, seed=73), S.GGML_Q8_0, 8, 64)
    assert lib.neon_cuda_matvec_q4_0_noalloc(q8.handle, dx.data_ptr(), 64, y0.data_ptr(), 8, 1, None) == -2
