"""Forced tile shapes of the one-position Q4_0 / Q8_0 kernel
(neon_cuda_set_stream_tiles), the knob of tuning sweeps: every allowed rows
per tile, whole rows and chunked rows (chunk sizes that are and are not
multiples of 8 blocks, a last chunk shorter than the rest), against the
oracle within the per-row bar; (0, 0) returns to the built-in planner bit for
bit. Collected after the other GPU suites (a variant not yet run on a GPU):
with -x, a failure here stops nothing else."""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, max_rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.newest]
torch = pytest.importorskip("torch")


@pytest.fixture(autouse=True)
def device():
    assert torch.cuda.is_available()
    N.init(0)
    yield
    N.set_stream_tiles(0, 0)


def run(dt, X, rows):
    dx = torch.from_numpy(X.copy()).cuda()
    dy = torch.full((rows + 3,), -3.0, device="cuda")
    dt.matvec(dx, dy)
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    assert np.all(y[rows:] == -3.0), "wrote past the rows"
    return y[:rows]


@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0], ids=lambda t: S.TYPE_NAMES[t])
@pytest.mark.parametrize("rows,cols", [(1000, 4096), (300, 14336)])
@pytest.mark.parametrize("rc,kc", [(2, 0), (4, 0), (8, 0), (16, 0), (32, 0), (8, 64), (8, 100), (16, 40), (2, 8),
                                   (32, 24)])
def test_forced_tiles_match_the_oracle(typ, rows, cols, rc, kc):
    W = S.weights(typ, rows, cols, seed=rows + rc + kc)
    X = S.activations(1, cols, seed=kc + 1)
    dt = N.DeviceTensor(W, typ, rows, cols)
    N.set_stream_tiles(rc, kc)
    try:
        y = run(dt, X[0], rows)
    except RuntimeError as e:  # a whole-row stage too large for shared memory is refused, not run
        assert "shared memory" in str(e) and kc == 0
        return
    assert max_rel_err(y, O.proj_all_positions(typ, W, rows, cols, X)[0]) <= MATVEC_RTOL


def test_default_plan_restored_bitwise():
    typ, rows, cols = S.GGML_Q4_0, 4096, 4096
    W = S.weights(typ, rows, cols, seed=3)
    X = S.activations(1, cols, seed=4)[0]
    dt = N.DeviceTensor(W, typ, rows, cols)
    a = run(dt, X, rows)
    N.set_stream_tiles(8, 32)
    run(dt, X, rows)
    N.set_stream_tiles(0, 0)
    b = run(dt, X, rows)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_bad_shapes_rejected():
    with pytest.raises(RuntimeError, match="rows per tile"):
        N.set_stream_tiles(3, 0)
    with pytest.raises(RuntimeError, match="blocks per chunk"):
        N.set_stream_tiles(8, -1)
