"""Parity of the CUDA matvec path (through the C ABI) with the reference.

Expected values come from the golden vectors the reference's own CPU path
produced, and from the oracle restatement (pinned bit-exact to the reference)
on fresh seeded inputs at the benchmark sizes. The bar:
  * Q8_0 activation quantisation: bit-exact (scales and quants);
  * matvec outputs: per row |y - y_ref| <= 1e-3 * max(|y_ref|, 0.01*rms(y_ref))
    (MATVEC_RTOL in conftest.py) -- only the fp32 summation order differs;
  * repeated calls, PDL on/off: bitwise identical.
"""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, load_golden, max_rel_err

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    N.init(0)
    N.set_pdl(True)
    yield


def dev_matvec(W, typ, rows, cols, X, y_stride=None, x_offset=0, y_fill=0.0):
    """Upload W, run neon_cuda_matvec on device copies of X, return Y (seq, y_stride)."""
    X = np.ascontiguousarray(X, np.float32)
    seq, xs = X.shape
    ys = rows if y_stride is None else y_stride
    dt = N.DeviceTensor(W, typ, rows, cols)
    dx = torch.zeros(x_offset + X.size, device="cuda")
    dx[x_offset:] = torch.from_numpy(X.reshape(-1)).cuda()
    dy = torch.full((seq * ys,), y_fill, device="cuda")
    before = N.launch_count()
    dt.matvec(dx[x_offset:], dy, seq=seq, x_stride=xs, y_stride=ys)
    torch.cuda.synchronize()
    assert N.launch_count() > before, "no kernel launched"
    return dy.cpu().numpy().reshape(seq, ys)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---------------------------------------------------------------------------
# golden vectors
# ---------------------------------------------------------------------------

def test_quantize_q8_0_bitexact_edge_cases():
    g = load_golden("quantize_q8_0.npz")
    for xk, dk, qk in (("x_edge", "d_edge", "q_edge"), ("x_rows", "d_rows", "q_rows")):
        X = g[xk]
        seq, cols = X.shape
        dx = torch.from_numpy(X).cuda()
        dd = torch.empty(seq * cols // 32, device="cuda")
        dq = torch.empty(seq * cols, dtype=torch.int8, device="cuda")
        N.quantize_q8_0(dx, cols, seq, dd, dq)
        torch.cuda.synchronize()
        assert np.array_equal(bits(dd.cpu().numpy()), bits(g[dk].reshape(-1))), xk
        assert np.array_equal(dq.cpu().numpy(), g[qk].reshape(-1)), xk


def test_golden_matvec_device_api():
    g = load_golden("matvec.npz")
    for i in range(int(g["n"])):
        typ, rows, cols, seq = (int(v) for v in g[f"c{i}_meta"])
        Y = dev_matvec(g[f"c{i}_W"], typ, rows, cols, g[f"c{i}_X"])
        err = max_rel_err(Y, g[f"c{i}_Y"])
        assert err <= MATVEC_RTOL, f"case {i}: type {typ} {rows}x{cols} seq {seq} err {err}"


def test_golden_matvec_host_api():
    g = load_golden("matvec.npz")
    for i in range(int(g["n"])):
        typ, rows, cols, seq = (int(v) for v in g[f"c{i}_meta"])
        W = N.TensorInfo(f"case{i}", [cols, rows], typ, g[f"c{i}_W"])
        Y = np.zeros((seq, rows), np.float32)
        N.proj_all_positions(W, g[f"c{i}_X"], cols, Y, rows, seq)
        assert max_rel_err(Y, g[f"c{i}_Y"]) <= MATVEC_RTOL, f"case {i}"


def test_golden_multi_device_and_host():
    g = load_golden("multi.npz")
    X = g["X"]
    seq, cols = X.shape
    metas = [tuple(int(v) for v in g[f"t{j}_meta"]) for j in range(int(g["n"]))]
    # device API
    dts = [N.DeviceTensor(g[f"t{j}_W"], t, r, c) for j, (t, r, c) in enumerate(metas)]
    ys = [torch.zeros(seq * r, device="cuda") for (_, r, _) in metas]
    N.matvec_multi([(dt, y, None) for dt, y in zip(dts, ys)], torch.from_numpy(X).cuda(), seq=seq)
    torch.cuda.synchronize()
    for j, y in enumerate(ys):
        assert max_rel_err(y.cpu().numpy(), g[f"t{j}_Y"]) <= MATVEC_RTOL
    # host API with the reference's ProjTarget surface
    targets = []
    for j, (t, r, c) in enumerate(metas):
        W = N.TensorInfo(f"t{j}", [c, r], t, g[f"t{j}_W"])
        targets.append(N.ProjTarget(W, np.zeros((seq, r), np.float32), r))
    N.proj_all_positions_multi(targets, X, cols, seq)
    for j, tg in enumerate(targets):
        assert max_rel_err(tg.Y, g[f"t{j}_Y"]) <= MATVEC_RTOL


# ---------------------------------------------------------------------------
# benchmark sizes against the oracle
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("typ,rows,cols", [
    (S.GGML_Q4_0, 4096, 4096),
    (S.GGML_Q8_0, 4096, 4096),
    (S.GGML_Q8_0, 14336, 4096),
    (S.GGML_Q8_0, 4096, 14336),
    (S.GGML_Q4_0, 28672, 8192),
    (S.GGML_Q4_0, 8192, 28672),
])
def test_decode_shapes_all_rows(typ, rows, cols):
    W = S.weights(typ, rows, cols, seed=11)
    X = S.activations(1, cols, seed=12)
    Y = dev_matvec(W, typ, rows, cols, X)
    ref = O.proj_all_positions(typ, W, rows, cols, X)
    assert max_rel_err(Y, ref) <= MATVEC_RTOL


@pytest.mark.parametrize("typ,rows,cols", [
    (S.GGML_Q4_0, 4096, 4096),
    (S.GGML_Q8_0, 4096, 4096),
    (S.GGML_Q8_0, 14336, 4096),
    (S.GGML_Q8_0, 4096, 14336),
])
def test_prefill_128_sampled_rows(typ, rows, cols):
    seq = 128
    W = S.weights(typ, rows, cols, seed=21)
    X = S.activations(seq, cols, seed=22)
    Y = dev_matvec(W, typ, rows, cols, X)
    idx = np.sort(np.random.default_rng(23).choice(rows, 192, replace=False))
    ref = O.proj_all_positions(typ, np.ascontiguousarray(W[idx]), len(idx), cols, X)
    assert max_rel_err(Y[:, idx], ref) <= MATVEC_RTOL


# ---------------------------------------------------------------------------
# ragged shapes, strides, alignment
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
@pytest.mark.parametrize("rows,cols,seq", [(1, 32, 1), (3, 64, 1), (33, 96, 1), (129, 8192, 1),
                                           (5, 32, 7), (67, 2048, 5), (2, 12288, 1), (301, 800, 1),
                                           (77, 1152, 1), (1000, 3072, 1), (19, 28672, 1)])
def test_ragged(typ, rows, cols, seq):
    W = S.weights(typ, rows, cols, seed=rows * 7 + cols)
    X = S.activations(seq, cols, seed=seq + 3)
    ref = O.proj_all_positions(typ, W, rows, cols, X)
    assert max_rel_err(dev_matvec(W, typ, rows, cols, X), ref) <= MATVEC_RTOL


@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
def test_strides_and_unaligned_x(typ):
    rows, cols, seq = 48, 256, 3
    W = S.weights(typ, rows, cols, seed=5)
    Xw = S.activations(seq, cols + 7, seed=6)          # x_stride = cols + 7
    ref = O.proj_all_positions(typ, W, rows, cols, Xw, x_stride=cols + 7, y_stride=rows + 5)
    Y = dev_matvec(W, typ, rows, cols, Xw, y_stride=rows + 5, x_offset=1, y_fill=-3.0)
    assert max_rel_err(Y[:, :rows], ref[:, :rows]) <= MATVEC_RTOL
    assert np.all(Y[:, rows:] == -3.0), "padding between rows and y_stride was written"
    # one position with an unaligned X pointer
    X1 = Xw[:1, :cols]
    assert max_rel_err(dev_matvec(W, typ, rows, cols, X1, x_offset=3),
                       O.proj_all_positions(typ, W, rows, cols, X1)) <= MATVEC_RTOL


def test_repeat_and_pdl_bitwise_identical():
    rows, cols = 1024, 4096
    for typ in (S.GGML_Q4_0, S.GGML_Q8_0):
        W = S.weights(typ, rows, cols, seed=9)
        X = S.activations(1, cols, seed=10)
        a = dev_matvec(W, typ, rows, cols, X)
        b = dev_matvec(W, typ, rows, cols, X)
        N.set_pdl(False)
        try:
            c = dev_matvec(W, typ, rows, cols, X)
        finally:
            N.set_pdl(True)
        assert np.array_equal(bits(a), bits(b)) and np.array_equal(bits(a), bits(c))


# ---------------------------------------------------------------------------
# tensor-parallel shards
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
@pytest.mark.parametrize("n", [2, 4, 8])
def test_row_and_col_shards(typ, n):
    rows, cols = 1024, 2048
    W = S.weights(typ, rows, cols, seed=31)
    X = S.activations(1, cols, seed=32)
    full = O.proj_all_positions(typ, W, rows, cols, X)
    dx = torch.from_numpy(X[0]).cuda()
    parts = []
    for i in range(n):
        # output-dim split: rows [i*rows/n, (i+1)*rows/n)
        dt = N.DeviceTensor(W, typ, rows, cols, N.SHARD_ROWS, i, n)
        y = torch.zeros(dt.rows, device="cuda")
        dt.matvec(dx, y)
        r0 = rows * i // n
        torch.cuda.synchronize()
        assert dt.rows == rows // n
        assert max_rel_err(y.cpu().numpy(), full[0, r0:r0 + dt.rows]) <= MATVEC_RTOL
        # input-dim split: 32-blocks [i*nb/n, (i+1)*nb/n) against the matching X slice
        dc = N.DeviceTensor(W, typ, rows, cols, N.SHARD_COLS, i, n)
        k0 = (cols // 32) * i // n * 32
        yc = torch.zeros(rows, device="cuda")
        dc.matvec(dx[k0:k0 + dc.cols].contiguous(), yc)
        torch.cuda.synchronize()
        Wslice = np.ascontiguousarray(W.reshape(rows, cols // 32, -1)[:, k0 // 32:(k0 + dc.cols) // 32]
                                      .reshape(rows, -1))
        ref = O.proj_all_positions(typ, Wslice, rows, dc.cols, X[:, k0:k0 + dc.cols])
        assert max_rel_err(yc.cpu().numpy(), ref) <= MATVEC_RTOL
        parts.append(yc.cpu().numpy())
    assert max_rel_err(np.sum(parts, axis=0), full) <= MATVEC_RTOL


# ---------------------------------------------------------------------------
# errors mirror the reference's
# ---------------------------------------------------------------------------

def test_multi_mismatched_q4_0_cols_rejected():
    a = N.DeviceTensor(S.q4_0_weights(8, 64, 1), S.GGML_Q4_0, 8, 64)
    b = N.DeviceTensor(S.q4_0_weights(8, 128, 2), S.GGML_Q4_0, 8, 128)
    y = torch.zeros(8, device="cuda")
    with pytest.raises(RuntimeError, match="mismatched input dims"):
        N.matvec_multi([(a, y, None), (b, y, None)], torch.zeros(128, device="cuda"))


def test_bad_y_stride_rejected():
    a = N.DeviceTensor(S.q8_0_weights(8, 64, 1), S.GGML_Q8_0, 8, 64)
    with pytest.raises(RuntimeError, match="y_stride"):
        a.matvec(torch.zeros(128, device="cuda"), torch.zeros(16, device="cuda"), seq=2, y_stride=4)


def test_empty_seq_is_noop():
    a = N.DeviceTensor(S.q4_0_weights(8, 64, 1), S.GGML_Q4_0, 8, 64)
    before = N.launch_count()
    a.matvec(torch.zeros(64, device="cuda"), torch.zeros(8, device="cuda"), seq=0)
    assert N.launch_count() == before
