"""The bulk-copy ring variant of the dequantising kernel
(neon_cuda_set_dq_ring, matvec_dq_ring_kernel in csrc/neon_dequant.cuh)
against the oracle: every dequantised type at the decode shapes, ragged float
rows, long rows cut into several chunks, column shards, and the fused decode
step (norm folded into X staging, RoPE / SwiGLU / residual epilogues). The bar
is the register-buffer kernel's: MATVEC_RTOL per row, the oracle's greedy
tokens. Collected after the other GPU suites (the kernel is the newest): with
-x, a failure here stops nothing else."""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, max_rel_err, rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.newest]
torch = pytest.importorskip("torch")

DQ_TYPES = [t for t in S.ALL_TYPES if t not in (S.GGML_Q4_0, S.GGML_Q8_0)]
ids = lambda t: S.TYPE_NAMES[t]  # noqa: E731


@pytest.fixture(autouse=True)
def ring_on():
    assert torch.cuda.is_available()
    N.init(0)
    N.set_dq_ring(True)
    yield
    N.set_dq_ring(None)  # the default: the types the ring is faster for


def dev_matvec(W, typ, rows, cols, X, y_stride=None):
    seq = X.shape[0]
    ys = rows if y_stride is None else y_stride
    dt = N.DeviceTensor(W, typ, rows, cols)
    dx = torch.from_numpy(np.ascontiguousarray(X, np.float32).reshape(-1).copy()).cuda()
    dy = torch.full((seq * ys,), -7.0, device="cuda")
    dt.matvec(dx, dy, seq=seq, x_stride=cols, y_stride=ys)
    torch.cuda.synchronize()
    return dy.cpu().numpy().reshape(seq, ys)


@pytest.mark.parametrize("typ", DQ_TYPES, ids=ids)
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1000, 2048), (14336, 4096), (4096, 14336), (24, 28672),
                                       (8, 256)])
def test_matches_oracle(typ, rows, cols):
    W = S.weights(typ, rows, cols, seed=rows + cols + typ)
    X = S.activations(1, cols, seed=4)
    Y = dev_matvec(W, typ, rows, cols, X, y_stride=rows + 3)
    assert np.all(Y[:, rows:] == -7.0), "wrote outside the rows"
    err = max_rel_err(Y[:, :rows], O.proj_all_positions(typ, W, rows, cols, X))
    assert err <= MATVEC_RTOL, f"{S.TYPE_NAMES[typ]} {rows}x{cols}: {err}"


@pytest.mark.parametrize("typ", [S.GGML_F32, S.GGML_F16, S.GGML_BF16], ids=ids)
def test_ragged_float_rows(typ):
    rows, cols = 77, 1013
    W = S.weights(typ, rows, cols, seed=8)
    X = S.activations(1, cols, seed=9)
    assert max_rel_err(dev_matvec(W, typ, rows, cols, X), O.proj_all_positions(typ, W, rows, cols, X)) <= MATVEC_RTOL


def test_repeatable_and_close_to_the_register_kernel():
    typ, rows, cols = S.GGML_Q4_K, 4096, 4096
    W = S.weights(typ, rows, cols, seed=1)
    X = S.activations(1, cols, seed=2)
    a = dev_matvec(W, typ, rows, cols, X)
    b = dev_matvec(W, typ, rows, cols, X)
    N.set_dq_ring(False)
    c = dev_matvec(W, typ, rows, cols, X)
    assert np.array_equal(a, b)
    assert max_rel_err(a, c) <= MATVEC_RTOL


def test_column_shards_sum_to_whole():
    typ, rows, cols = S.GGML_Q6_K, 512, 4096
    W = S.weights(typ, rows, cols, seed=4)
    X = S.activations(1, cols, seed=5)
    parts = []
    for i in range(2):
        dt = N.DeviceTensor(W, typ, rows, cols, N.SHARD_COLS, i, 2)
        dx = torch.from_numpy(X[:, i * cols // 2:(i + 1) * cols // 2].copy()).cuda()
        dy = torch.zeros(rows, device="cuda")
        dt.matvec(dx, dy)
        torch.cuda.synchronize()
        parts.append(dy.cpu().numpy())
    assert max_rel_err(parts[0] + parts[1], O.proj_all_positions(typ, W, rows, cols, X)) <= MATVEC_RTOL


TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")


@pytest.mark.parametrize("wtype,etype", [(S.GGML_Q4_K, S.GGML_Q6_K), (S.GGML_Q5_0, S.GGML_Q4_1),
                                         (S.GGML_BF16, S.GGML_F16)], ids=lambda v: S.TYPE_NAMES[v])
def test_decoder_matches_oracle(wtype, etype):
    tensors = list(S.model_tensors(TINY, seed=19, wtype=wtype, embd_type=etype, tied=False))
    m = N.Model(TINY, tensors)
    o = O.Model(TINY, tensors, "port")
    prompt = S.prompt_tokens(9, TINY.n_vocab, 20)
    want_toks, want_logits = o.generate_greedy(prompt, 8)
    assert np.array_equal(m.generate(prompt, 8), want_toks)
    m.set_length(0)
    got = [m.forward(prompt)] + [m.forward([t]) for t in want_toks[:7]]
    for i, (a, b) in enumerate(zip(got, want_logits)):
        assert rel_l2(a, b) <= 1e-3, f"step {i}"
    m.free()
