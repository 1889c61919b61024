"""Parity of the dequantising kernel (F32, F16, BF16, Q4_1, Q5_0, Q5_1, Q4_K,
Q5_K, Q6_K weights x fp32 X) through the C ABI with the reference.

Expected values: the reference's own outputs (tests/golden/matvec_types.npz)
and the oracle restatement (pinned bit-exact to the reference) on seeded
inputs at the benchmark sizes. Decoded weights are the reference's bit for
bit; only the fp32 summation order differs, so the bar is the per-row
MATVEC_RTOL of conftest.py. A small decoder built from each type generates
the oracle's greedy tokens with logits within the same per-element bar."""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, load_golden, max_rel_err, rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

DQ_TYPES = [t for t in S.ALL_TYPES if t not in (S.GGML_Q4_0, S.GGML_Q8_0)]
ids = lambda t: S.TYPE_NAMES[t]  # noqa: E731


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    N.init(0)
    N.set_pdl(True)
    yield


def dev_matvec(W, typ, rows, cols, X, y_stride=None):
    X = np.ascontiguousarray(X, np.float32)
    seq = X.shape[0]
    ys = rows if y_stride is None else y_stride
    dt = N.DeviceTensor(W, typ, rows, cols)
    dx = torch.from_numpy(X.reshape(-1).copy()).cuda()
    dy = torch.full((seq * ys,), -7.0, device="cuda")
    before = N.launch_count()
    dt.matvec(dx, dy, seq=seq, x_stride=X.shape[1], y_stride=ys)
    torch.cuda.synchronize()
    assert N.launch_count() > before, "no kernel launched"
    return dy.cpu().numpy().reshape(seq, ys)


def test_golden_other_types_device_and_host_api():
    g = load_golden("matvec_types.npz")
    for i in range(int(g["n"])):
        typ, rows, cols, seq = (int(v) for v in g[f"c{i}_meta"])
        Y = dev_matvec(g[f"c{i}_W"], typ, rows, cols, g[f"c{i}_X"])
        assert max_rel_err(Y, g[f"c{i}_Y"]) <= MATVEC_RTOL, f"case {i}: {S.TYPE_NAMES[typ]} {rows}x{cols} seq {seq}"
        W = N.TensorInfo(f"case{i}", [cols, rows], typ, g[f"c{i}_W"])
        Yh = np.zeros((seq, rows), np.float32)
        N.proj_all_positions(W, g[f"c{i}_X"], cols, Yh, rows, seq)
        assert max_rel_err(Yh, g[f"c{i}_Y"]) <= MATVEC_RTOL, f"host case {i}"


def test_golden_mixed_multi():
    """Q4_K, Q6_K and Q4_0 targets sharing X in one proj_all_positions_multi call."""
    g = load_golden("matvec_types.npz")
    X = g["mX"]
    seq, cols = X.shape
    targets = []
    for j in range(int(g["m_n"])):
        typ, rows, c = (int(v) for v in g[f"m{j}_meta"])
        targets.append(N.ProjTarget(N.TensorInfo(f"m{j}", [c, rows], typ, g[f"m{j}_W"]),
                                    np.zeros((seq, rows), np.float32), rows))
    N.proj_all_positions_multi(targets, X, cols, seq)
    for j, tg in enumerate(targets):
        assert max_rel_err(tg.Y, g[f"m{j}_Y"]) <= MATVEC_RTOL, j


@pytest.mark.parametrize("typ", DQ_TYPES, ids=ids)
@pytest.mark.parametrize("rows,cols,seq", [
    (4096, 4096, 1),      # the decode shape
    (1000, 2048, 1),      # ragged last tile
    (14336, 4096, 1),     # ffn_gate / ffn_up
    (4096, 14336, 1),     # ffn_down: long rows, several chunks a row
    (96, 1024, 3),        # two positions per CTA
    (64, 2048, 9),        # four positions per CTA, ragged last position tile
])
def test_matches_oracle(typ, rows, cols, seq):
    W = S.weights(typ, rows, cols, seed=rows + cols + seq + typ)
    X = S.activations(seq, cols, seed=seq + 3)
    Y = dev_matvec(W, typ, rows, cols, X)
    err = max_rel_err(Y, O.proj_all_positions(typ, W, rows, cols, X))
    assert err <= MATVEC_RTOL, f"{S.TYPE_NAMES[typ]} {rows}x{cols} seq {seq}: {err}"


@pytest.mark.parametrize("typ", [S.GGML_Q6_K, S.GGML_F32], ids=ids)
def test_long_rows_one_position_per_cta(typ):
    # X of two positions of 28672 values does not fit shared memory next to the
    # chunk buffers: one position per CTA, grid.y over the positions
    rows, cols, seq = 24, 28672, 2
    W = S.weights(typ, rows, cols, seed=5)
    X = S.activations(seq, cols, seed=6)
    assert max_rel_err(dev_matvec(W, typ, rows, cols, X), O.proj_all_positions(typ, W, rows, cols, X)) <= MATVEC_RTOL


@pytest.mark.parametrize("typ", [S.GGML_F32, S.GGML_F16, S.GGML_BF16], ids=ids)
def test_ragged_float_input_dim(typ):
    rows, cols, seq = 77, 1000 + 13, 2
    W = S.weights(typ, rows, cols, seed=8)
    X = S.activations(seq, cols, seed=9)
    assert max_rel_err(dev_matvec(W, typ, rows, cols, X), O.proj_all_positions(typ, W, rows, cols, X)) <= MATVEC_RTOL


def test_strides_repeat_and_pdl_bitwise():
    typ, rows, cols = S.GGML_Q4_K, 512, 2048
    W = S.weights(typ, rows, cols, seed=1)
    X = S.activations(3, cols, seed=2)
    a = dev_matvec(W, typ, rows, cols, X, y_stride=rows + 5)
    b = dev_matvec(W, typ, rows, cols, X, y_stride=rows + 5)
    N.set_pdl(False)
    try:
        c = dev_matvec(W, typ, rows, cols, X, y_stride=rows + 5)
    finally:
        N.set_pdl(True)
    assert np.array_equal(a, b) and np.array_equal(a, c)
    assert np.all(a[:, rows:] == -7.0), "wrote outside the rows"
    assert max_rel_err(a[:, :rows], O.proj_all_positions(typ, W, rows, cols, X)) <= MATVEC_RTOL


def test_column_shards_sum_to_whole():
    typ, rows, cols = S.GGML_Q5_K, 256, 4096
    W = S.weights(typ, rows, cols, seed=4)
    X = S.activations(1, cols, seed=5)
    whole = O.proj_all_positions(typ, W, rows, cols, X)
    parts = []
    for i in range(4):
        dt = N.DeviceTensor(W, typ, rows, cols, N.SHARD_COLS, i, 4)
        assert dt.cols == cols // 4
        c0, c1 = cols * i // 4, cols * (i + 1) // 4
        dx = torch.from_numpy(X[:, c0:c1].copy()).cuda()
        dy = torch.zeros(rows, device="cuda")
        dt.matvec(dx, dy)
        torch.cuda.synchronize()
        parts.append(dy.cpu().numpy())
    assert max_rel_err(np.sum(parts, axis=0), whole) <= MATVEC_RTOL


TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")


@pytest.mark.parametrize("wtype,etype,tied", [
    (S.GGML_Q4_K, S.GGML_Q6_K, False),
    (S.GGML_Q5_K, S.GGML_Q5_K, True),
    (S.GGML_Q6_K, S.GGML_Q4_K, True),
    (S.GGML_Q5_0, S.GGML_Q4_1, True),
    (S.GGML_Q5_1, S.GGML_F16, True),
    (S.GGML_F16, S.GGML_BF16, False),
    (S.GGML_F32, S.GGML_Q8_0, True),
], ids=lambda v: S.TYPE_NAMES.get(v, str(v)) if not isinstance(v, bool) else ("tied" if v else "untied"))
def test_decoder_of_each_type_matches_oracle(wtype, etype, tied):
    """The fused decode step (norm folded into X staging, RoPE / SwiGLU /
    residual epilogues, CUDA-graph replay) on the dequantising kernel: the
    oracle's greedy tokens, and logits within 1e-3 relative L2 at every step --
    50x tighter than the whole-model bar of the Q4_0 decoder (conftest.py),
    since no activation is quantised here, but not the single-matvec
    per-element bar: fp32 reordering compounds over two layers of attention."""
    tensors = list(S.model_tensors(TINY, seed=17, wtype=wtype, embd_type=etype, tied=tied))
    m = N.Model(TINY, tensors)
    o = O.Model(TINY, tensors, "port")
    prompt = S.prompt_tokens(9, TINY.n_vocab, 18)
    want_toks, want_logits = o.generate_greedy(prompt, 8)
    assert np.array_equal(m.generate(prompt, 8), want_toks)
    m.set_length(0)
    got = [m.forward(prompt)] + [m.forward([t]) for t in want_toks[:7]]
    for i, (a, b) in enumerate(zip(got, want_logits)):
        assert rel_l2(a, b) <= 1e-3, f"step {i}"
        assert int(np.argmax(a)) == int(np.argmax(b)), f"step {i}"
    m.free()


def test_decoder_of_a_mixed_k_quant_model():
    """Q4_K projections with Q6_K attn_v, ffn_down and lm_head (a Q4_K_M
    conversion's mix): Q/K/V and each residual projection span two types, so
    the fused step splits them by type. The oracle's greedy tokens, logits
    within the same bar as the single-type decoders."""
    tensors = list(S.mixed_k_quant_tensors(TINY, seed=19))
    m = N.Model(TINY, tensors)
    o = O.Model(TINY, tensors, "port")
    prompt = S.prompt_tokens(9, TINY.n_vocab, 20)
    want_toks, want_logits = o.generate_greedy(prompt, 8)
    assert np.array_equal(m.generate(prompt, 8), want_toks)
    m.set_length(0)
    assert rel_l2(m.forward(prompt), want_logits[0]) <= 1e-3
    m.free()
