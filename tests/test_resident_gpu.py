"""The resident one-position kernel (matvec_resident_kernel, the default for
decode-sized Q4_0 / Q8_0 projections) against the oracle, through the C ABI.

  * several targets in one launch whose rows are odd (span pieces inside one
    CTA, scale windows at every 16-byte offset), against the oracle;
  * CTAs per SM 1, 2, 4: against the oracle, and bitwise repeatable;
  * the streaming kernel (resident kernel switched off) still matches the
    oracle on the same shapes, so both one-position paths stay covered;
  * the decode step's epilogues (norm folded, RoPE, cache rows, SwiGLU,
    accumulate) on either kernel: the oracle's greedy tokens.
"""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, MODEL_L2_RTOL, max_rel_err, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    N.init(0)
    yield
    N.set_resident(1)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def multi(typ, shapes, cols, X, resident):
    """One neon_cuda_matvec_multi call over targets of shapes[i] x cols."""
    N.set_resident(resident)
    try:
        Ws = [S.weights(typ, r, cols, seed=100 + i) for i, r in enumerate(shapes)]
        dts = [N.DeviceTensor(W, typ, r, cols) for W, r in zip(Ws, shapes)]
        ys = [torch.full((r,), float("nan"), device="cuda") for r in shapes]
        N.matvec_multi([(dt, y, None) for dt, y in zip(dts, ys)], torch.from_numpy(X[0]).cuda())
        torch.cuda.synchronize()
        return Ws, [y.cpu().numpy() for y in ys]
    finally:
        N.set_resident(1)


@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
@pytest.mark.parametrize("shapes,cols", [((33, 65, 7), 800), ((4096, 1024, 1024), 1024), ((5, 3, 1), 32),
                                         ((257, 130), 4096), ((2048, 2049), 288)])
def test_spans_with_odd_rows(typ, shapes, cols):
    X = S.activations(1, cols, seed=cols)
    Ws, got = multi(typ, shapes, cols, X, 2)
    for W, r, y in zip(Ws, shapes, got):
        ref = O.proj_all_positions(typ, W, r, cols, X)
        assert max_rel_err(y, ref) <= MATVEC_RTOL, f"{r}x{cols}"
    _, streamed = multi(typ, shapes, cols, X, 0)
    for W, r, y in zip(Ws, shapes, streamed):
        assert max_rel_err(y, O.proj_all_positions(typ, W, r, cols, X)) <= MATVEC_RTOL, f"streaming {r}x{cols}"


@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1000, 3072), (6144, 1024), (301, 800)])
def test_ctas_per_sm(typ, rows, cols):
    """Every CTAs-per-SM setting against the oracle (the setting may change
    the row-group width, so the fp32 sum order), and bitwise repeatable."""
    X = S.activations(1, cols, seed=rows)
    for k in (1, 2, 4):
        Ws, (y,) = multi(typ, (rows,), cols, X, k)
        assert max_rel_err(y, O.proj_all_positions(typ, Ws[0], rows, cols, X)) <= MATVEC_RTOL, f"k={k}"
        _, (y2,) = multi(typ, (rows,), cols, X, k)
        assert np.array_equal(bits(y), bits(y2)), f"k={k} not repeatable"


@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
@pytest.mark.parametrize("rows,cols", [(1, 32), (3, 64), (33, 96), (129, 8192), (301, 800), (77, 1152)])
def test_streaming_kernel_ragged(typ, rows, cols):
    X = S.activations(1, cols, seed=rows)
    Ws, got = multi(typ, (rows,), cols, X, 0)
    assert max_rel_err(got[0], O.proj_all_positions(typ, Ws[0], rows, cols, X)) <= MATVEC_RTOL


@pytest.mark.parametrize("resident", [1, 2, 0])
def test_decode_epilogues(resident):
    """A small decoder (norms folded into X staging, RoPE and cache-row
    epilogues on Q/K/V, SwiGLU on gate/up, accumulate on attn_output and
    ffn_down): the oracle's greedy tokens on both one-position kernels."""
    cfg = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=48, rope_base=1e4)
    tensors = list(S.model_tensors(cfg, seed=41))
    prompt = S.prompt_tokens(8, cfg.n_vocab, 42)
    N.set_resident(resident)
    try:
        m = N.Model(cfg, tensors)
        toks = m.generate(prompt, 12)
        m.set_length(0)
        logits = m.forward(prompt)
        m.free()
    finally:
        N.set_resident(1)
    o = O.Model(cfg, tensors, "port")
    want, want_logits = o.generate_greedy(prompt, 12)
    o.close()
    assert np.array_equal(toks, want)
    assert rel_l2(logits, want_logits[0]) <= MODEL_L2_RTOL
