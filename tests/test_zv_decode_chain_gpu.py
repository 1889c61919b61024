"""The decode projection chain (neon_cuda_set_decode_chain,
matvec_chain_kernel in csrc/neon_chain.cuh): attn_output, ffn gate/up,
ffn_down and the next layer's Q/K/V as the phases of one launch with grid
barriers between them. Each phase runs the streaming kernel's tile plan, X
staging, dot products and epilogues, so tokens and logits must equal the
launch-per-projection decode step's bit for bit -- in the captured decode
graph and in an eager one-token forward -- and a model it does not take
(K-quant projections) must decode as before. Collected after the other GPU
suites (a variant not yet run on a GPU): with -x, a failure here stops nothing
else."""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MODEL_L2_RTOL, rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.newest(1)]
torch = pytest.importorskip("torch")

TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")


@pytest.fixture(autouse=True)
def device():
    assert torch.cuda.is_available()
    N.init(0)
    yield
    N.set_decode_chain(False)


def decode(cfg, tensors, prompt, steps, chain):
    N.set_decode_chain(chain)
    m = N.Model(cfg, tensors)
    toks = m.generate(prompt, steps)
    m.set_length(0)
    logits = [m.forward(prompt)] + [m.forward([t]) for t in toks[:6]]  # one-token forwards run eagerly
    m.free()
    return toks, logits


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("cfg,n_prompt,steps", [
    (TINY, 9, 12),
    (TINY.with_(plain_ffn=True, n_ff=768), 9, 12),
    (TINY.with_(n_vocab=777, n_embd=384, n_ff=1024, n_head=6, n_kv_head=2, ctx_len=300, n_layer=3), 40, 16),
    (S.QWEN3_0_6B.with_(n_layer=4, ctx_len=96), 32, 16),
], ids=["tiny", "plain_ffn", "wide", "qwen3_4_layers"])
def test_bitwise_equal_to_the_launch_per_projection_step(cfg, n_prompt, steps):
    tensors = list(S.model_tensors(cfg, seed=31))
    prompt = S.prompt_tokens(n_prompt, cfg.n_vocab, 32)
    t0, l0 = decode(cfg, tensors, prompt, steps, False)
    t1, l1 = decode(cfg, tensors, prompt, steps, True)
    assert np.array_equal(t0, t1)
    for i, (a, b) in enumerate(zip(l0, l1)):
        assert np.array_equal(bits(a), bits(b)), f"step {i}"


def test_matches_the_oracle():
    tensors = list(S.model_tensors(TINY, seed=33))
    prompt = S.prompt_tokens(9, TINY.n_vocab, 34)
    want_toks, want_logits = O.Model(TINY, tensors, "port").generate_greedy(prompt, 8)
    toks, logits = decode(TINY, tensors, prompt, 8, True)
    assert np.array_equal(toks, want_toks)
    assert rel_l2(logits[0], want_logits[0]) <= MODEL_L2_RTOL


def test_models_it_does_not_take_decode_as_before():
    tensors = list(S.model_tensors(TINY, seed=35, wtype=S.GGML_Q4_K, embd_type=S.GGML_Q6_K))
    prompt = S.prompt_tokens(9, TINY.n_vocab, 36)
    t0, l0 = decode(TINY, tensors, prompt, 8, False)
    t1, l1 = decode(TINY, tensors, prompt, 8, True)
    assert np.array_equal(t0, t1) and all(np.array_equal(bits(a), bits(b)) for a, b in zip(l0, l1))
