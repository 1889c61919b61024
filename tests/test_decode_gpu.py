"""The device decode step (neon_cuda_model_*) against the reference's
transformer_forward: the golden generation of a small model, the oracle
restatement, and -- at full depth on the Qwen3-0.6B-shaped decoder -- the
reference's own build. The bar: identical greedy tokens; logits within
MODEL_L2_RTOL in relative L2 at every step (conftest.py explains why a
multi-layer Q8_0-quantised forward is not held to the per-element matvec bar);
the small model's first steps and K/V cache also within the per-element bar."""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, MODEL_L2_RTOL, load_golden, max_rel_err, rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available()
    N.init(0)


def test_tiny_golden_generation():
    g = load_golden("decode_tiny.npz")
    m = N.Model(TINY, S.model_tensors(TINY, seed=3))
    toks = m.generate(g["prompt"], 16)
    assert np.array_equal(toks, g["tokens"])
    assert m.length == len(g["prompt"]) + 16


def close(a, b, strict):
    """Per-element bar on the CUDA-core prompt path (the same arithmetic as the
    golden up to fp32 summation order); on the tensor-core path (the default),
    whose prompt attention sums in another order, the whole-model bar: a
    1e-7 difference can flip a Q8_0 activation at a rounding tie downstream
    (conftest.py)."""
    return max_rel_err(a, b) <= MATVEC_RTOL if strict else rel_l2(a, b) <= MODEL_L2_RTOL


PREFILL = [pytest.param(False, id="cuda_core_prefill"), pytest.param(True, id="tensor_core_prefill")]


@pytest.fixture
def prefill(request):
    N.set_prefill_mma(request.param)
    yield request.param
    N.set_prefill_mma(True)  # the default


@pytest.mark.parametrize("prefill", PREFILL, indirect=True)
def test_tiny_forward_logits_and_kv(prefill):
    strict = not prefill
    g = load_golden("decode_tiny.npz")
    m = N.Model(TINY, S.model_tensors(TINY, seed=3))
    logits = m.forward(g["prompt"])
    assert close(logits, g["logits"][0], strict)
    for i, t in enumerate(g["tokens"][:6]):
        logits = m.forward([t])
        assert close(logits, g["logits"][i + 1], strict), f"step {i}"
    o = O.Model(TINY, list(S.model_tensors(TINY, seed=3)), "port")
    o.forward(g["prompt"])
    for t in g["tokens"][:6]:
        o.forward([t])
    n = len(g["prompt"]) + 6
    for layer in range(TINY.n_layer):
        k1, v1 = m.read_kv(layer, n)
        k2, v2 = o.kv(layer, n)
        assert close(k1, k2, strict) and close(v1, v2, strict)


@pytest.mark.parametrize("prefill", PREFILL, indirect=True)
def test_rewind_and_eos(prefill):
    g = load_golden("decode_tiny.npz")
    m = N.Model(TINY, S.model_tensors(TINY, seed=3))
    m.forward(g["prompt"])
    m.set_length(3)  # keep the first 3 prompt positions, re-feed the rest
    logits = m.forward(g["prompt"][3:])
    assert close(logits, g["logits"][0], not prefill)
    # stopping before the eos token, as run_generation does
    m2 = N.Model(TINY, S.model_tensors(TINY, seed=3))
    eos = int(g["tokens"][5])
    toks = m2.generate(g["prompt"], 16, eos_id=eos)
    first = list(g["tokens"]).index(eos)
    assert np.array_equal(toks, g["tokens"][:first]) and m2.length == len(g["prompt"]) + first


def test_errors_match_reference_messages():
    m = N.Model(TINY, S.model_tensors(TINY, seed=3))
    with pytest.raises(RuntimeError, match="out of vocab range"):
        m.forward([TINY.n_vocab])
    with pytest.raises(RuntimeError, match="KV cache exhausted"):
        m.forward(np.zeros(TINY.ctx_len + 1, np.int32))
    with pytest.raises(RuntimeError, match="empty token batch"):
        m.forward([])
    with pytest.raises(RuntimeError, match="has shape"):
        m.set_tensor(S.ROLE_ATTN_Q, 0, S.q4_0_weights(32, 256, 1), S.GGML_Q4_0, 256, 32)
    with pytest.raises(RuntimeError, match="norm weight must be"):  # a ragged Q4_K row
        m.set_tensor(S.ROLE_FFN_NORM, 0, np.zeros(144, np.uint8), S.GGML_Q4_K, 256 - 32, 0)


@pytest.mark.parametrize("cfg,n_prompt,steps", [
    (TINY.with_(n_vocab=777, n_embd=384, n_ff=1024, n_head=6, n_kv_head=2, ctx_len=300), 200, 24),
    (TINY.with_(plain_ffn=True, n_ff=768, ctx_len=120), 40, 24),                 # SiLU-FFN without a gate
    (TINY.with_(n_head=8, n_kv_head=1, ctx_len=1100), 1060, 16),                 # long context: 17 CTAs merged, group 8
    (S.QWEN3_0_6B.with_(ctx_len=128 + 64 + 1), 128, 64),
])
def test_greedy_matches_reference(cfg, n_prompt, steps):
    """Identical greedy tokens to the reference's own transformer_forward."""
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    tensors = list(S.model_tensors(cfg, seed=21))
    prompt = S.prompt_tokens(n_prompt, cfg.n_vocab, 22)
    ref = O.Model(cfg, tensors, "reference")
    ref_toks, ref_logits = ref.generate_greedy(prompt, steps)
    ref.close()
    m = N.Model(cfg, tensors)
    toks = m.generate(prompt, steps)
    # the smallest top-2 logit margin of the reference run, for the record
    top2 = np.sort(ref_logits, axis=1)[:, -2:]
    margin = float(np.min(top2[:, 1] - top2[:, 0]))
    assert np.array_equal(toks, ref_toks), f"greedy tokens differ (min top-2 margin {margin:.3g})"
    # logits step by step on the same token stream
    m2 = N.Model(cfg, tensors)
    errs = [rel_l2(m2.forward(prompt), ref_logits[0])]
    for i, t in enumerate(ref_toks[:8]):
        errs.append(rel_l2(m2.forward([t]), ref_logits[i + 1]))
    print(f"{cfg.name}: min top-2 margin {margin:.3g}, logits rel-L2 max {max(errs):.2e}")
    assert max(errs) <= MODEL_L2_RTOL


def test_attention_splits_agree():
    """The decode attention at four work splits of a cluster of 16 CTAs per
    KV head (sized for 32-row shares; K and V in 32-row shared-memory
    rounds): 32-row shares over up to 8 CTAs, with each KV head's 4 query
    heads in one cluster and spread over 4 clusters; 96-row shares over 3
    CTAs in 3 rounds each; one CTA for the whole context in up to 8 rounds
    (no exchange). F32 projections and embedding keep activations
    unquantised, so the model is continuous and the comparison sees the
    attention's rounding alone: every decode step's logits within MATVEC_RTOL
    per element of the oracle's, and the splits within 1e-5 relative L2 of
    each other."""
    cfg = TINY.with_(n_head=8, n_kv_head=2, ctx_len=256 + 1)
    tensors = list(S.model_tensors(cfg, seed=31, wtype=S.GGML_F32, embd_type=S.GGML_F32))
    prompt = S.prompt_tokens(230, cfg.n_vocab, 32)
    toks = S.prompt_tokens(10, cfg.n_vocab, 33)
    o = O.Model(cfg, tensors, "port")
    o.forward(prompt)
    ref = [o.forward([t]) for t in toks]
    runs, errs = [], {}
    try:
        for lo, hi, split in ((32, 32, 1), (32, 32, 8), (96, 32, 1), (256, 32, 1)):
            N.set_attn_rows(lo, hi)
            N.set_attn_head_split(split)
            m = N.Model(cfg, tensors)
            m.forward(prompt)
            runs.append([m.forward([t]) for t in toks])
            m.free()
            errs[f"{lo}-{hi}/{split}"] = [max_rel_err(lg, want) for lg, want in zip(runs[-1], ref)]
    finally:
        N.set_attn_rows()
        N.set_attn_head_split()
    print({k: f"{max(v):.2e}" for k, v in errs.items()})
    assert all(max(v) <= MATVEC_RTOL for v in errs.values()), errs
    for other in runs[1:]:
        for a, b in zip(runs[0], other):
            assert rel_l2(a, b) <= 1e-5


def test_kv_cache_shift_matches_reference():
    """neon_cuda_model_kv_shift (fwd::kv_cache_shift): V rows move bit for bit,
    the kept K rows stay, the slid K rows equal the reference's (same rotation
    on K that already differs by fp32 summation order: the per-element bar), and
    generation continues with the reference's greedy tokens."""
    cfg = TINY.with_(rope_dim_count=48, ctx_len=80)
    tensors = list(S.model_tensors(cfg, seed=7))
    prompt = S.prompt_tokens(40, cfg.n_vocab, 8)
    kind = "reference" if O.ref_available() else "port"
    ref = O.Model(cfg, tensors, kind)
    ref.forward(prompt)
    ref.kv_shift(4, 13)
    m = N.Model(cfg, tensors)
    m.forward(prompt)
    pre = [m.read_kv(layer, 40) for layer in range(cfg.n_layer)]
    m.kv_shift(4, 0)  # no-op
    m.kv_shift(4, 13)
    assert m.length == ref.length == 27
    for layer in range(cfg.n_layer):
        k0, v0 = pre[layer]
        k1, v1 = m.read_kv(layer, m.length)
        k2, _ = ref.kv(layer, ref.length)
        assert np.array_equal(v1[:4], v0[:4]) and np.array_equal(v1[4:], v0[17:]), f"layer {layer} V"
        assert np.array_equal(k1[:4], k0[:4]), f"layer {layer} kept K"
        assert max_rel_err(k1, k2) <= MATVEC_RTOL, f"layer {layer} slid K"
    nxt = np.array([5], np.int32)
    ref_toks, _ = ref.generate_greedy(nxt, 12)
    ref.close()
    toks = m.generate(nxt, 12)
    assert np.array_equal(toks, ref_toks)


@pytest.mark.parametrize("norm_type", [S.GGML_F16, S.GGML_BF16, S.GGML_Q8_0, S.GGML_Q4_K],
                         ids=lambda t: S.TYPE_NAMES[t])
def test_norm_weight_types(norm_type):
    """RMSNorm weights of F16 / BF16 / block types (dequant_full in the
    reference, rawllm_forward.hpp:325-328), decoded at load time: the oracle's
    greedy tokens, and logits within the whole-model bar."""
    tensors = list(S.model_tensors(TINY, seed=17, norm_type=norm_type))
    prompt = S.prompt_tokens(11, TINY.n_vocab, 18)
    o = O.Model(TINY, tensors, "reference" if O.ref_available() else "port")
    want_toks, want_logits = o.generate_greedy(prompt, 6)
    m = N.Model(TINY, tensors)
    assert np.array_equal(m.generate(prompt, 6), want_toks)
    m.set_length(0)
    assert rel_l2(m.forward(prompt), want_logits[0]) <= MODEL_L2_RTOL
    m.free()
