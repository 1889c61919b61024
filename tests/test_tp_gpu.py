"""Tensor-parallel decode on two GPUs (one process per GPU, launched with
torch.distributed.run): the peer-memory all-reduce bit-exact against host
sums, the row-sharded matvec with its output all-gathered against the oracle
on every rank, and the split decoder against the reference's greedy tokens -- the small
model's golden generation and, for the Qwen3-0.6B-shaped decoder, the same
tokens as one GPU and as the reference's own transformer_forward. Skipped on
a host with fewer than two GPUs."""
import numpy as np
import pytest

import oracle as O
import synth as S
from conftest import MATVEC_RTOL, MODEL_L2_RTOL, load_golden, max_rel_err, rel_l2
from tp_launch import run_tp_worker

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

QWEN_PROMPT, QWEN_STEPS = 128, 32


@pytest.fixture(scope="module")
def tp2(tmp_path_factory):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    return run_tp_worker(tmp_path_factory.mktemp("tp2") / "rank0.npz", "--qwen-prompt", str(QWEN_PROMPT),
                         "--qwen-steps", str(QWEN_STEPS))


def test_allreduce_bit_exact(tp2):
    for k, v in tp2.items():
        if k.startswith("allreduce_"):
            assert float(v) == 0.0, k


def test_allgather_matvec_matches_oracle_on_every_rank(tp2):
    """neon_cuda_matvec_allgather: each rank's row shard, gathered, equals the
    whole matvec (oracle, per-row bar) on every rank and every call, and all
    ranks hold the same bits."""
    from tp_gpu_worker import ALLGATHER_CASES

    for name, typ, rows, cols in ALLGATHER_CASES:
        got = tp2[f"allgather_{name}"]  # [rank][call][rows]
        W = S.weights(typ, rows, cols, seed=rows + cols)
        ref = O.proj_all_positions(typ, W, rows, cols, S.activations(1, cols, seed=cols))[0]
        for r in range(got.shape[0]):
            for call in range(got.shape[1]):
                assert max_rel_err(got[r, call], ref) <= MATVEC_RTOL, f"{name} rank {r} call {call}"
                assert np.array_equal(got[r, call].view(np.uint32), got[0, 0].view(np.uint32)), f"{name} {r} {call}"


def test_tiny_golden_tokens_and_logits(tp2):
    g = load_golden("decode_tiny.npz")
    assert np.array_equal(tp2["tiny_tokens"], g["tokens"])
    for i, lg in enumerate(tp2["tiny_logits"]):
        assert rel_l2(lg, g["logits"][i]) <= MODEL_L2_RTOL, f"step {i}"
        assert int(np.argmax(lg)) == int(np.argmax(g["logits"][i]))
    # the fused collectives give the same bits as separate all-reduce launches
    assert np.array_equal(tp2["tiny_logits"], tp2["tiny_logits_unfused"])
    # each rank holds its own KV heads
    assert tuple(tp2["tiny_k0_shape"]) == (len(g["prompt"]), 2 // 2 * 64)


def test_qwen_split_matches_one_gpu_and_reference(tp2):
    assert np.array_equal(tp2["qwen_tokens"], tp2["qwen_tokens_1gpu"])
    assert np.array_equal(tp2["qwen_tokens"], tp2["qwen_tokens_unfused"])
    print(f"decode {QWEN_STEPS} tokens: 2 GPUs fused {float(tp2['qwen_tp_ms']):.2f} ms, "
          f"unfused {float(tp2['qwen_tp_unfused_ms']):.2f} ms, 1 GPU {float(tp2['qwen_1gpu_ms']):.2f} ms")
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    cfg = S.QWEN3_0_6B.with_(ctx_len=QWEN_PROMPT + QWEN_STEPS + 1)
    ref = O.Model(cfg, list(S.model_tensors(cfg, seed=21)), "reference")
    toks, _ = ref.generate_greedy(S.prompt_tokens(QWEN_PROMPT, cfg.n_vocab, 22), QWEN_STEPS)
    ref.close()
    assert np.array_equal(tp2["qwen_tokens"], toks)
