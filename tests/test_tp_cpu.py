"""Tensor parallelism, host side (no GPU): the library's shard plan and a
world-2 gloo emulation of the sharded decode.

The CUDA path splits the decoder as neon_cuda_tp_shard says; these tests check
that plan on the benchmark shapes (every tensor covered exactly once, heads and
FFN rows kept whole per rank, attn_output / ffn_down columns matching the
ranks' activations) and run the decode of a small model split over two gloo
ranks against the same model on one rank: same greedy tokens, logits within
the whole-model bar. The GPU runs of the same split are in test_tp_gpu.py.
"""
import socket

import numpy as np
import pytest

import neon_cuda as NC
import synth as S
from conftest import MODEL_L2_RTOL, rel_l2

TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")
CONFIGS = [TINY, S.QWEN3_0_6B, S.PHI4_MINI, S.LLAMA3_70B]
ROLES = range(12)


def _whole(cfg, role):
    return NC.tp_shard(cfg, role, 0, 1)


@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: c.name)
def test_shard_plan_partitions_every_tensor(cfg):
    for world in (1, 2, 4, 8):
        if cfg.n_kv_head % world:
            continue
        for role in ROLES:
            r0, r1, c0, c1 = _whole(cfg, role)
            assert r0 == 0 and c0 == 0
            parts = [NC.tp_shard(cfg, role, r, world) for r in range(world)]
            split_rows = any(p[:2] != (0, r1) for p in parts)
            split_cols = any(p[2:] != (0, c1) for p in parts)
            assert not (split_rows and split_cols), "a tensor is split along one dimension only"
            lo, hi = (0, 1) if split_rows else (2, 3)
            total = r1 if split_rows else c1
            if split_rows or split_cols:
                assert parts[0][lo] == 0 and parts[-1][hi] == total
                for a, b in zip(parts, parts[1:]):
                    assert a[hi] == b[lo], "shards must tile the dimension without gaps"
                assert all(p[hi] > p[lo] for p in parts), "no empty shard"
            if world == 1 or role in (S.ROLE_TOKEN_EMBD, S.ROLE_OUTPUT_NORM, S.ROLE_ATTN_NORM, S.ROLE_FFN_NORM):
                assert not split_rows and not split_cols


@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: c.name)
def test_shard_plan_keeps_heads_and_ffn_rows_together(cfg):
    hd = cfg.head_dim
    for world in (2, 4, 8):
        if cfg.n_kv_head % world:
            continue
        for r in range(world):
            q = NC.tp_shard(cfg, S.ROLE_ATTN_Q, r, world)
            k = NC.tp_shard(cfg, S.ROLE_ATTN_K, r, world)
            v = NC.tp_shard(cfg, S.ROLE_ATTN_V, r, world)
            o = NC.tp_shard(cfg, S.ROLE_ATTN_OUT, r, world)
            g = NC.tp_shard(cfg, S.ROLE_FFN_GATE, r, world)
            u = NC.tp_shard(cfg, S.ROLE_FFN_UP, r, world)
            d = NC.tp_shard(cfg, S.ROLE_FFN_DOWN, r, world)
            # whole KV heads with exactly their query heads (GQA groups stay on one rank)
            assert k == v and k[0] % hd == 0 and (k[1] - k[0]) == cfg.kv_dim // world
            group = cfg.n_head // cfg.n_kv_head
            assert q[0] == k[0] * group and q[1] == k[1] * group
            # attn_output consumes exactly this rank's attention output columns
            assert (o[2], o[3]) == (q[0], q[1]) and (o[0], o[1]) == (0, cfg.n_embd)
            # ffn_down consumes exactly this rank's gate/up rows, in whole 32-blocks
            assert g == u and (d[2], d[3]) == (g[0], g[1]) and g[0] % 32 == 0 and g[1] % 32 == 0
        sizes = [NC.tp_shard(cfg, S.ROLE_OUTPUT, r, world) for r in range(world)]
        assert sum(s[1] - s[0] for s in sizes) == cfg.n_vocab


def test_shard_plan_rejects_bad_rank():
    with pytest.raises(NC.NeonError):
        NC.tp_shard(TINY, S.ROLE_ATTN_Q, 2, 2)
    with pytest.raises(NC.NeonError):
        NC.tp_shard(TINY, 99, 0, 1)


def test_comm_floats_covers_prefill_and_vocab_shard():
    assert NC.model_comm_floats(S.QWEN3_0_6B, 1) >= 256 * S.QWEN3_0_6B.n_embd
    assert NC.model_comm_floats(TINY, 2) >= (TINY.n_vocab + 1) // 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp_decode_gloo_world2_matches_one_rank(tmp_path):
    import torch.multiprocessing as mp

    import tp_emulation as E

    seed, n_prompt, n_new = 3, 6, 8
    cfg_args = ((TINY.n_vocab, TINY.n_embd, TINY.n_layer, TINY.n_head, TINY.n_kv_head, TINY.head_dim, TINY.n_ff),
                dict(ctx_len=TINY.ctx_len, rope_base=TINY.rope_base, norm_eps=TINY.norm_eps, name="tiny"))
    mp.start_processes(E.worker, args=(2, _free_port(), str(tmp_path), cfg_args, seed, n_prompt, n_new), nprocs=2,
                       join=True, start_method="spawn")
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    # the replicated state stays identical across ranks
    np.testing.assert_array_equal(r0["tokens"], r1["tokens"])
    np.testing.assert_array_equal(r0["logits"], r1["logits"])

    one = E.RankModel(TINY, S.model_tensors(TINY, seed), 0, 1)
    toks, logits = one.generate(S.prompt_tokens(n_prompt, TINY.n_vocab, seed + 1), n_new, lambda x: x, lambda x: x)
    np.testing.assert_array_equal(r0["tokens"], toks)
    for i in range(n_new):
        assert rel_l2(r0["logits"][i], logits[i]) <= MODEL_L2_RTOL


def test_tp_decode_gloo_world2_kquant_model(tmp_path):
    """The same split of a Q4_K model with a Q6_K embedding: every column cut
    falls on a 256-value super-block (n_head 8 x head_dim 64 = 256 columns of
    attn_output per rank; 256 of ffn_down)."""
    import torch.multiprocessing as mp

    import tp_emulation as E

    cfg = TINY.with_(n_head=8, n_kv_head=2)
    seed, n_prompt, n_new = 4, 5, 5
    cfg_args = ((cfg.n_vocab, cfg.n_embd, cfg.n_layer, cfg.n_head, cfg.n_kv_head, cfg.head_dim, cfg.n_ff),
                dict(ctx_len=cfg.ctx_len, rope_base=cfg.rope_base, norm_eps=cfg.norm_eps, name="tiny-k"))
    mp.start_processes(E.worker, args=(2, _free_port(), str(tmp_path), cfg_args, seed, n_prompt, n_new,
                                       S.GGML_Q4_K, S.GGML_Q6_K), nprocs=2, join=True, start_method="spawn")
    r0 = np.load(tmp_path / "rank0.npz")
    one = E.RankModel(cfg, S.model_tensors(cfg, seed, wtype=S.GGML_Q4_K, embd_type=S.GGML_Q6_K), 0, 1)
    toks, logits = one.generate(S.prompt_tokens(n_prompt, cfg.n_vocab, seed + 1), n_new, lambda x: x, lambda x: x)
    np.testing.assert_array_equal(r0["tokens"], toks)
    for i in range(n_new):
        assert rel_l2(r0["logits"][i], logits[i]) <= 1e-4  # no activation quantisation: one fp32 sum reordered


# Whether a K-quant model of each benchmark shape can be split: every column
# cut of attn_output and ffn_down on a 256-value super-block. The head split
# fixes attn_output's cuts at (heads per rank) x head_dim columns.
KQ_SPLITTABLE = {
    ("Qwen3-0.6B-shaped", 2): True, ("Qwen3-0.6B-shaped", 4): True, ("Qwen3-0.6B-shaped", 8): False,
    ("Phi-4-mini-shaped", 2): True, ("Phi-4-mini-shaped", 4): True, ("Phi-4-mini-shaped", 8): False,
    ("Llama-3-70B-shaped", 2): True, ("Llama-3-70B-shaped", 4): True, ("Llama-3-70B-shaped", 8): True,
}


@pytest.mark.parametrize("cfg", [S.QWEN3_0_6B, S.PHI4_MINI, S.LLAMA3_70B], ids=lambda c: c.name)
@pytest.mark.parametrize("world", [2, 4, 8])
def test_kquant_column_cuts_of_the_benchmark_shapes(cfg, world):
    cuts = set()
    for role in (S.ROLE_ATTN_OUT, S.ROLE_FFN_DOWN):
        for r in range(world):
            _, _, c0, c1 = NC.tp_shard(cfg, role, r, world)
            cuts |= {c0, c1}
    assert all(c % 256 == 0 for c in cuts) == KQ_SPLITTABLE[(cfg.name, world)]
