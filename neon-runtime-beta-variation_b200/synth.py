"""Seeded synthetic GGUF tensors for the quantized-matvec workloads.

No dataset or checkpoint is involved anywhere in this project: every weight and
activation is generated here from a fixed seed, with the value distributions
the benchmark configurations state.

* Q4_0 block (18 bytes, GGUF layout of rawllm_loader.hpp:367-386): an fp16
  scale ``d = fp16(|N(0,1)| * 0.02)`` then 16 bytes uniform in 0..255, i.e.
  32 nibbles uniform in 0..15 with value ``(q - 8) * d``.
* Q8_0 block (34 bytes): ``d = fp16(|N(0,1)| * 0.01)`` then 32 int8 uniform
  in [-127, 127].
* The other GGUF weight types (matvec parity tests only): fp16 scales drawn the
  same way, every quant field uniform random bytes; Q4_1 / Q5_1 minimums put
  the block's middle value near zero; Q6_K int8 sub-block scales uniform in
  [-64, 64]; F32 / F16 / BF16 values ``N(0, 1) * 0.02``.
* Activations: fp32 ``N(0, 1)``.
"""
from __future__ import annotations

import numpy as np

GGML_F32 = 0
GGML_F16 = 1
GGML_Q4_0 = 2
GGML_Q4_1 = 3
GGML_Q5_0 = 6
GGML_Q5_1 = 7
GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q5_K = 13
GGML_Q6_K = 14
GGML_BF16 = 30

BLOCK = 32
# bytes and values of one block of each weight type (rawllm_loader.hpp:367-386,
# rawllm_forward.hpp:289-299)
BLOCK_BYTES = {GGML_Q4_0: 18, GGML_Q8_0: 34, GGML_Q4_1: 20, GGML_Q5_0: 22, GGML_Q5_1: 24,
               GGML_Q4_K: 144, GGML_Q5_K: 176, GGML_Q6_K: 210, GGML_F32: 4, GGML_F16: 2, GGML_BF16: 2}
BLOCK_ELEMS = {GGML_Q4_0: 32, GGML_Q8_0: 32, GGML_Q4_1: 32, GGML_Q5_0: 32, GGML_Q5_1: 32,
               GGML_Q4_K: 256, GGML_Q5_K: 256, GGML_Q6_K: 256, GGML_F32: 1, GGML_F16: 1, GGML_BF16: 1}
ALL_TYPES = (GGML_F32, GGML_F16, GGML_BF16, GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q8_0,
             GGML_Q4_K, GGML_Q5_K, GGML_Q6_K)
TYPE_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_BF16: "BF16", GGML_Q4_0: "Q4_0", GGML_Q4_1: "Q4_1",
              GGML_Q5_0: "Q5_0", GGML_Q5_1: "Q5_1", GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K", GGML_Q5_K: "Q5_K",
              GGML_Q6_K: "Q6_K"}


def row_bytes(ggml_type: int, cols: int) -> int:
    """Bytes of one GGUF row (rawllm_loader.hpp:367-386)."""
    be = BLOCK_ELEMS[ggml_type]
    if cols % be:
        raise ValueError(f"cols={cols} is not a multiple of {be}")
    return cols // be * BLOCK_BYTES[ggml_type]


def q4_0_weights(rows: int, cols: int, seed: int, scale: float = 0.02) -> np.ndarray:
    """rows x cols Q4_0 tensor as GGUF bytes, shape (rows, row_bytes) uint8."""
    rng = np.random.default_rng(seed)
    nb = cols // BLOCK
    d = (np.abs(rng.standard_normal((rows, nb), dtype=np.float32)) * scale).astype(np.float16)
    qs = rng.integers(0, 256, size=(rows, nb, 16), dtype=np.uint8)
    out = np.empty((rows, nb, 18), np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = qs
    return out.reshape(rows, nb * 18)


def q8_0_weights(rows: int, cols: int, seed: int, scale: float = 0.01) -> np.ndarray:
    """rows x cols Q8_0 tensor as GGUF bytes, shape (rows, row_bytes) uint8."""
    rng = np.random.default_rng(seed)
    nb = cols // BLOCK
    d = (np.abs(rng.standard_normal((rows, nb), dtype=np.float32)) * scale).astype(np.float16)
    qs = rng.integers(-127, 128, size=(rows, nb, 32), dtype=np.int8)
    out = np.empty((rows, nb, 34), np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = qs.view(np.uint8)
    return out.reshape(rows, nb * 34)


_POOL_BLOCKS = 1 << 23  # 8M blocks: 144 MB of Q4_0, 272 MB of Q8_0
_pools = {}


def pooled_weights(ggml_type: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """rows x cols GGUF bytes cut from a seeded pool of 8M random 32-value
    blocks' worth of the type (same per-block distributions as `weights`) at a seeded
    offset: a read-only view when the tensor fits in the pool, else a copy
    that repeats the pool. For benchmark models of tens of GB, where drawing
    every block would take minutes; tensors are not independent of one another."""
    be = max(BLOCK, BLOCK_ELEMS[ggml_type])  # pool unit: a 32-value block (256 for the K-quants)
    bb = BLOCK_BYTES[ggml_type] * (BLOCK if BLOCK_ELEMS[ggml_type] == 1 else 1)
    n_pool = _POOL_BLOCKS * BLOCK // be
    if ggml_type not in _pools:
        pool = weights(ggml_type, n_pool // 256, 256 * be, seed=987654321).reshape(-1)
        pool.flags.writeable = False
        _pools[ggml_type] = pool
    pool = _pools[ggml_type]
    if cols % be:
        raise ValueError(f"cols={cols} is not a multiple of {be}")
    n = rows * (cols // be)
    rng = np.random.default_rng(seed)
    if n <= n_pool:
        off = int(rng.integers(0, n_pool - n + 1)) * bb
        return pool[off:off + n * bb].reshape(rows, (cols // be) * bb)
    out = np.empty(n * bb, np.uint8)
    pos, src = 0, int(rng.integers(0, n_pool)) * bb
    while pos < out.size:
        k = min(out.size - pos, pool.size - src)
        out[pos:pos + k] = pool[src:src + k]
        pos += k
        src = 0
    return out.reshape(rows, (cols // be) * bb)


def _f16_bytes(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float16).view(np.uint8)


def other_weights(ggml_type: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """rows x cols tensor of one of the remaining GGUF types as raw bytes,
    shape (rows, row_bytes) uint8 (distributions in the module docstring)."""
    rng = np.random.default_rng(seed)
    if ggml_type in (GGML_F32, GGML_F16, GGML_BF16):
        v = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
        if ggml_type == GGML_F32:
            return v.view(np.uint8).reshape(rows, cols * 4)
        if ggml_type == GGML_F16:
            return v.astype(np.float16).view(np.uint8).reshape(rows, cols * 2)
        u = v.view(np.uint32)
        bf = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
        return bf.view(np.uint8).reshape(rows, cols * 2)
    be, bb = BLOCK_ELEMS[ggml_type], BLOCK_BYTES[ggml_type]
    nb = cols // be
    out = rng.integers(0, 256, size=(rows, nb, bb), dtype=np.uint8)
    absn = lambda scale: np.abs(rng.standard_normal((rows, nb), dtype=np.float32)) * np.float32(scale)
    if ggml_type in (GGML_Q4_1, GGML_Q5_1):
        d = absn(0.02).astype(np.float16)
        mid = 8 if ggml_type == GGML_Q4_1 else 16
        m = (-mid * d.astype(np.float32)).astype(np.float16)
        out[:, :, 0:2] = _f16_bytes(d).reshape(rows, nb, 2)
        out[:, :, 2:4] = _f16_bytes(m).reshape(rows, nb, 2)
    elif ggml_type == GGML_Q5_0:
        out[:, :, 0:2] = _f16_bytes(absn(0.01)).reshape(rows, nb, 2)
    elif ggml_type in (GGML_Q4_K, GGML_Q5_K):
        out[:, :, 0:2] = _f16_bytes(absn(0.0005)).reshape(rows, nb, 2)
        out[:, :, 2:4] = _f16_bytes(absn(0.004)).reshape(rows, nb, 2)
    elif ggml_type == GGML_Q6_K:
        out[:, :, 192:208] = rng.integers(-64, 65, size=(rows, nb, 16), dtype=np.int8).view(np.uint8)
        out[:, :, 208:210] = _f16_bytes(absn(0.0005)).reshape(rows, nb, 2)
    else:
        raise ValueError(f"unsupported ggml type {ggml_type}")
    return out.reshape(rows, nb * bb)


def weights(ggml_type: int, rows: int, cols: int, seed: int) -> np.ndarray:
    if ggml_type == GGML_Q4_0:
        return q4_0_weights(rows, cols, seed)
    if ggml_type == GGML_Q8_0:
        return q8_0_weights(rows, cols, seed)
    if ggml_type in BLOCK_BYTES:
        return other_weights(ggml_type, rows, cols, seed)
    raise ValueError(f"unsupported ggml type {ggml_type}")


def activations(seq: int, cols: int, seed: int) -> np.ndarray:
    """fp32 N(0,1) activations, shape (seq, cols)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((seq, cols), dtype=np.float32)


def algorithmic_bytes(ggml_type: int, rows: int, cols: int, seq: int = 1) -> int:
    """Bytes a matvec must move at minimum: the quantized weight payload and
    scales once, plus fp32 X read and fp32 Y written for every position."""
    return rows * row_bytes(ggml_type, cols) + seq * (cols + rows) * 4


# ---------------------------------------------------------------------------
# Whole decoder models (NANITY_ARCHITECTURE_SPEC.md tensor list, GGUF ne shapes)
# ---------------------------------------------------------------------------

# Tensor roles, numbered as include/neon_cuda.h's NEON_ROLE_* values.
ROLE_TOKEN_EMBD, ROLE_OUTPUT_NORM, ROLE_OUTPUT = 0, 1, 2
ROLE_ATTN_NORM, ROLE_ATTN_Q, ROLE_ATTN_K, ROLE_ATTN_V, ROLE_ATTN_OUT = 3, 4, 5, 6, 7
ROLE_FFN_NORM, ROLE_FFN_GATE, ROLE_FFN_UP, ROLE_FFN_DOWN = 8, 9, 10, 11


class ModelConfig:
    """Hyperparameters of a NANITY decoder (engine::Config, rawllm_common.hpp:113-145)."""

    FIELDS = ("n_vocab", "n_embd", "n_layer", "n_head", "n_kv_head", "head_dim", "n_ff", "ctx_len",
              "rope_base", "rope_scale", "rope_dim_count", "norm_eps", "plain_ffn")

    def __init__(self, n_vocab, n_embd, n_layer, n_head, n_kv_head, head_dim, n_ff, ctx_len=4096,
                 rope_base=10000.0, rope_scale=1.0, rope_dim_count=0, norm_eps=1e-5, name="", plain_ffn=False):
        self.n_vocab, self.n_embd, self.n_layer = n_vocab, n_embd, n_layer
        self.n_head, self.n_kv_head, self.head_dim, self.n_ff = n_head, n_kv_head, head_dim, n_ff
        self.ctx_len, self.rope_base, self.rope_scale = ctx_len, rope_base, rope_scale
        self.rope_dim_count, self.norm_eps, self.name = rope_dim_count, norm_eps, name
        # engine::Config::use_swiglu == false: act = silu(ffn_up x), no ffn_gate
        self.plain_ffn = plain_ffn

    @property
    def q_dim(self):
        return self.n_head * self.head_dim

    @property
    def kv_dim(self):
        return self.n_kv_head * self.head_dim

    def with_(self, **kw):
        d = {f: getattr(self, f) for f in self.FIELDS}
        d["name"] = self.name
        d.update(kw)
        return ModelConfig(**d)


# The decoder shapes of the benchmark configurations.
QWEN3_0_6B = ModelConfig(151936, 1024, 28, 16, 8, 128, 3072, ctx_len=512, rope_base=1e6, norm_eps=1e-6,
                         name="Qwen3-0.6B-shaped")
PHI4_MINI = ModelConfig(200064, 3072, 32, 24, 8, 128, 8192, ctx_len=1152, rope_base=1e4, norm_eps=1e-5,
                        name="Phi-4-mini-shaped")
LLAMA3_70B = ModelConfig(128256, 8192, 80, 64, 8, 128, 28672, ctx_len=2432, rope_base=5e5, norm_eps=1e-5,
                         name="Llama-3-70B-shaped")


def norm_weights(ggml_type: int, n: int, seed: int) -> np.ndarray:
    """An RMSNorm weight of n values as raw bytes of `ggml_type`: 1 + 0.1 N(0,1)
    for the float types (F16 and BF16 rounded to nearest even), random blocks
    (other_weights / weights) for a block type."""
    if ggml_type not in (GGML_F32, GGML_F16, GGML_BF16):
        return weights(ggml_type, 1, n, seed).reshape(-1)
    v = np.float32(1) + np.random.default_rng(seed).standard_normal(n, dtype=np.float32) * np.float32(0.1)
    if ggml_type == GGML_F32:
        return v.view(np.uint8)
    if ggml_type == GGML_F16:
        return v.astype(np.float16).view(np.uint8)
    u = v.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).view(np.uint8)


def model_tensors(cfg: ModelConfig, seed: int, wtype: int = GGML_Q4_0, embd_type: int = GGML_Q8_0,
                  tied: bool = True, pooled: bool = False, norm_type=None):
    """Seeded random-init tensors of a decoder, in GGUF layout:
    yields (role, layer, raw bytes uint8, ggml type, ne0, ne1); ne1 = 0 for 1-D.
    Projections are `wtype` with the benchmark's block distributions, the
    embedding (also the lm_head when tied) is `embd_type`, norm weights fp32 1,
    or random norm_weights of `norm_type` when one is given.
    `pooled`: tensors cut from one random block pool (pooled_weights)."""
    weights_fn = pooled_weights if pooled else weights
    def sub(role, layer):
        return seed * 1000003 + role * 10007 + layer + 1

    ones = np.ones(cfg.n_embd, np.float32).view(np.uint8)
    def norm(role, layer):
        if norm_type is None:
            return ones, GGML_F32
        return norm_weights(norm_type, cfg.n_embd, sub(role, layer)), norm_type

    yield ROLE_TOKEN_EMBD, -1, weights_fn(embd_type, cfg.n_vocab, cfg.n_embd, sub(0, 0)), embd_type, cfg.n_embd, cfg.n_vocab
    yield (ROLE_OUTPUT_NORM, -1, *norm(ROLE_OUTPUT_NORM, 0), cfg.n_embd, 0)
    if not tied:
        yield ROLE_OUTPUT, -1, weights_fn(wtype, cfg.n_vocab, cfg.n_embd, sub(2, 0)), wtype, cfg.n_embd, cfg.n_vocab
    shapes = {ROLE_ATTN_Q: (cfg.q_dim, cfg.n_embd), ROLE_ATTN_K: (cfg.kv_dim, cfg.n_embd),
              ROLE_ATTN_V: (cfg.kv_dim, cfg.n_embd), ROLE_ATTN_OUT: (cfg.n_embd, cfg.q_dim),
              ROLE_FFN_GATE: (cfg.n_ff, cfg.n_embd), ROLE_FFN_UP: (cfg.n_ff, cfg.n_embd),
              ROLE_FFN_DOWN: (cfg.n_embd, cfg.n_ff)}
    if cfg.plain_ffn:
        del shapes[ROLE_FFN_GATE]
    for li in range(cfg.n_layer):
        yield (ROLE_ATTN_NORM, li, *norm(ROLE_ATTN_NORM, li), cfg.n_embd, 0)
        yield (ROLE_FFN_NORM, li, *norm(ROLE_FFN_NORM, li), cfg.n_embd, 0)
        for role, (rows, cols) in shapes.items():
            yield role, li, weights_fn(wtype, rows, cols, sub(role, li)), wtype, cols, rows


def mixed_k_quant_tensors(cfg: ModelConfig, seed: int):
    """A decoder with the type mix of a Q4_K_M conversion: Q4_K projections and
    embedding, Q6_K attn_v, ffn_down and lm_head (untied), fp32 norms -- so
    one layer's Q/K/V and its residual projections span two types. Same tuple
    layout as model_tensors."""
    q6 = {ROLE_ATTN_V, ROLE_FFN_DOWN, ROLE_OUTPUT}
    for role, layer, raw, typ, ne0, ne1 in model_tensors(cfg, seed, wtype=GGML_Q4_K, embd_type=GGML_Q4_K, tied=False):
        if role in q6:
            raw = weights(GGML_Q6_K, ne1, ne0, seed * 7919 + role * 131 + layer + 3)
            typ = GGML_Q6_K
        yield role, layer, raw, typ, ne0, ne1


def prompt_tokens(n: int, n_vocab: int, seed: int) -> np.ndarray:
    """Seeded random prompt token ids."""
    return np.random.default_rng(seed).integers(0, n_vocab, size=n, dtype=np.int32)
