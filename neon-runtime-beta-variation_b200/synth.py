"""Seeded synthetic GGUF tensors for the quantized-matvec workloads.

No dataset or checkpoint is involved anywhere in this project: every weight and
activation is generated here from a fixed seed, with the value distributions
the benchmark configurations state.

* Q4_0 block (18 bytes, GGUF layout of rawllm_loader.hpp:367-386): an fp16
  scale ``d = fp16(|N(0,1)| * 0.02)`` then 16 bytes uniform in 0..255, i.e.
  32 nibbles uniform in 0..15 with value ``(q - 8) * d``.
* Q8_0 block (34 bytes): ``d = fp16(|N(0,1)| * 0.01)`` then 32 int8 uniform
  in [-127, 127].
* Activations: fp32 ``N(0, 1)``.
"""
from __future__ import annotations

import numpy as np

GGML_F32 = 0
GGML_F16 = 1
GGML_Q4_0 = 2
GGML_Q8_0 = 8

BLOCK = 32
BLOCK_BYTES = {GGML_Q4_0: 18, GGML_Q8_0: 34}


def row_bytes(ggml_type: int, cols: int) -> int:
    """Bytes of one GGUF row (rawllm_loader.hpp:367-386)."""
    if cols % BLOCK:
        raise ValueError(f"cols={cols} is not a multiple of {BLOCK}")
    return cols // BLOCK * BLOCK_BYTES[ggml_type]


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


def weights(ggml_type: int, rows: int, cols: int, seed: int) -> np.ndarray:
    if ggml_type == GGML_Q4_0:
        return q4_0_weights(rows, cols, seed)
    if ggml_type == GGML_Q8_0:
        return q8_0_weights(rows, cols, seed)
    raise ValueError(f"unsupported ggml type {ggml_type}")


def activations(seq: int, cols: int, seed: int) -> np.ndarray:
    """fp32 N(0,1) activations, shape (seq, cols)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((seq, cols), dtype=np.float32)


def algorithmic_bytes(ggml_type: int, rows: int, cols: int, seq: int = 1) -> int:
    """Bytes a matvec must move at minimum: the quantized weight payload and
    scales once, plus fp32 X read and fp32 Y written for every position."""
    return rows * row_bytes(ggml_type, cols) + seq * (cols + rows) * 4
