"""Synthetic workload generators: GGUF layouts and the stated distributions."""
import numpy as np

import oracle as O
import synth as S


def test_row_bytes():
    assert S.row_bytes(S.GGML_Q4_0, 4096) == 2304
    assert S.row_bytes(S.GGML_Q8_0, 4096) == 4352
    assert S.algorithmic_bytes(S.GGML_Q4_0, 4096, 4096) == 9469952


def test_q4_0_layout_and_distribution():
    W = S.q4_0_weights(64, 4096, seed=1)
    assert W.shape == (64, 2304) and W.dtype == np.uint8
    blocks = W.reshape(64, 128, 18)
    d = blocks[:, :, 0:2].copy().view(np.float16).astype(np.float32)
    assert (d >= 0).all() and 0.01 < d.mean() < 0.02   # |N(0,1)|*0.02 has mean 0.016
    nib = np.concatenate([blocks[:, :, 2:] & 15, blocks[:, :, 2:] >> 4])
    assert nib.min() == 0 and nib.max() == 15 and abs(nib.mean() - 7.5) < 0.05


def test_q8_0_layout_and_dequant():
    W = S.q8_0_weights(8, 256, seed=2)
    blocks = W.reshape(8, 8, 34)
    q = blocks[:, :, 2:].copy().view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    d = blocks[:, :, 0:2].copy().view(np.float16).astype(np.float32)
    # a dot with a one-hot X returns d * q of that element (dequant_q8_0)
    X = np.zeros((1, 256), np.float32); X[0, 37] = 1.0
    Y = O.proj_all_positions(S.GGML_Q8_0, W, 8, 256, X)
    assert np.array_equal(Y[0], d[:, 1, 0] * q[:, 1, 5].astype(np.float32))


def test_seeded():
    assert np.array_equal(S.activations(2, 64, 5), S.activations(2, 64, 5))
    assert not np.array_equal(S.q4_0_weights(2, 64, 5), S.q4_0_weights(2, 64, 6))


def test_row_bytes_of_every_type():
    # nbytes_for (rawllm_loader.hpp:367-386) for a 4096-value row
    want = {S.GGML_F32: 16384, S.GGML_F16: 8192, S.GGML_BF16: 8192, S.GGML_Q4_0: 2304, S.GGML_Q4_1: 2560,
            S.GGML_Q5_0: 2816, S.GGML_Q5_1: 3072, S.GGML_Q8_0: 4352, S.GGML_Q4_K: 2304, S.GGML_Q5_K: 2816,
            S.GGML_Q6_K: 3360}
    for t, n in want.items():
        assert S.row_bytes(t, 4096) == n == O.lib().oracle_row_bytes(t, 4096), S.TYPE_NAMES[t]


def test_pooled_weights_every_type():
    """The block pool of the large benchmark models: GGUF rows of the type,
    seeded, and (past the pool's size) repeated from a seeded offset."""
    for t in (S.GGML_Q4_K,):  # the 256-value super-block path (Q4_0 / Q8_0 pools serve the bench)
        a = S.pooled_weights(t, 96, 4096, seed=3)
        assert a.shape == (96, S.row_bytes(t, 4096))
        assert np.array_equal(a, S.pooled_weights(t, 96, 4096, seed=3))
        assert not np.array_equal(a, S.pooled_weights(t, 96, 4096, seed=4))
    be = 256
    n_pool = (1 << 23) * 32 // be  # super-blocks in the Q4_K pool
    rows = n_pool // (8192 // be) + 3  # more blocks than the pool holds
    big = S.pooled_weights(S.GGML_Q4_K, rows, 8192, seed=5)
    assert big.shape == (rows, S.row_bytes(S.GGML_Q4_K, 8192))
