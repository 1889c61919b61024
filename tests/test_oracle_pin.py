"""Pins the oracle restatement against the reference's OWN CPU path
(rawllm_forward.hpp compiled into oracle/_ref/ by oracle/Makefile) on fresh
seeded inputs: fp16 decode over all 65536 codes, the block integer dot over
50,000 random blocks (the validation rawllm_forward.hpp:348-350 describes but
does not ship), activation quantisation, the dequantisers of all eleven weight
types (dequantize_row, :301-321) on synthetic and on fully random bytes, and
the full matvecs of every type. Bit-exact."""
import numpy as np
import pytest

import oracle as O
import synth as S

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_fp16_all_codes():
    L, R = O.lib(), O.ref()
    a = np.array([L.oracle_fp16_to_fp32(h) for h in range(65536)], np.float32)
    b = np.array([R.ref_fp16_to_fp32(h) for h in range(65536)], np.float32)
    assert np.array_equal(bits(a), bits(b))


def test_block_isum_50k_blocks():
    L, R = O.lib(), O.ref()
    rng = np.random.default_rng(7)
    qs = rng.integers(0, 256, (50000, 16), dtype=np.uint8)
    xq = rng.integers(-127, 128, (50000, 32), dtype=np.int8)
    for i in range(50000):
        a = L.oracle_block_isum(qs[i], xq[i])
        assert a == R.ref_block_isum(qs[i], xq[i]) == R.ref_block_isum_scalar(qs[i], xq[i])


def test_quantize_random_scales():
    R = O.ref()
    rng = np.random.default_rng(8)
    X = (rng.standard_normal((16, 1024)) * np.exp(rng.uniform(-30, 30, (16, 1)))).astype(np.float32)
    d, q = O.quantize_rows_q8_0(X)
    d2 = np.empty_like(d)
    q2 = np.empty_like(q)
    R.ref_quantize_rows_q8_0(X.reshape(-1), 1024, 1024, 16, d2.reshape(-1), q2.reshape(-1))
    assert np.array_equal(bits(d), bits(d2)) and np.array_equal(q, q2)


@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
@pytest.mark.parametrize("rows,cols,seq", [(256, 4096, 1), (96, 2048, 4), (7, 32, 1)])
def test_proj_all_positions_matches_reference(typ, rows, cols, seq):
    pool = O.RefPool(4)
    W = S.weights(typ, rows, cols, seed=rows + cols)
    X = S.activations(seq, cols, seed=seq)
    Y = np.zeros((seq, rows), np.float32)
    pool.proj_all_positions(typ, W, rows, cols, X, Y)
    assert np.array_equal(bits(O.proj_all_positions(typ, W, rows, cols, X)), bits(Y))
    pool.close()


@pytest.mark.parametrize("typ", S.ALL_TYPES, ids=lambda t: S.TYPE_NAMES[t])
def test_dequantize_row_all_types(typ):
    cols = 1024
    W = S.weights(typ, 48, cols, seed=5)
    # random bytes everywhere, scales included (NaN / Inf / subnormal scales)
    R = np.random.default_rng(typ).integers(0, 256, W.shape, dtype=np.uint8)
    for M in (W, R):
        for r in range(M.shape[0]):
            assert np.array_equal(bits(O.dequantize_row(typ, M[r], cols)),
                                  bits(O.ref_dequantize_row(typ, M[r], cols))), (S.TYPE_NAMES[typ], r)


@pytest.mark.parametrize("typ", [t for t in S.ALL_TYPES if t not in (S.GGML_Q4_0, S.GGML_Q8_0)],
                         ids=lambda t: S.TYPE_NAMES[t])
@pytest.mark.parametrize("rows,cols,seq", [(64, 2048, 1), (33, 512, 3)])
def test_proj_all_positions_other_types(typ, rows, cols, seq):
    pool = O.RefPool(4)
    W = S.weights(typ, rows, cols, seed=rows + cols + typ)
    X = S.activations(seq, cols, seed=seq + 40)
    Y = np.zeros((seq, rows), np.float32)
    pool.proj_all_positions(typ, W, rows, cols, X, Y)
    assert np.array_equal(bits(O.proj_all_positions(typ, W, rows, cols, X)), bits(Y))
    pool.close()


def test_float_types_any_input_dim():
    # F32 / F16 / BF16 have a block size of 1: any cols is accepted
    pool = O.RefPool(2)
    for typ in (S.GGML_F32, S.GGML_F16, S.GGML_BF16):
        W = S.weights(typ, 5, 45, seed=typ)
        X = S.activations(2, 45, seed=1)
        Y = np.zeros((2, 5), np.float32)
        pool.proj_all_positions(typ, W, 5, 45, X, Y)
        assert np.array_equal(bits(O.proj_all_positions(typ, W, 5, 45, X)), bits(Y))
    pool.close()
