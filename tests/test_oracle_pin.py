"""Pins the oracle restatement against the reference's OWN CPU path
(rawllm_forward.hpp compiled into oracle/_ref/ by oracle/Makefile) on fresh
seeded inputs: fp16 decode over all 65536 codes, the block integer dot over
50,000 random blocks (the validation rawllm_forward.hpp:348-350 describes but
does not ship), activation quantisation and the full matvecs. Bit-exact."""
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
