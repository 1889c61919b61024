"""The oracle restatement (oracle/neon_oracle.c) against the golden vectors the
reference's own CPU path produced (tests/golden/make_golden.py). Bit-exact."""
import numpy as np

import oracle as O
from conftest import load_golden


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_quantize_rows_q8_0_edge_cases_bitexact():
    g = load_golden("quantize_q8_0.npz")
    d, q = O.quantize_rows_q8_0(g["x_edge"])
    assert np.array_equal(bits(d), bits(g["d_edge"]))
    assert np.array_equal(q, g["q_edge"])


def test_quantize_rows_q8_0_multirow_bitexact():
    g = load_golden("quantize_q8_0.npz")
    d, q = O.quantize_rows_q8_0(g["x_rows"])
    assert np.array_equal(bits(d), bits(g["d_rows"]))
    assert np.array_equal(q, g["q_rows"])


def test_block_isum_exact():
    g = load_golden("block_isum.npz")
    L = O.lib()
    got = np.array([L.oracle_block_isum(g["qs"][i], g["xq"][i]) for i in range(len(g["qs"]))], np.int32)
    assert np.array_equal(got, g["isum"])


def test_proj_all_positions_bitexact():
    g = load_golden("matvec.npz")
    for i in range(int(g["n"])):
        typ, rows, cols, seq = (int(v) for v in g[f"c{i}_meta"])
        Y = O.proj_all_positions(typ, g[f"c{i}_W"], rows, cols, g[f"c{i}_X"])
        assert np.array_equal(bits(Y), bits(g[f"c{i}_Y"])), f"case {i} type {typ} {rows}x{cols} seq {seq}"


def test_proj_all_positions_multi_bitexact():
    g = load_golden("multi.npz")
    X = g["X"]
    for j in range(int(g["n"])):
        typ, rows, cols = (int(v) for v in g[f"t{j}_meta"])
        Y = O.proj_all_positions(typ, g[f"t{j}_W"], rows, cols, X)
        assert np.array_equal(bits(Y), bits(g[f"t{j}_Y"]))


def test_bad_cols_rejected():
    W = np.zeros(18, np.uint8)
    rc = O.lib().oracle_proj_all_positions(2, W, 1, 31, np.zeros(31, np.float32), 31,
                                           np.zeros(1, np.float32), 1, 1, np.zeros(1, np.float32),
                                           np.zeros(31, np.int8), np.zeros(31, np.float32))
    assert rc == -1


def test_other_types_bitexact():
    """F32/F16/BF16, Q4_1/Q5_0/Q5_1 and the K-quants: dequantize_row + dot_f32
    (rawllm_forward.hpp:597-605) against the reference's outputs."""
    g = load_golden("matvec_types.npz")
    for i in range(int(g["n"])):
        typ, rows, cols, seq = (int(v) for v in g[f"c{i}_meta"])
        Y = O.proj_all_positions(typ, g[f"c{i}_W"], rows, cols, g[f"c{i}_X"])
        assert np.array_equal(bits(Y), bits(g[f"c{i}_Y"])), f"case {i} type {typ} {rows}x{cols} seq {seq}"
    for j in range(int(g["m_n"])):
        typ, rows, cols = (int(v) for v in g[f"m{j}_meta"])
        Y = O.proj_all_positions(typ, g[f"m{j}_W"], rows, cols, g["mX"])
        assert np.array_equal(bits(Y), bits(g[f"m{j}_Y"]))
