"""Generate the golden vectors in tests/golden/ from the reference itself.

    make -C oracle ref && python tests/golden/make_golden.py && python tests/golden/make_golden.py --decode
    python tests/golden/make_golden.py --types
    python tests/golden/make_golden.py --quant      # needs gguf-py (the exporters' quantiser)

Every expected output here is produced by the reference's own CPU path --
rawllm_forward.hpp compiled with the reference's flags into
oracle/_ref/libneon_ref.so (oracle/Makefile) -- on seeded synthetic inputs.
The reference ships no golden vectors or known-answer tests of its own for
this path, so these fixtures are what pins both the C restatement in
oracle/neon_oracle.c and the CUDA kernels.

Outputs (numpy .npz, a few hundred KB in all):
  quantize_q8_0.npz  X -> (d, q) of quantize_rows_q8_0, incl. edge cases
  block_isum.npz     4096 random Q4_0 blocks x Q8_0 blocks -> isum
  matvec.npz         Q4_0 / Q8_0 proj_all_positions cases (W bytes, X, Y)
  multi.npz          a proj_all_positions_multi case shaped like Q/K/V
  decode_tiny.npz    greedy generation of transformer_forward on a small model
  matvec_types.npz   proj_all_positions of the nine other weight types (F32,
                     F16, BF16, Q4_1, Q5_0, Q5_1, Q4_K, Q5_K, Q6_K) and a
                     proj_all_positions_multi case mixing K-quants with Q4_0
  quant_gguf.npz     float rows and what gguf-py's gguf.quants.quantize writes
                     for them (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, F16, BF16): the
                     quantiser of the reference's exporters
                     (train_nanity_fixed.py:1162-1169, nanity_convert.py:472-484)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "neon-runtime-beta-variation_b200"))

import oracle as O  # noqa: E402
import synth as S  # noqa: E402

# (type, rows, cols, seq): small shapes, ragged row counts, the smallest
# input dim (32), several positions, and one full 4096-wide row set.
MATVEC_CASES = [
    (S.GGML_Q4_0, 64, 256, 1),
    (S.GGML_Q4_0, 37, 4096, 1),
    (S.GGML_Q4_0, 5, 32, 1),
    (S.GGML_Q4_0, 24, 1024, 3),
    (S.GGML_Q4_0, 130, 96, 2),
    (S.GGML_Q8_0, 64, 256, 1),
    (S.GGML_Q8_0, 19, 4096, 1),
    (S.GGML_Q8_0, 3, 32, 1),
    (S.GGML_Q8_0, 24, 1024, 3),
    (S.GGML_Q8_0, 70, 160, 2),
]


def quantize_inputs() -> np.ndarray:
    rng = np.random.default_rng(101)
    blocks = []
    blocks.append(rng.standard_normal(32).astype(np.float32))               # ordinary
    blocks.append(np.zeros(32, np.float32))                                  # amax = 0 -> d = 0
    blocks.append((rng.standard_normal(32) * 1e-39).astype(np.float32))      # denormal inputs
    blocks.append((rng.standard_normal(32) * 1e-43).astype(np.float32))      # 1/d overflows
    blocks.append((rng.standard_normal(32) * 3e37).astype(np.float32))       # near FLT_MAX
    b = rng.standard_normal(32).astype(np.float32); b[3] = np.inf; blocks.append(b)
    b = rng.standard_normal(32).astype(np.float32); b[7] = np.nan; blocks.append(b)
    b = rng.standard_normal(32).astype(np.float32); b[:] = np.nan; blocks.append(b)
    b = np.zeros(32, np.float32); b[0] = -127.0; b[1:] = np.arange(-15.5, 15.5, 1.0, dtype=np.float32)
    blocks.append(b)                                                         # exact halfway cases
    b = np.full(32, 2.5, np.float32); b[0] = 127.0; b[1] = -2.5; blocks.append(b)
    b = rng.integers(-127, 128, 32).astype(np.float32) * np.float32(0.37); blocks.append(b)
    blocks.append(np.full(32, -0.0, np.float32))
    x = np.concatenate(blocks)
    # plus 3 rows x 4096 of N(0,1) for the seq > 1 layout
    more = rng.standard_normal((3, 4096)).astype(np.float32)
    return x, more


def main() -> None:
    R = O.ref()
    if R is None:
        raise SystemExit("oracle/_ref/libneon_ref.so is missing: run `make -C oracle ref` first")
    pool = O.RefPool(4)

    # --- quantize_rows_q8_0
    x_edge, x_rows = quantize_inputs()
    X1 = x_edge.reshape(1, -1)
    d1 = np.empty((1, X1.shape[1] // 32), np.float32)
    q1 = np.empty(X1.shape, np.int8)
    R.ref_quantize_rows_q8_0(X1.reshape(-1), X1.shape[1], X1.shape[1], 1, d1.reshape(-1), q1.reshape(-1))
    d3 = np.empty((3, 128), np.float32)
    q3 = np.empty((3, 4096), np.int8)
    R.ref_quantize_rows_q8_0(x_rows.reshape(-1), 4096, 4096, 3, d3.reshape(-1), q3.reshape(-1))
    np.savez_compressed(os.path.join(HERE, "quantize_q8_0.npz"), x_edge=X1, d_edge=d1, q_edge=q1,
                        x_rows=x_rows, d_rows=d3, q_rows=q3)

    # --- block isum (exact integer dot of 4096 random block pairs)
    rng = np.random.default_rng(202)
    qs = rng.integers(0, 256, (4096, 16), dtype=np.uint8)
    xq = rng.integers(-127, 128, (4096, 32), dtype=np.int8)
    xq[0] = 127; xq[1] = -127; qs[0] = 0xFF; qs[1] = 0x00
    isum = np.array([R.ref_block_isum(qs[i], xq[i]) for i in range(len(qs))], np.int32)
    np.savez_compressed(os.path.join(HERE, "block_isum.npz"), qs=qs, xq=xq, isum=isum)

    # --- proj_all_positions cases
    out = {}
    for i, (typ, rows, cols, seq) in enumerate(MATVEC_CASES):
        W = S.weights(typ, rows, cols, seed=1000 + i)
        X = S.activations(seq, cols, seed=2000 + i)
        Y = np.zeros((seq, rows), np.float32)
        pool.proj_all_positions(typ, W, rows, cols, X, Y)
        out[f"c{i}_meta"] = np.array([typ, rows, cols, seq], np.int64)
        out[f"c{i}_W"] = W
        out[f"c{i}_X"] = X
        out[f"c{i}_Y"] = Y
    out["n"] = np.array(len(MATVEC_CASES))
    np.savez_compressed(os.path.join(HERE, "matvec.npz"), **out)

    # --- proj_all_positions_multi: Q/K/V-shaped (q_dim 128, kv_dim 64), mixed types
    cols, seq = 256, 2
    specs = [(S.GGML_Q4_0, 128), (S.GGML_Q4_0, 64), (S.GGML_Q8_0, 64)]
    X = S.activations(seq, cols, seed=3000)
    targets, out = [], {}
    for j, (typ, rows) in enumerate(specs):
        W = S.weights(typ, rows, cols, seed=3100 + j)
        Y = np.zeros((seq, rows), np.float32)
        targets.append((typ, W, rows, cols, Y))
        out[f"t{j}_meta"] = np.array([typ, rows, cols], np.int64)
        out[f"t{j}_W"] = W
    pool.proj_all_positions_multi(targets, X)
    for j, t in enumerate(targets):
        out[f"t{j}_Y"] = t[4]
    out["X"] = X
    out["n"] = np.array(len(specs))
    np.savez_compressed(os.path.join(HERE, "multi.npz"), **out)
    pool.close()
    print("golden vectors written to", HERE)


if __name__ == "__main__" and not {"--decode", "--types", "--quant"} & set(sys.argv):
    main()


def decode_golden() -> None:
    """decode_tiny.npz: greedy generation of the reference's transformer_forward
    on a small seeded model (the prompt, 16 tokens, the logits of every step and
    a checksum of the regenerated weights)."""
    import hashlib

    cfg = TINY_CFG
    tensors = list(S.model_tensors(cfg, seed=TINY_SEED))
    h = hashlib.sha256()
    for role, layer, raw, typ, ne0, ne1 in tensors:
        h.update(np.ascontiguousarray(raw).tobytes())
    m = O.Model(cfg, tensors, "reference", threads=4)
    prompt = S.prompt_tokens(8, cfg.n_vocab, TINY_SEED + 1)
    toks, logits = m.generate_greedy(prompt, 16)
    m.close()
    np.savez_compressed(os.path.join(HERE, "decode_tiny.npz"), prompt=prompt, tokens=toks, logits=logits,
                        weights_sha256=np.frombuffer(h.digest(), np.uint8))


TINY_CFG = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")
TINY_SEED = 3

if __name__ == "__main__" and "--decode" in sys.argv:
    decode_golden()


# (type, rows, cols, seq) of the other weight types: ragged row counts, one
# and several positions, and ragged float rows (block size 1).
TYPE_CASES = []
for _t in (S.GGML_Q4_1, S.GGML_Q5_0, S.GGML_Q5_1):
    TYPE_CASES += [(_t, 37, 512, 1), (_t, 9, 96, 2)]
for _t in (S.GGML_Q4_K, S.GGML_Q5_K, S.GGML_Q6_K):
    TYPE_CASES += [(_t, 21, 512, 1), (_t, 6, 256, 3)]
for _t in (S.GGML_F32, S.GGML_F16, S.GGML_BF16):
    TYPE_CASES += [(_t, 33, 512, 1), (_t, 13, 45, 2)]


def types_golden() -> None:
    pool = O.RefPool(4)
    out = {}
    for i, (typ, rows, cols, seq) in enumerate(TYPE_CASES):
        W = S.weights(typ, rows, cols, seed=4000 + i)
        X = S.activations(seq, cols, seed=5000 + i)
        Y = np.zeros((seq, rows), np.float32)
        pool.proj_all_positions(typ, W, rows, cols, X, Y)
        out[f"c{i}_meta"] = np.array([typ, rows, cols, seq], np.int64)
        out[f"c{i}_W"] = W
        out[f"c{i}_X"] = X
        out[f"c{i}_Y"] = Y
    out["n"] = np.array(len(TYPE_CASES))
    # a K-quant model's Q/K/V: Q4_K, Q6_K and a Q4_0 target sharing X
    cols, seq = 512, 2
    specs = [(S.GGML_Q4_K, 64), (S.GGML_Q6_K, 32), (S.GGML_Q4_0, 32)]
    X = S.activations(seq, cols, seed=6000)
    targets = []
    for j, (typ, rows) in enumerate(specs):
        W = S.weights(typ, rows, cols, seed=6100 + j)
        targets.append((typ, W, rows, cols, np.zeros((seq, rows), np.float32)))
        out[f"m{j}_meta"] = np.array([typ, rows, cols], np.int64)
        out[f"m{j}_W"] = W
    pool.proj_all_positions_multi(targets, X)
    for j, t in enumerate(targets):
        out[f"m{j}_Y"] = t[4]
    out["mX"] = X
    out["m_n"] = np.array(len(specs))
    pool.close()
    np.savez_compressed(os.path.join(HERE, "matvec_types.npz"), **out)
    print("wrote", os.path.join(HERE, "matvec_types.npz"))


if __name__ == "__main__" and "--types" in sys.argv:
    types_golden()


QUANT_TYPES = (S.GGML_Q8_0, S.GGML_Q4_0, S.GGML_Q4_1, S.GGML_Q5_0, S.GGML_Q5_1, S.GGML_F16, S.GGML_BF16)


def quant_inputs() -> np.ndarray:
    """8 x 256 float32: edge blocks (exact .5 ties after scaling, negative and
    positive extremes, all-zero, constant, tiny and large scales) then random rows."""
    rng = np.random.default_rng(77)
    blocks = []
    b = np.zeros(32, np.float32); b[0] = 127.0; b[1:] = np.arange(-15.5, 15.5, 1.0); blocks.append(b)   # Q8_0 ties
    b = np.zeros(32, np.float32); b[0] = -8.0; b[1:] = np.arange(-7.75, 7.75, 0.5); blocks.append(b)      # Q4_0 ties
    b = np.zeros(32, np.float32); b[5] = 16.0; b[6:] = np.arange(-12.5, 13.5, 1.0)[:26]; blocks.append(b)
    blocks.append(np.zeros(32, np.float32))                                                          # d = 0
    blocks.append(np.full(32, 0.375, np.float32))                                                    # max == min
    blocks.append((rng.standard_normal(32) * 1e-6).astype(np.float32))                               # fp16-subnormal d
    blocks.append((rng.standard_normal(32) * 3e4).astype(np.float32))                                # large
    b = rng.standard_normal(32).astype(np.float32); b[3] = -4.0; b[9] = 4.0; blocks.append(b)        # |max| tie, sign
    edge = np.concatenate(blocks).reshape(1, -1)                                                     # 1 x 256
    rows = (rng.standard_normal((7, 256)) * rng.uniform(0.001, 2, (7, 1))).astype(np.float32)
    return np.concatenate([edge, rows]).astype(np.float32)


def quant_golden() -> None:
    import gguf
    from gguf.constants import GGMLQuantizationType as Q

    X = quant_inputs()
    out = {"x": X, "types": np.array(QUANT_TYPES, np.int64)}
    for t in QUANT_TYPES:
        out[f"q{t}"] = np.ascontiguousarray(gguf.quants.quantize(X, Q(t))).view(np.uint8).reshape(X.shape[0], -1)
    np.savez_compressed(os.path.join(HERE, "quant_gguf.npz"), **out)
    print("wrote", os.path.join(HERE, "quant_gguf.npz"), "with gguf", __import__("importlib.metadata").metadata.version("gguf"))


if __name__ == "__main__" and "--quant" in sys.argv:
    quant_golden()
