"""The C++ drop-in header (host/neon_proj_cuda.hpp): compiles against the C ABI
with TensorInfo/ProjTarget-shaped types, links libneon_cuda.so, and on a GPU
reproduces the oracle through proj_all_positions[_multi]."""
import os
import subprocess

import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, PKG, ROOT, max_rel_err

SRC = os.path.join(ROOT, "tests", "cpp", "shim_driver.cpp")


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    N.load()  # builds libneon_cuda.so if needed
    exe = str(tmp_path_factory.mktemp("shim") / "shim_driver")
    subprocess.check_call(["g++", "-std=c++17", "-O2", SRC, "-I", os.path.join(ROOT, "include"),
                           "-I", os.path.join(PKG, "host"), "-L", PKG, "-lneon_cuda",
                           f"-Wl,-rpath,{PKG}", "-o", exe])
    return exe


def test_shim_compiles_and_links(driver):
    assert os.access(driver, os.X_OK)


NAMES = {S.ROLE_TOKEN_EMBD: "token_embd.weight", S.ROLE_OUTPUT_NORM: "output_norm.weight",
         S.ROLE_OUTPUT: "output.weight", S.ROLE_ATTN_NORM: "attn_norm.weight", S.ROLE_ATTN_Q: "attn_q.weight",
         S.ROLE_ATTN_K: "attn_k.weight", S.ROLE_ATTN_V: "attn_v.weight", S.ROLE_ATTN_OUT: "attn_output.weight",
         S.ROLE_FFN_NORM: "ffn_norm.weight", S.ROLE_FFN_GATE: "ffn_gate.weight", S.ROLE_FFN_UP: "ffn_up.weight",
         S.ROLE_FFN_DOWN: "ffn_down.weight"}


def gguf_name(role, layer):
    """The tensor names ModelWeights::build looks up (rawllm_forward.hpp:847-866)."""
    return NAMES[role] if layer < 0 else f"blk.{layer}.{NAMES[role]}"


def test_shim_tensor_names_map_to_roles(driver):
    names = [gguf_name(r, -1 if r < S.ROLE_ATTN_NORM else 17) for r in NAMES]
    names += ["blk.x.attn_q.weight", "blk.3.attn_q.bias", "rope_freqs.weight", "blk..ffn_up.weight"]
    out = subprocess.run([driver, "roles", *names], capture_output=True, text=True, check=True).stdout.split("\n")
    for i, r in enumerate(NAMES):
        assert out[i] == f"{r} {-1 if r < S.ROLE_ATTN_NORM else 17}"
    assert out[len(NAMES):len(NAMES) + 4] == ["none"] * 4


def test_shim_reference_error_before_device_use(driver):
    out = subprocess.run([driver, "badshape"], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert "blk.3.attn_k.weight input dim (100) isn't a multiple of its quant block size (32)" in out.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0])
def test_shim_single_matches_oracle(driver, tmp_path, typ):
    rows, cols, seq = 96, 1024, 2
    W = S.weights(typ, rows, cols, seed=41)
    X = S.activations(seq, cols, seed=42)
    W.tofile(tmp_path / "W.bin")
    X.tofile(tmp_path / "X.bin")
    subprocess.check_call([driver, "single", str(typ), str(rows), str(cols), str(seq), str(tmp_path / "W.bin"),
                           str(tmp_path / "X.bin"), str(tmp_path / "Y.out")])
    Y = np.fromfile(tmp_path / "Y.out", np.float32).reshape(seq, rows)
    assert max_rel_err(Y, O.proj_all_positions(typ, W, rows, cols, X)) <= MATVEC_RTOL


@pytest.mark.gpu
def test_shim_multi_matches_oracle(driver, tmp_path):
    cols, seq = 512, 1
    specs = [(S.GGML_Q4_0, 256), (S.GGML_Q4_0, 128), (S.GGML_Q4_0, 128)]  # Q/K/V-shaped
    X = S.activations(seq, cols, seed=43)
    X.tofile(tmp_path / "X.bin")
    args, Ws = [], []
    for i, (typ, rows) in enumerate(specs):
        W = S.weights(typ, rows, cols, seed=50 + i)
        W.tofile(tmp_path / f"W{i}.bin")
        Ws.append(W)
        args += [str(typ), str(rows), str(tmp_path / f"W{i}.bin")]
    subprocess.check_call([driver, "multi", str(cols), str(seq), str(tmp_path / "X.bin"),
                           str(tmp_path / "Y.out"), *args])
    Y = np.fromfile(tmp_path / "Y.out", np.float32)
    off = 0
    for (typ, rows), W in zip(specs, Ws):
        ref = O.proj_all_positions(typ, W, rows, cols, X)
        assert max_rel_err(Y[off:off + rows * seq], ref) <= MATVEC_RTOL
        off += rows * seq


@pytest.mark.gpu
@pytest.mark.parametrize("plain,wtype,etype,quantize", [
    (False, S.GGML_Q4_0, S.GGML_Q8_0, None), (True, S.GGML_Q4_0, S.GGML_Q8_0, None),
    (False, S.GGML_Q4_K, S.GGML_Q6_K, None),       # a nanity_convert.py --quant Q4_K model
    (False, S.GGML_F32, S.GGML_F32, S.GGML_Q8_0),  # F32 tensors (a .nctr's) quantised on load
], ids=["q4_0", "q4_0-plain", "q4_k", "f32-to-q8_0"])
def test_shim_decoder_from_loader_matches_reference(driver, tmp_path, plain, wtype, etype, quantize):
    """neon_cuda::Decoder built from a loader's GGUF-named tensors and an
    engine::Config gives the reference's greedy tokens."""
    from conftest import MODEL_L2_RTOL, rel_l2

    cfg = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, plain_ffn=plain)
    tensors = list(S.model_tensors(cfg, seed=7, wtype=wtype, embd_type=etype))
    lines = []
    for i, (role, layer, raw, typ, ne0, ne1) in enumerate(tensors):
        np.ascontiguousarray(raw).tofile(tmp_path / f"t{i}.bin")
        lines.append(f"{gguf_name(role, layer)} {typ} {ne0} {ne1} t{i}.bin")
    (tmp_path / "manifest.txt").write_text("\n".join(lines) + "\n")
    (tmp_path / "config.txt").write_text(
        f"{cfg.n_vocab} {cfg.n_embd} {cfg.n_layer} {cfg.n_head} {cfg.n_kv_head} {cfg.head_dim} {cfg.n_ff} "
        f"{cfg.ctx_len} 0 {cfg.rope_base} {cfg.rope_scale} {cfg.rope_dim_count} {cfg.norm_eps} {0 if plain else 1}\n")
    prompt = S.prompt_tokens(8, cfg.n_vocab, 8)
    prompt.astype(np.int32).tofile(tmp_path / "prompt.bin")
    out = subprocess.run([driver, "decode", str(tmp_path), "16"] + ([str(quantize)] if quantize is not None else []),
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    toks = np.fromfile(tmp_path / "tokens.bin", np.int32)
    logits = np.fromfile(tmp_path / "logits.bin", np.float32)
    if quantize is not None:  # the reference runs the tensors an exporter would have written
        N.init(0)
        tensors = [(r, l, N.quantize(raw, t, ne1, ne0, quantize) if ne1 else raw, quantize if ne1 else t, ne0, ne1)
                   for r, l, raw, t, ne0, ne1 in tensors]
    kind = "reference" if O.ref_available() else "port"
    ref = O.Model(cfg, tensors, kind)
    ref_toks, ref_logits = ref.generate_greedy(prompt, 16)
    ref.close()
    assert np.array_equal(toks, ref_toks)
    assert rel_l2(logits, ref_logits[0]) <= MODEL_L2_RTOL
