"""On-load quantisation on the device, and .nctr / .gguf models on the GPU.

* neon_cuda_quantize_rows / _host: byte for byte what gguf-py's
  gguf.quants.quantize (the reference exporters' quantiser) writes
  (tests/golden/quant_gguf.npz);
* neon_cuda_upload_quantized: the quantised tensor's matvec against the oracle
  on those bytes, whole and column-sharded;
* a .nctr model (F32, as export_nctr writes it) decoded on the device as is
  and quantised on load to Q8_0 / Q4_0: the oracle's greedy tokens on the same
  weights, logits within 1e-3 relative L2 (Q4_0: the whole-model bar, its
  activations are quantised);
* a .gguf model written by gguf-py and read by neon_cuda.load_gguf, likewise."""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, MODEL_L2_RTOL, load_golden, max_rel_err, rel_l2
from nctr_file import write_nctr

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

QTYPES = (S.GGML_Q8_0, S.GGML_Q4_0, S.GGML_Q4_1, S.GGML_Q5_0, S.GGML_Q5_1, S.GGML_F16, S.GGML_BF16)
ids = lambda t: S.TYPE_NAMES[t]  # noqa: E731
TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available()
    N.init(0)


@pytest.mark.parametrize("dst", QTYPES, ids=ids)
def test_device_quantize_matches_gguf(dst):
    g = load_golden("quant_gguf.npz")
    x = g["x"]
    assert np.array_equal(N.quantize(x, S.GGML_F32, x.shape[0], x.shape[1], dst), g[f"q{dst}"])
    # the device-buffer entry point on a stream
    dx = torch.from_numpy(x.copy()).cuda()
    dy = torch.zeros(g[f"q{dst}"].size, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream()
    N._check(N.load().neon_cuda_quantize_rows(dx.data_ptr(), S.GGML_F32, x.shape[0], x.shape[1], dst,
                                              dy.data_ptr(), s.cuda_stream))
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy(), g[f"q{dst}"].reshape(-1))


@pytest.mark.parametrize("dst", [S.GGML_Q8_0, S.GGML_Q4_0, S.GGML_Q5_1, S.GGML_BF16], ids=ids)
def test_upload_quantized_matvec(dst):
    rows, cols = 1000, 2048
    x = (np.random.default_rng(dst).standard_normal((rows, cols)) * 0.05).astype(np.float32)
    q = N.quantize(x, S.GGML_F32, rows, cols, dst)
    X = S.activations(1, cols, seed=3)
    want = O.proj_all_positions(dst, q, rows, cols, X)
    dt = N.upload_quantized(x, S.GGML_F32, rows, cols, dst)
    assert (dt.rows, dt.cols, dt.type) == (rows, cols, dst)
    dx = torch.from_numpy(X.copy()).cuda()
    dy = torch.zeros(rows, device="cuda")
    dt.matvec(dx, dy)
    torch.cuda.synchronize()
    assert max_rel_err(dy.cpu().numpy(), want) <= MATVEC_RTOL
    # column shards of the quantised tensor add up to the whole
    parts = []
    for i in range(2):
        sh = N.upload_quantized(x, S.GGML_F32, rows, cols, dst, N.SHARD_COLS, i, 2)
        dxs = torch.from_numpy(X[:, i * cols // 2:(i + 1) * cols // 2].copy()).cuda()
        dys = torch.zeros(rows, device="cuda")
        sh.matvec(dxs, dys)
        torch.cuda.synchronize()
        parts.append(dys.cpu().numpy())
    assert max_rel_err(parts[0] + parts[1], want) <= MATVEC_RTOL


@pytest.mark.parametrize("quant", [None, S.GGML_Q8_0, S.GGML_Q4_0], ids=["F32", "Q8_0", "Q4_0"])
def test_nctr_model_decodes_like_the_oracle(tmp_path, quant):
    path = str(tmp_path / "m.nctr")
    write_nctr(path, TINY, has_output=True)
    c, tensors = N.load_nctr(path)
    m = N.Model(c, tensors, quantize=quant)
    if quant is None:
        oracle_tensors = tensors
    else:  # the oracle runs the tensor the exporter would have written (device quantiser == gguf-py)
        oracle_tensors = [(r, l, N.quantize(np.asarray(raw), t, ne1, ne0, quant) if ne1 else raw,
                           quant if ne1 else t, ne0, ne1) for r, l, raw, t, ne0, ne1 in tensors]
    o = O.Model(TINY.with_(ctx_len=c.ctx_len), oracle_tensors, "port")
    prompt = S.prompt_tokens(9, TINY.n_vocab, 19)
    want_toks, want_logits = o.generate_greedy(prompt, 6)
    assert np.array_equal(m.generate(prompt, 6), want_toks)
    m.set_length(0)
    got = [m.forward(prompt)] + [m.forward([t]) for t in want_toks[:5]]
    bar = MODEL_L2_RTOL if quant == S.GGML_Q4_0 else 1e-3
    for i, (a, b) in enumerate(zip(got, want_logits)):
        assert rel_l2(a, b) <= bar, f"step {i}"
    m.free()


@pytest.mark.parametrize("ntype", [None, S.GGML_F16], ids=["f32-norms", "f16-norms"])
def test_gguf_model_decodes_like_the_oracle(tmp_path, ntype):
    """A .gguf file written by gguf-py, read by neon_cuda.load_gguf, decoded on
    the device: the oracle's greedy tokens on the same tensors (norm weights
    F32, or F16 as some converters write them)."""
    pytest.importorskip("gguf")
    from gguf_file import write_gguf

    path = str(tmp_path / "m.gguf")
    write_gguf(path, TINY, wtype=S.GGML_Q4_K, embd_type=S.GGML_Q6_K, tied=False, norm_type=ntype)
    c, tensors = N.load_gguf(path)
    m = N.Model(c, tensors)
    o = O.Model(TINY.with_(ctx_len=c.ctx_len), tensors, "port")
    prompt = S.prompt_tokens(9, TINY.n_vocab, 21)
    want_toks, want_logits = o.generate_greedy(prompt, 6)
    assert np.array_equal(m.generate(prompt, 6), want_toks)
    m.set_length(0)
    assert rel_l2(m.forward(prompt), want_logits[0]) <= 1e-3
    m.free()
