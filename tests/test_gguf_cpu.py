""".gguf models read by the package (neon_cuda.load_gguf) against the
reference's own loader::GGUFLoader (rawllm_loader.hpp, compiled into
oracle/_ref): files written with gguf-py's GGUFWriter give the same tensors,
shapes, types, data and validated configuration, and the same error messages;
the oracle's decode over the reader's tensors equals the reference's."""
import ctypes as C

import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S

gguf = pytest.importorskip("gguf")
from gguf_file import tensor_name, write_gguf  # noqa: E402

TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")
ref_only = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def ref_lib():
    R = O.ref()
    R.ref_gguf_open.argtypes = [C.c_char_p]
    R.ref_gguf_open.restype = C.c_void_p
    R.ref_gguf_free.argtypes = [C.c_void_p]
    R.ref_gguf_count.argtypes = [C.c_void_p]
    R.ref_gguf_count.restype = C.c_size_t
    u64 = C.POINTER(C.c_uint64)
    R.ref_gguf_tensor.argtypes = [C.c_void_p, C.c_size_t, C.c_char_p, C.c_size_t, u64, u64, C.POINTER(C.c_int),
                                  C.POINTER(C.c_int64), u64]
    R.ref_gguf_config.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_int),
                                  C.POINTER(C.c_int)]
    return R


MODELS = [(S.GGML_Q4_0, S.GGML_Q8_0, True, None), (S.GGML_Q4_K, S.GGML_Q6_K, False, None),
          (S.GGML_F16, S.GGML_F16, True, None), (S.GGML_Q4_0, S.GGML_Q8_0, True, S.GGML_F16),
          (S.GGML_Q4_K, S.GGML_Q6_K, False, S.GGML_BF16)]
ids = ["q4_0", "q4_k", "f16", "q4_0-f16-norms", "q4_k-bf16-norms"]


@pytest.mark.parametrize("wtype,etype,tied,ntype", MODELS, ids=ids)
def test_reader_returns_the_written_tensors(tmp_path, wtype, etype, tied, ntype):
    path = str(tmp_path / "m.gguf")
    written = write_gguf(path, TINY, wtype=wtype, embd_type=etype, tied=tied, alignment=64, norm_type=ntype)
    c, tensors = N.load_gguf(path)
    got = {(r, l): (raw, t, ne0, ne1) for r, l, raw, t, ne0, ne1 in tensors}
    assert len(got) == len(written)
    for r, l, raw, t, ne0, ne1 in written:
        g = got[(r, l)]
        assert g[1:] == (t, ne0, ne1)
        assert np.array_equal(np.asarray(g[0]), np.ascontiguousarray(raw).view(np.uint8).reshape(-1))
    for f in ("n_vocab", "n_embd", "n_layer", "n_head", "n_kv_head", "head_dim", "n_ff"):
        assert getattr(c, f) == getattr(TINY, f)
    assert c.ctx_len == TINY.ctx_len and not c.plain_ffn and (c.bos_id, c.eos_id) == (1, 2)
    assert c.rope_base == np.float32(TINY.rope_base) and c.norm_eps == np.float32(TINY.norm_eps)


@ref_only
@pytest.mark.parametrize("wtype,etype,tied,ntype", MODELS, ids=ids)
def test_reader_matches_reference_loader(tmp_path, wtype, etype, tied, ntype):
    R = ref_lib()
    path = str(tmp_path / "m.gguf")
    write_gguf(path, TINY, wtype=wtype, embd_type=etype, tied=tied, norm_type=ntype)
    c, tensors = N.load_gguf(path)
    h = R.ref_gguf_open(path.encode())
    assert h, R.ref_last_error()
    try:
        n = R.ref_gguf_count(h)
        ref = {}
        for i in range(n):
            name = C.create_string_buffer(128)
            a, b, nb = C.c_uint64(), C.c_uint64(), C.c_uint64()
            typ, off = C.c_int(), C.c_int64()
            R.ref_gguf_tensor(h, i, name, 128, C.byref(a), C.byref(b), C.byref(typ), C.byref(off), C.byref(nb))
            ref[name.value.decode()] = (a.value, b.value, typ.value, off.value, nb.value)
        base = None
        for r, l, raw, t, ne0, ne1 in tensors:
            a, b, typ, off, nb = ref[tensor_name(r, l)]
            addr = np.asarray(raw).__array_interface__["data"][0]
            if base is None:
                base = addr - off
            assert (a, b, typ, nb) == (ne0, ne1, t, raw.size) and addr - base == off
        cfgbuf = (C.c_uint32 * 16)()
        hdr_ctx, bos, eos = C.c_uint32(), C.c_int(), C.c_int()
        assert R.ref_gguf_config(h, cfgbuf, C.byref(hdr_ctx), C.byref(bos), C.byref(eos)) == 0
        ints = list(cfgbuf)
        assert ints[:8] == [c.n_vocab, c.n_embd, c.n_layer, c.n_head, c.n_kv_head, c.head_dim, c.n_ff, c.ctx_len]
        assert (hdr_ctx.value, bos.value, eos.value) == (c.context_length, c.bos_id, c.eos_id)
    finally:
        R.ref_gguf_free(h)


def _corrupt_magic(path):
    with open(path, "r+b") as f:
        f.write(b"GGUX")


def _truncate(path):
    with open(path, "r+b") as f:
        f.truncate(f.seek(0, 2) - 100)


@ref_only
@pytest.mark.parametrize("kw,post", [
    (dict(), _corrupt_magic), (dict(), _truncate), (dict(arch="llama"), None), (dict(spec_version=2), None),
    (dict(drop_key="nanity.attention.head_count_kv"), None), (dict(vocab_size=999), None),
    (dict(bad_shape=(S.ROLE_FFN_UP, 1)), None),
], ids=["magic", "truncated", "arch", "spec", "missing-key", "vocab-size", "shape"])
def test_errors_match_reference_loader(tmp_path, kw, post):
    R = ref_lib()
    path = str(tmp_path / "bad.gguf")
    write_gguf(path, TINY, **kw)
    if post:
        post(path)
    h = R.ref_gguf_open(path.encode())
    if h:  # opened: the error comes from validate_config
        cfgbuf = (C.c_uint32 * 16)()
        x, y, z = C.c_uint32(), C.c_int(), C.c_int()
        assert R.ref_gguf_config(h, cfgbuf, C.byref(x), C.byref(y), C.byref(z)) != 0
        R.ref_gguf_free(h)
    ref_msg = R.ref_last_error().decode()
    with pytest.raises(RuntimeError) as e:
        N.load_gguf(path)
    assert str(e.value) == ref_msg


@ref_only
@pytest.mark.parametrize("ntype", [None, S.GGML_F16], ids=["f32-norms", "f16-norms"])
def test_oracle_decode_over_gguf_tensors_matches_reference(tmp_path, ntype):
    path = str(tmp_path / "m.gguf")
    write_gguf(path, TINY, wtype=S.GGML_Q4_K, embd_type=S.GGML_Q6_K, tied=False, norm_type=ntype)
    c, tensors = N.load_gguf(path)
    cfg = TINY.with_(ctx_len=c.ctx_len)
    mo, mr = O.Model(cfg, tensors, "port"), O.Model(cfg, tensors, "reference", threads=2)
    p = S.prompt_tokens(6, cfg.n_vocab, 4)
    ta, la = mo.generate_greedy(p, 4)
    tb, lb = mr.generate_greedy(p, 4)
    assert np.array_equal(ta, tb) and np.array_equal(la.view(np.uint32), lb.view(np.uint32))
