""".nctr models (the reference's F32 export container): the package's reader
(neon_cuda.load_nctr) against the reference's own loader::NCTRLoader
(rawllm_nctr_loader.hpp, compiled into oracle/_ref): the same tensors, names,
shapes, offsets, configuration, tokenizer ids and error messages; and the
decode step of the oracle over the file's tensors against the reference's."""
import ctypes as C
import os

import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from nctr_file import write_nctr

TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")
NAMES = {0: "token_embd", 1: "output_norm", 2: "output", 3: "attn_norm", 4: "attn_q", 5: "attn_k", 6: "attn_v",
         7: "attn_output", 8: "ffn_norm", 9: "ffn_gate", 10: "ffn_up", 11: "ffn_down"}
ref_only = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def ref_lib():
    R = O.ref()
    R.ref_nctr_open.argtypes = [C.c_char_p]
    R.ref_nctr_open.restype = C.c_void_p
    R.ref_nctr_free.argtypes = [C.c_void_p]
    R.ref_nctr_count.argtypes = [C.c_void_p]
    R.ref_nctr_count.restype = C.c_size_t
    u64 = C.POINTER(C.c_uint64)
    R.ref_nctr_tensor.argtypes = [C.c_void_p, C.c_size_t, C.c_char_p, C.c_size_t, u64, u64, C.POINTER(C.c_int),
                                  u64, u64]
    R.ref_nctr_config.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_int),
                                  C.POINTER(C.c_int), C.POINTER(C.c_size_t)]
    return R


@pytest.mark.parametrize("cfg,has_output", [(TINY, False), (TINY.with_(plain_ffn=True), True),
                                            (TINY.with_(ctx_len=5000), False)])
def test_reader_matches_written_file(tmp_path, cfg, has_output):
    path = str(tmp_path / "m.nctr")
    written = write_nctr(path, cfg, has_output=has_output)
    c, tensors = N.load_nctr(path)
    assert len(tensors) == len(written) == 2 + has_output + cfg.n_layer * (8 + (0 if cfg.plain_ffn else 1))
    for (r, l, raw, t, ne0, ne1), w in zip(tensors, written):
        assert (r, l, t, ne0, ne1) == (w[0], w[1], S.GGML_F32, w[4], w[5])
        assert np.array_equal(np.asarray(raw), np.ascontiguousarray(w[2]).view(np.uint8).reshape(-1))
    for f in ("n_vocab", "n_embd", "n_layer", "n_head", "n_kv_head", "head_dim", "n_ff", "rope_dim_count"):
        assert getattr(c, f) == getattr(cfg, f)
    assert c.plain_ffn == cfg.plain_ffn and c.context_length == cfg.ctx_len and c.ctx_len == min(cfg.ctx_len, 4096)
    assert (c.bos_id, c.eos_id, c.n_tokens) == (1, 2, cfg.n_vocab)


@ref_only
@pytest.mark.parametrize("cfg,has_output", [(TINY, False), (TINY.with_(plain_ffn=True), True),
                                            (TINY.with_(ctx_len=5000), False)])
def test_reader_matches_reference_loader(tmp_path, cfg, has_output):
    R = ref_lib()
    path = str(tmp_path / "m.nctr")
    write_nctr(path, cfg, has_output=has_output)
    c, tensors = N.load_nctr(path)
    h = R.ref_nctr_open(path.encode())
    assert h, R.ref_last_error()
    try:
        assert R.ref_nctr_count(h) == len(tensors)
        mm = np.memmap(path, np.uint8, mode="r")
        for i, (r, l, raw, t, ne0, ne1) in enumerate(tensors):
            name = C.create_string_buffer(128)
            a, b, off, nb = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
            typ = C.c_int()
            R.ref_nctr_tensor(h, i, name, 128, C.byref(a), C.byref(b), C.byref(typ), C.byref(off), C.byref(nb))
            want = NAMES[r] + ".weight" if l < 0 else f"blk.{l}.{NAMES[r]}.weight"
            assert name.value.decode() == want
            assert (a.value, b.value, typ.value, nb.value) == (ne0, ne1, t, raw.size)
            assert np.array_equal(np.asarray(mm[off.value:off.value + nb.value]), np.asarray(raw))
        cfgbuf = (C.c_uint32 * 16)()
        hdr_ctx, bos, eos, ntok = C.c_uint32(), C.c_int(), C.c_int(), C.c_size_t()
        assert R.ref_nctr_config(h, cfgbuf, C.byref(hdr_ctx), C.byref(bos), C.byref(eos), C.byref(ntok)) == 0
        ints = list(cfgbuf)
        assert ints[:8] == [c.n_vocab, c.n_embd, c.n_layer, c.n_head, c.n_kv_head, c.head_dim, c.n_ff, c.ctx_len]
        assert ints[10] == c.rope_dim_count and ints[12] == int(c.plain_ffn)
        assert (hdr_ctx.value, bos.value, eos.value, ntok.value) == (c.context_length, c.bos_id, c.eos_id,
                                                                      c.n_tokens)
    finally:
        R.ref_nctr_free(h)


@ref_only
@pytest.mark.parametrize("kw", [dict(magic=b"GGUF"), dict(spec_version=2), dict(truncate=100)])
def test_errors_match_reference_loader(tmp_path, kw):
    R = ref_lib()
    path = str(tmp_path / "bad.nctr")
    write_nctr(path, TINY, **kw)
    assert not R.ref_nctr_open(path.encode())
    ref_msg = R.ref_last_error().decode()
    with pytest.raises(RuntimeError) as e:
        N.load_nctr(path)
    assert str(e.value) == ref_msg


@ref_only
def test_oracle_decode_over_nctr_tensors_matches_reference(tmp_path):
    path = str(tmp_path / "m.nctr")
    write_nctr(path, TINY, has_output=True)
    c, tensors = N.load_nctr(path)
    cfg = TINY.with_(ctx_len=c.ctx_len)
    mo, mr = O.Model(cfg, tensors, "port"), O.Model(cfg, tensors, "reference", threads=2)
    p = S.prompt_tokens(6, cfg.n_vocab, 4)
    ta, la = mo.generate_greedy(p, 4)
    tb, lb = mr.generate_greedy(p, 4)
    assert np.array_equal(ta, tb) and np.array_equal(la.view(np.uint32), lb.view(np.uint32))


REF_TREE = O.ref_tree()


@pytest.mark.skipif(not REF_TREE or not os.path.exists(os.path.join(REF_TREE, "rawllm_nctr_loader.hpp")),
                    reason="reference tree not present")
@pytest.mark.parametrize("plain_ffn,has_output", [(False, False), (True, True)])
def test_cpp_decoder_roles_from_reference_nctr_loader(tmp_path, plain_ffn, has_output):
    """The C++ adapter compiles with the reference's loader::NCTRLoader and maps
    every .nctr tensor to the role neon_cuda::Decoder uploads it as (and the
    header to the model configuration)."""
    import subprocess

    from conftest import PKG, ROOT
    exe = str(tmp_path / "nctr_roles")
    N.load()
    subprocess.check_call(["g++", "-std=c++17", "-O1", os.path.join(ROOT, "tests", "cpp", "nctr_roles.cpp"),
                           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(PKG, "host"), "-I", REF_TREE,
                           "-L", PKG, "-lneon_cuda", f"-Wl,-rpath,{PKG}", "-lpthread", "-o", exe])
    cfg = TINY.with_(plain_ffn=plain_ffn)
    path = str(tmp_path / "m.nctr")
    write_nctr(path, cfg, has_output=has_output)
    lines = subprocess.run([exe, path], capture_output=True, text=True, check=True).stdout.splitlines()
    c, tensors = N.load_nctr(path)
    assert lines[0].split()[1:] == [str(v) for v in (c.n_vocab, c.n_embd, c.n_layer, c.n_head, c.n_kv_head,
                                                     c.head_dim, c.n_ff, c.ctx_len, int(c.plain_ffn))]
    assert len(lines) - 1 == len(tensors)
    for line, (r, l, raw, t, ne0, ne1) in zip(lines[1:], tensors):
        f = line.split()
        assert [int(v) for v in f[1:]] == [r, l, ne0, ne1, t, raw.size], line
