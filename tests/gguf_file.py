"""Writes NANITY .gguf files for the tests with gguf-py's GGUFWriter (the
writer export_gguf and nanity_convert.py use: train_nanity_fixed.py:1180-1250,
nanity_convert.py) -- the nanity.* metadata validate_config reads and a seeded
synthetic model's tensors (no checkpoint exists here). Test infrastructure."""
from __future__ import annotations

import numpy as np

import synth as S

NAMES = {S.ROLE_TOKEN_EMBD: "token_embd", S.ROLE_OUTPUT_NORM: "output_norm", S.ROLE_OUTPUT: "output",
         S.ROLE_ATTN_NORM: "attn_norm", S.ROLE_ATTN_Q: "attn_q", S.ROLE_ATTN_K: "attn_k", S.ROLE_ATTN_V: "attn_v",
         S.ROLE_ATTN_OUT: "attn_output", S.ROLE_FFN_NORM: "ffn_norm", S.ROLE_FFN_GATE: "ffn_gate",
         S.ROLE_FFN_UP: "ffn_up", S.ROLE_FFN_DOWN: "ffn_down"}


def tensor_name(role, layer):
    return f"{NAMES[role]}.weight" if layer < 0 else f"blk.{layer}.{NAMES[role]}.weight"


def write_gguf(path, cfg, seed=5, wtype=S.GGML_Q4_0, embd_type=S.GGML_Q8_0, tied=True, arch="nanity",
               spec_version=1, drop_key=None, bad_shape=None, vocab_size=None, alignment=None, norm_type=None):
    """A NANITY .gguf of `cfg`; returns the tensor list (role, layer, bytes,
    type, ne0, ne1) as synth.model_tensors made it (norm weights of
    `norm_type` when given: 1-D tensors of that type)."""
    import gguf
    from gguf.constants import GGMLQuantizationType as Q

    w = gguf.GGUFWriter(path, arch=arch)
    keys = [("nanity.spec_version", spec_version), ("nanity.embedding_length", cfg.n_embd),
            ("nanity.block_count", cfg.n_layer), ("nanity.attention.head_count", cfg.n_head),
            ("nanity.attention.head_count_kv", cfg.n_kv_head), ("nanity.attention.key_length", cfg.head_dim),
            ("nanity.feed_forward_length", cfg.n_ff), ("nanity.context_length", cfg.ctx_len)]
    for k, v in keys:
        if k != drop_key:
            w.add_uint32(k, int(v))
    w.add_float32("nanity.attention.layer_norm_rms_epsilon", cfg.norm_eps)
    w.add_float32("nanity.rope.freq_base", cfg.rope_base)
    if vocab_size is not None:
        w.add_uint32("nanity.vocab_size", vocab_size)
    if alignment is not None:
        w.add_custom_alignment(alignment)
    w.add_token_list([f"t{i}" for i in range(cfg.n_vocab)])
    w.add_bos_token_id(1)
    w.add_eos_token_id(2)
    tensors = list(S.model_tensors(cfg, seed=seed, wtype=wtype, embd_type=embd_type, tied=tied, norm_type=norm_type))
    for role, layer, raw, typ, ne0, ne1 in tensors:
        name = tensor_name(role, layer)
        a = np.ascontiguousarray(raw).view(np.uint8)
        if (role, layer) == bad_shape:
            ne1 = ne1 // 2  # half the rows: a shape validate_config refuses
            a = a.reshape(-1)[:a.size // 2]
        if typ == S.GGML_F32:
            arr = a.view(np.float32).reshape((ne1, ne0) if ne1 else (ne0,))
            w.add_tensor(name, arr)
        elif ne1 == 0:  # a 1-D tensor of another type: its bytes, shape from the type's block size
            w.add_tensor(name, a.view(np.float16) if typ == S.GGML_F16 else a, raw_dtype=None if typ == S.GGML_F16
                         else Q(typ))
        else:
            w.add_tensor(name, a.reshape(ne1, -1), raw_dtype=Q(typ))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors
