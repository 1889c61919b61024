"""Writes .nctr files for the tests: the container export_nctr produces
(train_nanity_fixed.py:1259-1433) -- a 116-byte NCTRHeader, a JSON manifest,
a JSON tokenizer section, the positional tensor table of 20-byte slots and the
F32 tensor data -- filled with a seeded synthetic model (no checkpoint exists
here). Test infrastructure."""
from __future__ import annotations

import json
import struct

import numpy as np

import synth as S

HEADER = struct.Struct("<4s10Iff I f II 6Q")


def write_nctr(path, cfg, seed=5, has_output=False, spec_version=1, magic=b"NCTR", truncate=0, vocab_tokens=None):
    """A .nctr of `cfg` (synth.ModelConfig) with F32 tensors; returns the
    tensor list (role, layer, float32 bytes, type, ne0, ne1) in file order."""
    tensors = list(S.model_tensors(cfg, seed=seed, wtype=S.GGML_F32, embd_type=S.GGML_F32, tied=not has_output))
    # the file's positional order (rawllm_nctr_loader.hpp:217-235)
    order = {S.ROLE_TOKEN_EMBD: 0, S.ROLE_OUTPUT_NORM: 1, S.ROLE_OUTPUT: 2}
    per_layer = [S.ROLE_ATTN_NORM, S.ROLE_ATTN_Q, S.ROLE_ATTN_K, S.ROLE_ATTN_V, S.ROLE_ATTN_OUT, S.ROLE_FFN_NORM,
                 S.ROLE_FFN_GATE, S.ROLE_FFN_UP, S.ROLE_FFN_DOWN]
    tensors.sort(key=lambda t: (t[1] + 1, order.get(t[0], per_layer.index(t[0]) if t[0] in per_layer else 99)))
    manifest = json.dumps({"nctr_manifest_version": 1, "note": "synthetic test model", "seed": seed}).encode()
    toks = vocab_tokens if vocab_tokens is not None else [f"t{i}" for i in range(cfg.n_vocab)]
    tokenizer = json.dumps({"tokens": toks, "merges": [], "bos_id": 1, "eos_id": 2, "unk_id": 0}).encode()
    blobs, table, cursor = [], [], 0
    for t in tensors:
        raw = np.ascontiguousarray(t[2]).view(np.uint8).reshape(-1).tobytes()
        table.append(struct.pack("<IQQ", 0, cursor, len(raw)))
        blobs.append(raw)
        cursor += len(raw)
    man_off = HEADER.size
    tok_off = man_off + len(manifest)
    table_off = tok_off + len(tokenizer)
    data_off = table_off + len(table) * 20
    flags = (0 if cfg.plain_ffn else 1) | (2 if has_output else 0)
    header = HEADER.pack(magic, 1, spec_version, cfg.n_vocab, cfg.n_embd, cfg.n_layer, cfg.n_head, cfg.n_kv_head,
                         cfg.head_dim, cfg.n_ff, cfg.ctx_len, cfg.rope_base, cfg.rope_scale, cfg.rope_dim_count,
                         cfg.norm_eps, flags, 32, man_off, len(manifest), tok_off, len(tokenizer), table_off,
                         data_off)
    data = header + manifest + tokenizer + b"".join(table) + b"".join(blobs)
    with open(path, "wb") as f:
        f.write(data[:len(data) - truncate] if truncate else data)
    return tensors
