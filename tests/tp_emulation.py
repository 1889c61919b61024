"""CPU emulation of the tensor-parallel decode, for the gloo tests.

Each rank keeps exactly the parts of the model that the library's shard plan
(neon_cuda_tp_shard, a host-only C function) assigns it, computes every
projection with the oracle's restatement of proj_all_positions (Q8_0
activations, the reference's block arithmetic), the element-wise steps of
transformer_forward (rawllm_forward.hpp:987-1236) in numpy, and sums the
column-split attn_output / ffn_down partials with a torch.distributed
all-reduce, as the CUDA path does with its peer-memory all-reduce. Run with
world 1 it is the unsharded model, so world 1 vs world N isolates what the
split changes: the order of one fp32 sum per residual update.
"""
from __future__ import annotations

import os

import numpy as np

import neon_cuda as NC
import oracle as O
import synth as S


def dequant_row(raw: np.ndarray, typ: int, cols: int, row: int) -> np.ndarray:
    """Row `row` of GGUF bytes `raw` (any weight type), decoded by the oracle."""
    rb = S.row_bytes(typ, cols)
    return O.dequantize_row(typ, np.ascontiguousarray(raw).reshape(-1)[row * rb:(row + 1) * rb], cols)


def shard(raw: np.ndarray, typ: int, ne0: int, ne1: int, rng):
    """Rows [r0, r1) x columns [c0, c1) of GGUF bytes -> (bytes, rows, cols).
    Columns are cut on the type's blocks (32 values; 256 for the K-quants)."""
    r0, r1, c0, c1 = rng
    be, bb = max(32, S.BLOCK_ELEMS[typ]), S.BLOCK_BYTES[typ] * (32 if S.BLOCK_ELEMS[typ] == 1 else 1)
    if c0 % be or c1 % be:
        raise ValueError(f"columns [{c0}, {c1}) do not fall on {be}-value blocks")
    a = np.ascontiguousarray(raw).reshape(ne1, ne0 // be, bb)[r0:r1, c0 // be:c1 // be]
    return np.ascontiguousarray(a).reshape(-1), r1 - r0, c1 - c0


class RankModel:
    def __init__(self, cfg, tensors, rank: int, world: int):
        self.cfg, self.rank, self.world = cfg, rank, world
        self.layers = [dict() for _ in range(cfg.n_layer)]
        self.g = {}
        for role, layer, raw, typ, ne0, ne1 in tensors:
            if typ == S.GGML_F32:
                w = np.frombuffer(np.ascontiguousarray(raw).tobytes(), np.float32)
                (self.g if layer < 0 else self.layers[layer])[role] = w
                continue
            if role == S.ROLE_TOKEN_EMBD:
                self.g["embd"] = (raw, typ, ne0)
                if "head" not in self.g or self.g["head_tied"]:
                    rng = NC.tp_shard(cfg, S.ROLE_OUTPUT, rank, world)
                    self.g["head"] = shard(raw, typ, ne0, ne1, rng) + (typ,)
                    self.g["head_tied"] = True
                    self.g["vocab0"] = rng[0]
                continue
            rng = NC.tp_shard(cfg, role, rank, world)
            entry = shard(raw, typ, ne0, ne1, rng) + (typ,)
            if role == S.ROLE_OUTPUT:
                self.g["head"], self.g["head_tied"], self.g["vocab0"] = entry, False, rng[0]
            else:
                self.layers[layer][role] = entry
        self.n_head_l = cfg.n_head // world
        self.n_kv_l = cfg.n_kv_head // world
        self.K = [[] for _ in range(cfg.n_layer)]
        self.V = [[] for _ in range(cfg.n_layer)]
        hd = cfg.head_dim
        self.freqs = np.array([np.float32(cfg.rope_base) ** np.float32(-2.0 * i / hd) for i in range(hd // 2)],
                              np.float32)
        self.rope_half = (cfg.rope_dim_count or hd) // 2

    @staticmethod
    def proj(entry, x):
        raw, rows, cols, typ = entry
        return O.proj_all_positions(typ, raw, rows, cols, x.reshape(1, -1))[0]

    def rms(self, x, w):
        ss = float(np.sum(x.astype(np.float64) ** 2))
        scale = np.float32(1.0) / np.sqrt(np.float32(ss / x.size) + np.float32(self.cfg.norm_eps))
        return (x * scale * w).astype(np.float32)

    def rope(self, v, n_heads, pos):
        hd = self.cfg.head_dim
        v = v.reshape(n_heads, hd).copy()
        th = np.float32(pos / self.cfg.rope_scale) * self.freqs[:self.rope_half]
        c, s = np.cos(th).astype(np.float32), np.sin(th).astype(np.float32)
        x0, x1 = v[:, 0:2 * self.rope_half:2].copy(), v[:, 1:2 * self.rope_half:2].copy()
        v[:, 0:2 * self.rope_half:2] = x0 * c - x1 * s
        v[:, 1:2 * self.rope_half:2] = x0 * s + x1 * c
        return v.reshape(-1)

    def step(self, tok: int, pos: int, allreduce, allgather) -> np.ndarray:
        cfg, hd = self.cfg, self.cfg.head_dim
        raw, typ, ne0 = self.g["embd"]
        h = dequant_row(raw, typ, ne0, tok)
        group = cfg.n_head // cfg.n_kv_head
        for li, L in enumerate(self.layers):
            xn = self.rms(h, L[S.ROLE_ATTN_NORM])
            q = self.rope(self.proj(L[S.ROLE_ATTN_Q], xn), self.n_head_l, pos)
            k = self.rope(self.proj(L[S.ROLE_ATTN_K], xn), self.n_kv_l, pos)
            v = self.proj(L[S.ROLE_ATTN_V], xn)
            self.K[li].append(k.reshape(self.n_kv_l, hd))
            self.V[li].append(v.reshape(self.n_kv_l, hd))
            Kc, Vc = np.stack(self.K[li]), np.stack(self.V[li])  # (L, n_kv_l, hd)
            att = np.zeros(self.n_head_l * hd, np.float32)
            for hh in range(self.n_head_l):
                kvh = hh // group
                sc = (Kc[:, kvh, :].astype(np.float64) @ q[hh * hd:(hh + 1) * hd]) / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                att[hh * hd:(hh + 1) * hd] = (p / p.sum()) @ Vc[:, kvh, :]
            h = h + allreduce(self.proj(L[S.ROLE_ATTN_OUT], att))
            xn = self.rms(h, L[S.ROLE_FFN_NORM])
            g = self.proj(L[S.ROLE_FFN_GATE], xn)
            u = self.proj(L[S.ROLE_FFN_UP], xn)
            act = (g / (1.0 + np.exp(-g.astype(np.float64))) * u).astype(np.float32)
            h = (h + allreduce(self.proj(L[S.ROLE_FFN_DOWN], act))).astype(np.float32)
        logits_l = self.proj(self.g["head"], self.rms(h, self.g[S.ROLE_OUTPUT_NORM]))
        return allgather(logits_l)

    def generate(self, prompt, n_new, allreduce, allgather):
        logits = None
        pos = 0
        for t in prompt:
            logits = self.step(int(t), pos, allreduce, allgather)
            pos += 1
        toks, all_logits = [], []
        for _ in range(n_new):
            all_logits.append(logits)
            tok = int(np.argmax(logits))
            toks.append(tok)
            logits = self.step(tok, pos, allreduce, allgather)
            pos += 1
        return np.array(toks, np.int32), np.stack(all_logits)


def worker(rank: int, world: int, port: int, out_dir: str, cfg_args, seed: int, n_prompt: int, n_new: int,
           wtype: int = S.GGML_Q4_0, embd_type: int = S.GGML_Q8_0):
    """torch.multiprocessing entry: one gloo rank of the emulated TP decode."""
    import torch
    import torch.distributed as dist

    os.environ.setdefault("OMP_NUM_THREADS", "1")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = S.ModelConfig(*cfg_args[0], **cfg_args[1])

        def allreduce(x):
            t = torch.from_numpy(np.ascontiguousarray(x, np.float32).copy())
            dist.all_reduce(t)
            return t.numpy()

        def allgather(x):
            parts = [None] * world
            dist.all_gather_object(parts, np.asarray(x, np.float32))
            return np.concatenate(parts)

        m = RankModel(cfg, S.model_tensors(cfg, seed, wtype=wtype, embd_type=embd_type), rank, world)
        prompt = S.prompt_tokens(n_prompt, cfg.n_vocab, seed + 1)
        toks, logits = m.generate(prompt, n_new, allreduce, allgather)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), tokens=toks, logits=logits)
    finally:
        dist.destroy_process_group()
