"""One rank of the tensor-parallel GPU tests (launched by test_tp_gpu.py under
torch.distributed.run, one process per GPU; gloo carries only the IPC handles
and the host-side checks).

Writes rank 0's observations to --out (npz): the all-reduce results against
their exact host sums, every rank's output of the all-gathered row-sharded
matvecs, the small model's greedy tokens and per-step logits,
and the Qwen3-0.6B-shaped decoder's tokens split over the ranks and on one GPU.
"""
from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "neon-runtime-beta-variation_b200"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import neon_cuda as NC  # noqa: E402
import synth as S  # noqa: E402

TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")


def allreduce_cases(comm, rank, world, dev):
    """(name, max |got - want|) for sums whose host value is exact (rank order)."""
    out = []
    for name, n, off, add in (("n4096", 4096, 0, True), ("n1", 1, 0, False), ("ragged", 1000003, 0, True),
                              ("unaligned", 777, 1, True), ("prefill", 256 * 1024, 0, False)):
        g = torch.Generator().manual_seed(1234 + 17 * rank + n)
        x_h = torch.randn(n + off, generator=g)
        base_h = torch.randn(n + off, generator=torch.Generator().manual_seed(99 + n))
        x = x_h.to(dev)
        o = base_h.to(dev)
        xs, os_ = x[off:], o[off:]
        dist.barrier()
        comm.allreduce(xs, os_, n=n, add=add, stream=torch.cuda.current_stream(dev))
        torch.cuda.synchronize(dev)
        comm.check()
        parts = [None] * world
        dist.all_gather_object(parts, x_h[off:].numpy())
        s = parts[0].astype(np.float32).copy()
        for p in parts[1:]:
            s = (s + p).astype(np.float32)
        want = (base_h[off:].numpy() + s).astype(np.float32) if add else s
        out.append((name, float(np.max(np.abs(os_.cpu().numpy() - want)))))
    return out


ALLGATHER_CASES = (("q4_0_4096", S.GGML_Q4_0, 4096, 4096), ("q8_0_ragged", S.GGML_Q8_0, 1001, 1024),
                   ("q4_k", S.GGML_Q4_K, 512, 2048), ("tiny", S.GGML_Q4_0, 3, 64))


def allgather_cases(comm, rank, world, dev, res):
    """Row-sharded matvecs with the output all-gathered: every rank's y for
    three calls in a row (the first two on the same X, the third after an
    all-reduce on the same communicator); rank 0 keeps its own and rank 1's."""
    for name, typ, rows, cols in ALLGATHER_CASES:
        W = S.weights(typ, rows, cols, seed=rows + cols)
        dt = NC.DeviceTensor(W, typ, rows, cols, NC.SHARD_ROWS, rank, world)
        row0 = rows * rank // world
        X = S.activations(1, cols, seed=cols)
        x = torch.from_numpy(X[0]).to(dev)
        ys = []
        for call in range(3):
            if call == 2:
                t = torch.ones(8, device=dev)
                comm.allreduce(t, t, stream=torch.cuda.current_stream(dev))
            y = torch.full((rows,), float("nan"), device=dev)
            dist.barrier()
            comm.matvec_allgather(dt, x, y, rows, row0, stream=torch.cuda.current_stream(dev))
            torch.cuda.synchronize(dev)
            ys.append(y.cpu().numpy())
        comm.check()
        parts = [None] * world
        dist.all_gather_object(parts, np.stack(ys))
        res[f"allgather_{name}"] = np.stack(parts)  # [rank][call][rows]
        dt.free()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--qwen-prompt", type=int, default=128)
    ap.add_argument("--qwen-steps", type=int, default=32)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    NC.init(local)
    res = {}
    qwen = S.QWEN3_0_6B.with_(ctx_len=a.qwen_prompt + a.qwen_steps + 1)
    floats = max(NC.model_comm_floats(TINY, world), NC.model_comm_floats(qwen, world), 1000003)
    comm = NC.Comm.from_process_group(floats)
    comm.set_timeout(20.0)
    try:
        for name, err in allreduce_cases(comm, rank, world, dev):
            res[f"allreduce_{name}"] = np.array(err)
        allgather_cases(comm, rank, world, dev, res)

        # small model: greedy tokens, then logits step by step
        from conftest import load_golden  # noqa: E402

        g = load_golden("decode_tiny.npz")
        m = NC.Model(TINY, S.model_tensors(TINY, seed=3), comm)
        dist.barrier()
        res["tiny_tokens"] = m.generate(g["prompt"], 16)
        for fused in (True, False):
            NC.set_fused_collectives(fused)
            m.set_length(0)
            dist.barrier()
            logits = [m.forward(g["prompt"])]
            for t in g["tokens"][:8]:
                logits.append(m.forward([t]))
            res["tiny_logits" if fused else "tiny_logits_unfused"] = np.stack(logits)
        NC.set_fused_collectives(True)
        k, v = m.read_kv(0, len(g["prompt"]))
        res["tiny_k0_shape"] = np.array(k.shape)
        m.free()

        # Qwen3-0.6B-shaped decoder split over the ranks
        tensors = list(S.model_tensors(qwen, seed=21))
        prompt = S.prompt_tokens(a.qwen_prompt, qwen.n_vocab, 22)
        m = NC.Model(qwen, tensors, comm)
        for fused in (False, True):
            NC.set_fused_collectives(fused)
            m.set_length(0)
            dist.barrier()
            toks = m.generate(prompt, a.qwen_steps)
            if fused:
                res["qwen_tokens"], res["qwen_tp_ms"] = toks, np.array(m.decode_ms)
            else:
                res["qwen_tokens_unfused"], res["qwen_tp_unfused_ms"] = toks, np.array(m.decode_ms)
        m.free()
        comm.check()
        dist.barrier()
        if rank == 0:
            m1 = NC.Model(qwen, tensors)
            res["qwen_tokens_1gpu"] = m1.generate(prompt, a.qwen_steps)
            res["qwen_1gpu_ms"] = np.array(m1.decode_ms)
            m1.free()
            np.savez(a.out, **res)
        dist.barrier()
    finally:
        comm.free()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
