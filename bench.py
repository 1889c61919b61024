#!/usr/bin/env python
"""Benchmark of the quantized decode matvec path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl neon|reference]

Workload (the Q4_0 x fp32 matvec configuration the metric is quoted on): W
4096x4096 Q4_0 (blocks of 32 along K: fp16 d = |N(0,1)|*0.02 and 16 bytes of
nibbles uniform 0..15), x fp32 N(0,1), batch 1, seeded. The GPU keeps a
rotation of 48 distinct weight tensors (455 MB, 3.6x the 126 MB L2) so every
call streams its weights from HBM. One step = 1024 matvec calls, each on the
next tensor of the rotation. Metric: algorithmic bytes (weights + scales + x +
y) per second, whole job.

  value     device-resident: the step's 1024 launches replayed from a CUDA
            graph, timed with CUDA events on the launch stream.
  e2e       through the public host-buffer API (neon_cuda.proj_all_positions:
            pinned host x in, host y out, blocking per call, like the
            reference's fwd::proj_all_positions).
  roofline  the Q4_0 decode kernel against the measured HBM copy bandwidth.
  cpu_baseline
            the reference's own CPU path (oracle/_ref, rawllm_forward.hpp
            compiled with its flags) on this host's cores, bounded sample.

With --gpus N under torchrun the same matrices are split by rows over the N
ranks (strong scaling): each call is the row-sharded matvec with the output
all-gathered on every rank (neon_cuda_matvec_allgather, the fused NVLink
all-gather); value = the whole matrices' bytes / max-over-ranks time. The
`decode` list carries batch-1 decode tokens/s (Qwen3-0.6B-shaped at 1 GPU,
Phi-4-mini-shaped at 1 and 2, Llama-3-70B-shaped tensor parallel over all N)
and, at 1 GPU, `sweep` the other Q4_0 / Q8_0 matvec shapes.
--impl reference times the reference's CPU path alone (rank 0 only).
The tuning switches (--resident, --tiles, --dq-ring / --no-dq-ring,
--attn-rows, --attn-head-split, --cuda-core-prefill; see --help) time the
library's variants; the matvec line names --resident, --tiles, --dq-ring and
--cuda-core-prefill in config.variants, a decode workload's line also the
attention switches.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "neon-runtime-beta-variation_b200")
sys.path.insert(0, PKG)

import numpy as np  # noqa: E402

import synth as S  # noqa: E402

UNIT = "GB/s"
CALLS_PER_STEP = 1024
ROTATION_BYTES = 3 * 126e6  # weights rotated per step: 3x the L2
FALLBACK_HBM_GBS = 6650.0
KERNEL = "matvec_resident_kernel"

# name -> (ggml type, rows, cols); the first is the headline workload.
WORKLOADS = {
    "q4_0_4096x4096": (S.GGML_Q4_0, 4096, 4096),
    "q8_0_4096x4096": (S.GGML_Q8_0, 4096, 4096),
    "q8_0_14336x4096": (S.GGML_Q8_0, 14336, 4096),
    "q8_0_4096x14336": (S.GGML_Q8_0, 4096, 14336),
    "q4_0_28672x8192": (S.GGML_Q4_0, 28672, 8192),
    "q4_0_8192x28672": (S.GGML_Q4_0, 8192, 28672),
    # the other weight types (dequantising kernel)
    **{f"{S.TYPE_NAMES[t].lower()}_4096x4096": (t, 4096, 4096)
       for t in (S.GGML_Q4_1, S.GGML_Q5_0, S.GGML_Q5_1, S.GGML_Q4_K, S.GGML_Q5_K, S.GGML_Q6_K,
                 S.GGML_F16, S.GGML_BF16, S.GGML_F32)},
    "q4_k_14336x4096": (S.GGML_Q4_K, 14336, 4096),
    "q6_k_4096x14336": (S.GGML_Q6_K, 4096, 14336),
}
# --type-sweep: every weight type at the decode shape, plus two FFN shapes
TYPE_SWEEP = ["q4_0_4096x4096", "q8_0_4096x4096"] + [k for k in WORKLOADS if not k.startswith(("q4_0", "q8_0"))]
TYPE, ROWS, COLS = WORKLOADS["q4_0_4096x4096"]
ROTATION = 48
METRIC = "Q4_0 matvec HBM GB/s vs peak"
TYPE_NAME = "Q4_0"


# decode workloads: name -> (model config, prompt tokens, generated tokens)
DECODE_WORKLOADS = {
    "decode_qwen3": (S.QWEN3_0_6B, 128, 256),
    "decode_phi4": (S.PHI4_MINI, 512, 512),
    "decode_llama70b": (S.LLAMA3_70B, 2048, 256),
}
DECODE_METRIC = "batch-1 decode tokens/s"


def select_workload(name):
    global TYPE, ROWS, COLS, ROTATION, METRIC, TYPE_NAME, KERNEL
    if name in DECODE_WORKLOADS:
        return
    TYPE, ROWS, COLS = WORKLOADS[name]
    TYPE_NAME = S.TYPE_NAMES[TYPE]
    KERNEL = one_position_kernel(TYPE, ROWS, COLS)
    METRIC = f"{TYPE_NAME} matvec HBM GB/s vs peak"
    ROTATION = max(2, int(-(-ROTATION_BYTES // (ROWS * S.row_bytes(TYPE, COLS)))))


def one_position_kernel(t, rows, cols):
    """The kernel the library runs for one position of this workload on one
    GPU: Q4_0 / Q8_0 matrices of up to ~10 MB take the resident kernel (their
    per-CTA share fits shared memory beside the next launch's; the plan is
    csrc/neon_resident.cuh, checked at these shapes by
    tests/test_resident_plan_cpu.py), larger ones the streaming kernel, the
    other types the dequantising kernel."""
    if t not in (S.GGML_Q4_0, S.GGML_Q8_0):
        return "matvec_dq_kernel"
    return "matvec_resident_kernel" if rows * S.row_bytes(t, cols) <= 10_000_000 else "matvec_stream_kernel"


def profile_summary_path():
    kind = {"matvec_stream_kernel": "stream", "matvec_resident_kernel": "resident"}.get(KERNEL, "dq")
    return os.path.join(ROOT, "profiles", f"matvec_{kind}_{TYPE_NAME.lower()}_{ROWS}x{COLS}.txt")


def weight_distribution(t):
    if t == S.GGML_Q4_0:
        return "fp16 d=|N(0,1)|*0.02, nibbles U(0..15)"
    if t == S.GGML_Q8_0:
        return "fp16 d=|N(0,1)|*0.01, int8 U(-127..127)"
    if t in (S.GGML_F32, S.GGML_F16, S.GGML_BF16):
        return "values N(0,1)*0.02"
    return "fp16 scales |N(0,1)|*s, quant bytes U(0..255)"


def compute_dtype(t):
    if t == S.GGML_Q4_0:
        return "int8/fp32 (q4_0 x q8_0 dp4a, fp32 scales)"
    if t == S.GGML_Q8_0:
        return "fp32 (q8_0 int8 weights x fp32 x, fp32 accumulate)"
    return f"fp32 ({S.TYPE_NAMES[t].lower()} weights decoded exactly x fp32 x, fp32 accumulate)"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["neon", "reference"], default="neon")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(DECODE_WORKLOADS), default="q4_0_4096x4096")
    p.add_argument("--prompt", type=int, default=None, help="decode workloads: prompt tokens (default: the config's)")
    p.add_argument("--new-tokens", type=int, default=None, help="decode workloads: generated tokens")
    p.add_argument("--no-fused-collectives", action="store_true",
                   help="decode workloads at N>1: one all-reduce launch per column-split projection")
    p.add_argument("--layers", type=int, default=None,
                   help="decode workloads: fewer layers (kernel shapes unchanged; for profiling)")
    p.add_argument("--no-decode", action="store_true", help="matvec workloads: skip the decode sub-measurements")
    p.add_argument("--no-sweep", action="store_true",
                   help="matvec workloads: skip the sweep of the other Q4_0 / Q8_0 benchmark shapes")
    p.add_argument("--weights", choices=["q4_0", "q4_k"], default="q4_0",
                   help="decode workloads: Q4_0 projections + Q8_0 embedding (default), or Q4_K + Q6_K "
                        "(what nanity_convert.py --quant Q4_K writes)")
    p.add_argument("--prefill-mma", action="store_true",
                   help="multi-position calls on the tensor-core prefill kernels (the default; neon_cuda_set_prefill_mma)")
    p.add_argument("--cuda-core-prefill", action="store_true",
                   help="multi-position calls on the CUDA-core kernel instead (neon_cuda_set_prefill_mma(0))")
    p.add_argument("--dq-ring", action="store_true",
                   help="one-position calls of every dequantising type on the bulk-copy ring kernel "
                        "(neon_cuda_set_dq_ring; default: the types it is faster for)")
    p.add_argument("--no-dq-ring", action="store_true",
                   help="one-position calls of every dequantising type on the register-buffer kernel")
    p.add_argument("--tiles", default=None, metavar="RC:KC",
                   help="one-position Q4_0 / Q8_0 tile shape: RC rows per tile, KC blocks per row chunk "
                        "(0 = whole rows); neon_cuda_set_stream_tiles")
    p.add_argument("--resident", type=int, default=None, metavar="K",
                   help="one-position Q4_0 / Q8_0 launches that fit shared memory on the resident kernel with K "
                        "CTAs per SM (0: streaming kernel only); neon_cuda_set_resident (default: the library's)")
    p.add_argument("--attn-rows", default=None, metavar="MIN:SHARE",
                   help="decode attention: at least MIN cache rows per CTA, the cluster sized for SHARE rows of "
                        "ctx_len per CTA (multiples of 32); neon_cuda_set_attn_rows (default: the library's)")
    p.add_argument("--attn-head-split", type=int, default=None, metavar="H",
                   help="decode attention: each KV head's query heads over at most H clusters when SMs are idle "
                        "(neon_cuda_set_attn_head_split; default: the library's)")
    p.add_argument("--batch", type=int, default=1,
                   help="matvec workloads: positions per call; > 1 times the prefill path (one JSON line)")
    p.add_argument("--tile-sweep", action="store_true",
                   help="time the one-position Q4_0 / Q8_0 workloads under every tile shape of the sweep "
                        "(one JSON line each) instead of the headline")
    p.add_argument("--type-sweep", action="store_true",
                   help="time the matvec of every weight type (one JSON line each) instead of the headline")
    p.add_argument("--no-large-decode", action="store_true",
                   help="matvec workloads: skip the Llama-3-70B-shaped split decode sub-measurement")
    args = p.parse_args()
    select_workload(args.workload)
    global LAYERS, WTYPE, EMBD_TYPE
    LAYERS = args.layers
    if args.weights == "q4_k":
        WTYPE, EMBD_TYPE = S.GGML_Q4_K, S.GGML_Q6_K
    return args


def workload_config():
    dist = weight_distribution(TYPE)
    return {
        "workload": f"{TYPE_NAME} x fp32 matvec, W {ROWS}x{COLS}, batch 1 ({dist}, x N(0,1), seeded)",
        "rows": ROWS, "cols": COLS, "batch": 1,
        "rotation_tensors": ROTATION, "calls_per_step": CALLS_PER_STEP,
        "l2": f"inputs larger than L2: {ROTATION} distinct weight tensors "
              f"({ROTATION * S.row_bytes(TYPE, COLS) * ROWS / 1e6:.0f} MB) rotated, L2 126 MB",
        "bytes_per_call": S.algorithmic_bytes(TYPE, ROWS, COLS),
    }


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic():
    """DRAM bytes per launch of the kernel from the committed ncu summary."""
    try:
        with open(profile_summary_path()) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(float(line.split(":", 1)[1].split()[0]))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", ",".join(str(g) for g in gpu_ids)],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.f.flush()

    def summary(self, t0, t1):
        rows = []
        try:
            with open(self.f.name) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                        ts += float("0." + parts[0].split(".")[1]) if "." in parts[0] else 0.0
                        rows.append((ts, int(parts[2]), int(parts[3]), parts[5:9]))
                    except ValueError:
                        continue
        finally:
            os.unlink(self.f.name)
        inside = [r for r in rows if t0 - 0.05 <= r[0] <= t1 + 0.05]
        note = "samples inside the timed region"
        if not inside and rows:
            inside = sorted(rows, key=lambda r: min(abs(r[0] - t0), abs(r[0] - t1)))[:4]
            note = "timed region shorter than the 50 ms sampling period; nearest samples"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": reasons, "samples": len(inside), "note": note}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own path on this host
# ---------------------------------------------------------------------------

def cpu_reference_gbs(host_weights, x, seconds, max_calls=None):
    """GB/s of the reference's proj_all_positions over the rotation, on a
    util::ThreadPool of all host cores, for about `seconds` of CPU work."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    if O.ref_available():
        pool = O.RefPool(os.cpu_count() or 1)
        kind, cores = "reference", pool.n

        def call(W, Y):
            pool.proj_all_positions(TYPE, W, ROWS, COLS, x, Y)
    else:
        pool, kind, cores = None, "port", 1

        def call(W, Y):
            Y[:] = O.proj_all_positions(TYPE, W, ROWS, COLS, x)
    Y = np.zeros((1, ROWS), np.float32)
    call(host_weights[0], Y)  # warm
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and (max_calls is None or n < max_calls):
        call(host_weights[n % len(host_weights)], Y)
        n += 1
    dt = time.perf_counter() - t0
    if pool is not None:
        pool.close()
    gbs = n * S.algorithmic_bytes(TYPE, ROWS, COLS) / dt / 1e9
    return {"value": round(gbs, 3), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{n} calls of proj_all_positions on {TYPE_NAME} {ROWS}x{COLS} over a rotation of "
                      f"{len(host_weights)} tensors in {dt:.1f} s"}


def host_rotation(rank, n):
    return [S.weights(TYPE, ROWS, COLS, seed=100000 * rank + i) for i in range(n)]


LAYERS = None  # --layers
WTYPE, EMBD_TYPE = S.GGML_Q4_0, S.GGML_Q8_0  # --weights: decode models' projection / embedding types


def decode_config(name, prompt=None, new_tokens=None):
    cfg, n_prompt, n_new = DECODE_WORKLOADS[name]
    n_prompt = n_prompt if prompt is None else prompt
    n_new = n_new if new_tokens is None else new_tokens
    cfg = cfg.with_(ctx_len=n_prompt + n_new + 1)
    if LAYERS:
        cfg = cfg.with_(n_layer=LAYERS)
    return cfg, n_prompt, n_new


def decode_desc(cfg, n_prompt, n_new):
    return (f"{cfg.name} decoder ({cfg.n_layer} layers, hidden {cfg.n_embd}, {cfg.n_head}/{cfg.n_kv_head} heads, "
            f"head_dim {cfg.head_dim}, ffn {cfg.n_ff}, vocab {cfg.n_vocab}), random-init {S.TYPE_NAMES[WTYPE]} "
            f"projections, {S.TYPE_NAMES[EMBD_TYPE]} tied embedding/lm_head, fp32 norms; greedy decode of {n_new} "
            f"tokens after a {n_prompt}-token seeded-random prompt")


def is_big(cfg):
    return cfg.n_embd * cfg.n_ff * cfg.n_layer > 4e9


def model_bytes(cfg):
    """GGUF bytes of the synthetic decoder's projections and tied embedding."""
    def rb(rows, cols, t):
        return rows * S.row_bytes(t, cols)

    per_layer = (rb(cfg.q_dim, cfg.n_embd, WTYPE) + 2 * rb(cfg.kv_dim, cfg.n_embd, WTYPE)
                 + rb(cfg.n_embd, cfg.q_dim, WTYPE) + (1 if cfg.plain_ffn else 2) * rb(cfg.n_ff, cfg.n_embd, WTYPE)
                 + rb(cfg.n_embd, cfg.n_ff, WTYPE))
    return cfg.n_layer * per_layer + rb(cfg.n_vocab, cfg.n_embd, EMBD_TYPE)


def measure_decode_gpu(name, prompt=None, new_tokens=None, comm=None, barrier=None, max_over_ranks=None):
    """Device-timed greedy decode through neon_cuda.Model.generate (CUDA graph
    per token), on one GPU or split over the ranks of `comm` (tensor
    parallel); returns (result dict, model config, prompt tokens)."""
    import neon_cuda as N

    barrier = barrier or (lambda: None)
    max_over_ranks = max_over_ranks or (lambda v: v)
    cfg, n_prompt, n_new = decode_config(name, prompt, new_tokens)
    big = is_big(cfg)
    t0 = time.perf_counter()
    m = N.Model(cfg, S.model_tensors(cfg, seed=5, pooled=big, wtype=WTYPE, embd_type=EMBD_TYPE), comm)
    load_s = time.perf_counter() - t0
    prompt_toks = S.prompt_tokens(n_prompt, cfg.n_vocab, 6)
    barrier()
    t0 = time.perf_counter()
    toks = m.generate(prompt_toks, n_new)
    wall = max_over_ranks(time.perf_counter() - t0)
    ms = max_over_ranks(m.decode_ms)
    prefill_ms = max_over_ranks(m.forward_ms)
    m.free()
    world = comm.world if comm is not None else 1
    return {"workload": decode_desc(cfg, n_prompt, n_new) + (" (weights cut from a seeded block pool)" if big else ""),
            "n_gpus": world, "parallelism": f"tp{world}",
            "tokens_per_s": round(n_new * 1e3 / ms, 2),
            "ms_per_token": round(ms / n_new, 4), "generated": int(len(toks)),
            "timing": "CUDA events around the replayed per-token graphs, max over ranks",
            "e2e_tokens_per_s": round(n_new / wall, 2),
            "e2e": "neon_cuda.Model.generate wall clock incl. prompt prefill and token read-back",
            "prefill_ms": round(prefill_ms, 2), "prefill_tokens_per_s": round(n_prompt * 1e3 / prefill_ms, 1)
            if prefill_ms > 0 else None,
            "prefill": "the prompt pass (multi-position kernels), CUDA events, max over ranks",
            "load_s": round(load_s, 2)}, cfg, prompt_toks


def decode_roofline(d, cfg, world):
    """Effective HBM rate of a decode step: the bytes one rank streams per
    token (its share of the weights, plus K and V of the average context)
    over the device time per token, against the measured copy bandwidth."""
    peak, kind = measured_peak()
    kv = 2 * cfg.n_layer * cfg.kv_dim * 4 / world
    ctx_avg = cfg.ctx_len - 1 - (d["generated"] / 2 if d.get("generated") else 0)
    per_token = model_bytes(cfg) / world + kv * ctx_avg
    gbs = per_token / (d["ms_per_token"] * 1e-3) / 1e9
    d["hbm"] = {"bytes_per_token_per_gpu": int(per_token), "achieved_gbs_per_gpu": round(gbs, 1),
                "peak_gbs": peak, "peak_source": kind, "frac": round(gbs / peak, 4)}
    return d


def measure_decode_cpu(cfg, prompt_toks, steps, threads=None):
    """The reference's own transformer_forward (oracle/_ref) on the host:
    prompt prefill, then `steps` greedy decode steps; tokens/s of the decode."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    kind = "reference" if O.ref_available() else "port"
    m = O.Model(cfg, S.model_tensors(cfg, seed=5, pooled=is_big(cfg), wtype=WTYPE, embd_type=EMBD_TYPE), kind,
                threads=threads)
    logits = m.forward(prompt_toks)
    nxt = int(np.argmax(logits))
    t0 = time.perf_counter()
    for _ in range(steps):
        logits = m.forward(np.array([nxt], np.int32))
        nxt = int(np.argmax(logits))
    dt = time.perf_counter() - t0
    cores = m.pool.n if m.pool is not None else 1
    m.close()
    return {"tokens_per_s": round(steps / dt, 3), "kind": kind, "cores": cores,
            "sample": f"{steps} greedy decode steps of the reference's transformer_forward after the "
                      f"{len(prompt_toks)}-token prompt"}


def run_decode(args):
    """--workload decode_*: one line, metric batch-1 decode tokens/s; under
    torchrun the decoder is split over the N ranks (tensor parallel)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    import neon_cuda as N

    N.init(local)
    N.set_prefill_mma(not getattr(args, "cuda_core_prefill", False))
    if getattr(args, "dq_ring", False):
        N.set_dq_ring(True)
    if getattr(args, "tiles", None):
        N.set_stream_tiles(*(int(v) for v in args.tiles.split(":")))
    if args.resident is not None:
        N.set_resident(args.resident)
    if args.attn_rows:
        N.set_attn_rows(*(int(v) for v in args.attn_rows.split(":")))
    if args.attn_head_split:
        N.set_attn_head_split(args.attn_head_split)
    N.set_fused_collectives(not args.no_fused_collectives)
    comm = None
    barrier, max_over_ranks = (lambda: None), (lambda v: v)
    if world > 1:
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        cfg0, _, _ = decode_config(args.workload, args.prompt, args.new_tokens)
        comm = N.Comm.from_process_group(N.model_comm_floats(cfg0, world))
        comm.set_timeout(30.0)
        barrier = dist.barrier

        def max_over_ranks(v):
            t = torch.tensor([float(v)], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
    sampler = ClockSampler([local]) if rank == 0 else None
    time.sleep(0.2)
    t0 = time.time()
    res, cfg, prompt_toks = measure_decode_gpu(args.workload, args.prompt, args.new_tokens, comm, barrier,
                                               max_over_ranks)
    t1 = time.time()
    if sampler:
        sampler.stop()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = measure_decode_cpu_bounded(cfg, prompt_toks)
    if rank == 0:
        line = {"metric": DECODE_METRIC, "value": res["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
                "steps": res["generated"], "warmup": 0, "ms_per_step": res["ms_per_token"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8/fp32 (q4_0 x q8_0 dp4a, fp32 scales)",
                "data": "synthetic", "config": {"workload": res["workload"], "parallelism": res["parallelism"],
                                                "variants": [v for v, on in (("cuda_core_prefill", args.cuda_core_prefill),)
                                                             if on]
                                                + ([f"resident {args.resident}"] if args.resident is not None
                                                   else [])
                                                + ([f"attn rows {args.attn_rows}"] if args.attn_rows else [])
                                                + ([f"attn head split {args.attn_head_split}"]
                                                   if args.attn_head_split else [])},
                "e2e": {"value": res["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 4, "api": res["e2e"]},
                "load_s": res["load_s"], "prefill_ms": res.get("prefill_ms"),
                "prefill_tokens_per_s": res.get("prefill_tokens_per_s"),
                "roofline": decode_roofline(dict(res), cfg, world)["hbm"],
                "cpu_baseline": cpu, "clocks": sampler.summary(t0, t1)}
        print(json.dumps(line), flush=True)
    if comm is not None:
        barrier()
        comm.free()
        dist.destroy_process_group()


def measure_decode_cpu_bounded(cfg, prompt_toks):
    """The reference's CPU decode on a bounded sample: the full prompt when the
    model is small, else a 16-token prompt and 2 steps (stated in `sample`);
    skipped when the host has too little memory for the model."""
    big = is_big(cfg)
    need = model_bytes(cfg)
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 0
    if big and avail < need * 1.5:
        return {"skipped": f"host memory {avail / 1e9:.0f} GB too small for the reference CPU model "
                           f"({need / 1e9:.0f} GB)"}
    if big:
        return measure_decode_cpu(cfg.with_(ctx_len=32), prompt_toks[:16], steps=2)
    return measure_decode_cpu(cfg, prompt_toks, steps=8)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload in DECODE_WORKLOADS:
        cfg, n_prompt, n_new = decode_config(args.workload, args.prompt, args.new_tokens)
        prompt_toks = S.prompt_tokens(n_prompt, cfg.n_vocab, 6)
        steps = max(1, min(args.steps, 16))
        cpu = measure_decode_cpu(cfg, prompt_toks, steps)
        line = {"impl": "reference", "metric": DECODE_METRIC, "value": cpu["tokens_per_s"], "unit": "tokens/s",
                "n_gpus": 0, "steps": steps, "warmup": 0, "ms_per_step": round(1e3 / cpu["tokens_per_s"], 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8/fp32",
                "data": "synthetic", "config": {"workload": decode_desc(cfg, n_prompt, n_new), "parallelism": "cpu"},
                "cpu_baseline": {**cpu, "value": cpu["tokens_per_s"], "unit": "tokens/s"},
                "e2e": {"value": cpu["tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    cpu_n = min(16, ROTATION)
    weights = host_rotation(0, cpu_n)
    x = S.activations(1, COLS, seed=7)
    K, W = max(1, args.steps), max(0, args.warmup)
    budget = 120.0
    per_step_calls = cpu_n
    res = cpu_reference_gbs(weights, x, seconds=0.5)  # warm-up + calibration
    est_call_s = S.algorithmic_bytes(TYPE, ROWS, COLS) / (res["value"] * 1e9)
    per_step_calls = max(1, min(cpu_n, int(budget / max(1, K + W) / est_call_s)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    pool = O.RefPool(os.cpu_count() or 1) if O.ref_available() else None
    Y = np.zeros((1, ROWS), np.float32)

    def step():
        for j in range(per_step_calls):
            if pool is not None:
                pool.proj_all_positions(TYPE, weights[j], ROWS, COLS, x, Y)
            else:
                Y[:] = O.proj_all_positions(TYPE, weights[j], ROWS, COLS, x)
    for _ in range(W):
        step()
    t0 = time.perf_counter()
    for _ in range(K):
        step()
    dt = time.perf_counter() - t0
    value = K * per_step_calls * S.algorithmic_bytes(TYPE, ROWS, COLS) / dt / 1e9
    cores = pool.n if pool is not None else 1
    kind = "reference" if pool is not None else "port"
    if pool is not None:
        pool.close()
    cfg = workload_config()
    cfg["calls_per_step"] = per_step_calls
    cfg["rotation_tensors"] = cpu_n
    cfg["l2"] = (f"host: {cpu_n} distinct weight tensors "
                 f"({cpu_n * S.row_bytes(TYPE, COLS) * ROWS / 1e6:.0f} MB) rotated")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": 0,
        "steps": K, "warmup": W, "ms_per_step": round(dt / K * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": ("int8/fp32 (q4_0 x q8_0 integer block dot, fp32 scales)" if TYPE == S.GGML_Q4_0
                  else f"fp32 ({TYPE_NAME.lower()} rows dequantised, AVX2 fp32 dot)"),
        "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": f"{K} steps x {per_step_calls} calls of the reference's "
                                   f"fwd::proj_all_positions (util::ThreadPool of {cores})"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

SWEEP_WORKLOADS = ["q8_0_4096x4096", "q8_0_14336x4096", "q8_0_4096x14336", "q4_0_28672x8192", "q4_0_8192x28672"]


def measure_sweep(N, torch, stream, steps=20, warmup=3):
    """The other one-position Q4_0 / Q8_0 benchmark shapes (the Q8_0 sweep of
    the matvec configurations and the Llama-3-70B FFN shapes), each timed as
    the headline is (a CUDA graph of 1024 calls over a rotation larger than
    L2), with its own roofline fraction. Restores the headline workload."""
    head = (TYPE, ROWS, COLS, ROTATION, METRIC, TYPE_NAME, KERNEL)
    peak, peak_kind = measured_peak()
    out = []
    try:
        for name in SWEEP_WORKLOADS:
            select_workload(name)
            tensors = [N.DeviceTensor(w, TYPE, ROWS, COLS) for w in host_rotation(0, ROTATION)]
            gbs, us = time_matvec_graph(N, torch, stream, tensors, steps, warmup)
            out.append({"workload": name, "rows": ROWS, "cols": COLS, "type": TYPE_NAME, "kernel": KERNEL,
                        "value": round(gbs, 1), "unit": UNIT, "us_per_call": round(us, 3),
                        "frac": round(gbs / peak, 4), "peak": peak, "peak_source": peak_kind,
                        "bytes_per_call": S.algorithmic_bytes(TYPE, ROWS, COLS), "rotation_tensors": ROTATION,
                        "steps": steps, "warmup": warmup})
            del tensors
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
    finally:
        g = globals()
        for k, v in zip(("TYPE", "ROWS", "COLS", "ROTATION", "METRIC", "TYPE_NAME", "KERNEL"), head):
            g[k] = v
    return out


def run_neon(args):
    import torch
    import torch.distributed as dist

    import neon_cuda as N

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    N.init(local)
    N.set_prefill_mma(not getattr(args, "cuda_core_prefill", False))
    if getattr(args, "dq_ring", False):
        N.set_dq_ring(True)
    if getattr(args, "tiles", None):
        N.set_stream_tiles(*(int(v) for v in args.tiles.split(":")))
    if getattr(args, "resident", None) is not None:
        N.set_resident(args.resident)
    if getattr(args, "attn_rows", None):
        N.set_attn_rows(*(int(v) for v in args.attn_rows.split(":")))
    if getattr(args, "attn_head_split", None):
        N.set_attn_head_split(args.attn_head_split)
    dev = torch.device("cuda", local)

    # One GPU: a rotation of whole matrices. N > 1 (strong scaling): every rank
    # keeps its row shard of the SAME matrices (N times as many, so that each
    # rank's shards still exceed L2) and each call is the row-sharded matvec
    # with its output all-gathered on every rank (neon_cuda_matvec_allgather).
    tp = world > 1
    comm_mv = None
    row0 = ROWS * rank // world
    if tp:
        comm_mv = N.Comm.from_process_group(4096)
        comm_mv.set_timeout(30.0)
        rot = ROTATION * world
        host_w = None
        tensors = [N.DeviceTensor(S.weights(TYPE, ROWS, COLS, seed=i), TYPE, ROWS, COLS, N.SHARD_ROWS, rank, world)
                   for i in range(rot)]
    else:
        rot = ROTATION
        host_w = host_rotation(rank, ROTATION)
        tensors = [N.DeviceTensor(w, TYPE, ROWS, COLS) for w in host_w]
    x_host = S.activations(1, COLS, seed=7)
    dx = torch.from_numpy(x_host).to(dev)
    assert x_host.shape == (1, COLS)
    ys = torch.zeros((rot, ROWS), device=dev)
    stream = torch.cuda.Stream(device=dev)

    def call(j, s, x=dx, y=None):
        t = tensors[j % rot]
        y = ys[j % rot] if y is None else y
        if tp:
            comm_mv.matvec_allgather(t, x, y, ROWS, row0, stream=s)
        else:
            t.matvec(x, y, stream=s)

    def launch_step(s):
        for j in range(CALLS_PER_STEP):
            call(j, s)

    with torch.cuda.stream(stream):
        call(0, stream)
    stream.synchronize()

    # capture one step (1024 calls) in a CUDA graph
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch_step(stream)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    K, W = args.steps, max(3, args.warmup)
    with torch.cuda.stream(stream):
        for _ in range(W):
            graph.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler([local]) if rank == 0 else None
    time.sleep(0.2 if sampler else 0)
    launches_before = N.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(K):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if sampler:
        sampler.stop()
    assert N.launch_count() == launches_before, "graph replay should not go through the launch API"
    gpu_launches = K * CALLS_PER_STEP * (2 if tp else 1)
    bytes_call = S.algorithmic_bytes(TYPE, ROWS, COLS)  # the whole matrix, x and y of one call
    total_bytes = (1 if tp else world) * K * CALLS_PER_STEP * bytes_call
    value = total_bytes / (ms / 1e3) / 1e9
    per_call_s = ms / 1e3 / (K * CALLS_PER_STEP)
    achieved = bytes_call / world / per_call_s / 1e9  # one GPU's share of the bytes over the call's time

    # end to end: host buffers in and out every call (pinned), blocking
    x_pin = torch.from_numpy(x_host.copy()).pin_memory()
    y_pin = torch.zeros(ROWS, dtype=torch.float32).pin_memory()
    e2e_steps = max(1, min(args.e2e_steps, K))
    if tp:
        dx_e = torch.empty(COLS, device=dev)
        dy_e = torch.empty(ROWS, device=dev)

        def e2e_call(j):
            with torch.cuda.stream(stream):
                dx_e.copy_(x_pin[0], non_blocking=True)
                call(j, stream, dx_e, dy_e)
                y_pin.copy_(dy_e, non_blocking=True)
            stream.synchronize()
        api = "neon_cuda_matvec_allgather per call: pinned host x in, host y out, blocking"
    else:
        x_np, y_np = x_pin.numpy(), y_pin.numpy()
        infos = [N.TensorInfo(f"rot{i}", [COLS, ROWS], TYPE, host_w[i]) for i in range(rot)]
        for i in range(rot):  # upload happens once, at "load" time, outside the timed region
            N.proj_all_positions(infos[i], x_np, COLS, y_np, ROWS, 1)

        def e2e_call(j):
            N.proj_all_positions(infos[j % rot], x_np, COLS, y_np, ROWS, 1)
        api = "neon_cuda.proj_all_positions (host buffers, blocking per call)"
    e2e_call(0)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for j in range(CALLS_PER_STEP):
            e2e_call(j)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = (1 if tp else world) * e2e_steps * CALLS_PER_STEP * bytes_call / e2e_s / 1e9
    if tp:
        comm_mv.check()

    sweep = None
    if world == 1 and not args.no_sweep:
        sweep = measure_sweep(N, torch, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_gbs(host_w, x_host, args.cpu_seconds)
    decode = None
    if not args.no_decode:
        # batch-1 decode tokens/s: the Qwen3-0.6B-shaped decoder on one GPU,
        # and the Llama-3-70B-shaped decoder split over all N ranks
        del tensors, graph
        graph = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        decode = []
        def max_over(v):
            if world == 1:
                return v
            t = torch.tensor([float(v)], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        if world == 1:
            d, dcfg, dprompt = measure_decode_gpu("decode_qwen3")
            if not args.no_cpu_baseline:
                dcpu = measure_decode_cpu(dcfg, dprompt, steps=8)
                d["cpu_reference_tokens_per_s"] = dcpu["tokens_per_s"]
                d["cpu_reference_cores"] = dcpu["cores"]
                d["cpu_reference_kind"] = dcpu["kind"]
            d["parity"] = ("greedy tokens identical to the reference's transformer_forward over 64 steps "
                           "(tests/test_decode_gpu.py)")
            decode.append(decode_roofline(d, dcfg, 1))
        if world <= 2:
            # the Phi-4-mini-shaped decoder, at 1 and 2 GPUs
            pcomm = None
            if world > 1:
                pcfg0, _, _ = decode_config("decode_phi4")
                pcomm = N.Comm.from_process_group(N.model_comm_floats(pcfg0, world))
                pcomm.set_timeout(30.0)
            d, dcfg, _ = measure_decode_gpu("decode_phi4", comm=pcomm, barrier=barrier, max_over_ranks=max_over)
            d["parity"] = ("greedy tokens identical to the reference's transformer_forward (Phi-4-mini-shaped, "
                           "tests/test_decode_gpu.py)")
            decode.append(decode_roofline(d, dcfg, world))
            if pcomm is not None:
                barrier()
                pcomm.free()
        if not args.no_large_decode:
            comm = None
            if world > 1:
                cfg0, _, _ = decode_config("decode_llama70b")
                comm = N.Comm.from_process_group(N.model_comm_floats(cfg0, world))
                comm.set_timeout(30.0)
            d, dcfg, _ = measure_decode_gpu("decode_llama70b", comm=comm, barrier=barrier, max_over_ranks=max_over)
            d["parity"] = ("split decode: greedy tokens identical to one GPU and to the reference on the "
                           "Qwen3-shaped decoder at 2 GPUs (tests/test_tp_gpu.py)")
            decode.append(decode_roofline(d, dcfg, world))
            if comm is not None:
                barrier()
                comm.free()

    if rank == 0:
        peak, peak_kind = measured_peak()
        traffic = profile_traffic()
        clocks = sampler.summary(t_wall0, t_wall1) if sampler else {}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 5), "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": compute_dtype(TYPE),
            "data": "synthetic",
            "config": {**workload_config(), "rotation_tensors": rot,
                       "parallelism": (f"tp{world}: row shards, output all-gathered on every rank every call "
                                       "(neon_cuda_matvec_allgather)") if tp else "one GPU",
                       "variants": [v for v, on in (("dq_ring", args.dq_ring),
                                                    ("cuda_core_prefill", args.cuda_core_prefill)) if on]
                       + ([f"tiles {args.tiles}"] if args.tiles else [])
                       + ([f"resident {args.resident}"] if args.resident is not None else []),
                       "launch": f"CUDA graph of 1024 calls per step ({2 if tp else 1} PDL launches per call)"},
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                    "h2d_bytes_per_step": CALLS_PER_STEP * COLS * 4,
                    "d2h_bytes_per_step": CALLS_PER_STEP * ROWS * 4,
                    "api": api, "steps": e2e_steps},
            "roofline": {"bound": "hbm", "kernel": (KERNEL.replace("matvec_dq_kernel", "matvec_dq_ring_kernel")
                                                    if args.dq_ring else KERNEL),
                         "achieved": round(achieved, 1),
                         "peak": peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6.65 TB/s",
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic if not tp else None,
                         "algorithmic_bytes_per_launch": bytes_call // world,
                         "note": ("one GPU's shard bytes over the time of a whole call (its matvec and the "
                                  "all-gather launch)") if tp else "bytes of one launch over its time in the graph"},
            "cpu_baseline": cpu,
            "sweep": sweep,
            "decode": decode,
            "gpu_launches": gpu_launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if args.no_decode:
        del graph
    if comm_mv is not None:
        barrier()
        comm_mv.free()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args):
    """Several positions per call (prefill): `--batch` positions of X against
    the workload's matrix, a CUDA graph of calls over a rotation larger than
    L2, device-timed. One JSON line: TFLOP/s (2 * batch * rows * cols per call)
    against the measured dense bf16 tensor peak, and the HBM fraction."""
    import torch

    import neon_cuda as N

    torch.cuda.set_device(0)
    N.init(0)
    N.set_prefill_mma(not args.cuda_core_prefill)
    dev = torch.device("cuda", 0)
    B = args.batch
    calls = 64
    tensors = [N.DeviceTensor(w, TYPE, ROWS, COLS) for w in host_rotation(0, ROTATION)]
    X = S.activations(B, COLS, seed=7)
    dx = torch.from_numpy(X).to(dev)
    ys = torch.zeros((ROTATION, B * ROWS), device=dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        tensors[0].matvec(dx, ys[0], seq=B, stream=stream)
    stream.synchronize()
    launches0 = N.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for j in range(calls):
            tensors[j % ROTATION].matvec(dx, ys[j % ROTATION], seq=B, stream=stream)
    per_call_launches = (N.launch_count() - launches0) // calls
    K, W = args.steps, max(3, args.warmup)
    with torch.cuda.stream(stream):
        for _ in range(W):
            graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(K):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    per_call_s = ms / 1e3 / (K * calls)
    flops = 2.0 * B * ROWS * COLS
    bytes_call = S.algorithmic_bytes(TYPE, ROWS, COLS, seq=B)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tc_peak, tc_kind = float(json.load(f)["bf16_tflops"]), "measured dense bf16 (MEASURED_PEAKS.json)"
    except Exception:
        tc_peak, tc_kind = 1590.0, "fallback 1.59 PFLOP/s bf16"
    hbm, _ = measured_peak()
    tflops = flops / per_call_s / 1e12
    print(json.dumps({
        "metric": f"{TYPE_NAME} prefill TFLOP/s (batch {B})", "value": round(tflops, 2), "unit": "TFLOP/s",
        "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True,
        "kernel": ("CUDA cores (multi-position kernel)" if args.cuda_core_prefill else "tensor cores (int8 / TF32 mma.sync)"),
        "config": {**workload_config(), "batch": B, "calls_per_step": calls},
        "us_per_call": round(per_call_s * 1e6, 2), "launches_per_call": per_call_launches,
        "roofline": {"tensor": {"achieved": round(tflops, 2), "peak": tc_peak, "peak_source": tc_kind,
                                "frac": round(tflops / tc_peak, 4)},
                     "hbm": {"achieved": round(bytes_call / per_call_s / 1e9, 1), "peak": hbm,
                             "frac": round(bytes_call / per_call_s / 1e9 / hbm, 4)}},
    }), flush=True)


def time_matvec_graph(N, torch, stream, tensors, K, W):
    """Device GB/s of the selected workload: a CUDA graph of CALLS_PER_STEP
    one-position launches over `tensors` (a rotation larger than L2), K
    replays timed with CUDA events after W warm-up replays (the headline's
    method). Returns (GB/s, microseconds per call)."""
    dev = torch.device("cuda", 0)
    dx = torch.from_numpy(S.activations(1, COLS, seed=7)).to(dev)
    ys = torch.zeros((len(tensors), ROWS), device=dev)
    n = len(tensors)
    with torch.cuda.stream(stream):
        tensors[0].matvec(dx, ys[0], stream=stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for j in range(CALLS_PER_STEP):
            tensors[j % n].matvec(dx, ys[j % n], stream=stream)
    with torch.cuda.stream(stream):
        for _ in range(W):
            graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(K):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    del graph
    torch.cuda.synchronize()
    bytes_call = S.algorithmic_bytes(TYPE, ROWS, COLS)
    return K * CALLS_PER_STEP * bytes_call / (ms / 1e3) / 1e9, ms * 1e3 / (K * CALLS_PER_STEP)


def run_type_sweep(args):
    """One JSON line per weight type: device GB/s of a CUDA graph of 1024
    one-position launches over a rotation of tensors larger than L2, timed
    with CUDA events (the headline's method), and the fraction of the HBM peak."""
    import torch

    import neon_cuda as N

    torch.cuda.set_device(0)
    N.init(0)
    N.set_dq_ring(True if args.dq_ring else (False if args.no_dq_ring else None))
    if args.tiles:
        N.set_stream_tiles(*(int(v) for v in args.tiles.split(":")))
    peak, peak_kind = measured_peak()
    stream = torch.cuda.Stream(device=torch.device("cuda", 0))
    K, W = args.steps, max(3, args.warmup)
    for name in TYPE_SWEEP:
        select_workload(name)
        tensors = [N.DeviceTensor(w, TYPE, ROWS, COLS) for w in host_rotation(0, ROTATION)]
        gbs, us = time_matvec_graph(N, torch, stream, tensors, K, W)
        del tensors
        torch.cuda.empty_cache()
        kernel = KERNEL.replace("matvec_dq_kernel", "matvec_dq_ring_kernel") if args.dq_ring else KERNEL
        print(json.dumps({"workload": name, "type": TYPE_NAME, "kernel": kernel, "rows": ROWS, "cols": COLS,
                          "value": round(gbs, 1), "unit": UNIT, "frac": round(gbs / peak, 4),
                          "peak": peak, "peak_source": peak_kind, "us_per_call": round(us, 3),
                          "bytes_per_call": S.algorithmic_bytes(TYPE, ROWS, COLS), "rotation_tensors": ROTATION,
                          "steps": K, "warmup": W}),
              flush=True)


# (rows per tile, chunks per row; 0 = whole rows) of the tile sweep, after the planner's own choice
TILE_SWEEP_SHAPES = [(2, 0), (4, 0), (8, 0), (16, 0), (32, 0), (4, 2), (8, 2), (8, 4), (16, 4), (16, 8), (32, 8)]
TILE_SWEEP_WORKLOADS = ["q4_0_4096x4096", "q4_0_28672x8192", "q4_0_8192x28672", "q8_0_4096x4096",
                        "q8_0_14336x4096", "q8_0_4096x14336"]


def run_tile_sweep(args):
    """One JSON line per (workload, tile shape) of the one-position Q4_0 / Q8_0
    kernel, timed as the type sweep times a workload: the planner's choice
    (resident kernel where it applies, and the streaming kernel alone), then
    every forced shape of TILE_SWEEP_SHAPES that fits shared memory
    (neon_cuda_set_stream_tiles; the streaming kernel)."""
    import torch

    import neon_cuda as N

    torch.cuda.set_device(0)
    N.init(0)
    peak, peak_kind = measured_peak()
    stream = torch.cuda.Stream(device=torch.device("cuda", 0))
    K, W = args.steps, max(3, args.warmup)
    for name in TILE_SWEEP_WORKLOADS:
        select_workload(name)
        nb = COLS // 32
        tensors = [N.DeviceTensor(w, TYPE, ROWS, COLS) for w in host_rotation(0, ROTATION)]
        runs = [("planner", 0, 0, 2), ("planner, streaming kernel only", 0, 0, 0)]
        for rc, nch in TILE_SWEEP_SHAPES:
            kc = 0 if nch == 0 else ((nb + nch - 1) // nch + 7) // 8 * 8
            runs.append((f"rc {rc}, kc {kc or nb}", rc, kc, 0))
        for label, rc, kc, resident in runs:
            N.set_stream_tiles(rc, kc)
            N.set_resident(resident)
            line = {"workload": name, "tiles": label, "rows": ROWS, "cols": COLS, "unit": UNIT, "steps": K,
                    "warmup": W, "peak": peak, "peak_source": peak_kind}
            try:
                gbs, us = time_matvec_graph(N, torch, stream, tensors, K, W)
                line.update({"value": round(gbs, 1), "frac": round(gbs / peak, 4), "us_per_call": round(us, 3)})
            except RuntimeError as e:  # a stage that does not fit shared memory is refused before any launch
                line["skipped"] = str(e).splitlines()[0][:160]
            print(json.dumps(line), flush=True)
        del tensors
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    N.set_stream_tiles(0, 0)
    N.set_resident(2)


def main():
    args = parse_args()
    if args.tile_sweep and args.impl != "reference":
        run_tile_sweep(args)
    elif args.type_sweep and args.impl != "reference":
        run_type_sweep(args)
    elif args.batch > 1 and args.impl != "reference" and args.workload not in DECODE_WORKLOADS:
        run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload in DECODE_WORKLOADS:
        run_decode(args)
    else:
        run_neon(args)


if __name__ == "__main__":
    main()
