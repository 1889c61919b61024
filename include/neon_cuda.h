/*
 * neon_cuda.h -- C ABI of the B200 (sm_100a) backend for NEON's quantized
 * decode matvec path.
 *
 * The NEON runtime (NANITY-project/NEON-Runtime-Beta-Variation) computes every
 * projection of its decode loop with fwd::proj_all_positions[_multi]
 * (rawllm_forward.hpp:522-726) over raw GGUF/.nctr tensor bytes that
 * loader::TensorInfo::data_ptr points at (rawllm_loader.hpp:34-41). This
 * library replaces that CPU path, and the unwired HIP backend
 * (rawllm_rocm.hpp), with hand-written CUDA kernels. The weights are uploaded
 * to HBM once per tensor; every later call streams them from there.
 *
 * Conventions
 *  - Every function returns NEON_OK (0) or a negative NEON_ERR_* code; the
 *    message of the last failure on the calling thread is
 *    neon_cuda_last_error(). Where the reference throws std::runtime_error,
 *    the same condition returns NEON_ERR_INVALID here, with the same wording.
 *  - `stream` arguments are cudaStream_t values passed as void* (NULL is the
 *    legacy default stream). Device-pointer entry points are asynchronous on
 *    that stream; the host-buffer entry points (neon_cuda_proj_*) block, like
 *    the reference.
 *  - A tensor lives on the device that was current when it was uploaded;
 *    launches switch to that device for their duration.
 *  - Calls that use library scratch (multi-position Q4_0 calls) must not run
 *    concurrently from several host threads on one device, the same rule the
 *    reference's thread_local scratch imposes (rawllm_forward.hpp:545-546).
 */
#ifndef NEON_CUDA_H
#define NEON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NEON_API __attribute__((visibility("default")))
#else
#define NEON_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define NEON_OK 0
#define NEON_ERR_INVALID (-1)     /* bad argument (reference: std::runtime_error) */
#define NEON_ERR_UNSUPPORTED (-2) /* quant type or shape this backend does not run */
#define NEON_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define NEON_ERR_NOMEM (-4)       /* device allocation failed */

/* GGML tensor types, values of loader::GGMLType (rawllm_loader.hpp:23-32):
 * the eleven that fwd::dequantize_row decodes (rawllm_forward.hpp:301-321).
 * Q4_0 and Q8_0 run the streaming integer / fp32 kernels; the others run the
 * dequantising kernel. Q8_1, Q2_K, Q3_K and IQ4_NL, which the reference does
 * not dequantise either, return NEON_ERR_UNSUPPORTED. */
#define NEON_GGML_F32 0
#define NEON_GGML_F16 1
#define NEON_GGML_Q4_0 2
#define NEON_GGML_Q4_1 3
#define NEON_GGML_Q5_0 6
#define NEON_GGML_Q5_1 7
#define NEON_GGML_Q8_0 8
#define NEON_GGML_Q4_K 12
#define NEON_GGML_Q5_K 13
#define NEON_GGML_Q6_K 14
#define NEON_GGML_BF16 30

/* Shard modes of neon_cuda_upload for tensor parallelism. */
#define NEON_SHARD_NONE 0 /* whole tensor */
#define NEON_SHARD_ROWS 1 /* rows [i*rows/n, (i+1)*rows/n): output-dim split */
#define NEON_SHARD_COLS 2 /* blocks [i*nb/n, (i+1)*nb/n) of every row: input-dim split (32-value
                             blocks; 256-value super-blocks for Q4_K/Q5_K/Q6_K) */

/* Opaque handle of a device-resident weight tensor. */
typedef struct neon_tensor* neon_tensor_t;

/* One target of a multi-projection call: the weights, where its output goes and
 * the output row stride in floats. Mirrors fwd::ProjTarget
 * (rawllm_forward.hpp:626-630). */
typedef struct {
    neon_tensor_t W;
    float* Y;
    size_t y_stride;
} neon_proj_target_t;

/* Message of the last failed call on this thread ("" if none). */
NEON_API const char* neon_cuda_last_error(void);

/* Library version, e.g. "0.1.0". */
NEON_API const char* neon_cuda_version(void);

/* Number of visible CUDA devices (0 when none). */
NEON_API int neon_cuda_device_count(int* count);

/* Make `device` current for the calling thread and set up the library's
 * per-device state. Replaces rocm::GpuContext / Mi300xProps::get
 * (rawllm_rocm.hpp:33-173). */
NEON_API int neon_cuda_init(int device);

/* Copy one GGUF tensor (rows x cols, `rows` rows of bytes_for_type(type, cols)
 * bytes, the layout TensorInfo::data_ptr points at, rawllm_loader.hpp:170-176)
 * into HBM on the current device, repacked into the coalesced device layout
 * (Q4_0 / Q8_0: payload and scale planes; other types: the GGUF rows at a
 * 16-byte pitch). `cols` must be a multiple of the type's block size (32, or
 * 256 for the K-quants; any cols for F32/F16/BF16), as proj_all_positions
 * requires (rawllm_forward.hpp:528-533).
 * With a shard mode, only shard `shard_index` of `shard_count` is kept.
 * Replaces the per-call host->device weight copy of matvec_rocblas
 * (rawllm_rocm.hpp:346-367): here weights move once, at load time. */
NEON_API int neon_cuda_upload(const uint8_t* host_bytes, int ggml_type, size_t rows, size_t cols,
                     int shard_mode, int shard_index, int shard_count, neon_tensor_t* out);

/* On-load quantisation. The reference's runtime takes weights as stored; its
 * exporters quantise them with gguf-py's gguf.quants.quantize
 * (train_nanity_fixed.py:1162-1169 export_gguf, nanity_convert.py:472-484),
 * and a .nctr file is F32 only (export_nctr, train_nanity_fixed.py:1259-1433).
 * These take rows of F32 / F16 / BF16 values (a .nctr tensor, or a float GGUF
 * tensor) to Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, F16 or BF16 on the device, byte for
 * byte as gguf-py 0.19.0 writes them (finite inputs; block types need cols a
 * multiple of 32).
 *   neon_cuda_quantize_rows: device buffers, rows of bytes_for_type(src, cols)
 *     in, rows of bytes_for_type(dst, cols) out, on `stream`.
 *   neon_cuda_quantize_host: the same from host bytes to host bytes, blocking.
 *   neon_cuda_upload_quantized: neon_cuda_upload of the quantised tensor
 *     (shard modes as neon_cuda_upload), without a host round trip. */
NEON_API int neon_cuda_quantize_rows(const void* d_src, int src_type, size_t rows, size_t cols, int dst_type,
                                     void* d_dst, void* stream);
NEON_API int neon_cuda_quantize_host(const void* host_src, int src_type, size_t rows, size_t cols, int dst_type,
                                     void* host_dst);
NEON_API int neon_cuda_upload_quantized(const void* host_src, int src_type, size_t rows, size_t cols, int dst_type,
                                        int shard_mode, int shard_index, int shard_count, neon_tensor_t* out);

/* Rows, cols (of the kept shard), type and device bytes of a tensor. */
NEON_API int neon_cuda_tensor_info(neon_tensor_t W, size_t* rows, size_t* cols, int* ggml_type,
                          size_t* device_bytes);

/* Free a tensor's device memory. NULL is a no-op. */
NEON_API int neon_cuda_free(neon_tensor_t W);

/* Q8_0 activation quantisation on the device, bit-exact with
 * quantize_rows_q8_0 (rawllm_forward.hpp:360-381): for seq rows of cols floats
 * (row stride x_stride), d_out gets seq*cols/32 fp32 scales and q_out seq*cols
 * int8 values. Device pointers. */
NEON_API int neon_cuda_quantize_q8_0(const float* dX, size_t x_stride, size_t cols, size_t seq,
                            float* d_out, int8_t* q_out, void* stream);

/* Y[t*y_stride + r] = W_r . X_t for r < rows, t < seq, on device buffers.
 * The device counterpart of fwd::proj_all_positions (rawllm_forward.hpp:522-609):
 * Q4_0 weights use the fused Q4_0 x Q8_0 integer dot against X quantised to
 * Q8_0 (bit-exact activations); every other type is decoded (bit-exact values,
 * dequantize_row) and multiplied with fp32 X. */
NEON_API int neon_cuda_matvec(neon_tensor_t W, const float* dX, size_t x_stride, float* dY,
                     size_t y_stride, size_t seq, void* stream);

/* Several tensors that share one input X, in as few launches as their types
 * allow (one for the Q/K/V or gate/up sets of the decode loop). The device
 * counterpart of fwd::proj_all_positions_multi (rawllm_forward.hpp:632-726),
 * including its rule that all Q4_0 targets of one call share `cols`. */
NEON_API int neon_cuda_matvec_multi(const neon_proj_target_t* targets, size_t n_targets,
                           const float* dX, size_t x_stride, size_t seq, void* stream);

/* Host-buffer forms with the reference's blocking semantics: X and Y are host
 * pointers (pinned or pageable); X is copied in, the matvec runs, Y is copied
 * out, and the call returns when Y is written. The drop-in replacement for
 * fwd::proj_all_positions / proj_all_positions_multi (rawllm_forward.hpp:522-525,
 * 632-634) once the tensors are uploaded. */
NEON_API int neon_cuda_proj_all_positions(neon_tensor_t W, const float* hX, size_t x_stride, float* hY,
                                 size_t y_stride, size_t seq);
NEON_API int neon_cuda_proj_all_positions_multi(const neon_proj_target_t* targets, size_t n_targets,
                                       const float* hX, size_t x_stride, size_t seq);

/* Wait for all work the library queued on `stream`. */
NEON_API int neon_cuda_sync(void* stream);

/* Number of kernels this library has launched in this process (all devices). */
NEON_API uint64_t neon_cuda_launch_count(void);

/* Allocation-free Q4_0 matvec, for callers that cannot let a library allocate
 * device memory (a server that has reserved all of HBM for its own pools, a
 * framework allocator that holds the free memory, a loop that cannot take
 * cudaMalloc's device-wide synchronisation). Same arguments as
 * neon_cuda_matvec on a Q4_0 tensor; results are bit-identical to its default
 * multi-position path (seq > 1) and within the matvec tolerance of its
 * one-position streaming kernel (seq == 1). The Q8_0 activations live in a fixed
 * 1.25 MiB array compiled into the library (held by every GPU that loads it)
 * instead of allocated scratch: seq*cols may not exceed 1,048,576. The first
 * call on a device looks up that array's address; make it before any stream
 * capture. Calls share the array, so calls that overlap on the GPU race.
 * This entry point has no counterpart in the reference. */
NEON_API int neon_cuda_matvec_q4_0_noalloc(neon_tensor_t W, const float* dX, size_t x_stride, float* dY,
                                           size_t y_stride, size_t seq, void* stream);

/* ------------------------------------------------------------------------ */
/* Decode step on the device                                                */
/* ------------------------------------------------------------------------ */

/* Tensor roles of a NANITY decoder (NANITY_ARCHITECTURE_SPEC.md section 4;
 * fwd::ModelWeights / LayerWeights, rawllm_forward.hpp:823-834). */
#define NEON_ROLE_TOKEN_EMBD 0 /* token_embd.weight  [n_embd, n_vocab] */
#define NEON_ROLE_OUTPUT_NORM 1 /* output_norm.weight [n_embd] */
#define NEON_ROLE_OUTPUT 2     /* output.weight      [n_embd, n_vocab], optional (tied) */
#define NEON_ROLE_ATTN_NORM 3  /* blk.i.attn_norm.weight [n_embd] */
#define NEON_ROLE_ATTN_Q 4     /* blk.i.attn_q.weight    [n_embd, q_dim] */
#define NEON_ROLE_ATTN_K 5     /* blk.i.attn_k.weight    [n_embd, kv_dim] */
#define NEON_ROLE_ATTN_V 6     /* blk.i.attn_v.weight    [n_embd, kv_dim] */
#define NEON_ROLE_ATTN_OUT 7   /* blk.i.attn_output.weight [q_dim, n_embd] */
#define NEON_ROLE_FFN_NORM 8   /* blk.i.ffn_norm.weight  [n_embd] */
#define NEON_ROLE_FFN_GATE 9   /* blk.i.ffn_gate.weight  [n_embd, n_ff] */
#define NEON_ROLE_FFN_UP 10    /* blk.i.ffn_up.weight    [n_embd, n_ff] */
#define NEON_ROLE_FFN_DOWN 11  /* blk.i.ffn_down.weight  [n_ff, n_embd] */

/* Hyperparameters, the fields of engine::Config (rawllm_common.hpp:113-145)
 * the forward pass reads. ctx_len is the KV-cache capacity in positions.
 * plain_ffn = !use_swiglu: 0 (the NANITY default) is SwiGLU,
 * act = silu(ffn_gate x) * ffn_up x; 1 is the plain SiLU-FFN variant,
 * act = silu(ffn_up x), with no ffn_gate tensor (rawllm_forward.hpp:1167-1190). */
typedef struct {
    uint32_t n_vocab, n_embd, n_layer, n_head, n_kv_head, head_dim, n_ff, ctx_len;
    float rope_base, rope_scale;
    uint32_t rope_dim_count; /* 0: rotate all of head_dim */
    float norm_eps;
    uint32_t plain_ffn;
} neon_model_config_t;

typedef struct neon_model* neon_model_t;

/* A decoder on the current device: its KV cache (fp32, like fwd::KVCache,
 * rawllm_forward.hpp:905-927), activations and RoPE table. Tensors are added
 * with neon_cuda_model_set_tensor. Replaces get_engine_state's ModelWeights
 * + KVCache (NEON-3.cpp:535-564). */
NEON_API int neon_cuda_model_create(const neon_model_config_t* cfg, neon_model_t* out);

/* Upload one tensor (GGUF bytes; ne1 = 0 for a 1-D norm weight). Projection,
 * embedding and lm_head tensors may be any NEON_GGML_* type above (ffn_gate
 * and ffn_up of one layer share theirs). A norm weight may be any of them too
 * whose block divides n_embd: it is decoded to F32 once, here, as the
 * reference's dequant_full does on every forward (rawllm_forward.hpp:325-328,
 * at :1077, :1161, :1226). */
NEON_API int neon_cuda_model_set_tensor(neon_model_t m, int role, int layer, const uint8_t* host_bytes,
                                        size_t nbytes, int ggml_type, size_t ne0, size_t ne1);

/* Quantise every later float (F32 / F16 / BF16) projection, embedding or
 * lm_head tensor given to neon_cuda_model_set_tensor to `ggml_type` (Q8_0,
 * Q4_0, Q4_1, Q5_0, Q5_1, F16 or BF16) on the device first, byte for byte as
 * the exporters' gguf-py would have (neon_cuda_quantize_rows): a .nctr model,
 * F32 only, then runs as the Q8_0 / Q4_0 GGUF its publisher could have
 * exported. -1 turns it off (the default: tensors run as given). */
NEON_API int neon_cuda_model_set_quantize(neon_model_t m, int ggml_type);

/* fwd::transformer_forward (rawllm_forward.hpp:987-1236): process `n` new
 * tokens at positions length .. length+n-1, append their K/V to the cache,
 * advance length, and write the n_vocab logits of the last token to
 * logits_host (may be NULL). Blocks until done. */
NEON_API int neon_cuda_model_forward(neon_model_t m, const int32_t* tokens, size_t n, float* logits_host);

/* run_generation's loop (NEON-3.cpp:676-759) with greedy sampling (the first
 * maximum, NEON-3.cpp:471-474), device-resident: the prompt is processed,
 * then every decode step runs from one CUDA graph with the sampled token fed
 * back on the device. Writes up to max_new tokens (stopping before eos_id,
 * as the reference does; eos_id < 0: never) and their count. */
NEON_API int neon_cuda_model_generate(neon_model_t m, const int32_t* prompt, size_t n_prompt, size_t max_new,
                                      int32_t eos_id, int32_t* out_tokens, size_t* n_out);

/* KV-cache length (KVCache::length), and rewinding it (run_generation's
 * prefix reuse, NEON-3.cpp:690-703). */
NEON_API int neon_cuda_model_length(neon_model_t m, size_t* length);
NEON_API int neon_cuda_model_set_length(neon_model_t m, size_t length);

/* fwd::kv_cache_shift (rawllm_forward.hpp:949-969), run_generation's sliding
 * window (ensure_cache_room, NEON-3.cpp:590-630): positions [keep,
 * keep+discard) are forgotten, the K rows after them rotated by -discard
 * positions and both K and V moved down; length shrinks by discard. A no-op
 * when discard is 0 or the cache holds no more than keep+discard positions. */
NEON_API int neon_cuda_model_kv_shift(neon_model_t m, size_t keep, size_t discard);

/* Copy the K and V rows of `layer` for positions [0, n) to the host
 * (n x n_kv_head*head_dim floats each). */
NEON_API int neon_cuda_model_read_kv(neon_model_t m, int layer, size_t n, float* k_host, float* v_host);

/* Device time (CUDA events, ms) of the last neon_cuda_model_forward -- for
 * neon_cuda_model_generate, its prompt pass. */
NEON_API int neon_cuda_model_forward_ms(neon_model_t m, float* ms);

/* Time of the last neon_cuda_model_generate's decode steps, device-measured
 * (CUDA events around the replayed graphs), in milliseconds. */
NEON_API int neon_cuda_model_decode_ms(neon_model_t m, float* ms);

NEON_API int neon_cuda_model_free(neon_model_t m);

/* ---- Tensor parallelism: one rank (process) per GPU ------------------------
 * The reference declares an fp32 all-reduce across devices
 * (rocm::MultiGpuCtx::all_reduce_sum, rawllm_rocm.hpp:531-562) but runs
 * transformer_forward on one device. Here a decoder can be split over up to 8
 * ranks: attention by KV head, the FFN by 32-row groups, the lm_head by
 * vocabulary rows (neon_cuda_tp_shard), with attn_output and ffn_down summed
 * across ranks by the communicator's one-shot all-reduce over peer memory.
 *
 * Setup on every rank, with the rank's device current:
 *   neon_cuda_comm_create(rank, world, floats, &c)  floats >= neon_cuda_model_comm_floats()
 *   neon_cuda_comm_ipc_handle(c, buf, &bytes)       exchange the handles between
 *                                                   the ranks (any transport)
 *   neon_cuda_comm_connect(c, all_handles, bytes)   handles of ranks 0..world-1, back to back
 *   neon_cuda_model_create_tp(&cfg, c, &m)          then set_tensor with WHOLE tensors:
 *                                                   each rank keeps its shard
 * Every rank must then make the same calls in the same order (forward,
 * generate, set_length): each collective waits for all ranks, at most the
 * communicator's timeout (default 4 s), after which it reports an error and
 * the communicator must be recreated. Never run two ranks on one GPU. */
typedef struct neon_comm* neon_comm_t;

/* Row-sharded tensor-parallel matvec with the output all-gathered, one
 * position: every rank passes its row shard W of an n_total-row matrix (rows
 * [row0, row0 + W's rows) of it, e.g. a NEON_SHARD_ROWS upload) and the same
 * X; afterwards dY[0 .. n_total) holds the whole product on every rank. The
 * shard's matvec stores each row straight into every rank's communicator
 * buffer over NVLink (an 8-byte word carrying the value and the call number),
 * and a second launch copies the n_total words of this rank's buffer into dY
 * once they all carry this call (bounded waits; a peer that never writes
 * leaves the communicator's error set, see neon_cuda_comm_check). The ranks'
 * shards must tile [0, n_total) exactly, n_total <= 65536, and every rank
 * must make the same sequence of collective calls. No counterpart in the
 * reference (its HIP backend's only collective is all_reduce_sum,
 * rawllm_rocm.hpp:531-562); the all-gather at the row-shard boundary of the
 * tensor-parallel matvec. */
NEON_API int neon_cuda_matvec_allgather(neon_comm_t c, neon_tensor_t W, const float* dX, float* dY, size_t n_total,
                                        size_t row0, void* stream);

NEON_API int neon_cuda_comm_create(int rank, int world, size_t max_floats, neon_comm_t* out);
/* CUDA IPC handle of this rank's buffer; handle_out NULL: only the size. */
NEON_API int neon_cuda_comm_ipc_handle(neon_comm_t c, void* handle_out, size_t* handle_bytes);
NEON_API int neon_cuda_comm_connect(neon_comm_t c, const void* all_handles, size_t handle_bytes);
/* Connect the n communicators of ranks 0..n-1 created in THIS process (one
 * per device; peer access is enabled as needed). */
NEON_API int neon_cuda_comm_connect_local(neon_comm_t* comms, int n);
NEON_API int neon_cuda_comm_set_timeout(neon_comm_t c, double seconds);
/* dOut[i] = (add ? dOut[i] : 0) + sum over ranks, in rank order, of dIn[i],
 * for i < n, asynchronous on `stream`. */
NEON_API int neon_cuda_comm_allreduce(neon_comm_t c, const float* dIn, float* dOut, size_t n, int add, void* stream);
/* NEON_OK, or NEON_ERR_CUDA when a collective gave up waiting for a peer. */
NEON_API int neon_cuda_comm_check(neon_comm_t c);
NEON_API int neon_cuda_comm_free(neon_comm_t c);

/* Receive-slot size (floats) a communicator needs for this model and world. */
NEON_API int neon_cuda_model_comm_floats(const neon_model_config_t* cfg, int world, size_t* n);
/* The part of a tensor of `role` that `rank` of `world` keeps: rows
 * [range[0], range[1]) and columns [range[2], range[3]) of its GGUF shape
 * [ne0 = columns, ne1 = rows]. Host-only; needs no GPU. */
NEON_API int neon_cuda_tp_shard(const neon_model_config_t* cfg, int role, int rank, int world, size_t range[4]);
/* A decoder over the ranks of `comm` (NULL: one device, as
 * neon_cuda_model_create). neon_cuda_model_read_kv then returns this rank's
 * KV heads only; logits and tokens are whole on every rank. */
NEON_API int neon_cuda_model_create_tp(const neon_model_config_t* cfg, neon_comm_t comm, neon_model_t* out);
/* Launch option of the sharded decode step: fused collectives (default on)
 * -- attn_output / ffn_down store their partial rows, each word tagged with
 * the call number, straight into every rank's buffer, and a small reduce
 * launch adds them into the residual -- or, off, the projection writes
 * locally and a fenced one-shot all-reduce follows. Both give bit-identical
 * results. Set it before the first generate. */
NEON_API int neon_cuda_set_fused_collectives(int enabled);

/* Multi-position Q4_0 and Q8_0 calls (prefill) on the tensor cores, tiles of
 * 64 rows x 64 positions: Q4_0 as int8 MMA (mma.sync m16n8k32), each output
 * bit-exact with the reference's dot_q4_0_q8_0; Q8_0 as TF32 MMA with X split
 * into two TF32 terms (fp32 accuracy). On by default (measured on B200: Q4_0
 * 4096x4096 at 128 positions 48 TFLOP/s against 30 on the CUDA-core kernel);
 * 0 runs the CUDA-core kernel. The switch is process-wide. */
NEON_API int neon_cuda_set_prefill_mma(int enabled);

/* One-position calls of the dequantising types (F32, F16, BF16, Q4_1, Q5_0,
 * Q5_1, Q4_K, Q5_K, Q6_K) on a bulk-copy ring: a copy warp per CTA streams
 * row tiles into a ring of shared-memory stages (several tiles in flight per
 * CTA) and the compute warps decode from it, with the same decoders and
 * per-sub-block dot products as the register-buffer kernel. enabled = 1 for
 * every such type, 0 for none, -1 (the default) for the types it measured
 * faster for on B200 (Q4_1, F16, BF16). Process-wide. */
NEON_API int neon_cuda_set_dq_ring(int enabled);

/* Tile shape of later one-position Q4_0 / Q8_0 launches, for tuning sweeps:
 * rows_per_tile (2, 4, 8, 16 or 32) rows per tile, each row in chunks of
 * blocks_per_chunk 32-value blocks (0: whole rows). (0, 0) returns to the
 * built-in planner, the default. A shape whose stage does not fit shared
 * memory makes the call fail with NEON_ERR_UNSUPPORTED. Process-wide. */
NEON_API int neon_cuda_set_stream_tiles(int rows_per_tile, int blocks_per_chunk);

/* One-position Q4_0 / Q8_0 launches whose weights fit shared memory (up to a
 * few MB per SM, decode-sized projections) run on the resident kernel: each
 * CTA copies its whole contiguous row range into shared memory at start,
 * before the dependency wait, and lets the next launch start at once, so the
 * weight streams of consecutive launches overlap. ctas_per_sm sets how many
 * of one launch's CTAs share an SM (default 1); 0 sends every one-position
 * launch to the streaming kernel. Results agree with the streaming kernel
 * within the matvec tolerance (the same block dots, summed in another
 * order). Process-wide. */
NEON_API int neon_cuda_set_resident(int ctas_per_sm);

/* Decode attention work split: a model's cluster of CTAs per KV head is the
 * smallest (up to 16) whose share of ctx_len is at most share_rows rows (read
 * when a model is created; default 128); at a step the cluster's CTAs take
 * the context in shares of at least min_rows (read when a step is launched
 * or captured; default 32). Multiples of 32 from 32 to 16384. Tuning and
 * tests only; no counterpart in the reference. Process-wide. */
NEON_API int neon_cuda_set_attn_rows(int min_rows, int share_rows);

/* Decode attention: when a model's clusters (one per KV head) leave SMs idle
 * -- few KV heads per rank under tensor parallelism -- each KV head's query
 * heads are spread over up to max_split clusters (a power of two from 1 to
 * 8; default 8; 1: one cluster per KV head), each reading the same K and V
 * rows for its share of the heads. Read when a model is created. Tuning and
 * tests only; no counterpart in the reference. Process-wide. */
NEON_API int neon_cuda_set_attn_head_split(int max_split);

/* Launch option: programmatic dependent launch (PDL) lets a matvec fetch its
 * weights while the previous kernel on the stream finishes; on by default. */
NEON_API int neon_cuda_set_pdl(int enabled);

#ifdef __cplusplus
}
#endif

#endif /* NEON_CUDA_H */
