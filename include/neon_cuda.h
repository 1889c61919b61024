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

/* GGML tensor types, values of loader::GGMLType (rawllm_loader.hpp:23-32).
 * This backend runs Q4_0 and Q8_0; other values return NEON_ERR_UNSUPPORTED. */
#define NEON_GGML_F32 0
#define NEON_GGML_F16 1
#define NEON_GGML_Q4_0 2
#define NEON_GGML_Q8_0 8

/* Shard modes of neon_cuda_upload for tensor parallelism. */
#define NEON_SHARD_NONE 0 /* whole tensor */
#define NEON_SHARD_ROWS 1 /* rows [i*rows/n, (i+1)*rows/n): output-dim split */
#define NEON_SHARD_COLS 2 /* 32-blocks [i*nb/n, (i+1)*nb/n) of every row: input-dim split */

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
 * into HBM on the current device, repacked into the coalesced device layout.
 * With a shard mode, only shard `shard_index` of `shard_count` is kept.
 * Replaces the per-call host->device weight copy of matvec_rocblas
 * (rawllm_rocm.hpp:346-367): here weights move once, at load time. */
NEON_API int neon_cuda_upload(const uint8_t* host_bytes, int ggml_type, size_t rows, size_t cols,
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
 * Q8_0 (bit-exact activations); Q8_0 weights multiply fp32 X. */
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
 * cudaMalloc's device-wide synchronisation). Same arguments and results as
 * neon_cuda_matvec on a Q4_0 tensor, but the Q8_0 activations live in a fixed
 * 1.25 MiB array compiled into the library (held by every GPU that loads it)
 * instead of allocated scratch: seq*cols may not exceed 1,048,576. The first
 * call on a device looks up that array's address; make it before any stream
 * capture. Calls share the array, so calls that overlap on the GPU race.
 * This entry point has no counterpart in the reference. */
NEON_API int neon_cuda_matvec_q4_0_noalloc(neon_tensor_t W, const float* dX, size_t x_stride, float* dY,
                                           size_t y_stride, size_t seq, void* stream);

/* Launch option: programmatic dependent launch (PDL) lets a matvec fetch its
 * weights while the previous kernel on the stream finishes; on by default. */
NEON_API int neon_cuda_set_pdl(int enabled);

#ifdef __cplusplus
}
#endif

#endif /* NEON_CUDA_H */
