// neon_decode.cu -- the decode step of a NANITY decoder on one device.
//
// Reference: fwd::transformer_forward (rawllm_forward.hpp:987-1236) and the
// greedy loop of run_generation (NEON-3.cpp:676-759). One decode position is
// five launches per layer:
//   q, k, v = proj_multi(rms_norm(h, attn_norm))   streaming matvec; the norm is
//        RoPE'd q -> q, RoPE'd k / v -> cache[pos]   folded into its X staging,
//                                                  RoPE and the cache writes
//                                                  into its epilogue
//   att = causal GQA attention(q, cache)           attention_kernel
//   h += proj(att, attn_output)                    matvec, accumulate epilogue
//   act = silu(g) * u, (g, u) = proj(rms_norm(h, ffn_norm))
//                                                  one matvec over the gate/up
//                                                  rows interleaved at upload
//   h += proj(act, ffn_down)                       matvec, accumulate epilogue
// then logits = proj(rms_norm(h, output_norm), output ?? token_embd) and, in
// generation, the first maximum (argmax_kernel), fed back on the device. A
// prompt (several positions) runs the same steps unfused: rmsnorm_kernel,
// multi-position matvecs, rope_kv_kernel, swiglu_pairs_kernel.
//
// Element-wise arithmetic mirrors the reference's optimised build: RoPE with
// the reference's cos/sin values (host libm, uploaded as a table) and g++'s
// FMA contraction, fast_expf's Schraudolph constants, silu as x/(1+e), the
// RMSNorm scale in fp32 from a double sum of squares. Reductions (dot
// products, softmax sums, the double sum) run as parallel trees, so sums
// differ from the reference's sequential order by fp32 rounding only.
#include "neon_cuda.h"
#include "neon_internal.h"
#include "neon_attn_layout.h"

namespace neon {
// epilogue kinds of the one-position matvec kernel (see neon_kernels.cuh)
enum : int { kEpiStore = 0, kEpiRope = 1, kEpiAtPos = 2, kEpiSwiglu = 3, kEpiSilu = 5 };
}  // namespace neon

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

using neon_internal::cuda_error;
static int cuda_error_if(cudaError_t e, const char* what) { return e == cudaSuccess ? NEON_OK : cuda_error(e, what); }
using neon_internal::error;

namespace {

constexpr int kThreads = 256;
constexpr int kMaxChunk = 256;      // positions per forward chunk (prefill)
constexpr int kMaxCtx = 16384;      // attention scores live in shared memory

// neon_cuda_set_attn_rows: the decode attention's cache rows per CTA at
// least (read when a step is launched), and the share of ctx_len per CTA the
// cluster size is chosen for (read when a model is created); multiples of 32.
std::atomic<int> g_attn_min_rows{32}, g_attn_share_rows{128};
// neon_cuda_set_attn_head_split: clusters per KV head at most (read when a
// model is created)
std::atomic<int> g_attn_head_split{8};

#define DEC_TRY(call)                                              \
    do {                                                           \
        cudaError_t _e = (call);                                   \
        if (_e != cudaSuccess) return cuda_error(_e, #call);       \
    } while (0)

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------

// engine::fast_expf (rawllm_common.hpp:88-100): 2^(x/ln2) through the float
// bit pattern; kA*x + kB is one FMA in the reference build, truncated to int.
__device__ __forceinline__ float fast_expf_dev(float x) {
    if (x < -88.f || x > 88.f) return expf(x);
    return __int_as_float(__float2int_rz(__fmaf_rn(12102203.9f, x, 1064872507.f)));
}

// Programmatic dependent launch (see neon_kernels.cuh): wait for the previous
// kernel's results, and let the next kernel start its prologue.
__device__ __forceinline__ void pdl_wait_d() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_d() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions for kThreads threads (scratch: 32 entries).
__device__ float block_sum_f(float v, float* scratch) {
    v = warp_sum_f(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) scratch[w] = v;
    __syncthreads();
    float r = l < (int)(blockDim.x >> 5) ? scratch[l] : 0.f;
    r = warp_sum_f(r);
    return r;
}

__device__ float block_max_f(float v, float* scratch) {
    v = warp_max_f(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) scratch[w] = v;
    __syncthreads();
    float r = l < (int)(blockDim.x >> 5) ? scratch[l] : -INFINITY;
    r = warp_max_f(r);
    return r;
}

__device__ double block_sum_d(double v, double* scratch) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) scratch[w] = v;
    __syncthreads();
    double r = l < (int)(blockDim.x >> 5) ? scratch[l] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------

// h[t] = dequantised row tokens[t] of the embedding (dequant_q8_0 /
// dequant_q4_0, rawllm_forward.hpp:143-162; transformer_forward :1023-1033).
// One thread per 32-block. An out-of-range id sets bit 1 of *err and reads row 0.
__global__ void embed_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dpl, int type, int nb,
                             const int* __restrict__ tokens, int n_vocab, float* __restrict__ h,
                             unsigned* err) {
    pdl_wait_d();
    pdl_trigger_d();
    const int t = blockIdx.y;
    int tok = tokens[t];
    if (tok < 0 || tok >= n_vocab) {
        if (threadIdx.x == 0) atomicOr(err, 2u);
        tok = 0;
    }
    float* out = h + (long long)t * nb * 32;
    for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += gridDim.x * blockDim.x) {
        const long long i = (long long)tok * nb + b;
        const float d = __half2float(__ushort_as_half(dpl[i]));
        if (type == NEON_GGML_Q8_0) {
            const int8_t* q = reinterpret_cast<const int8_t*>(qs + i * 32);
#pragma unroll
            for (int j = 0; j < 32; ++j) out[b * 32 + j] = __fmul_rn(d, (float)q[j]);
        } else {
            const uint8_t* q = qs + i * 16;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                out[b * 32 + j] = __fmul_rn(d, __fsub_rn((float)(q[j] & 0xF), 8.f));
                out[b * 32 + j + 16] = __fmul_rn(d, __fsub_rn((float)(q[j] >> 4), 8.f));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Prefill attention on the tensor cores (neon_cuda_set_prefill_mma), the
// attention loop of transformer_forward (rawllm_forward.hpp:1108-1150) for a
// tile of 64 positions of one query head: pass 1 takes each position's
// maximum of the scaled scores s = (q . k) * scale over keys 0..pos; pass 2
// recomputes the same scores, p = fast_expf(s - max), their sums, and P.V,
// and the outputs are (P.V) / sum. Both products are TF32 MMAs (mma.sync
// m16n8k8) with every operand split into two TF32 terms and the three
// significant partial products kept: fp32 accuracy, in another order of
// additions than the reference's dot_f32 / axpy. Two passes rather than an
// online softmax: the reference applies fast_expf, a piecewise-linear
// exponential, to s minus the maximum over ALL keys, and rescaled partial
// sums of fast_expf values would not be its numbers. head_dim <= 128.
// ---------------------------------------------------------------------------
constexpr int kApRows = 64;   // positions per CTA (4 warps x 16)
constexpr int kApKeys = 64;   // keys per tile
constexpr int kApMaxHd = 128;

__device__ __forceinline__ uint32_t ap_tf32(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return r;
}
__device__ __forceinline__ void ap_split(float v, uint32_t& hi, uint32_t& lo) {
    hi = ap_tf32(v);
    lo = ap_tf32(__fsub_rn(v, __uint_as_float(hi)));
}
__device__ __forceinline__ void ap_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// c += a * b for a = ah + al, b = bh + bl (the al*bl term dropped), small terms first
__device__ __forceinline__ void ap_mma3(float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                        uint32_t bh0, uint32_t bh1, uint32_t bl0, uint32_t bl1) {
    ap_mma(c, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
    ap_mma(c, al[0], al[1], al[2], al[3], bh0, bh1);
    ap_mma(c, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
}

// Dynamic shared memory: Q and K tiles at a pitch of hd+4 floats, V at hd+8,
// P at 68 (conflict-free fragment reads).
__host__ __device__ inline int ap_smem_bytes(int hd) {
    return (int)sizeof(float) * (kApRows * (hd + 4) + kApKeys * (hd + 4) + kApKeys * (hd + 8) + kApRows * (kApKeys + 4));
}

__global__ void __launch_bounds__(128) attn_prefill_mma_kernel(const float* __restrict__ q, const float* __restrict__ Kc,
                                                               const float* __restrict__ Vc, float* __restrict__ out,
                                                               const int* __restrict__ d_pos, int seq, int q_dim,
                                                               int kv_dim, int hd, int group, float scale) {
    extern __shared__ float ap_sm[];
    const int qp = hd + 4, vp = hd + 8, pp = kApKeys + 4;
    float* Qs = ap_sm;
    float* Ks = Qs + kApRows * qp;
    float* Vs = Ks + kApKeys * qp;
    float* Ps = Vs + kApKeys * vp;
    const int h = blockIdx.x, t0 = blockIdx.y * kApRows;
    const int kvh = h / group;
    const int base = *d_pos;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int r0 = warp * 16 + g, r1 = r0 + 8;  // this lane's two rows of the tile
    const bool ok0 = t0 + r0 < seq, ok1 = t0 + r1 < seq;
    const int pos0 = base + t0 + r0, pos1 = base + t0 + r1;
    const int nq = min(kApRows, seq - t0);
    const int kend = base + t0 + nq;  // keys [0, kend) are seen by some position of the tile
    const int ntiles = (kend + kApKeys - 1) / kApKeys;
    const int nd = hd / 8;

    for (int i = tid; i < kApRows * hd; i += blockDim.x) {
        const int r = i / hd, d = i % hd;
        Qs[r * qp + d] = t0 + r < seq ? q[(long long)(t0 + r) * q_dim + (long long)h * hd + d] : 0.f;
    }
    auto load_tile = [&](int kt, bool with_v) {
        for (int i = tid; i < kApKeys * hd; i += blockDim.x) {
            const int r = i / hd, d = i % hd, key = kt * kApKeys + r;
            const long long src = (long long)key * kv_dim + (long long)kvh * hd + d;
            Ks[r * qp + d] = key < kend ? Kc[src] : 0.f;
            if (with_v) Vs[r * vp + d] = key < kend ? Vc[src] : 0.f;
        }
    };
    // the scaled scores of this lane's rows r0, r1 against keys 8j+2tq(+1) of a tile
    auto scores = [&](float (&sc)[8][4]) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[j][e] = 0.f;
        for (int ks = 0; ks < nd; ++ks) {
            uint32_t ah[4], al[4];
            ap_split(Qs[r0 * qp + 8 * ks + tq], ah[0], al[0]);
            ap_split(Qs[r1 * qp + 8 * ks + tq], ah[1], al[1]);
            ap_split(Qs[r0 * qp + 8 * ks + tq + 4], ah[2], al[2]);
            ap_split(Qs[r1 * qp + 8 * ks + tq + 4], ah[3], al[3]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t bh0, bl0, bh1, bl1;
                ap_split(Ks[(8 * j + g) * qp + 8 * ks + tq], bh0, bl0);
                ap_split(Ks[(8 * j + g) * qp + 8 * ks + tq + 4], bh1, bl1);
                ap_mma3(sc[j], ah, al, bh0, bh1, bl0, bl1);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[j][e] = __fmul_rn(sc[j][e], scale);
    };

    // pass 1: row maxima over each position's keys 0..pos
    float m0 = -INFINITY, m1 = -INFINITY;
    for (int kt = 0; kt < ntiles; ++kt) {
        __syncthreads();
        load_tile(kt, false);
        __syncthreads();
        float sc[8][4];
        scores(sc);
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kt * kApKeys + 8 * j + 2 * tq + (e & 1);
                if (e < 2) {
                    if (ok0 && key <= pos0) m0 = fmaxf(m0, sc[j][e]);
                } else if (ok1 && key <= pos1) {
                    m1 = fmaxf(m1, sc[j][e]);
                }
            }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }

    // pass 2: p = fast_expf(s - max), sums, P.V
    float acc[kApMaxHd / 8][4];
#pragma unroll
    for (int n = 0; n < kApMaxHd / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
    float l0 = 0.f, l1 = 0.f;
    for (int kt = 0; kt < ntiles; ++kt) {
        __syncthreads();
        load_tile(kt, true);
        __syncthreads();
        float sc[8][4];
        scores(sc);
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 8 * j + 2 * tq + (e & 1), key = kt * kApKeys + col;
                const bool on = e < 2 ? (ok0 && key <= pos0) : (ok1 && key <= pos1);
                const float p = on ? fast_expf_dev(__fsub_rn(sc[j][e], e < 2 ? m0 : m1)) : 0.f;
                if (e < 2) l0 += p;
                else l1 += p;
                Ps[(e < 2 ? r0 : r1) * pp + col] = p;
            }
        __syncwarp();  // a warp reads back only its own 16 rows of P
        for (int ks = 0; ks < kApKeys / 8; ++ks) {
            uint32_t ah[4], al[4];
            ap_split(Ps[r0 * pp + 8 * ks + tq], ah[0], al[0]);
            ap_split(Ps[r1 * pp + 8 * ks + tq], ah[1], al[1]);
            ap_split(Ps[r0 * pp + 8 * ks + tq + 4], ah[2], al[2]);
            ap_split(Ps[r1 * pp + 8 * ks + tq + 4], ah[3], al[3]);
#pragma unroll
            for (int n = 0; n < kApMaxHd / 8; ++n) {
                if (n >= nd) break;
                uint32_t bh0, bl0, bh1, bl1;
                ap_split(Vs[(8 * ks + tq) * vp + 8 * n + g], bh0, bl0);
                ap_split(Vs[(8 * ks + tq + 4) * vp + 8 * n + g], bh1, bl1);
                ap_mma3(acc[n], ah, al, bh0, bh1, bl0, bl1);
            }
        }
        __syncwarp();  // P is rewritten by this warp for the next tile
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    const float inv0 = ok0 ? __fdiv_rn(1.0f, l0) : 0.f, inv1 = ok1 ? __fdiv_rn(1.0f, l1) : 0.f;
#pragma unroll
    for (int n = 0; n < kApMaxHd / 8; ++n) {
        if (n >= nd) break;
        const int d = 8 * n + 2 * tq;
        if (ok0) {
            float* o0 = out + (long long)(t0 + r0) * q_dim + (long long)h * hd + d;
            o0[0] = __fmul_rn(acc[n][0], inv0);
            o0[1] = __fmul_rn(acc[n][1], inv0);
        }
        if (ok1) {
            float* o1 = out + (long long)(t0 + r1) * q_dim + (long long)h * hd + d;
            o1[0] = __fmul_rn(acc[n][2], inv1);
            o1[1] = __fmul_rn(acc[n][3], inv1);
        }
    }
}

// Causal GQA attention of a multi-position forward (transformer_forward
// :1115-1151) on the CUDA cores, register-tiled like an fp32 GEMM: a CTA of
// 256 threads takes query head blockIdx.x at 64 positions (blockIdx.y) and
// walks the key tiles of 64 cached rows; thread (ty, tx) of a 16 x 16 grid
// owns rows 4ty..4ty+3 and, for the scores, keys 4tx..4tx+3 of a tile, for
// the output dims (HD/16)tx.. of the head. Q and the K tile sit transposed in
// shared memory (a score is one fmaf chain over the head dim, in order), V in
// its own layout, p transposed for the p*v loop. The reference's two passes:
// the row maxima over each position's keys 0..pos first, then
// p = fast_expf(score - max), l = sum p and o = sum p * v; out = o * (1 / l).
// 112 KB of shared memory: two CTAs per SM.
constexpr int kPfRows = 64, kPfKeys = 64, kPfThreads = 256;
template <int HD>
constexpr int pf_smem_bytes() {
    return (int)sizeof(float) * (HD * kPfRows + HD * kPfKeys + kPfKeys * HD + kPfKeys * kPfRows);
}

template <int HD>
__global__ void __launch_bounds__(kPfThreads, 2) attn_prefill_f32_kernel(const float* __restrict__ q,
                                                                         const float* __restrict__ Kc,
                                                                         const float* __restrict__ Vc,
                                                                         float* __restrict__ out,
                                                                         const int* __restrict__ d_pos, int seq,
                                                                         int q_dim, int kv_dim, int group,
                                                                         float scale) {
    constexpr int DPT = HD / 16;  // output dims per thread
    extern __shared__ __align__(16) float pf_sm[];
    float* qt = pf_sm;                 // [HD][64]: Q of the tile's positions, transposed
    float* kt = qt + HD * kPfRows;     // [HD][64]: the key tile, transposed
    float* vs = kt + HD * kPfKeys;     // [64][HD]
    float* pt = vs + kPfKeys * HD;     // [64 keys][64 rows]: p, transposed
    const int h = blockIdx.x, t0 = blockIdx.y * kPfRows, kvh = h / group;
    const int base = *d_pos;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int nq = min(kPfRows, seq - t0);
    const int kend = base + t0 + nq;  // keys [0, kend) are seen by some position of the tile
    const int ntiles = (kend + kPfKeys - 1) / kPfKeys;

    // Q: float4 along the head dim from each position's row, stored transposed
    for (int i = tid; i < kPfRows * (HD / 4); i += kPfThreads) {
        const int r = i % kPfRows, d4 = i / kPfRows;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nq) v = *reinterpret_cast<const float4*>(q + (long long)(t0 + r) * q_dim + (long long)h * HD + 4 * d4);
        qt[(4 * d4 + 0) * kPfRows + r] = v.x;
        qt[(4 * d4 + 1) * kPfRows + r] = v.y;
        qt[(4 * d4 + 2) * kPfRows + r] = v.z;
        qt[(4 * d4 + 3) * kPfRows + r] = v.w;
    }
    auto load_k = [&](int t) {
        for (int i = tid; i < kPfKeys * (HD / 4); i += kPfThreads) {
            const int r = i % kPfKeys, d4 = i / kPfKeys, key = t * kPfKeys + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (key < kend) v = *reinterpret_cast<const float4*>(Kc + (long long)key * kv_dim + (long long)kvh * HD + 4 * d4);
            kt[(4 * d4 + 0) * kPfKeys + r] = v.x;
            kt[(4 * d4 + 1) * kPfKeys + r] = v.y;
            kt[(4 * d4 + 2) * kPfKeys + r] = v.z;
            kt[(4 * d4 + 3) * kPfKeys + r] = v.w;
        }
    };
    auto load_v = [&](int t) {
        for (int i = tid; i < kPfKeys * (HD / 4); i += kPfThreads) {
            const int r = i / (HD / 4), d4 = i % (HD / 4), key = t * kPfKeys + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (key < kend) v = *reinterpret_cast<const float4*>(Vc + (long long)key * kv_dim + (long long)kvh * HD + 4 * d4);
            *reinterpret_cast<float4*>(vs + r * HD + 4 * d4) = v;
        }
    };
    // the scaled scores of rows 4ty.. against keys 4tx.. of the tile in kt
    auto scores = [&](float (&s)[4][4]) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; ++d) {
            const float4 qa = *reinterpret_cast<const float4*>(qt + d * kPfRows + 4 * ty);
            const float4 kb = *reinterpret_cast<const float4*>(kt + d * kPfKeys + 4 * tx);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = __fmaf_rn(qv[i], kv[j], s[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = __fmul_rn(s[i][j], scale);
    };
    int pos[4];
    bool live[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        live[i] = 4 * ty + i < nq;
        pos[i] = base + t0 + 4 * ty + i;
    }

    // pass 1: row maxima
    float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int t = 0; t < ntiles; ++t) {
        __syncthreads();
        load_k(t);
        __syncthreads();
        float s[4][4];
        scores(s);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (live[i] && t * kPfKeys + 4 * tx + j <= pos[i]) m[i] = fmaxf(m[i], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int o = 8; o; o >>= 1) m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));

    // pass 2: p, l and o = sum p * v
    float acc[4][DPT], l[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < DPT; ++c) acc[i][c] = 0.f;
    for (int t = 0; t < ntiles; ++t) {
        __syncthreads();
        load_k(t);
        load_v(t);
        __syncthreads();
        float s[4][4];
        scores(s);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float p4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const bool on = live[i] && t * kPfKeys + 4 * tx + j <= pos[i];
                p4[i] = on ? fast_expf_dev(__fsub_rn(s[i][j], m[i])) : 0.f;
                l[i] += p4[i];
            }
            *reinterpret_cast<float4*>(pt + (4 * tx + j) * kPfRows + 4 * ty) = make_float4(p4[0], p4[1], p4[2], p4[3]);
        }
        __syncthreads();
#pragma unroll 4
        for (int k = 0; k < kPfKeys; ++k) {
            const float4 pa = *reinterpret_cast<const float4*>(pt + k * kPfRows + 4 * ty);
            const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
            float vv[DPT];
#pragma unroll
            for (int c = 0; c < DPT; c += 4) {
                const float4 v4 = *reinterpret_cast<const float4*>(vs + k * HD + DPT * tx + c);
                vv[c] = v4.x, vv[c + 1] = v4.y, vv[c + 2] = v4.z, vv[c + 3] = v4.w;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < DPT; ++c) acc[i][c] = __fmaf_rn(pv[i], vv[c], acc[i][c]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int o = 8; o; o >>= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], o);
        if (!live[i]) continue;
        const float inv = __fdiv_rn(1.0f, l[i]);
        float* o = out + (long long)(t0 + 4 * ty + i) * q_dim + (long long)h * HD + DPT * tx;
#pragma unroll
        for (int c = 0; c < DPT; c += 4)
            *reinterpret_cast<float4*>(o + c) = make_float4(__fmul_rn(acc[i][c], inv), __fmul_rn(acc[i][c + 1], inv),
                                                            __fmul_rn(acc[i][c + 2], inv), __fmul_rn(acc[i][c + 3], inv));
    }
}


// out = x * (1/sqrt(mean(x^2) + eps)) * w per row; one CTA per row
// (fwd::rms_norm, rawllm_forward.hpp:730-735).
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           float* __restrict__ out, int n, float eps) {
    __shared__ double dscratch[32];
    const float* xr = x + (long long)blockIdx.x * n;
    float* o = out + (long long)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fma((double)xr[i], (double)xr[i], ss);
    ss = block_sum_d(ss, dscratch);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / (double)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

// RoPE on q and k of position pos = *d_pos + blockIdx.x (fwd::rope_apply,
// rawllm_forward.hpp:767-782, with the reference's cos/sin from `cs`), then
// K/V cache rows at pos (transformer_forward :1104-1107).
__global__ void rope_kv_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                               const float2* __restrict__ cs, const int* __restrict__ d_pos, int n_head, int n_kv,
                               int hd, int rope_half, int q_dim, int kv_dim, float* __restrict__ Kc,
                               float* __restrict__ Vc) {
    const int t = blockIdx.x;
    const int pos = *d_pos + t;
    const int half = hd / 2;
    const float2* csp = cs + (long long)pos * rope_half;
    float* qt = q + (long long)t * q_dim;
    for (int idx = threadIdx.x; idx < n_head * half; idx += blockDim.x) {
        const int h = idx / half, i = idx % half;
        if (i < rope_half) {
            const float2 c = csp[i];
            float* p = qt + h * hd + 2 * i;
            const float x0 = p[0], x1 = p[1];
            p[0] = __fmaf_rn(x0, c.x, -__fmul_rn(x1, c.y));
            p[1] = __fmaf_rn(x0, c.y, __fmul_rn(x1, c.x));
        }
    }
    const float* kt = k + (long long)t * kv_dim;
    float* kc = Kc + (long long)pos * kv_dim;
    for (int idx = threadIdx.x; idx < n_kv * half; idx += blockDim.x) {
        const int h = idx / half, i = idx % half;
        const float x0 = kt[h * hd + 2 * i], x1 = kt[h * hd + 2 * i + 1];
        if (i < rope_half) {
            const float2 c = csp[i];
            kc[h * hd + 2 * i] = __fmaf_rn(x0, c.x, -__fmul_rn(x1, c.y));
            kc[h * hd + 2 * i + 1] = __fmaf_rn(x0, c.y, __fmul_rn(x1, c.x));
        } else {
            kc[h * hd + 2 * i] = x0;
            kc[h * hd + 2 * i + 1] = x1;
        }
    }
    const float* vt = v + (long long)t * kv_dim;
    float* vc = Vc + (long long)pos * kv_dim;
    for (int j = threadIdx.x; j < kv_dim; j += blockDim.x) vc[j] = vt[j];
}

// Causal GQA attention of query head blockIdx.x at position *d_pos +
// blockIdx.y over cache positions [0, pos] (transformer_forward :1115-1151):
// scores = (q . k_s) * scale, p_s = fast_expf(score - max), out = sum_s
// (p_s / sum p) v_s. Scores live in shared memory (L floats).
__global__ void __launch_bounds__(kThreads) attention_kernel(const float* __restrict__ q, const float* __restrict__ Kc,
                                                             const float* __restrict__ Vc, float* __restrict__ out,
                                                             const int* __restrict__ d_pos, int q_dim, int kv_dim,
                                                             int hd, int group, float scale) {
    extern __shared__ float sc[];
    __shared__ float scratch[32];
    __shared__ float part[kThreads];
    const int h = blockIdx.x, t = blockIdx.y;
    const int L = *d_pos + t + 1;
    const int kvh = h / group;
    const float* qv = q + (long long)t * q_dim + (long long)h * hd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    // scores: warp per position, lanes split head_dim
    float qr[8];
    const int per = hd / 32;  // head_dim is a multiple of 32, at most 256
#pragma unroll
    for (int j = 0; j < 8; ++j) qr[j] = j < per ? qv[lane + 32 * j] : 0.f;
    for (int s = warp; s < L; s += nw) {
        const float* kr = Kc + (long long)s * kv_dim + (long long)kvh * hd;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < per) acc = __fmaf_rn(qr[j], kr[lane + 32 * j], acc);
        acc = warp_sum_f(acc);
        if (lane == 0) sc[s] = __fmul_rn(acc, scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int s = threadIdx.x; s < L; s += blockDim.x) m = fmaxf(m, sc[s]);
    m = block_max_f(m, scratch);
    float sum = 0.f;
    for (int s = threadIdx.x; s < L; s += blockDim.x) {
        const float p = fast_expf_dev(__fsub_rn(sc[s], m));
        sc[s] = p;
        sum += p;
    }
    sum = block_sum_f(sum, scratch);
    const float inv = __fdiv_rn(1.0f, sum);
    // out[d] = sum_s (p_s * inv) * v_s[d]; the CTA's threads split (d, s mod parts)
    const int parts = blockDim.x / hd;
    const int d = threadIdx.x % hd, pidx = threadIdx.x / hd;
    float acc = 0.f;
    if (pidx < parts) {
        const float* vb = Vc + (long long)kvh * hd + d;
        for (int s = pidx; s < L; s += parts) acc = __fmaf_rn(__fmul_rn(sc[s], inv), vb[(long long)s * kv_dim], acc);
    }
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < hd) {
        float r = 0.f;
        for (int p = 0; p < parts; ++p) r += part[p * hd + threadIdx.x];
        out[(long long)t * q_dim + (long long)h * hd + threadIdx.x] = r;
    }
}


// ---------------------------------------------------------------------------
// Decode attention (transformer_forward's attention at one position,
// rawllm_forward.hpp:1115-1151): a thread-block cluster of cs CTAs per KV
// head. At context length L = *d_pos + 1, CTA r of the cluster takes cache
// rows [r * rows, (r + 1) * rows) (attn_rows_per_cta); the first n_act CTAs
// have rows, the others leave after the cluster's opening barrier.
//
// K and V rows land in shared memory by TMA tensor copies of 32-row x
// bw-float boxes with the matching swizzle, so that a lane per cache row
// reads its row's 16-byte chunks without bank conflicts. A CTA's rows come in
// rounds of round_rows through two slots: its K rounds, then its V rounds,
// item t in slot t % 2, each slot refilled as soon as its item is consumed,
// so that the V rows arrive while the K rows are scored (the slots stay
// small enough for two CTAs per SM, which keeps every KV head's cluster
// resident at once). The rows before *d_pos were written by earlier decode
// steps, whose kernels have all finished before any kernel of this step
// starts (each step opens with the embedding kernel, which waits for the
// step before); the first two items' copies of them are issued before the
// dependency wait and overlap the kernel before. Only the box that holds the
// new row, written by the kernel before, waits.
//
// Pass 1 (per round): warp tasks (32-row box, dim block), a lane per row, the
// group's query rows read as broadcasts: the partial dot per (row, head, dim
// block); the score is the blocks' partials added in order, times the scale.
// Each CTA sends its per-head maxima to every active CTA of the cluster
// (st.async into the peer's shared memory, counted on the peer's mbarrier),
// so that all form p = fast_expf(score - max over ALL positions) exactly as
// transformer_forward does (:1123-1137): fast_expf is an approximation, and
// rescaling by per-CTA maxima would not reproduce its values. Pass 2: a warp
// per row stride, a lane per float4 column: o = sum p * v, l = sum p. Each
// CTA keeps (o, l) in its shared memory and signals CTA 0, which reads them
// through distributed shared memory and adds them in rank order:
// out = (sum o) * (1 / sum l).
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr_d(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Bounded wait on an mbarrier phase (2 s of %globaltimer, then bit 2 of the
// error word); `cluster`: acquire at cluster scope (data from other CTAs).
__device__ __forceinline__ bool mbar_wait_d(uint64_t* bar, uint32_t parity, unsigned int* err, bool cluster = false) {
    uint32_t done = 0;
    unsigned long long t0 = 0;
    for (int it = 0;; ++it) {
        if (cluster)
            asm volatile(
                "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, "
                "0, p; }"
                : "=r"(done)
                : "r"(smem_addr_d(bar)), "r"(parity)
                : "memory");
        else
            asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                         : "=r"(done)
                         : "r"(smem_addr_d(bar)), "r"(parity)
                         : "memory");
        if (done) return true;
        unsigned long long t;
        asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
        if (it == 0) t0 = t;
        else if (t - t0 > 2000000000ull) {
            atomicOr(err, 4u);
            return false;
        }
    }
}

static_assert(kThreads == kAttnThreads, "the attention layout assumes kThreads threads");

// A box of the layer's K or V cache (a 2D tensor, rows x kv_dim): columns x ..
// x + bw, rows y .. y + 32, into shared memory, completion counted in bytes on
// `bar`. Rows past the cache's end arrive as zeros.
__device__ __forceinline__ void tma_box(float* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr_d(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_addr_d(bar))
        : "memory");
}

// Offset (floats) of 16-byte chunk c of row r in a dim block of BW-float rows
// as a TMA box with the BW*4-byte swizzle leaves it: the chunk index XOR bits
// 7.. of the row's byte offset (the block starts 1024-byte aligned).
template <int BW>
__device__ __forceinline__ int attn_swz(int r, int c) {
    constexpr int kW = BW * 4, kM = kW / 16 - 1;
    return r * BW + ((c ^ ((r * kW >> 7) & kM)) << 2);
}

template <int GP, int BW>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(
    const float* __restrict__ q, const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
    const __grid_constant__ CUtensorMap tmk_r, const __grid_constant__ CUtensorMap tmv_r, const int* __restrict__ d_pos,
    int hd, int group, int hsplit, float scale, int min_rows, int round_rows, int score_rows, float* __restrict__ out,
    unsigned int* err) {
    extern __shared__ __align__(1024) float sm[];
    uint32_t rank, cs;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(cs));
    // cluster c = blockIdx.x / cs: KV head c / hsplit, its query heads
    // [h0, h0 + GP) (those below group are real; the rest are zero rows)
    const int kvh = blockIdx.x / (cs * hsplit);
    const int h0 = (int)((blockIdx.x / cs) % hsplit) * GP;
    const int nh = min(GP, group - h0);  // real query heads of this cluster
    const long long qrow0 = ((long long)kvh * group + h0) * hd;  // its first query / output element
    const int pos = __ldcg(d_pos), L = pos + 1;
    const int rows = attn_rows_per_cta(L, (int)cs, min_rows);
    const int n_act = (L + rows - 1) / rows;
    const int s0 = (int)rank * rows;
    const int len = s0 < L ? min(rows, L - s0) : 0;
    const int nbk = hd / BW;
    const AttnSmem lay = attn_smem_layout(hd, GP, BW, round_rows, score_rows, (int)cs);
    float* const slot0 = sm + lay.k;  // the two slots of K or V rows
    float* const slot1 = sm + lay.v;
    auto slot = [&](int t) { return (t & 1) ? slot1 : slot0; };
    float* ps = sm + lay.ps;  // [nbk][round_rows][GP]
    float* sc = sm + lay.sc;  // [score_rows][GP]
    float* qs = sm + lay.q;   // [GP][hd]
    float* wm = sm + lay.wm;  // [warps][GP]
    float* wl = sm + lay.wl;
    float* cmax = sm + lay.cmax;  // [cs][GP]
    // slot 0, slot 1, the cluster's maxima, (CTA 0) the peers' partials, (peers) CTA 0 has read them
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + lay.bar);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool aligned = (smem_addr_d(sm) & 1023u) == 0;  // the swizzled boxes need it
    if (threadIdx.x == 0) {
        if (!aligned) atomicOr(err, 8u);
        for (int i = 0; i < 5; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr_d(&bars[i])),
                         "r"(i == 3 ? (uint32_t)max(1, n_act - 1) : 1u)
                         : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (len > 0 && n_act > 1)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr_d(&bars[2])),
                         "r"((uint32_t)(n_act * GP * 4))
                         : "memory");
    }
    __syncthreads();
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    if (len == 0 || !aligned) {
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
        return;
    }
    const int nr = (len + round_rows - 1) / round_rows, n_items = 2 * nr;
    // item t (K round t, then V round t - nr) into slot t % 2, issued by warp 0:
    // an item without row pos as one round-sized box per dim block (the round
    // maps; rows past the CTA's share land in slot rows nothing reads), the
    // item with it as 32-row boxes. mode 0: every box, 1: the boxes without
    // row pos (before the dependency wait), 2: the box with it
    auto issue = [&](int t, int mode) {
        const bool is_v = t >= nr;
        const int r0 = (is_v ? t - nr : t) * round_rows;
        const int nrb = (min(round_rows, len - r0) + kAttnBoxRows - 1) / kAttnBoxRows;
        const bool pos_item = pos < s0 + r0 + nrb * kAttnBoxRows;  // rows < len <= pos + 1 - s0
        uint64_t* bar = &bars[t & 1];
        float* base = slot(t);
        if (mode != 2 && lane == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr_d(bar)),
                         "r"((uint32_t)(nbk * (pos_item ? nrb * kAttnBoxRows : round_rows) * BW * 4))
                         : "memory");
        __syncwarp();
        if (!pos_item) {
            if (mode != 2 && lane < nbk)
                tma_box(base + lane * round_rows * BW, is_v ? &tmv_r : &tmk_r, kvh * hd + lane * BW, s0 + r0, bar);
            return;
        }
        for (int i = lane; i < nrb * nbk; i += 32) {
            const int rb = i / nbk, nb = i - rb * nbk, y = s0 + r0 + rb * kAttnBoxRows;
            const bool has_pos = pos < y + kAttnBoxRows;
            if ((mode == 1 && has_pos) || (mode == 2 && !has_pos)) continue;
            tma_box(base + (nb * round_rows + rb * kAttnBoxRows) * BW, is_v ? &tmv : &tmk, kvh * hd + nb * BW, y, bar);
        }
    };
    // slot t % 2 is read: refill it with item t + 2 (after the barrier that closes the reads)
    auto refill = [&](int t) {
        if (warp == 0 && t + 2 < n_items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(t + 2, 0);
        }
    };
    if (warp == 0) {
#pragma unroll 1
        for (int t = 0; t < 2; ++t) issue(t, 1);
    }
    pdl_wait_d();
    pdl_trigger_d();
    if (warp == 0) {
#pragma unroll 1
        for (int t = 0; t < 2; ++t) issue(t, 2);
    }
    for (int i = threadIdx.x; i < GP * hd; i += kAttnThreads)
        qs[i] = i < nh * hd ? q[qrow0 + i] : 0.f;
    __syncthreads();

    // pass 1, per round: partial dots per (row, head, dim block), then the scores
    const int gq = threadIdx.x % GP;  // the head of this thread's (row, head) pairs
    float run_max = -INFINITY;
    bool ok = true;
    for (int j = 0; j < nr; ++j) {
        const int r0 = j * round_rows, rl = min(round_rows, len - r0);
        const int nrb = (rl + kAttnBoxRows - 1) / kAttnBoxRows;
        ok = mbar_wait_d(&bars[j & 1], (uint32_t)((j >> 1) & 1), err) && ok;
        const float* Ks = slot(j);
        for (int t = warp; t < nrb * nbk; t += kAttnWarps) {
            const int rb = t / nbk, nb = t - rb * nbk, r = rb * kAttnBoxRows + lane;
            if (r < rl) {
                const float* kb = Ks + nb * round_rows * BW;
                const float* qb = qs + nb * BW;
                // two chains per head (the x, z and the y, w products), added at the end
                float acc[GP], acc2[GP];
#pragma unroll
                for (int g = 0; g < GP; ++g) acc[g] = acc2[g] = 0.f;
#pragma unroll 2
                for (int c = 0; c < BW / 4; ++c) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kb + attn_swz<BW>(r, c));
#pragma unroll
                    for (int g = 0; g < GP; ++g) {
                        const float4 q4 = *reinterpret_cast<const float4*>(qb + g * hd + c * 4);
                        acc[g] = __fmaf_rn(q4.x, k4.x, acc[g]);
                        acc2[g] = __fmaf_rn(q4.y, k4.y, acc2[g]);
                        acc[g] = __fmaf_rn(q4.z, k4.z, acc[g]);
                        acc2[g] = __fmaf_rn(q4.w, k4.w, acc2[g]);
                    }
                }
#pragma unroll
                for (int g = 0; g < GP; ++g) acc[g] += acc2[g];
                float* dst = ps + (nb * round_rows + r) * GP;
                if constexpr (GP >= 4) {
#pragma unroll
                    for (int g = 0; g < GP; g += 4)
                        *reinterpret_cast<float4*>(dst + g) = make_float4(acc[g], acc[g + 1], acc[g + 2], acc[g + 3]);
                } else {
#pragma unroll
                    for (int g = 0; g < GP; ++g) dst[g] = acc[g];
                }
            }
        }
        __syncthreads();
        refill(j);
        for (int r = threadIdx.x / GP; r < rl; r += kAttnThreads / GP) {
            float d = ps[r * GP + gq];
            for (int nb = 1; nb < nbk; ++nb) d += ps[(nb * round_rows + r) * GP + gq];
            const float s = __fmul_rn(d, scale);
            sc[(r0 + r) * GP + gq] = s;
            run_max = fmaxf(run_max, s);
        }
        __syncthreads();  // ps is free for the next round
    }
    // this CTA's maximum per head, then the cluster's
#pragma unroll
    for (int o = 16; o >= GP; o >>= 1) run_max = fmaxf(run_max, __shfl_xor_sync(0xffffffffu, run_max, o));
    if (lane < GP) wm[warp * GP + lane] = run_max;
    __syncthreads();
    float m = wm[gq];
#pragma unroll
    for (int w = 1; w < kAttnWarps; ++w) m = fmaxf(m, wm[w * GP + gq]);
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // every CTA's barriers are set up
    if (n_act > 1) {
        if ((int)threadIdx.x < n_act * GP) {  // head gq's maximum to CTA threadIdx.x / GP
            const uint32_t peer = threadIdx.x / GP;
            uint32_t dst, bar;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                         : "=r"(dst)
                         : "r"(smem_addr_d(&cmax[rank * GP + gq])), "r"(peer));
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(smem_addr_d(&bars[2])), "r"(peer));
            asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(dst),
                         "r"(__float_as_uint(m)), "r"(bar)
                         : "memory");
        }
        ok = mbar_wait_d(&bars[2], 0, err, true) && ok;
        m = cmax[gq];
        for (int r = 1; r < n_act; ++r) m = fmaxf(m, cmax[r * GP + gq]);
    }
    // p = fast_expf(score - max) in place, l = sum p
    float lsum = 0.f;
    for (int r = threadIdx.x / GP; r < len; r += kAttnThreads / GP) {
        const float p = fast_expf_dev(__fsub_rn(sc[r * GP + gq], m));
        sc[r * GP + gq] = p;
        lsum += p;
    }
#pragma unroll
    for (int o = 16; o >= GP; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane < GP) wl[warp * GP + lane] = lsum;
    __syncthreads();

    // pass 2, per round: o = sum over rows of p * v, a lane per float4 column
    const int nc = hd / 4;
    constexpr int kCB = BW / 4;  // 16-byte chunks per block row
    float4 acc[2][GP];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int g = 0; g < GP; ++g) acc[i][g] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int c0 = lane, c1 = lane + 32;
    const int vo0 = (c0 / kCB) * round_rows * BW, vo1 = (c1 / kCB) * round_rows * BW;
    auto pv = [&](float4(&a)[GP], const float* Vs, int vo, int c, int r, const float* p) {
        const float4 v4 = *reinterpret_cast<const float4*>(Vs + vo + attn_swz<BW>(r, c % kCB));
#pragma unroll
        for (int g = 0; g < GP; ++g) {
            a[g].x = __fmaf_rn(p[g], v4.x, a[g].x);
            a[g].y = __fmaf_rn(p[g], v4.y, a[g].y);
            a[g].z = __fmaf_rn(p[g], v4.z, a[g].z);
            a[g].w = __fmaf_rn(p[g], v4.w, a[g].w);
        }
    };
    for (int j = 0; j < nr; ++j) {
        const int t = nr + j, r0 = j * round_rows, rl = min(round_rows, len - r0);
        ok = mbar_wait_d(&bars[t & 1], (uint32_t)((t >> 1) & 1), err) && ok;
        const float* Vs = slot(t);
#pragma unroll 2
        for (int r = warp; r < rl; r += kAttnWarps) {
            float p[GP];
            const float* pr = sc + (r0 + r) * GP;
            if constexpr (GP >= 4) {
#pragma unroll
                for (int g = 0; g < GP; g += 4) {
                    const float4 p4 = *reinterpret_cast<const float4*>(pr + g);
                    p[g] = p4.x, p[g + 1] = p4.y, p[g + 2] = p4.z, p[g + 3] = p4.w;
                }
            } else {
#pragma unroll
                for (int g = 0; g < GP; ++g) p[g] = pr[g];
            }
            if (c0 < nc) pv(acc[0], Vs, vo0, c0, r, p);
            if (c1 < nc) pv(acc[1], Vs, vo1, c1, r, p);
        }
        if (j + 1 < nr) {
            __syncthreads();  // the slot is read
            refill(t);
        }
    }
    (void)ok;  // a copy or exchange that timed out set bit 2 of the error word; the results are then not used
    // the warps' sums -> red (slot 0: the last item is in slot 1, and the
    // barrier after the one before it closed slot 0's reads), then this CTA's
    // o and l into ps and lsum, where CTA 0 reads them
    float* red = sm + lay.red;
#pragma unroll
    for (int g = 0; g < GP; ++g) {
        if (c0 < nc) *reinterpret_cast<float4*>(red + (warp * GP + g) * hd + c0 * 4) = acc[0][g];
        if (c1 < nc) *reinterpret_cast<float4*>(red + (warp * GP + g) * hd + c1 * 4) = acc[1][g];
    }
    __syncthreads();
    const int ne = GP * hd;
    float* mine = ps;               // [GP][hd]
    float* mine_l = sm + lay.lsum;  // [GP]
    if ((int)threadIdx.x < GP) {
        float v = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) v += wl[w * GP + threadIdx.x];
        mine_l[threadIdx.x] = v;
    }
#pragma unroll 1
    for (int e = threadIdx.x; e < ne; e += kAttnThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) v += red[w * ne + e];
        mine[e] = v;
    }
    __syncthreads();
    if (rank != 0) {
        if (threadIdx.x == 0) {
            uint32_t ready;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(ready) : "r"(smem_addr_d(&bars[3])));
            asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(ready) : "memory");
            mbar_wait_d(&bars[4], 0, err);  // CTA 0 has read this CTA's partial
        }
        return;
    }
    // CTA 0: out = (sum o) * (1 / sum l) over the active CTAs in rank order,
    // four elements of one head per thread
    if (n_act > 1) mbar_wait_d(&bars[3], 0, err, true);  // every active CTA's partial is in place
#pragma unroll 1
    for (int e = 4 * threadIdx.x; e < nh * hd; e += 4 * kAttnThreads) {
        const int g = e / hd;  // hd % 4 == 0: the four share a head
        float4 num = *reinterpret_cast<const float4*>(&mine[e]);
        float den = mine_l[g];
        for (int r = 1; r < n_act; ++r) {
            const float4 v = *static_cast<const float4*>(__cluster_map_shared_rank(&mine[e], r));
            num.x += v.x, num.y += v.y, num.z += v.z, num.w += v.w;
            den += *static_cast<const float*>(__cluster_map_shared_rank(&mine_l[g], r));
        }
        const float inv = __fdiv_rn(1.0f, den);
        *reinterpret_cast<float4*>(&out[qrow0 + e]) =
            make_float4(__fmul_rn(num.x, inv), __fmul_rn(num.y, inv), __fmul_rn(num.z, inv), __fmul_rn(num.w, inv));
    }
    if (n_act > 1) {
        __syncthreads();  // the peers' partials are read: release them
        if ((int)threadIdx.x >= 1 && (int)threadIdx.x < n_act) {
            uint32_t done;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(done) : "r"(smem_addr_d(&bars[4])), "r"(threadIdx.x));
            asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(done) : "memory");
        }
    }
}

// act[t][i] = silu(y[t][2i]) * y[t][2i+1] over the interleaved gate/up rows,
// silu(x) = x / (1 + fast_expf(-x)) (rawllm_forward.hpp:740, :1186).
__global__ void swiglu_pairs_kernel(const float* __restrict__ y, float* __restrict__ act, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float x = y[2 * i];
        act[i] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, fast_expf_dev(-x))), y[2 * i + 1]);
    }
}

// fwd::kv_cache_shift's rotation (rawllm_forward.hpp:949-969): the tail K rows
// of one layer, rotated by -discard positions (rope_rotate_by_delta, :794-809,
// with the host's cos/sin of that one angle per pair), into `dst`.
__global__ void kv_shift_rotate_kernel(const float* __restrict__ src, float* __restrict__ dst, const float2* __restrict__ cs,
                                       long long tail, int kv_dim, int hd, int rope_half) {
    const int half = hd / 2;
    const long long n = tail * (kv_dim / 2);
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (long long)gridDim.x * blockDim.x) {
        const long long row = idx / (kv_dim / 2);
        const int pr = (int)(idx - row * (kv_dim / 2));  // pair index within the row
        const int i = pr % half;
        const float* s = src + row * kv_dim + 2 * pr;
        float* d = dst + row * kv_dim + 2 * pr;
        const float x0 = s[0], x1 = s[1];
        if (i < rope_half) {
            const float2 c = cs[i];
            d[0] = __fmaf_rn(x0, c.x, -__fmul_rn(x1, c.y));
            d[1] = __fmaf_rn(x0, c.y, __fmul_rn(x1, c.x));
        } else {
            d[0] = x0;
            d[1] = x1;
        }
    }
}

// act[i] = silu(y[i]): the plain SiLU-FFN variant (rawllm_forward.hpp:1189).
__global__ void silu_kernel(const float* __restrict__ y, float* __restrict__ act, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float x = y[i];
        act[i] = __fdiv_rn(x, __fadd_rn(1.0f, fast_expf_dev(-x)));
    }
}

// Orderable 32-bit image of a float: larger float, larger unsigned.
__device__ __forceinline__ unsigned int float_order(float v) {
    const unsigned int u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Greedy sampling: the first maximum of the logits (std::max_element,
// NEON-3.cpp:471-474) over the whole grid. Each CTA folds its best (value,
// index + index0) into *key as (order(value) << 32) | ~index with atomicMax --
// the larger value wins, among equal values the lower index. With `finalize`,
// the last CTA to finish writes the token to *d_tok and out[*d_step], advances
// *d_step (and *d_pos when `advance`) and clears *key; without it (a
// vocabulary shard of a tensor-parallel lm_head) *key is left for the ranks'
// key exchange. The last CTA always clears *counter for the next launch.
__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ logits, int n, int index0,
                                                     unsigned long long* key, unsigned int* counter, int* d_tok,
                                                     int* out, int* d_step, int* d_pos, int advance, int finalize) {
    __shared__ float bv[8];
    __shared__ int bi[8];
    __shared__ bool last;
    pdl_wait_d();
    pdl_trigger_d();
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = logits[i];
        if (v > best) { best = v; idx = i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { bv[w] = best; bi[w] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
            if (bv[k] > best || (bv[k] == best && bi[k] < idx)) { best = bv[k]; idx = bi[k]; }
        if (idx != 0x7fffffff)
            atomicMax(key, ((unsigned long long)float_order(best) << 32) |
                               (unsigned long long)(0xFFFFFFFFu - (unsigned)(idx + index0)));
        __threadfence();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0 && !finalize) *counter = 0u;
    if (last && threadIdx.x == 0 && finalize) {
        const unsigned long long k = atomicAdd(key, 0ull);
        const int tok = k ? (int)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull)) : 0;  // all NaN: element 0
        *d_tok = tok;
        out[*d_step] = tok;
        *d_step += 1;
        if (advance) *d_pos += 1;
        *key = 0ull;
        *counter = 0u;
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// the model
// ---------------------------------------------------------------------------

struct neon_model {
    neon_model_config_t cfg{};
    int device = 0;
    // q_dim / kv_dim / n_ff_l are this rank's shares (the whole model on one device)
    size_t q_dim = 0, kv_dim = 0, rope_half = 0;
    // tensor parallelism over `world` ranks: this rank keeps query heads
    // [rank*n_head_l, ..), KV heads [rank*n_kv_l, ..), FFN rows [ff0, ff0+n_ff_l)
    // and vocabulary rows [vocab0, vocab0+vocab_l)
    neon_comm_impl* comm = nullptr;  // null: one device
    int rank = 0, world = 1;
    size_t n_head_l = 0, n_kv_l = 0, ff0 = 0, n_ff_l = 0, vocab0 = 0, vocab_l = 0;
    neon_tensor_t head = nullptr;    // lm_head shard (tensor parallel only)
    bool head_from_output = false;   // `head` was cut from output.weight, not the tied embedding
    int quantize_to = -1;            // neon_cuda_model_set_quantize: float matrices quantised on load to this type
    float* part = nullptr;           // partial sums of the column-split projections
    float* shift_scratch = nullptr;  // ctx_len x kv_dim, for neon_cuda_model_kv_shift
    float2* shift_cs = nullptr;      // rope_half (cos, sin) of the shift angle
    // decode attention (attn_decode_kernel, attn_plan): a cluster of att_cs CTAs per KV head, K and
    // V rows in rounds of att_round, scores for att_score_rows rows
    // (att_gp: query heads per cluster, padded; att_hsplit: clusters per KV head)
    int att_gp = 1, att_cs = 1, att_round = kAttnBoxRows, att_score_rows = kAttnMinScores, att_smem = 0;
    int att_hsplit = 1;
    float* logits_full = nullptr;    // all-gathered logits (tensor parallel only)
    neon_tensor_t embd = nullptr, output = nullptr;
    float* output_norm = nullptr;
    struct Layer {
        float *attn_norm = nullptr, *ffn_norm = nullptr;
        neon_tensor_t w[5] = {};  // q, k, v, out, down
        neon_tensor_t gateup = nullptr;  // gate and up rows interleaved (2*n_ff rows); up alone for a plain FFN
        std::vector<uint8_t> gate_bytes, up_bytes;  // held until both halves are set
        int gate_type = -1, up_type = -1;
    };
    std::vector<Layer> layers;
    float *K = nullptr, *V = nullptr;   // [layer][ctx][kv_dim]
    float2* rope_cs = nullptr;          // [ctx][rope_half]
    float *h = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *gu = nullptr, *act = nullptr, *logits = nullptr;
    int *d_tokens = nullptr, *d_tok = nullptr, *d_pos = nullptr, *d_step = nullptr, *d_out = nullptr;
    unsigned* d_err = nullptr;
    unsigned long long* am_key = nullptr;  // argmax scratch
    unsigned int* am_count = nullptr;
    size_t out_cap = 0;
    size_t length = 0;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t step_graph = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cudaEvent_t evf0 = nullptr, evf1 = nullptr;  // around the last forward pass
    float forward_ms = 0.f;
    float decode_ms = 0.f;
    std::vector<void*> allocs;
    // per layer: the K and V caches as 2D tensors for attn_decode_kernel, in boxes of 32 rows (tm_k,
    // tm_v) and of one round (tm_kr, tm_vr)
    std::vector<CUtensorMap> tm_k, tm_v, tm_kr, tm_vr;
};

namespace {

int dev_alloc(neon_model* m, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return error(NEON_ERR_NOMEM, std::string("cudaMalloc in the decode engine: ") + cudaGetErrorString(e));
    m->allocs.push_back(*p);
    return NEON_OK;
}

struct ModelDevice {  // makes the model's device current for a scope
    int prev = -1;
    explicit ModelDevice(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~ModelDevice() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, what);
    return neon_internal::launched(1);
}

// Tensor-parallel shard of a GGUF tensor [ne0 = cols, ne1 = rows] kept by
// `rank` of `world`: rows [r[0], r[1]) and columns [r[2], r[3]). Attention is
// split by KV head (with its query heads), the FFN by 32-row groups of n_ff,
// the lm_head by vocabulary rows; attn_output and ffn_down are split along
// their input (the matching columns), so each rank's result is a partial sum
// of the residual update. Norms and token_embd stay whole on every rank.
int tp_shard(const neon_model_config_t& c, int role, int rank, int world, size_t r[4]) {
    if (world < 1 || rank < 0 || rank >= world) return error(NEON_ERR_INVALID, "bad rank / world");
    const size_t q_dim = (size_t)c.n_head * c.head_dim, kv_dim = (size_t)c.n_kv_head * c.head_dim;
    const size_t nbff = c.n_ff / 32, W = (size_t)world, i = (size_t)rank;
    const size_t ff0 = 32 * (nbff * i / W), ff1 = 32 * (nbff * (i + 1) / W);
    size_t rows = 0, cols = 0;
    switch (role) {
        case NEON_ROLE_OUTPUT_NORM: case NEON_ROLE_ATTN_NORM: case NEON_ROLE_FFN_NORM: rows = 1; cols = c.n_embd; break;
        case NEON_ROLE_TOKEN_EMBD: case NEON_ROLE_OUTPUT: rows = c.n_vocab; cols = c.n_embd; break;
        case NEON_ROLE_ATTN_Q: rows = q_dim; cols = c.n_embd; break;
        case NEON_ROLE_ATTN_K: case NEON_ROLE_ATTN_V: rows = kv_dim; cols = c.n_embd; break;
        case NEON_ROLE_ATTN_OUT: rows = c.n_embd; cols = q_dim; break;
        case NEON_ROLE_FFN_GATE: case NEON_ROLE_FFN_UP: rows = c.n_ff; cols = c.n_embd; break;
        case NEON_ROLE_FFN_DOWN: rows = c.n_embd; cols = c.n_ff; break;
        default: return error(NEON_ERR_INVALID, "unknown tensor role " + std::to_string(role));
    }
    r[0] = 0; r[1] = rows; r[2] = 0; r[3] = cols;
    switch (role) {
        case NEON_ROLE_OUTPUT: case NEON_ROLE_ATTN_Q: case NEON_ROLE_ATTN_K: case NEON_ROLE_ATTN_V:
            r[0] = rows * i / W; r[1] = rows * (i + 1) / W; break;  // head-aligned: n_kv_head % world == 0
        case NEON_ROLE_ATTN_OUT: r[2] = cols * i / W; r[3] = cols * (i + 1) / W; break;
        case NEON_ROLE_FFN_GATE: case NEON_ROLE_FFN_UP: r[0] = ff0; r[1] = ff1; break;
        case NEON_ROLE_FFN_DOWN: r[2] = ff0; r[3] = ff1; break;
        default: break;
    }
    return NEON_OK;
}

// Launch with programmatic dependent launch when enabled (the kernel waits for
// its predecessor with griddepcontrol.wait before reading its results).
template <typename... KArgs, typename... Args>
int launch_k(const char* what, void (*kern)(KArgs...), dim3 grid, int threads, size_t smem, cudaStream_t st,
             Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (neon_internal::pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    if (e != cudaSuccess) return cuda_error(e, what);
    return neon_internal::launched(1);
}

// h = the embedding rows of `seq` tokens (device ids): the split-layout
// kernel for Q4_0 / Q8_0, the library's decoder for the other types.
int launch_embed(neon_model* m, const int* toks, int seq) {
    const auto& c = m->cfg;
    const neon_tensor_t E = m->embd;
    if (E->pitch)
        return neon_internal::embed_rows(E, toks, seq, (int)c.n_embd, (int)c.n_vocab, m->h, m->d_err, m->stream);
    const int nb = (int)(c.n_embd / 32);
    return launch_k("embed_kernel", embed_kernel, dim3((nb + 127) / 128, seq), 128, 0, m->stream, E->qs, E->d, E->type,
                    nb, toks, (int)c.n_vocab, m->h, m->d_err);
}

// The decode attention kernel for a padded group (head dims are multiples of
// 32: 128-byte swizzled boxes).
using AttnKernel = void (*)(const float*, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, const int*, int, int, int,
                            float, int, int, int, float*, unsigned int*);
AttnKernel attn_kernel_for(int gp) {
    switch (gp) {
        case 1: return attn_decode_kernel<1, 32>;
        case 2: return attn_decode_kernel<2, 32>;
        case 4: return attn_decode_kernel<4, 32>;
        default: return attn_decode_kernel<8, 32>;
    }
}

// The layers' K and V caches as 2D tensors for the decode attention's TMA
// copies: ctx_len rows of kv_dim floats each, boxes of 32 columns (128 bytes,
// the 128-byte swizzle; a box's first column, kvh * head_dim + 32 * block, is
// 128-byte aligned) by kAttnBoxRows rows, and by att_round rows (a whole
// round in one copy per dim block). cuTensorMapEncodeTiled
// comes from the driver through the runtime's entry-point query, so the
// library does not link libcuda.
int build_kv_maps(neon_model* m) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return error(NEON_ERR_CUDA, "decode attention: cuTensorMapEncodeTiled is not available");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const auto& c = m->cfg;
    if (attn_block_width((int)c.head_dim) != 32)
        return error(NEON_ERR_UNSUPPORTED, "decode attention: head_dim must be a multiple of 32");
    m->tm_k.assign(c.n_layer, CUtensorMap{});
    m->tm_v.assign(c.n_layer, CUtensorMap{});
    m->tm_kr.assign(c.n_layer, CUtensorMap{});
    m->tm_vr.assign(c.n_layer, CUtensorMap{});
    for (uint32_t li = 0; li < c.n_layer; ++li) {
        for (int which = 0; which < 4; ++which) {
            float* base = (which & 1 ? m->V : m->K) + (size_t)li * c.ctx_len * m->kv_dim;
            CUtensorMap* tm = which == 0 ? &m->tm_k[li] : which == 1 ? &m->tm_v[li] : which == 2 ? &m->tm_kr[li] : &m->tm_vr[li];
            const cuuint64_t dims[2] = {(cuuint64_t)m->kv_dim, (cuuint64_t)c.ctx_len};
            const cuuint64_t strides[1] = {(cuuint64_t)m->kv_dim * sizeof(float)};
            const cuuint32_t box[2] = {32u, (cuuint32_t)(which < 2 ? kAttnBoxRows : m->att_round)};
            const cuuint32_t estr[2] = {1, 1};
            const CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS)
                return error(NEON_ERR_CUDA, "decode attention: cuTensorMapEncodeTiled failed (" +
                                                std::to_string((int)r) + ")");
        }
    }
    return NEON_OK;
}

// How many clusters of cs CTAs of the decode attention with `smem` bytes
// each the device holds at once (0: none; cs > 8 needs the non-portable
// cluster size).
int attn_max_clusters(AttnKernel k, int cs, int smem) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmemMax) != cudaSuccess ||
        (cs > 8 && cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3((unsigned)cs);
    q.blockDim = dim3(kAttnThreads);
    q.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = (unsigned)cs;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.attrs = qa;
    q.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, k, &q) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return clusters;
}

// The decode attention's split (attn_plan), with the largest cluster the
// device schedules (16, else 8, ...); then, while the grid leaves SMs idle,
// each KV head's query heads over 2, 4, ... clusters (the same K and V rows,
// a fraction of the score and p*v arithmetic per CTA), as long as every
// cluster of the launch stays resident at once.
int plan_attention(neon_model* m) {
    const auto& c = m->cfg;
    const int group = (int)(c.n_head / c.n_kv_head), gp = attn_group_pad(group);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device);
    for (int cs_max = kAttnMaxCluster; cs_max >= 1; cs_max /= 2) {
        AttnPlan p;
        if (!attn_plan((int)c.ctx_len, group, (int)c.head_dim, cs_max, g_attn_share_rows.load(), &p)) break;
        if (attn_max_clusters(attn_kernel_for(p.gp), p.cs, p.smem_bytes) < 1) continue;
        int hsplit = 1;
        for (int h = 2; h <= gp && h <= g_attn_head_split.load(); h *= 2) {
            AttnPlan ph;
            if ((h - 1) * (gp / h) >= group ||  // a cluster without a real query head
                (int)m->n_kv_l * h * p.cs > sms ||
                !attn_plan((int)c.ctx_len, gp / h, (int)c.head_dim, cs_max, g_attn_share_rows.load(), &ph) ||
                ph.cs != p.cs || attn_max_clusters(attn_kernel_for(ph.gp), ph.cs, ph.smem_bytes) < (int)m->n_kv_l * h)
                break;
            hsplit = h;
            p = ph;
        }
        m->att_gp = p.gp;
        m->att_hsplit = hsplit;
        m->att_cs = p.cs;
        m->att_round = p.round_rows;
        m->att_score_rows = p.score_rows;
        m->att_smem = p.smem_bytes;
        return NEON_OK;
    }
    return error(NEON_ERR_UNSUPPORTED, "decode attention: no cluster split of ctx_len fits the device");
}

// attn_decode_kernel: a cluster of att_cs CTAs per KV head, PDL when enabled.
int launch_attn_decode(neon_model* m, uint32_t li) {
    const auto& c = m->cfg;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(m->n_kv_l * m->att_hsplit * m->att_cs));
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = (size_t)m->att_smem;
    cfg.stream = m->stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)m->att_cs;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
    if (neon_internal::pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    const float scale = 1.0f / std::sqrt((float)c.head_dim);
    const int min_rows = std::min(g_attn_min_rows.load(), m->att_score_rows);
    cudaError_t e = cudaLaunchKernelEx(&cfg, attn_kernel_for(m->att_gp), (const float*)m->q, m->tm_k[li], m->tm_v[li],
                                       m->tm_kr[li], m->tm_vr[li], (const int*)m->d_pos, (int)c.head_dim, (int)(c.n_head / c.n_kv_head),
                                       m->att_hsplit, scale,
                                       min_rows, m->att_round, m->att_score_rows, m->att, m->d_err);
    if (e != cudaSuccess) return cuda_error(e, "attn_decode_kernel");
    return neon_internal::launched(1);
}

int rmsnorm(neon_model* m, const float* x, const float* w, float* out, int rows) {
    rmsnorm_kernel<<<rows, kThreads, 0, m->stream>>>(x, w, out, (int)m->cfg.n_embd, m->cfg.norm_eps);
    return check_launch("rmsnorm_kernel");
}

int proj(neon_model* m, std::initializer_list<neon_proj_target_t> t, const float* x, size_t x_stride, size_t seq,
         int accumulate) {
    std::vector<neon_proj_target_t> v(t);
    return neon_internal::matvec(v.data(), v.size(), x, x_stride, seq, m->stream, accumulate);
}

// h += W x for `seq` positions (attn_output, ffn_down). Tensor parallel: W is
// this rank's column shard, its partial sum goes through the all-reduce, and
// h += sum over ranks in rank order (identical on every rank).
int residual_proj(neon_model* m, neon_tensor_t W, const float* x, size_t x_stride, size_t seq) {
    const size_t n_embd = m->cfg.n_embd;
    if (m->world == 1) return proj(m, {{W, m->h, n_embd}}, x, x_stride, seq, 1);
    int rc = proj(m, {{W, m->part, n_embd}}, x, x_stride, seq, 0);
    if (!rc) rc = neon_internal::comm_allreduce(m->comm, m->part, m->h, (long long)(seq * n_embd), 1, m->stream);
    return rc;
}

// All layers for `seq` positions starting at *d_pos, tokens in `toks` (device).
int run_layers(neon_model* m, const int* toks, int seq) {
    const auto& c = m->cfg;
    int rc = launch_embed(m, toks, seq);
    const size_t n_embd = c.n_embd, q_dim = m->q_dim, kv_dim = m->kv_dim, n_ff = m->n_ff_l;
    const float scale = 1.0f / std::sqrt((float)c.head_dim);
    const int group = (int)(c.n_head / c.n_kv_head);
    const size_t attn_smem = sizeof(float) * c.ctx_len;
    for (uint32_t li = 0; li < c.n_layer && !rc; ++li) {
        auto& L = m->layers[li];
        float* Kl = m->K + (size_t)li * c.ctx_len * kv_dim;
        float* Vl = m->V + (size_t)li * c.ctx_len * kv_dim;
        rc = rmsnorm(m, m->h, L.attn_norm, m->xn, seq);
        if (!rc) rc = proj(m, {{L.w[0], m->q, q_dim}, {L.w[1], m->k, kv_dim}, {L.w[2], m->v, kv_dim}}, m->xn, n_embd, seq, 0);
        if (!rc) {
            rope_kv_kernel<<<seq, kThreads, 0, m->stream>>>(m->q, m->k, m->v, m->rope_cs, m->d_pos, (int)m->n_head_l,
                                                            (int)m->n_kv_l, (int)c.head_dim, (int)m->rope_half,
                                                            (int)q_dim, (int)kv_dim, Kl, Vl);
            rc = check_launch("rope_kv_kernel");
        }
        if (!rc && (c.head_dim == 64 || c.head_dim == 128)) {
            // register-tiled fp32 tiles of 64 positions per query head
            const dim3 grid((unsigned)m->n_head_l, (unsigned)((seq + kPfRows - 1) / kPfRows));
            if (c.head_dim == 128)
                attn_prefill_f32_kernel<128><<<grid, kPfThreads, pf_smem_bytes<128>(), m->stream>>>(
                    m->q, Kl, Vl, m->att, m->d_pos, seq, (int)q_dim, (int)kv_dim, group, scale);
            else
                attn_prefill_f32_kernel<64><<<grid, kPfThreads, pf_smem_bytes<64>(), m->stream>>>(
                    m->q, Kl, Vl, m->att, m->d_pos, seq, (int)q_dim, (int)kv_dim, group, scale);
            rc = check_launch("attn_prefill_f32_kernel");
        } else if (!rc && neon_internal::prefill_mma() && c.head_dim <= (uint32_t)kApMaxHd && c.head_dim % 8 == 0) {
            // tensor-core tiles of 64 positions per query head
            attn_prefill_mma_kernel<<<dim3((unsigned)m->n_head_l, (unsigned)((seq + kApRows - 1) / kApRows)), 128,
                                      ap_smem_bytes((int)c.head_dim), m->stream>>>(
                m->q, Kl, Vl, m->att, m->d_pos, seq, (int)q_dim, (int)kv_dim, (int)c.head_dim, group, scale);
            rc = check_launch("attn_prefill_mma_kernel");
        } else if (!rc) {
            attention_kernel<<<dim3((unsigned)m->n_head_l, seq), kThreads, attn_smem, m->stream>>>(
                m->q, Kl, Vl, m->att, m->d_pos, (int)q_dim, (int)kv_dim, (int)c.head_dim, group, scale);
            rc = check_launch("attention_kernel");
        }
        if (!rc) rc = residual_proj(m, L.w[3], m->att, q_dim, seq);
        if (!rc) rc = rmsnorm(m, m->h, L.ffn_norm, m->xn, seq);
        const size_t gu_rows = m->cfg.plain_ffn ? n_ff : 2 * n_ff;
        if (!rc) rc = proj(m, {{L.gateup, m->gu, gu_rows}}, m->xn, n_embd, seq, 0);
        if (!rc) {
            const long long n = (long long)seq * n_ff;
            const int grid = (int)std::min<long long>((n + 255) / 256, 4096);
            if (m->cfg.plain_ffn) {
                silu_kernel<<<grid, 256, 0, m->stream>>>(m->gu, m->act, n);
                rc = check_launch("silu_kernel");
            } else {
                swiglu_pairs_kernel<<<grid, 256, 0, m->stream>>>(m->gu, m->act, n);
                rc = check_launch("swiglu_pairs_kernel");
            }
        }
        if (!rc) rc = residual_proj(m, L.w[4], m->act, n_ff, seq);
    }
    return rc;
}

// logits of residual row x: rms_norm(output_norm) folded into the lm_head matvec
int run_head(neon_model* m, const float* x) {
    neon_tensor_t W = m->world > 1 ? m->head : m->output ? m->output : m->embd;
    neon_proj_target_t t{W, m->logits, m->vocab_l};
    neon_internal::MatvecExt ext;
    ext.norm_w = m->output_norm;
    ext.norm_eps = m->cfg.norm_eps;
    return neon_internal::matvec(&t, 1, x, m->cfg.n_embd, 1, m->stream, 0, &ext);
}

// One decode position (token in *d_tok, position *d_pos): the fused step.
//
// Tensor parallel with fused collectives: attn_output and ffn_down store their
// partial rows as LL words straight into every rank's slot, and a small
// reduce launch adds the ranks' rows into the residual.
int run_step(neon_model* m) {
    const auto& c = m->cfg;
    int rc = launch_embed(m, m->d_tok, 1);
    const size_t n_embd = c.n_embd, q_dim = m->q_dim, kv_dim = m->kv_dim, n_ff = m->n_ff_l;
    const bool fused = m->world > 1 && neon_internal::fused_collectives();
    float* hc = m->h;
    // h += W x: fused producer + LL reduce, or matvec + all-reduce, or one device's accumulate
    auto residual = [&](neon_tensor_t W, const float* x, size_t x_stride) {
        if (!fused) {
            if (m->world == 1) return proj(m, {{W, hc, n_embd}}, x, x_stride, 1, 1);
            int r = proj(m, {{W, m->part, n_embd}}, x, x_stride, 1, 0);
            if (!r) r = neon_internal::comm_allreduce(m->comm, m->part, hc, (long long)n_embd, 1, m->stream);
            return r;
        }
        const neon_proj_target_t t{W, m->part, n_embd};
        neon_internal::MatvecExt ext;
        ext.peer_mode = 1;
        ext.peer = neon_internal::comm_peer_set(m->comm);
        bool streamed = false;  // a long producer: the reduce polls its words while its tail runs
        ext.launched_stream = &streamed;
        int r = neon_internal::matvec(&t, 1, x, x_stride, 1, m->stream, 0, &ext);
        if (!r) r = neon_internal::comm_ll_reduce(m->comm, hc, (long long)n_embd, m->stream, !streamed);
        return r;
    };
    for (uint32_t li = 0; li < c.n_layer && !rc; ++li) {
        auto& L = m->layers[li];
        float* Kl = m->K + (size_t)li * c.ctx_len * kv_dim;
        float* Vl = m->V + (size_t)li * c.ctx_len * kv_dim;
        {
            // q, k, v = W x with x = rms_norm(h); RoPE on q and k; k and v into the cache
            const neon_proj_target_t t[3] = {{L.w[0], m->q, q_dim}, {L.w[1], Kl, kv_dim}, {L.w[2], Vl, kv_dim}};
            const int epi[3] = {neon::kEpiRope, neon::kEpiRope, neon::kEpiAtPos};
            const long long stride[3] = {0, (long long)kv_dim, (long long)kv_dim};
            neon_internal::MatvecExt ext;
            ext.norm_w = L.attn_norm;
            ext.norm_eps = c.norm_eps;
            ext.d_pos = m->d_pos;
            ext.rope_cs = m->rope_cs;
            ext.rope_half = (int)m->rope_half;
            ext.head_dim = (int)c.head_dim;
            ext.epi = epi;
            ext.pos_stride = stride;
            rc = neon_internal::matvec(t, 3, hc, n_embd, 1, m->stream, 0, &ext);
        }
        if (!rc) rc = launch_attn_decode(m, li);
        if (!rc) rc = residual(L.w[3], m->att, q_dim);
        if (!rc) {
            // act = silu(gate) * up, (gate, up) = W x with x = rms_norm(h); or silu(up)
            const neon_proj_target_t t{L.gateup, m->act, n_ff};
            const int epi = m->cfg.plain_ffn ? neon::kEpiSilu : neon::kEpiSwiglu;
            const long long stride = 0;
            neon_internal::MatvecExt ext;
            ext.norm_w = L.ffn_norm;
            ext.norm_eps = c.norm_eps;
            ext.epi = &epi;
            ext.pos_stride = &stride;
            rc = neon_internal::matvec(&t, 1, hc, n_embd, 1, m->stream, 0, &ext);
        }
        if (!rc) rc = residual(L.w[4], m->act, n_ff);
    }
    return rc;
}

int launch_argmax(neon_model* m, int advance) {
    const int grid = std::max(1, std::min<int>(148, (int)((m->vocab_l + 1023) / 1024)));
    int rc = launch_k("argmax_kernel", argmax_kernel, dim3(grid), 256, 0, m->stream, m->logits, (int)m->vocab_l,
                      (int)m->vocab0, m->am_key, m->am_count, m->d_tok, m->d_out, m->d_step, m->d_pos, advance,
                      (int)(m->world == 1));
    if (!rc && m->world > 1)
        rc = neon_internal::comm_argmax(m->comm, m->am_key, m->d_tok, m->d_out, m->d_step, m->d_pos, advance, m->stream);
    return rc;
}

int check_ready(neon_model* m) {
    if (!m->embd || !m->output_norm) return error(NEON_ERR_INVALID, "forward(): token_embd.weight / output_norm.weight not set");
    if (m->world > 1 && !m->head) return error(NEON_ERR_INVALID, "forward(): lm_head shard not set");
    for (uint32_t i = 0; i < m->cfg.n_layer; ++i) {
        auto& L = m->layers[i];
        if (!L.attn_norm || !L.ffn_norm)
            return error(NEON_ERR_INVALID, "forward(): layer " + std::to_string(i) + " is missing a norm weight");
        for (auto* w : L.w)
            if (!w) return error(NEON_ERR_INVALID, "forward(): layer " + std::to_string(i) + " is missing a projection");
        if (!L.gateup)
            return error(NEON_ERR_INVALID, "forward(): layer " + std::to_string(i) + " is missing ffn_gate or ffn_up");
    }
    return NEON_OK;
}

int sync_and_check(neon_model* m) {
    DEC_TRY(cudaStreamSynchronize(m->stream));
    unsigned e = 0;
    DEC_TRY(cudaMemcpy(&e, m->d_err, sizeof(e), cudaMemcpyDeviceToHost));
    if (e & 2u) {
        DEC_TRY(cudaMemset(m->d_err, 0, sizeof(unsigned)));
        return error(NEON_ERR_INVALID, "forward(): token id out of vocab range");
    }
    if (e & 4u) {
        DEC_TRY(cudaMemset(m->d_err, 0, sizeof(unsigned)));
        return error(NEON_ERR_CUDA, "decode attention: a shared-memory copy of the KV cache never completed");
    }
    if (e & 8u) {
        DEC_TRY(cudaMemset(m->d_err, 0, sizeof(unsigned)));
        return error(NEON_ERR_CUDA, "decode attention: dynamic shared memory not 1024-byte aligned");
    }
    if (m->world > 1) {
        const int rc = neon_cuda_comm_check(static_cast<neon_comm*>(m->comm));
        if (rc) return rc;
    }
    return neon_internal::check_device_error(m->device);
}

// Tokens [0, n) of `tokens_dev` at positions length..; logits of the last.
int forward_device(neon_model* m, const int32_t* tokens_host, size_t n) {
    for (size_t off = 0; off < n; off += kMaxChunk) {
        const int seq = (int)std::min<size_t>(kMaxChunk, n - off);
        const int pos = (int)(m->length + off);
        DEC_TRY(cudaMemcpyAsync(m->d_tokens, tokens_host + off, seq * sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
        DEC_TRY(cudaMemcpyAsync(m->d_pos, &pos, sizeof(int), cudaMemcpyHostToDevice, m->stream));
        int rc;
        if (seq == 1) {
            DEC_TRY(cudaMemcpyAsync(m->d_tok, tokens_host + off, sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
            rc = run_step(m);
        } else {
            rc = run_layers(m, m->d_tokens, seq);
        }
        if (rc) return rc;
        if (off + seq == n) {
            rc = run_head(m, m->h + (size_t)(seq - 1) * m->cfg.n_embd);
            if (!rc && m->world > 1)
                rc = neon_internal::comm_allgather(m->comm, m->logits, m->logits_full, (long long)m->cfg.n_vocab, m->stream);
            if (rc) return rc;
        }
        DEC_TRY(cudaStreamSynchronize(m->stream));  // pos / tokens are reused by the next chunk
    }
    return NEON_OK;
}

}  // namespace

extern "C" {

int neon_cuda_model_comm_floats(const neon_model_config_t* cfg, int world, size_t* n) {
    if (!cfg || !n || world < 1) return error(NEON_ERR_INVALID, "bad argument");
    *n = std::max<size_t>((size_t)kMaxChunk * cfg->n_embd, ((size_t)cfg->n_vocab + world - 1) / world);
    return NEON_OK;
}

int neon_cuda_tp_shard(const neon_model_config_t* cfg, int role, int rank, int world, size_t range[4]) {
    if (!cfg || !range) return error(NEON_ERR_INVALID, "null argument");
    return tp_shard(*cfg, role, rank, world, range);
}

int neon_cuda_model_create(const neon_model_config_t* cfg, neon_model_t* out) {
    return neon_cuda_model_create_tp(cfg, nullptr, out);
}

int neon_cuda_model_create_tp(const neon_model_config_t* cfg, neon_comm_t comm, neon_model_t* out) {
    if (!cfg || !out) return error(NEON_ERR_INVALID, "null argument");
    *out = nullptr;
    const auto& c = *cfg;
    if (c.n_embd == 0 || c.n_layer == 0 || c.n_head == 0 || c.n_kv_head == 0 || c.head_dim == 0 || c.n_ff == 0 ||
        c.n_vocab == 0 || c.ctx_len == 0)
        return error(NEON_ERR_INVALID, "NANITY: one or more required hyperparameters is zero.");
    if (c.n_head % c.n_kv_head != 0)
        return error(NEON_ERR_INVALID, "NANITY: attention.head_count must be an exact multiple of attention.head_count_kv");
    if (c.head_dim % 32 != 0 || c.head_dim > 256 || c.n_embd % 32 != 0 || c.n_ff % 32 != 0)
        return error(NEON_ERR_UNSUPPORTED, "head_dim must be a multiple of 32 up to 256; n_embd and n_ff multiples of 32");
    if (c.ctx_len > (uint32_t)kMaxCtx) return error(NEON_ERR_UNSUPPORTED, "ctx_len above 16384");
    if (c.n_head / c.n_kv_head > 8) return error(NEON_ERR_UNSUPPORTED, "more than 8 query heads per KV head");
    if (c.rope_dim_count > c.head_dim) return error(NEON_ERR_INVALID, "rope dimension count above head_dim");
    const int world = comm ? comm->peers.world : 1, rank = comm ? comm->peers.rank : 0;
    if (comm) {
        if (!comm->connected) return error(NEON_ERR_INVALID, "communicator not connected");
        int dev = -1;
        cudaGetDevice(&dev);
        if (dev != comm->device) return error(NEON_ERR_INVALID, "the communicator lives on another device");
        if (c.n_kv_head % (uint32_t)world != 0)
            return error(NEON_ERR_UNSUPPORTED, "tensor parallelism needs n_kv_head divisible by the number of ranks");
        if (c.n_ff / 32 < (uint32_t)world || c.n_vocab < (uint32_t)world)
            return error(NEON_ERR_UNSUPPORTED, "n_ff / 32 and n_vocab must be at least the number of ranks");
        size_t need = 0;
        neon_cuda_model_comm_floats(cfg, world, &need);
        if ((size_t)comm->peers.max_floats < need)
            return error(NEON_ERR_INVALID, "communicator buffer below neon_cuda_model_comm_floats() = " + std::to_string(need));
    }
    auto* m = new neon_model();
    m->cfg = c;
    cudaGetDevice(&m->device);
    m->comm = world > 1 ? comm : nullptr;
    m->world = world;
    m->rank = rank;
    {
        size_t r[4];
        tp_shard(c, NEON_ROLE_ATTN_Q, rank, world, r);
        m->q_dim = r[1] - r[0];
        tp_shard(c, NEON_ROLE_ATTN_K, rank, world, r);
        m->kv_dim = r[1] - r[0];
        tp_shard(c, NEON_ROLE_FFN_GATE, rank, world, r);
        m->ff0 = r[0];
        m->n_ff_l = r[1] - r[0];
        tp_shard(c, NEON_ROLE_OUTPUT, rank, world, r);
        m->vocab0 = r[0];
        m->vocab_l = r[1] - r[0];
    }
    m->n_head_l = c.n_head / world;
    m->n_kv_l = c.n_kv_head / world;
    m->rope_half = c.rope_dim_count ? c.rope_dim_count / 2 : c.head_dim / 2;
    m->layers.resize(c.n_layer);
    int rc = NEON_OK;
    const size_t S = kMaxChunk;
    auto A = [&](void** p, size_t bytes) {
        if (!rc) rc = dev_alloc(m, p, bytes);
    };
    const size_t kv_bytes = sizeof(float) * (size_t)c.n_layer * c.ctx_len * m->kv_dim;
    A((void**)&m->K, kv_bytes);
    A((void**)&m->V, kv_bytes);
    A((void**)&m->rope_cs, sizeof(float2) * (size_t)c.ctx_len * std::max<size_t>(1, m->rope_half));
    A((void**)&m->h, sizeof(float) * S * c.n_embd);
    A((void**)&m->xn, sizeof(float) * S * c.n_embd);
    A((void**)&m->q, sizeof(float) * S * m->q_dim);
    A((void**)&m->k, sizeof(float) * S * m->kv_dim);
    A((void**)&m->v, sizeof(float) * S * m->kv_dim);
    A((void**)&m->att, sizeof(float) * S * m->q_dim);
    A((void**)&m->gu, sizeof(float) * S * 2 * m->n_ff_l);
    A((void**)&m->act, sizeof(float) * S * m->n_ff_l);
    if (world > 1) {
        A((void**)&m->part, sizeof(float) * S * c.n_embd);
        A((void**)&m->logits_full, sizeof(float) * c.n_vocab);
    }
    A((void**)&m->am_key, sizeof(unsigned long long));
    A((void**)&m->am_count, sizeof(unsigned int));
    A((void**)&m->logits, sizeof(float) * m->vocab_l);
    A((void**)&m->d_tokens, sizeof(int) * S);
    A((void**)&m->d_tok, sizeof(int));
    A((void**)&m->d_pos, sizeof(int));
    A((void**)&m->d_step, sizeof(int));
    A((void**)&m->d_err, sizeof(unsigned));
    if (!rc) rc = plan_attention(m);
    if (!rc) rc = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) == cudaSuccess ? NEON_OK : error(NEON_ERR_CUDA, "cudaStreamCreate");
    if (!rc) rc = (cudaEventCreate(&m->ev0) == cudaSuccess && cudaEventCreate(&m->ev1) == cudaSuccess &&
                   cudaEventCreate(&m->evf0) == cudaSuccess && cudaEventCreate(&m->evf1) == cudaSuccess)
                      ? NEON_OK
                      : error(NEON_ERR_CUDA, "cudaEventCreate");
    if (!rc) {
        // RoPE cos/sin of every position with the host libm, as rope_apply computes
        // them (rawllm_forward.hpp:755-782): theta = ((float)pos / scale) * freq.
        std::vector<float> freqs(c.head_dim / 2);
        for (size_t i = 0; i < c.head_dim / 2; ++i) freqs[i] = std::pow(c.rope_base, -2.0f * (float)i / (float)c.head_dim);
        std::vector<float2> tab((size_t)c.ctx_len * std::max<size_t>(1, m->rope_half));
        for (size_t p = 0; p < c.ctx_len; ++p) {
            const float fpos = (float)p / c.rope_scale;
            for (size_t i = 0; i < m->rope_half; ++i) {
                const float theta = fpos * freqs[i];
                tab[p * m->rope_half + i] = make_float2(std::cos(theta), std::sin(theta));
            }
        }
        if (cudaMemcpy(m->rope_cs, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemset(m->d_err, 0, sizeof(unsigned)) != cudaSuccess || cudaMemset(m->K, 0, kv_bytes) != cudaSuccess ||
            cudaMemset(m->am_key, 0, sizeof(unsigned long long)) != cudaSuccess ||
            cudaMemset(m->am_count, 0, sizeof(unsigned int)) != cudaSuccess ||
            cudaMemset(m->V, 0, kv_bytes) != cudaSuccess)
            rc = error(NEON_ERR_CUDA, "model initialisation copies failed");
    }
    if (!rc) rc = build_kv_maps(m);
    if (!rc && c.ctx_len * sizeof(float) > 48 * 1024) {
        if (cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(c.ctx_len * sizeof(float))) != cudaSuccess)
            rc = error(NEON_ERR_CUDA, "cudaFuncSetAttribute(attention_kernel)");
    }
    if (!rc && c.head_dim <= (uint32_t)kApMaxHd &&
        cudaFuncSetAttribute(attn_prefill_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ap_smem_bytes((int)c.head_dim)) != cudaSuccess)
        rc = error(NEON_ERR_CUDA, "cudaFuncSetAttribute(attn_prefill_mma_kernel)");
    if (!rc && (cudaFuncSetAttribute(attn_prefill_f32_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     pf_smem_bytes<128>()) != cudaSuccess ||
                cudaFuncSetAttribute(attn_prefill_f32_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     pf_smem_bytes<64>()) != cudaSuccess))
        rc = error(NEON_ERR_CUDA, "cudaFuncSetAttribute(attn_prefill_f32_kernel)");
    if (rc) {
        neon_cuda_model_free(m);
        return rc;
    }
    *out = m;
    return NEON_OK;
}

int neon_cuda_set_attn_head_split(int max_split) {
    if (max_split < 1 || max_split > kAttnMaxGroup || (max_split & (max_split - 1)))
        return error(NEON_ERR_INVALID, "attention head split: a power of two from 1 to 8");
    g_attn_head_split.store(max_split);
    return NEON_OK;
}

int neon_cuda_set_attn_rows(int min_rows, int share_rows) {
    if (min_rows < kAttnBoxRows || share_rows < kAttnBoxRows || min_rows > kMaxCtx || share_rows > kMaxCtx ||
        min_rows % kAttnBoxRows || share_rows % kAttnBoxRows)
        return error(NEON_ERR_INVALID, "attention rows: multiples of 32 from 32 to 16384");
    g_attn_min_rows.store(min_rows);
    g_attn_share_rows.store(share_rows);
    return NEON_OK;
}

int neon_cuda_model_set_quantize(neon_model_t m, int ggml_type) {
    if (!m) return error(NEON_ERR_INVALID, "null argument");
    if (ggml_type >= 0 && ggml_type != NEON_GGML_Q8_0 && ggml_type != NEON_GGML_Q4_0 && ggml_type != NEON_GGML_Q4_1 &&
        ggml_type != NEON_GGML_Q5_0 && ggml_type != NEON_GGML_Q5_1 && ggml_type != NEON_GGML_F16 &&
        ggml_type != NEON_GGML_BF16)
        return error(NEON_ERR_UNSUPPORTED, "on-load quantisation to type " + std::to_string(ggml_type) +
                                               " is not available (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, F16, BF16 are)");
    m->quantize_to = ggml_type < 0 ? -1 : ggml_type;
    return NEON_OK;
}

int neon_cuda_model_set_tensor(neon_model_t m, int role, int layer, const uint8_t* host_bytes, size_t nbytes,
                               int ggml_type, size_t ne0, size_t ne1) {
    if (!m || !host_bytes) return error(NEON_ERR_INVALID, "null argument");
    ModelDevice md(m->device);
    const auto& c = m->cfg;
    const bool matrix = role != NEON_ROLE_OUTPUT_NORM && role != NEON_ROLE_ATTN_NORM && role != NEON_ROLE_FFN_NORM;
    if (matrix && m->quantize_to >= 0 && m->quantize_to != ggml_type &&
        (ggml_type == NEON_GGML_F32 || ggml_type == NEON_GGML_F16 || ggml_type == NEON_GGML_BF16) && ne1 > 0) {
        // a float matrix (a .nctr tensor, an F32/F16 GGUF tensor): quantise it
        // on the device first, as the exporters' gguf-py would have
        const size_t in_row = neon_internal::gguf_row_bytes(ggml_type, ne0);
        const size_t out_row = neon_internal::gguf_row_bytes(m->quantize_to, ne0);
        if (in_row == 0 || out_row == 0)
            return error(NEON_ERR_UNSUPPORTED, "on-load quantisation: input dim " + std::to_string(ne0) +
                                                   " is not a multiple of the block size");
        if (nbytes < in_row * ne1) return error(NEON_ERR_INVALID, "tensor bytes shorter than its shape");
        std::vector<uint8_t> q(out_row * ne1);
        int rc = neon_cuda_quantize_host(host_bytes, ggml_type, ne1, ne0, m->quantize_to, q.data());
        if (rc) return rc;
        return neon_cuda_model_set_tensor(m, role, layer, q.data(), q.size(), m->quantize_to, ne0, ne1);
    }
    if (role == NEON_ROLE_OUTPUT_NORM || role == NEON_ROLE_ATTN_NORM || role == NEON_ROLE_FFN_NORM) {
        // any type the reference dequantises (dequant_full, rawllm_forward.hpp:
        // 325-328, at :1077 / :1161 / :1226), decoded to F32 here, once
        const size_t rb = neon_internal::gguf_row_bytes(ggml_type, ne0);
        if (ne0 != c.n_embd || ne1 > 1 || rb == 0 || nbytes != rb)
            return error(NEON_ERR_INVALID, "NANITY: norm weight must be [n_embd] of a dequantisable type (F32, F16, "
                                           "BF16 or a block type whose block divides n_embd)");
        std::vector<float> w(ne0);
        if (!neon_internal::dequantize_row_host(ggml_type, host_bytes, ne0, w.data()))
            return error(NEON_ERR_UNSUPPORTED, "norm weight of type " + std::to_string(ggml_type) + " is not supported");
        float* p = nullptr;
        int rc = dev_alloc(m, (void**)&p, ne0 * sizeof(float));
        if (rc) return rc;
        DEC_TRY(cudaMemcpy(p, w.data(), ne0 * sizeof(float), cudaMemcpyHostToDevice));
        if (role == NEON_ROLE_OUTPUT_NORM) m->output_norm = p;
        else {
            if (layer < 0 || (uint32_t)layer >= c.n_layer) return error(NEON_ERR_INVALID, "layer index out of range");
            (role == NEON_ROLE_ATTN_NORM ? m->layers[layer].attn_norm : m->layers[layer].ffn_norm) = p;
        }
        return NEON_OK;
    }
    // projections: expected GGUF ne = [cols, rows] of the whole tensor; a
    // tensor-parallel rank keeps its shard (tp_shard)
    size_t sh[4];
    int rc0 = tp_shard(c, role, m->rank, m->world, sh);
    if (rc0) return rc0;
    size_t want0 = 0, want1 = 0;
    {
        size_t whole[4];
        tp_shard(c, role, 0, 1, whole);
        want0 = whole[3];
        want1 = whole[1];
    }
    if (ne0 != want0 || ne1 != want1)
        return error(NEON_ERR_INVALID, "NANITY: tensor of role " + std::to_string(role) + " has shape [" + std::to_string(ne0) +
                                           ", " + std::to_string(ne1) + "], expected [" + std::to_string(want0) + ", " +
                                           std::to_string(want1) + "].");
    if (role != NEON_ROLE_TOKEN_EMBD && role != NEON_ROLE_OUTPUT && (layer < 0 || (uint32_t)layer >= c.n_layer))
        return error(NEON_ERR_INVALID, "layer index out of range");
    {
        const size_t rb = neon_internal::gguf_row_bytes(ggml_type, ne0);
        if (rb == 0)
            return error(NEON_ERR_UNSUPPORTED, "NANITY: tensor of role " + std::to_string(role) + ": quant type " +
                                                   std::to_string(ggml_type) + " with input dim " + std::to_string(ne0) +
                                                   " is not supported");
        if (nbytes < rb * ne1) return error(NEON_ERR_INVALID, "tensor bytes shorter than its shape");
    }
    if (role == NEON_ROLE_FFN_GATE && c.plain_ffn)
        return error(NEON_ERR_INVALID, "ffn_gate given to a plain SiLU-FFN model (plain_ffn = 1)");
    if (role == NEON_ROLE_FFN_UP && c.plain_ffn) {
        // plain SiLU-FFN: the up rows alone (this rank's [ff0, ff0 + n_ff_l))
        const size_t row_b = neon_internal::gguf_row_bytes(ggml_type, ne0);
        if (row_b == 0) return error(NEON_ERR_UNSUPPORTED, "ffn_up: unsupported quant type or input dim");
        if (nbytes < row_b * ne1) return error(NEON_ERR_INVALID, "tensor bytes shorter than its shape");
        neon_tensor_t t = nullptr;
        int rc = neon_cuda_upload(host_bytes + sh[0] * row_b, ggml_type, sh[1] - sh[0], ne0, NEON_SHARD_NONE, 0, 1, &t);
        if (rc) return rc;
        auto& L = m->layers[layer];
        if (L.gateup) neon_cuda_free(L.gateup);
        L.gateup = t;
        return NEON_OK;
    }
    if (role == NEON_ROLE_FFN_GATE || role == NEON_ROLE_FFN_UP) {
        // held until both halves are present, then uploaded as one tensor whose
        // row 2i is gate row i and row 2i+1 up row i (same bytes, same math)
        // (a tensor-parallel rank keeps rows [ff0, ff0 + n_ff_l) of both)
        auto& L = m->layers[layer];
        const size_t row_b = neon_internal::gguf_row_bytes(ggml_type, ne0);
        if (row_b == 0) return error(NEON_ERR_UNSUPPORTED, "ffn_gate / ffn_up: unsupported quant type or input dim");
        if (nbytes < row_b * ne1) return error(NEON_ERR_INVALID, "tensor bytes shorter than its shape");
        const size_t r0 = sh[0], nr = sh[1] - sh[0];
        (role == NEON_ROLE_FFN_GATE ? L.gate_bytes : L.up_bytes)
            .assign(host_bytes + r0 * row_b, host_bytes + (r0 + nr) * row_b);
        (role == NEON_ROLE_FFN_GATE ? L.gate_type : L.up_type) = ggml_type;
        if (L.gate_bytes.empty() || L.up_bytes.empty()) return NEON_OK;
        if (L.gate_type != L.up_type) return error(NEON_ERR_UNSUPPORTED, "ffn_gate and ffn_up must share a quant type");
        std::vector<uint8_t> inter(2 * row_b * nr);
        for (size_t r = 0; r < nr; ++r) {
            std::memcpy(inter.data() + (2 * r) * row_b, L.gate_bytes.data() + r * row_b, row_b);
            std::memcpy(inter.data() + (2 * r + 1) * row_b, L.up_bytes.data() + r * row_b, row_b);
        }
        neon_tensor_t t = nullptr;
        int rc = neon_cuda_upload(inter.data(), ggml_type, 2 * nr, ne0, NEON_SHARD_NONE, 0, 1, &t);
        if (rc) return rc;
        if (L.gateup) neon_cuda_free(L.gateup);
        L.gateup = t;
        L.gate_bytes.clear();
        L.gate_bytes.shrink_to_fit();
        L.up_bytes.clear();
        L.up_bytes.shrink_to_fit();
        return NEON_OK;
    }
    int mode = NEON_SHARD_NONE;
    if (m->world > 1) {
        if (sh[0] != 0 || sh[1] != ne1) mode = NEON_SHARD_ROWS;
        else if (sh[2] != 0 || sh[3] != ne0) mode = NEON_SHARD_COLS;
    }
    if (mode == NEON_SHARD_COLS) {
        // the upload keeps blocks [nblk*r/W, nblk*(r+1)/W) of every row: that
        // must be exactly this rank's column range (256-value K-quant blocks
        // may not split where the 32-column plan does)
        const size_t be = std::max<size_t>(32, neon_internal::gguf_block_elems(ggml_type));
        const size_t nblk = ne0 / be;
        const size_t b0 = nblk * (size_t)m->rank / (size_t)m->world, b1 = nblk * (size_t)(m->rank + 1) / (size_t)m->world;
        if (ne0 % be != 0 || b0 * be != sh[2] || b1 * be != sh[3])
            return error(NEON_ERR_UNSUPPORTED, "tensor-parallel column split of role " + std::to_string(role) +
                                                   ": columns [" + std::to_string(sh[2]) + ", " + std::to_string(sh[3]) +
                                                   ") do not fall on this type's " + std::to_string(be) + "-value blocks");
    }
    if (m->world > 1 && (role == NEON_ROLE_OUTPUT || (role == NEON_ROLE_TOKEN_EMBD && !m->head_from_output))) {
        // the lm_head's vocabulary shard (of output.weight, or of the tied embedding)
        neon_tensor_t hs = nullptr;
        int rc = neon_cuda_upload(host_bytes, ggml_type, ne1, ne0, NEON_SHARD_ROWS, m->rank, m->world, &hs);
        if (rc) return rc;
        if (m->head) neon_cuda_free(m->head);
        m->head = hs;
        if (role == NEON_ROLE_OUTPUT) {
            m->head_from_output = true;
            return NEON_OK;
        }
    }
    neon_tensor_t t = nullptr;
    int rc = neon_cuda_upload(host_bytes, ggml_type, ne1, ne0, mode, m->rank, m->world, &t);
    if (rc) return rc;
    neon_tensor_t* slot = nullptr;
    if (role == NEON_ROLE_TOKEN_EMBD) slot = &m->embd;
    else if (role == NEON_ROLE_OUTPUT) slot = &m->output;
    else {
        // projection slots: q, k, v, out (roles 4-7), down (role 11)
        const int idx = role <= NEON_ROLE_ATTN_OUT ? role - NEON_ROLE_ATTN_Q : 4;
        slot = &m->layers[layer].w[idx];
    }
    if (*slot) neon_cuda_free(*slot);
    *slot = t;
    return NEON_OK;
}

int neon_cuda_model_forward(neon_model_t m, const int32_t* tokens, size_t n, float* logits_host) {
    if (!m || (!tokens && n)) return error(NEON_ERR_INVALID, "null argument");
    if (n == 0) return error(NEON_ERR_INVALID, "forward(): empty token batch");
    if (m->length + n > m->cfg.ctx_len)
        return error(NEON_ERR_INVALID, "forward(): KV cache exhausted (ctx_len=" + std::to_string(m->cfg.ctx_len) + " exceeded)");
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= m->cfg.n_vocab)
            return error(NEON_ERR_INVALID, "forward(): token id " + std::to_string(tokens[i]) + " out of vocab range");
    int rc = check_ready(m);
    if (rc) return rc;
    ModelDevice md(m->device);
    DEC_TRY(cudaEventRecord(m->evf0, m->stream));
    rc = forward_device(m, tokens, n);
    if (!rc) rc = cuda_error_if(cudaEventRecord(m->evf1, m->stream), "cudaEventRecord");
    if (!rc) rc = sync_and_check(m);
    if (rc) return rc;
    cudaEventElapsedTime(&m->forward_ms, m->evf0, m->evf1);
    m->length += n;
    if (logits_host)
        DEC_TRY(cudaMemcpy(logits_host, m->world > 1 ? m->logits_full : m->logits, sizeof(float) * m->cfg.n_vocab,
                           cudaMemcpyDeviceToHost));
    return NEON_OK;
}

int neon_cuda_model_generate(neon_model_t m, const int32_t* prompt, size_t n_prompt, size_t max_new, int32_t eos_id,
                             int32_t* out_tokens, size_t* n_out) {
    if (!m || !prompt || !out_tokens || !n_out) return error(NEON_ERR_INVALID, "null argument");
    *n_out = 0;
    if (n_prompt == 0) return error(NEON_ERR_INVALID, "forward(): empty token batch");
    if (m->length + n_prompt + max_new > m->cfg.ctx_len)
        return error(NEON_ERR_INVALID, "forward(): KV cache exhausted (ctx_len=" + std::to_string(m->cfg.ctx_len) + " exceeded)");
    int rc = neon_cuda_model_forward(m, prompt, n_prompt, nullptr);
    if (rc) return rc;
    ModelDevice md(m->device);
    if (m->out_cap < max_new + 1) {
        if (m->d_out) cudaFree(m->d_out);
        m->d_out = nullptr;
        DEC_TRY(cudaMalloc(&m->d_out, sizeof(int) * (max_new + 1)));
        m->out_cap = max_new + 1;
    }
    const int zero = 0, pos = (int)m->length;
    DEC_TRY(cudaMemcpyAsync(m->d_step, &zero, sizeof(int), cudaMemcpyHostToDevice, m->stream));
    DEC_TRY(cudaMemcpyAsync(m->d_pos, &pos, sizeof(int), cudaMemcpyHostToDevice, m->stream));
    // first token: from the prompt's logits
    rc = launch_argmax(m, 0);
    if (rc) return rc;
    if (max_new > 0) {
        // one decode step as a CUDA graph: embed(d_tok) .. logits .. argmax -> d_tok, pos += 1
        if (m->step_graph) {
            cudaGraphExecDestroy(m->step_graph);
            m->step_graph = nullptr;
        }
        cudaGraph_t g = nullptr;
        DEC_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        rc = run_step(m);
        if (!rc) rc = run_head(m, m->h);
        if (!rc) rc = launch_argmax(m, 1);
        cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return cuda_error(ce, "cudaStreamEndCapture");
        ce = cudaGraphInstantiate(&m->step_graph, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) return cuda_error(ce, "cudaGraphInstantiate");
        DEC_TRY(cudaEventRecord(m->ev0, m->stream));
        for (size_t s = 0; s < max_new; ++s) DEC_TRY(cudaGraphLaunch(m->step_graph, m->stream));
        DEC_TRY(cudaEventRecord(m->ev1, m->stream));
    }
    rc = sync_and_check(m);
    if (rc) return rc;
    if (max_new > 0) cudaEventElapsedTime(&m->decode_ms, m->ev0, m->ev1);
    std::vector<int32_t> toks(max_new + 1);
    DEC_TRY(cudaMemcpy(toks.data(), m->d_out, sizeof(int) * (max_new + 1), cudaMemcpyDeviceToHost));
    size_t n = 0;
    while (n < max_new && toks[n] != eos_id) {
        out_tokens[n] = toks[n];
        ++n;
    }
    *n_out = n;
    m->length += n;  // one forward per emitted token, as run_generation does
    return NEON_OK;
}

int neon_cuda_model_length(neon_model_t m, size_t* length) {
    if (!m || !length) return error(NEON_ERR_INVALID, "null argument");
    *length = m->length;
    return NEON_OK;
}

int neon_cuda_model_set_length(neon_model_t m, size_t length) {
    if (!m) return error(NEON_ERR_INVALID, "null model");
    if (length > m->cfg.ctx_len) return error(NEON_ERR_INVALID, "length above the KV-cache capacity");
    m->length = length;
    return NEON_OK;
}

int neon_cuda_model_kv_shift(neon_model_t m, size_t keep, size_t discard) {
    if (!m) return error(NEON_ERR_INVALID, "null model");
    if (discard == 0 || m->length <= keep + discard) return NEON_OK;  // as kv_cache_shift: nothing to slide
    ModelDevice md(m->device);
    const auto& c = m->cfg;
    const size_t kv_dim = m->kv_dim, tail = m->length - keep - discard;
    if (!m->shift_scratch) {
        int rc = dev_alloc(m, (void**)&m->shift_scratch, sizeof(float) * (size_t)c.ctx_len * kv_dim);
        if (!rc) rc = dev_alloc(m, (void**)&m->shift_cs, sizeof(float2) * std::max<size_t>(1, m->rope_half));
        if (rc) return rc;
    }
    // the one angle of the shift, per pair, with the host libm (rope_rotate_by_delta)
    std::vector<float2> cs(std::max<size_t>(1, m->rope_half));
    const float fdelta = -(float)discard / c.rope_scale;
    for (size_t i = 0; i < m->rope_half; ++i) {
        const float freq = std::pow(c.rope_base, -2.0f * (float)i / (float)c.head_dim);
        const float theta = fdelta * freq;
        cs[i] = make_float2(std::cos(theta), std::sin(theta));
    }
    DEC_TRY(cudaMemcpyAsync(m->shift_cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice, m->stream));
    const size_t row_bytes = kv_dim * sizeof(float);
    for (uint32_t li = 0; li < c.n_layer; ++li) {
        float* K = m->K + (size_t)li * c.ctx_len * kv_dim;
        float* V = m->V + (size_t)li * c.ctx_len * kv_dim;
        const long long pairs = (long long)tail * (long long)(kv_dim / 2);
        const int grid = (int)std::min<long long>((pairs + 255) / 256, 4096);
        kv_shift_rotate_kernel<<<grid, 256, 0, m->stream>>>(K + (keep + discard) * kv_dim, m->shift_scratch, m->shift_cs,
                                                             (long long)tail, (int)kv_dim, (int)c.head_dim,
                                                             (int)m->rope_half);
        int rc = check_launch("kv_shift_rotate_kernel");
        if (rc) return rc;
        DEC_TRY(cudaMemcpyAsync(K + keep * kv_dim, m->shift_scratch, tail * row_bytes, cudaMemcpyDeviceToDevice, m->stream));
        DEC_TRY(cudaMemcpyAsync(m->shift_scratch, V + (keep + discard) * kv_dim, tail * row_bytes, cudaMemcpyDeviceToDevice,
                                m->stream));
        DEC_TRY(cudaMemcpyAsync(V + keep * kv_dim, m->shift_scratch, tail * row_bytes, cudaMemcpyDeviceToDevice, m->stream));
    }
    DEC_TRY(cudaStreamSynchronize(m->stream));
    m->length = keep + tail;
    return NEON_OK;
}

int neon_cuda_model_read_kv(neon_model_t m, int layer, size_t n, float* k_host, float* v_host) {
    if (!m || !k_host || !v_host) return error(NEON_ERR_INVALID, "null argument");
    if (layer < 0 || (uint32_t)layer >= m->cfg.n_layer || n > m->cfg.ctx_len) return error(NEON_ERR_INVALID, "layer or n out of range");
    ModelDevice md(m->device);
    const size_t off = (size_t)layer * m->cfg.ctx_len * m->kv_dim;
    DEC_TRY(cudaMemcpy(k_host, m->K + off, sizeof(float) * n * m->kv_dim, cudaMemcpyDeviceToHost));
    DEC_TRY(cudaMemcpy(v_host, m->V + off, sizeof(float) * n * m->kv_dim, cudaMemcpyDeviceToHost));
    return NEON_OK;
}

int neon_cuda_model_forward_ms(neon_model_t m, float* ms) {
    if (!m || !ms) return error(NEON_ERR_INVALID, "null argument");
    *ms = m->forward_ms;
    return NEON_OK;
}

int neon_cuda_model_decode_ms(neon_model_t m, float* ms) {
    if (!m || !ms) return error(NEON_ERR_INVALID, "null argument");
    *ms = m->decode_ms;
    return NEON_OK;
}

int neon_cuda_model_free(neon_model_t m) {
    if (!m) return NEON_OK;
    ModelDevice md(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->step_graph) cudaGraphExecDestroy(m->step_graph);
    neon_cuda_free(m->embd);
    neon_cuda_free(m->output);
    neon_cuda_free(m->head);
    for (auto& L : m->layers) {
        for (auto* w : L.w) neon_cuda_free(w);
        neon_cuda_free(L.gateup);
    }
    for (void* p : m->allocs) cudaFree(p);
    if (m->d_out) cudaFree(m->d_out);
    if (m->ev0) cudaEventDestroy(m->ev0);
    if (m->ev1) cudaEventDestroy(m->ev1);
    if (m->evf0) cudaEventDestroy(m->evf0);
    if (m->evf1) cudaEventDestroy(m->evf1);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return NEON_OK;
}

}  // extern "C"
