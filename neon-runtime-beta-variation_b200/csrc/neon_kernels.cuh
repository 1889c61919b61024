// neon_kernels.cuh -- sm_100a kernels of the quantized decode matvec path.
//
// Reference path: fwd::proj_all_positions[_multi] (rawllm_forward.hpp:522-726),
// which for Q4_0 weights quantises X to Q8_0 (quantize_rows_q8_0, :360-381) and
// runs the fused integer block dot (dot_q4_0_q8_0, :419-434), and for Q8_0
// weights dequantises each row and takes an fp32 dot with X (:597-605).
//
// Device layout of an uploaded tensor (repack_kernel below), same bytes as GGUF
// but split into two planes so every lane load is aligned and coalesced:
//   payload plane  rows x nb x P bytes, P = 16 (Q4_0 nibbles) or 32 (Q8_0 int8)
//   scale plane    rows x nb fp16
// where nb = cols / 32. Row r, block b of the payload sits at (r*nb + b)*P.
//
// Work decomposition: a warp owns a tile of R consecutive rows; lane l handles
// blocks b = c + u*32 + l (u < U) of every row in the tile, so each 128-bit
// load instruction of a warp reads 512 (Q4_0) or 2x512 (Q8_0) contiguous bytes.
// The X operand of a block is read once from shared memory and reused for the
// R rows. Each lane keeps one fp32 partial per row; a butterfly shuffle
// finishes the row.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "neon_internal.h"

namespace neon {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSpans = 8;
// Q8_0 activation record in shared memory: 32 quants, fp32 d, int32 sum, pad
// (a 48-byte pitch keeps a warp's 128-bit reads conflict-free).
constexpr int kQ4Rec = 48;
// fp32 X block pitch in shared memory, in floats (144 bytes: conflict-free
// 128-bit reads when lane l reads block l).
constexpr int kQ8Pitch = 36;

// One projection target of a launch: rows [0, rows) of one uploaded tensor.
// Epilogues of the one-position kernel (decode step). Pair epilogues take
// rows (2i, 2i+1), which always share a tile (tiles start at even rows).
enum : int {
    kEpiStore = 0,   // y[r] = v (or += with accumulate)
    kEpiRope = 1,    // RoPE on pairs (fwd::rope_apply), then store at y + pos*pos_stride
    kEpiAtPos = 2,   // store at y + pos*pos_stride (the V cache row of the position)
    kEpiSwiglu = 3,  // rows interleave gate/up: y[i] = silu(v_2i) * v_2i+1
    kEpiPeer = 4,    // fused collective: row r into slot [parity][rank] of every rank
    kEpiSilu = 5,    // y[r] = silu(v): the plain SiLU-FFN variant's activation
    kEpiGather = 6,  // fused all-gather: row r (of a row shard starting at row pos_stride of the
                     // whole output) into the gather slot [parity] of every rank, at pos_stride + r
};

struct Span {
    const uint8_t* qs;   // payload plane
    const uint16_t* d;   // fp16 scale plane
    float* y;            // output, element (t, r) at y[t*y_stride + r]
    long long y_stride;
    long long pos_stride;  // kEpiRope / kEpiAtPos: y advances this far per position
    int rows;
    int tile0;           // index of this span's first row tile in the launch
    int epi;             // kEpi*
};

struct MatvecArgs {
    Span span[kMaxSpans];
    const float* x;      // fp32 activations, row t at x + t*x_stride
    long long x_stride;
    const int8_t* xq;    // Q8_0 activations (multi-position Q4_0): seq x cols
    const float* xd;     //   fp32 block scales: seq x nb
    const int* xs;       //   per-block sums of the 32 quants: seq x nb
    int n_spans;
    int n_tiles;
    int nb;
    int seq;
    int accumulate;      // 1: y += result (the residual add of the decode loop)
};

// ---------------------------------------------------------------------------
// small PTX helpers
// ---------------------------------------------------------------------------

// Streaming 128-bit load of weight bytes: read-only, not kept in L1.
__device__ __forceinline__ uint4 ld_weights_u4(const void* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

// Fetch the line holding p into L1 (no register is written): a load of it
// later in the kernel then hits L1 instead of paying an L2 round trip.
__device__ __forceinline__ void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

__device__ __forceinline__ uint16_t ld_weights_u16(const void* p) {
    uint16_t v;
    asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Programmatic dependent launch: let the next kernel on the stream start, and
// wait until the previous one has finished and its writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float fp16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));  // exact, subnormals included
}

// Four int8 packed in a word -> four exact floats, using the 2^23 trick:
// 0x4B0000uu reads as 8388608 + uu, and uu = q + 128 after flipping the sign bit.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
    const uint32_t u = w ^ 0x80808080u;
    f0 = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
    f1 = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
    f2 = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
    f3 = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// ---------------------------------------------------------------------------
// Q8_0 activation quantisation, bit-exact with quantize_rows_q8_0
// (rawllm_forward.hpp:360-381).
// ---------------------------------------------------------------------------

// (int)std::lround(v) clamped to [-127, 127]. lround rounds halfway cases away
// from zero, as roundf does. For a non-finite v glibc's lroundf returns
// LONG_MIN, whose low 32 bits -- what the (int) cast keeps -- are 0; finite v
// here is bounded by about 128 in magnitude.
__device__ __forceinline__ int q8_round_clamp(float v) {
    int q = (fabsf(v) <= 16777216.0f) ? (int)roundf(v) : 0;
    return min(max(q, -127), 127);
}

// One 32-element block held by one thread (x points at 32 floats):
// amax = max|x| (std::max ignores a NaN on its right, as fmaxf does),
// d = amax/127, id = d > 0 ? 1/d : 0, q = clamp(lround(x*id)).
__device__ __forceinline__ void quantize_block_thread(const float* x, uint32_t q[8], float& d,
                                                      int& qsum) {
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
    d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.f ? __frcp_rn(d) : 0.f;  // 1/d correctly rounded, as 1.0f / d
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int v = q8_round_clamp(__fmul_rn(x[4 * k + i], id));
            s += v;
            w |= (uint32_t)(v & 0xFF) << (8 * i);
        }
        q[k] = w;
    }
    qsum = s;
}

// Standalone quantiser: one warp per 32-block; lane j owns element j.
// Writes q (seq x cols int8), d (seq x nb fp32) and, if sums != nullptr, the
// per-block sum of the 32 quants (seq x nb int32).
__global__ void __launch_bounds__(kThreads) quantize_q8_0_kernel(
    const float* __restrict__ X, long long x_stride, int nb, int seq, int8_t* __restrict__ q_out,
    float* __restrict__ d_out, int* __restrict__ sums) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long total = (long long)nb * seq;
    for (long long gb = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5); gb < total;
         gb += (long long)gridDim.x * kWarps) {
        const int t = (int)(gb / nb), b = (int)(gb - (long long)t * nb);
        const float xv = X[(long long)t * x_stride + (long long)b * 32 + lane];
        float amax = fmaxf(0.f, fabsf(xv));  // a NaN lane contributes 0, like std::max
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d > 0.f ? __frcp_rn(d) : 0.f;  // 1/d correctly rounded, as 1.0f / d
        const int v = q8_round_clamp(__fmul_rn(xv, id));
        q_out[(long long)t * nb * 32 + (long long)b * 32 + lane] = (int8_t)v;
        if (sums) {
            int s = v;
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) sums[gb] = s;
        }
        if (lane == 0) d_out[gb] = d;
    }
}

// ---------------------------------------------------------------------------
// GGUF -> device layout repack (load time only)
// ---------------------------------------------------------------------------

// One thread per destination (row, block). src holds `rows` GGUF rows of
// src_row_bytes; destination keeps blocks [b0, b0 + nb_dst) of each row.
// P = payload bytes per block (16 or 32); source blocks are 2-byte aligned.
__global__ void repack_kernel(const uint8_t* __restrict__ src, long long src_row_bytes, int rows,
                              int b0, int nb_dst, int P, uint8_t* __restrict__ qs,
                              uint16_t* __restrict__ dplane) {
    const long long total = (long long)rows * nb_dst;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / nb_dst;
        const int b = (int)(i - r * nb_dst);
        const uint16_t* s = reinterpret_cast<const uint16_t*>(src + r * src_row_bytes +
                                                              (long long)(b0 + b) * (P + 2));
        dplane[i] = s[0];
        uint32_t w[8];
        for (int k = 0; k < P / 4; ++k) w[k] = (uint32_t)s[1 + 2 * k] | ((uint32_t)s[2 + 2 * k] << 16);
        uint4* dst = reinterpret_cast<uint4*>(qs + i * P);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        if (P == 32) dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// ---------------------------------------------------------------------------
// shared pieces of the matvec kernels
// ---------------------------------------------------------------------------

// Span owning `tile` (spans are sorted by tile0, at most kMaxSpans).
__device__ __forceinline__ int find_span(const MatvecArgs& a, int tile) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSpans; ++i)
        if (i < a.n_spans && a.span[i].tile0 <= tile) s = i;
    return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Exact Q4_0 x Q8_0 block dot: 16 nibble bytes (low nibble -> element j, high
// -> j+16) against 32 int8 quants whose sum is qsum. Nibbles are dotted
// unsigned and 8*qsum is subtracted, giving sum((nib-8)*q) exactly
// (block_isum_scalar, rawllm_forward.hpp:384-392).
// Two independent accumulators (low and high nibbles) halve the dependent
// dp4a chain; integer sums are exact, so the order does not matter.
__device__ __forceinline__ int q4_block_isum(const uint4 w, const uint4 x0, const uint4 x1, int qsum) {
    int lo = 0, hi = 0;
    lo = __dp4a((int)(w.x & 0x0F0F0F0Fu), (int)x0.x, lo);
    hi = __dp4a((int)((w.x >> 4) & 0x0F0F0F0Fu), (int)x1.x, hi);
    lo = __dp4a((int)(w.y & 0x0F0F0F0Fu), (int)x0.y, lo);
    hi = __dp4a((int)((w.y >> 4) & 0x0F0F0F0Fu), (int)x1.y, hi);
    lo = __dp4a((int)(w.z & 0x0F0F0F0Fu), (int)x0.z, lo);
    hi = __dp4a((int)((w.z >> 4) & 0x0F0F0F0Fu), (int)x1.z, hi);
    lo = __dp4a((int)(w.w & 0x0F0F0F0Fu), (int)x0.w, lo);
    hi = __dp4a((int)((w.w >> 4) & 0x0F0F0F0Fu), (int)x1.w, hi);
    return (lo + hi) - 8 * qsum;
}

// dp4a of four unsigned bytes of a with four signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// The same exact block sum as q4_block_isum, as a float, with fewer integer
// operations: the high nibbles are dotted in place (16 x their value), so
// 16 * isum = 16 * lo + hi16 - 128 * qsum, and `bias` = 0x4B400000 - 128 * qsum
// folds the qsum term and the float conversion's 1.5 * 2^23 bias into one
// add. |16 * isum| < 2^22, so the conversion is exact, and so is the scaling
// by 1/16: the result equals (float)q4_block_isum(w, x0, x1, qsum).
__device__ __forceinline__ float q4_block_dot16(const uint4 w, const uint4 x0, const uint4 x1, int bias) {
    int lo = 0, hi = 0;
    lo = dp4a_us(w.x & 0x0F0F0F0Fu, x0.x, lo);
    hi = dp4a_us(w.x & 0xF0F0F0F0u, x1.x, hi);
    lo = dp4a_us(w.y & 0x0F0F0F0Fu, x0.y, lo);
    hi = dp4a_us(w.y & 0xF0F0F0F0u, x1.y, hi);
    lo = dp4a_us(w.z & 0x0F0F0F0Fu, x0.z, lo);
    hi = dp4a_us(w.z & 0xF0F0F0F0u, x1.z, hi);
    lo = dp4a_us(w.w & 0x0F0F0F0Fu, x0.w, lo);
    hi = dp4a_us(w.w & 0xF0F0F0F0u, x1.w, hi);
    return __fmul_rn(__int_as_float(lo * 16 + hi + bias) - 12582912.0f, 0.0625f);
}

// Exact int -> float for |v| < 2^22 without the conversion pipe: the bits of
// 1.5*2^23 + v read as a float are 12582912 + v exactly.
__device__ __forceinline__ float small_int_to_f32(int v) {
    return __int_as_float(0x4B400000 + v) - 12582912.0f;
}

// Sum over one Q8_0 block of q[j] * x[j] in fp32 (w0, w1 = 32 int8).
__device__ __forceinline__ float q8_block_dot(const uint4 w0, const uint4 w1, const float4* xv) {
    const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float f0, f1, f2, f3;
        i8x4_to_f32(ws[k], f0, f1, f2, f3);
        const float4 xx = xv[k];
        s = fmaf(f0, xx.x, s);
        s = fmaf(f1, xx.y, s);
        s = fmaf(f2, xx.z, s);
        s = fmaf(f3, xx.w, s);
    }
    return s;
}

// Write the R row results of a warp tile (lane r stores row r).
template <int R>
__device__ __forceinline__ void store_tile(const float (&acc)[R], float* y, int row0, int rows, int lane) {
    float mine = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float v = warp_sum(acc[r]);
        if (lane == r) mine = v;
    }
    if (lane < R && row0 + lane < rows) y[row0 + lane] = mine;
}

// ---------------------------------------------------------------------------
// One position (decode): the streaming kernel.
//
// A CTA of kStreamWarps warps owns row tiles of RC rows
// (tiles t = blockIdx.x, blockIdx.x + gridDim.x, ...). A tile's input dim is
// cut into nch chunks of kc blocks; one (tile, chunk) pair is an "item". Warp 0
// copies items into a ring of shared-memory stages with cp.async.bulk, one
// mbarrier per stage counting the bytes. When the whole row fits one chunk,
// a tile's RC rows are contiguous in both planes and an item is two copies
// (payload, scales); otherwise each row is two copies. The first items are
// issued before the PDL wait: weights are never written by earlier kernels,
// so a launch streams its weights while the previous kernel is finishing.
//
// After the PDL wait the CTA stages X once: Q4_0 quantises it to Q8_0 records
// (bit-exact with quantize_rows_q8_0), 1, 2 or 4 threads per 32-block so that
// one L2 round trip brings all of X in; Q8_0 keeps fp32. Only then does the
// CTA let the next launch on the stream start (a trigger before this point
// lets several launches' CTAs pile up on the SMs).
//
// Dot products: see the work mapping above matvec_stream_kernel. Q8_0 tiles
// give each thread two rows so that one read of a block of X serves both.
//
// Stage layout: payload RC x kc_max x P bytes (row r at r*kc_max*P), then the
// scales: the 16-byte-aligned window around the wanted scales (the scale plane
// carries 16 bytes of tail padding so a window never leaves the allocation),
// one window per tile (contiguous case) or per row at a pitch of SPH halfs.
// ---------------------------------------------------------------------------
constexpr int kStreamWarps = 8;                      // compute warps
constexpr int kStreamThreads = kStreamWarps * 32;
constexpr int kStreamBlock = kStreamThreads + 32;    // + the copy warp
constexpr int kMaxRopeHalf = 128;  // head_dim <= 256
constexpr int kMaxStages = 3;

struct StreamArgs {
    Span span[kMaxSpans];
    const float* x;         // fp32 activations of the one position
    unsigned int* err;      // device error word: bit 0 = a bounded wait timed out
    int n_spans;
    int n_tiles;
    int nb;                 // blocks per row
    int kc;                 // blocks per chunk (the last chunk may be shorter)
    int nch;                // chunks per row
    int stages;             // ring depth
    int stage_bytes;        // bytes per stage
    int x_vec;              // x is 16-byte aligned: 128-bit loads
    int accumulate;         // 1: y += result (the residual add of the decode loop)
    const float* norm_w;    // non-null: X is replaced by rms_norm(X, norm_w, norm_eps) first
    float norm_eps;
    const int* d_pos;       // position of the token (RoPE / cache epilogues)
    const float2* rope_cs;  // [position][rope_half] (cos, sin)
    int rope_half;
    int head_dim;
    int peer_mode;          // 1: fused all-reduce producer, 2: fused all-gather producer (neon_internal::MatvecExt)
    PeerSet peer;
    // matvec_resident_kernel only: rows per CTA (even) and the rows of all
    // spans (each span starting at an even row, span[i].tile0)
    int rpc;
    int n_vrows;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Bulk copy global -> this CTA's shared memory; completion is counted in
// bytes on `bar`. dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Wait for phase `parity` of `bar`; give up after ~2 s, record the timeout in
// *err and return false (the caller leaves the kernel, CTA-uniformly).
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Barrier of the streaming kernel's compute warps only (named barrier 1,
// kStreamThreads threads): its copy warp never waits on it.
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, %0;" ::"n"(256) : "memory"); }
__device__ __forceinline__ bool compute_sync_or(bool v) {
    uint32_t r;
    asm volatile("{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.or.pred q, 1, %2, p; selp.u32 %0, 1, 0, q; }"
                 : "=r"(r)
                 : "r"((uint32_t)v), "n"(256)
                 : "memory");
    return r != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    const uint32_t addr = smem_u32(bar);
    uint32_t done = 0;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if (globaltimer_ns() - t0 > 2000000000ull) {
            if (err) atomicOr(err, 1u);
            return false;
        }
    }
}

template <class Args>
__device__ __forceinline__ int find_span_of(const Args& a, int tile) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSpans; ++i)
        if (i < a.n_spans && a.span[i].tile0 <= tile) s = i;
    return s;
}

__host__ __device__ constexpr int stream_scale_pitch(int kc) { return ((kc + 7) & ~7) + 8; }
__host__ __device__ constexpr int stream_x_bytes(int type, int nb) {
    return ((type == 2 ? nb * kQ4Rec : nb * kQ8Pitch * 4) + 127) & ~127;
}

// X loads of the staging functions: read-only through the non-coherent path
// (X was written by an earlier kernel), or with CG through L2 only, for X
// written earlier in the same launch by other CTAs.
template <bool CG>
__device__ __forceinline__ float ld_x(const float* p) {
    if constexpr (CG) return __ldcg(p);
    else return __ldg(p);
}
template <bool CG>
__device__ __forceinline__ float4 ld_x4(const float4* p) {
    if constexpr (CG) return __ldcg(p);
    else return __ldg(p);
}

// rms_norm's scale 1/sqrt(mean(x^2) + eps) of n floats (fwd::rms_norm,
// rawllm_forward.hpp:730-735): a double sum of squares over the whole CTA,
// so every CTA of the launch derives the same scale.
template <bool CG = false>
__device__ __forceinline__ float cta_rms_scale(const float* __restrict__ x, int n, float eps, double* scratch) {
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += kStreamThreads) {
        const double v = (double)ld_x<CG>(x + i);
        ss = fma(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) scratch[w] = ss;
    compute_sync();
    double r = l < kStreamWarps ? scratch[l] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    compute_sync();  // scratch may be reused right after
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(r / (double)n), eps)));
}

// Quantise X (nb blocks) into the CTA's Q8_0 records, TPB threads per block.
// Whole warps iterate together (the shuffles need every lane); the TPB
// threads of one block are always all active or all idle.
// With norm_w, each element is first replaced by (x * scale) * w, rms_norm's
// output (the reference multiplies in that order).
// Q8_0 record of the EPT elements xv[] a thread holds of block b (TPB
// threads per block, `part` this thread's share): amax over the TPB lanes,
// d = amax/127, q = clamp(lround(x / d)), and the block's sum of q.
template <int TPB>
__device__ __forceinline__ void quantize_store_q8(float (&xv)[32 / TPB], bool act, int b, int part,
                                                  unsigned char* rec) {
    constexpr int EPT = 32 / TPB;
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < EPT; ++j) amax = fmaxf(amax, fabsf(xv[j]));
#pragma unroll
    for (int o = 1; o < TPB; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.f ? __frcp_rn(d) : 0.f;  // 1/d correctly rounded, as 1.0f / d
    uint32_t q[EPT / 4];
    int s = 0;
#pragma unroll
    for (int k = 0; k < EPT / 4; ++k) {
        uint32_t w = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int v = q8_round_clamp(__fmul_rn(xv[4 * k + j], id));
            s += v;
            w |= (uint32_t)(v & 0xFF) << (8 * j);
        }
        q[k] = w;
    }
#pragma unroll
    for (int o = 1; o < TPB; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (act) {
        uint32_t* r32 = reinterpret_cast<uint32_t*>(rec + b * kQ4Rec) + part * (EPT / 4);
#pragma unroll
        for (int k = 0; k < EPT / 4; ++k) r32[k] = q[k];
        if (part == 0)
            *reinterpret_cast<uint2*>(rec + b * kQ4Rec + 32) = make_uint2(__float_as_uint(d), (uint32_t)s);
    }
}

// The EPT elements of X thread `part` of block b holds.
template <int TPB, bool CG = false>
__device__ __forceinline__ void load_x_part(const float* __restrict__ x, bool x_vec, bool act, int b, int part,
                                            float (&xv)[32 / TPB]) {
    constexpr int EPT = 32 / TPB;
    const long long e0 = (long long)b * 32 + part * EPT;
    if (act && x_vec) {
#pragma unroll
        for (int k = 0; k < EPT / 4; ++k) {
            const float4 v = ld_x4<CG>(reinterpret_cast<const float4*>(x + e0) + k);
            xv[4 * k] = v.x; xv[4 * k + 1] = v.y; xv[4 * k + 2] = v.z; xv[4 * k + 3] = v.w;
        }
    } else if (act) {
#pragma unroll
        for (int j = 0; j < EPT; ++j) xv[j] = ld_x<CG>(x + e0 + j);
    } else {
#pragma unroll
        for (int j = 0; j < EPT; ++j) xv[j] = 0.f;
    }
}

// Quantise X (nb blocks) into the CTA's Q8_0 records, TPB threads per block.
// Whole warps iterate together (the shuffles need every lane); the TPB
// threads of one block are always all active or all idle.
// With norm_w, each element is first replaced by (x * scale) * w, rms_norm's
// output (the reference multiplies in that order).
template <int TPB, bool CG = false>
__device__ __forceinline__ void stage_x_q8(const float* __restrict__ x, int nb, bool x_vec, unsigned char* rec,
                                           const float* __restrict__ norm_w, float scale) {
    constexpr int EPT = 32 / TPB;
    const int lane = threadIdx.x & 31;
    const int n = nb * TPB;
    for (int i0 = threadIdx.x - lane; i0 < n; i0 += kStreamThreads) {
        const int i = i0 + lane;
        const bool act = i < n;
        const int b = act ? i / TPB : 0, part = i % TPB;
        float xv[EPT];
        load_x_part<TPB, CG>(x, x_vec, act, b, part, xv);
        if (norm_w && act) {
            const float* wb = norm_w + (long long)b * 32 + part * EPT;
#pragma unroll
            for (int j = 0; j < EPT; ++j) xv[j] = __fmul_rn(__fmul_rn(xv[j], scale), __ldg(wb + j));
        }
        quantize_store_q8<TPB>(xv, act, b, part, rec);
    }
}

// rms_norm folded into the Q8_0 staging in one pass, when the CTA's threads
// cover X once (nb * TPB <= kStreamThreads): every thread loads its elements,
// the CTA reduces the double sum of squares, and the same registers are
// scaled, multiplied by the norm weight and quantised.
template <int TPB, bool CG = false>
__device__ __forceinline__ void stage_x_q8_norm(const float* __restrict__ x, int nb, bool x_vec, unsigned char* rec,
                                                const float* __restrict__ norm_w, float eps, double* scratch) {
    constexpr int EPT = 32 / TPB;
    const int i = threadIdx.x;
    const bool act = i < nb * TPB;
    const int b = act ? i / TPB : 0, part = i % TPB;
    const long long e0 = (long long)b * 32 + part * EPT;
    float xv[EPT];
    load_x_part<TPB, CG>(x, x_vec, act, b, part, xv);
    // the norm weights never change: fetched into L1 with X's loads, not after the reduction
    if (act) prefetch_l1(norm_w + e0);
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < EPT; ++j) ss = fma((double)xv[j], (double)xv[j], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) scratch[w] = ss;
    compute_sync();
    double r = l < kStreamWarps ? scratch[l] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(r / (double)(nb * 32)), eps)));
    if (act) {
#pragma unroll
        for (int j = 0; j < EPT; ++j) xv[j] = __fmul_rn(__fmul_rn(xv[j], scale), __ldg(norm_w + e0 + j));
    }
    quantize_store_q8<TPB>(xv, act, b, part, rec);
}

// Packed fp32x2 arithmetic of sm_100 (one instruction, two lanes of fp32).
__device__ __forceinline__ unsigned long long f32x2_fma(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long f32x2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// Bytes 0,1 (sel 0) or 2,3 (sel 1) of (w ^ 0x80808080) as the floats
// 8388608 + 128 + q, packed in one 64-bit register.
template <int HALF>
__device__ __forceinline__ unsigned long long i8x2_magic(uint32_t u) {
    unsigned long long v;
    if (HALF == 0)
        asm("{ .reg .b32 lo, hi; prmt.b32 lo, %1, 0x4B000000, 0x7650; prmt.b32 hi, %1, 0x4B000000, 0x7651; "
            "mov.b64 %0, {lo, hi}; }"
            : "=l"(v) : "r"(u));
    else
        asm("{ .reg .b32 lo, hi; prmt.b32 lo, %1, 0x4B000000, 0x7652; prmt.b32 hi, %1, 0x4B000000, 0x7653; "
            "mov.b64 %0, {lo, hi}; }"
            : "=l"(v) : "r"(u));
    return v;
}

// Sum over one Q8_0 block of q[j]*x[j] in fp32 with packed arithmetic:
// two interleaved partial sums (even and odd elements), added at the end.
// xv: the block's 32 floats as 16 packed pairs.
__device__ __forceinline__ float q8_block_dot_x2(const uint4 w0, const uint4 w1, const unsigned long long* xv) {
    const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const unsigned long long neg_magic = 0xCB000080CB000080ull;  // {-8388736.f, -8388736.f}
    unsigned long long acc = 0ull;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t u = ws[k] ^ 0x80808080u;
        acc = f32x2_fma(f32x2_add(i8x2_magic<0>(u), neg_magic), xv[2 * k], acc);
        acc = f32x2_fma(f32x2_add(i8x2_magic<1>(u), neg_magic), xv[2 * k + 1], acc);
    }
    return __uint_as_float((uint32_t)acc) + __uint_as_float((uint32_t)(acc >> 32));
}

__device__ __forceinline__ float silu_dev(float x) {
    // x / (1 + fast_expf(-x)) with engine::fast_expf (rawllm_common.hpp:88-100):
    // Schraudolph's exp, kA*x + kB as one FMA truncated to int.
    const float e = (-x < -88.f || -x > 88.f)
                        ? expf(-x)
                        : __int_as_float(__float2int_rz(__fmaf_rn(12102203.9f, -x, 1064872507.f)));
    return __fdiv_rn(x, __fadd_rn(1.0f, e));
}

// Writes the RC row results of a tile (rowv[], shared memory) through the
// span's epilogue; threads t < RC own row row0 + t. `pos` is the token's
// position, `rcs` its RoPE (cos, sin) row staged in shared memory, `yold` the
// row's previous output (read ahead of the dot products when accumulating).
// `t` is the row's place in the tile (by default the calling thread's index).
__device__ __forceinline__ void stream_epilogue(const StreamArgs& a, const Span& sp, int row0, int RC,
                                                const float* rowv, unsigned int peer_call, int pos,
                                                const float2* rcs, float yold, int t = -1) {
    if (t < 0) t = threadIdx.x;
    if (t >= RC) return;
    const int row = row0 + t;
    if (row >= sp.rows) return;
    const float v = rowv[t];
    switch (sp.epi) {
        case kEpiStore:
            sp.y[row] = a.accumulate ? yold + v : v;
            break;
        case kEpiAtPos:
            sp.y[(long long)pos * sp.pos_stride + row] = v;
            break;
        case kEpiRope: {
            // rotate (v_2i, v_2i+1) of a head by the position's angle
            // (fwd::rope_apply, rawllm_forward.hpp:767-782, with g++'s FMA
            // contraction); pairs at or beyond rope_half are stored unrotated
            float* dst = sp.y + (long long)pos * sp.pos_stride;
            if (t & 1) break;
            const float x0 = v, x1 = rowv[t + 1];
            const int i = (row % a.head_dim) / 2;
            if (i < a.rope_half) {
                const float2 c = rcs[i];
                dst[row] = __fmaf_rn(x0, c.x, -__fmul_rn(x1, c.y));
                dst[row + 1] = __fmaf_rn(x0, c.y, __fmul_rn(x1, c.x));
            } else {
                dst[row] = x0;
                dst[row + 1] = x1;
            }
            break;
        }
        case kEpiSwiglu:
            // silu(gate) * up (rawllm_forward.hpp:1186)
            if (!(t & 1)) sp.y[row / 2] = __fmul_rn(silu_dev(v), rowv[t + 1]);
            break;
        case kEpiSilu:
            // silu(up), the FFN without a gate (rawllm_forward.hpp:1189)
            sp.y[row] = silu_dev(v);
            break;
        case kEpiPeer: {
            // this rank's partial row sum, as an LL word, into its slot on every rank (NVLink stores)
            const long long off = ll_slot_off(a.peer.world, (int)(peer_call & 1u), a.peer.rank) / 8 + row;
            const unsigned long long w = ll_pack(v, peer_call);
            for (int p = 0; p < a.peer.world; ++p)
                st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(a.peer.base[p]) + off, w);
            break;
        }
        case kEpiGather: {
            // this rank's row, as an LL word, at its place in the whole output, into every rank's gather slot
            const long long off = ll_slot_off(a.peer.world, (int)(peer_call & 1u), 0) / 8 + sp.pos_stride + row;
            const unsigned long long w = ll_pack(v, peer_call);
            for (int p = 0; p < a.peer.world; ++p)
                st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(a.peer.base[p]) + off, w);
            break;
        }
    }
}

// Work mapping: a tile has RC rows; every thread owns R consecutive rows and a
// slice of the blocks of a chunk. G = RC/R row groups share the CTA's threads,
// TPG = kStreamThreads/G per group: WPG = TPG/32 whole warps per group when
// TPG >= 32 (a row split over several warps: K-split, finished through shared
// memory), else 32/TPG groups per warp (finished by a shuffle tree).
template <int TYPE, int RC, int R>
__global__ void __launch_bounds__(kStreamBlock) matvec_stream_kernel(const __grid_constant__ StreamArgs a) {
    constexpr int P = TYPE == 2 ? 16 : 32;
    constexpr int G = RC / R;
    constexpr int TPG = kStreamThreads / G;
    constexpr int WPG = TPG >= 32 ? TPG / 32 : 1;
    constexpr int LPG = TPG >= 32 ? 32 : TPG;
    static_assert(RC % R == 0 && kStreamThreads % G == 0, "bad tile shape");
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float red[2][RC * WPG];  // by tile parity: a tile's reduction never waits on the last epilogue
    __shared__ float rowv[2][RC];
    const int nb = a.nb, KC = a.kc, nch = a.nch, S = a.stages;
    const int SPH = stream_scale_pitch(KC);
    unsigned char* xsm = smem;
    unsigned char* ring = smem + stream_x_bytes(TYPE, nb);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * a.stage_bytes);
    uint64_t* empty = full + kMaxStages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = TPG >= 32 ? warp / WPG : warp * (32 / TPG) + lane / TPG;
    const int slice = TPG >= 32 ? (warp % WPG) * 32 + lane : lane % TPG;

    const int my_tiles = (int)blockIdx.x < a.n_tiles ? (a.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_items = my_tiles * nch;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStreamWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // The copy warp: item `item` of this CTA into its stage.
    auto issue = [&](int item) {
        const int stage = item % S;
        const int tile = (int)blockIdx.x + (item / nch) * (int)gridDim.x;
        const int chunk = item % nch;
        const Span& sp = a.span[find_span_of(a, tile)];
        const int row0 = (tile - sp.tile0) * RC;
        const int k0 = chunk * KC;
        const int kc = min(KC, nb - k0);
        const int nrows = min(RC, sp.rows - row0);
        unsigned char* pay = ring + stage * a.stage_bytes;
        uint16_t* sc = reinterpret_cast<uint16_t*>(pay + RC * KC * P);
        if (nch == 1) {
            const long long e = (long long)row0 * nb;
            const int off = (int)(e & 7);
            const uint32_t pbytes = (uint32_t)(nrows * nb * P);
            const uint32_t sbytes = 2u * (uint32_t)((off + nrows * nb + 7) & ~7);
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[stage], pbytes + sbytes);
                bulk_g2s(pay, sp.qs + e * P, pbytes, &full[stage]);
                bulk_g2s(sc, sp.d + (e - off), sbytes, &full[stage]);
            }
            return;
        }
        uint32_t bytes = 0;
        for (int r = lane; r < nrows; r += 32) {
            const long long e = (long long)(row0 + r) * nb + k0;
            const int off = (int)(e & 7);
            bytes += (uint32_t)(kc * P) + 2u * (uint32_t)((off + kc + 7) & ~7);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
        if (lane == 0) mbar_arrive_expect_tx(&full[stage], bytes);
        __syncwarp();
        for (int r = lane; r < nrows; r += 32) {
            const long long e = (long long)(row0 + r) * nb + k0;
            const int off = (int)(e & 7);
            bulk_g2s(pay + r * KC * P, sp.qs + e * P, (uint32_t)(kc * P), &full[stage]);
            bulk_g2s(sc + r * SPH, sp.d + (e - off), 2u * (uint32_t)((off + kc + 7) & ~7), &full[stage]);
        }
    };

    if (warp == kStreamWarps) {
        // Copy warp (never reads what earlier kernels wrote, so no PDL wait):
        // a stage is refilled as soon as every compute warp has released it.
        // The CTA lets the next launch start when its compute warps have
        // staged X; this warp, which lives until its last copy, signals now.
        pdl_launch_dependents();
        for (int item = 0; item < n_items; ++item) {
            const int stage = item % S;
            if (item >= S && !mbar_wait(&empty[stage], (uint32_t)(((item / S) - 1) & 1), a.err)) break;
            issue(item);
        }
        return;
    }
    pdl_wait();

    // Fused (LL) collective, producing side: this launch's call number, the
    // one after the last completed.
    const unsigned int peer_call =
        a.peer_mode ? *reinterpret_cast<volatile const unsigned int*>(a.peer.calls) + 1u : 0u;

    // the token's position and its RoPE row, read once per launch; the row
    // (rope_half <= kMaxRopeHalf <= kStreamThreads entries, one per thread) is
    // fetched into L1 alongside X's loads and copied to shared memory after
    // the X staging
    __shared__ float2 rcs[kMaxRopeHalf];
    static_assert(kMaxRopeHalf <= kStreamThreads, "one RoPE entry per thread");
    const int pos = a.d_pos ? *a.d_pos : 0;
    if (a.rope_cs && (int)threadIdx.x < a.rope_half) prefetch_l1(a.rope_cs + (long long)pos * a.rope_half + threadIdx.x);

    // Stage X once per CTA (normalised first when asked), then let the next
    // launch start.
    __shared__ double dscratch[32];
    const int tpb = TYPE == 2 ? kStreamThreads / nb : 0;
    if (TYPE == 2 && a.norm_w && tpb >= 1) {
        if (tpb >= 4) stage_x_q8_norm<4>(a.x, nb, a.x_vec, xsm, a.norm_w, a.norm_eps, dscratch);
        else if (tpb >= 2) stage_x_q8_norm<2>(a.x, nb, a.x_vec, xsm, a.norm_w, a.norm_eps, dscratch);
        else stage_x_q8_norm<1>(a.x, nb, a.x_vec, xsm, a.norm_w, a.norm_eps, dscratch);
    } else if (TYPE == 2) {
        const float nscale = a.norm_w ? cta_rms_scale(a.x, nb * 32, a.norm_eps, dscratch) : 1.f;
        if (tpb >= 4) stage_x_q8<4>(a.x, nb, a.x_vec, xsm, a.norm_w, nscale);
        else if (tpb >= 2) stage_x_q8<2>(a.x, nb, a.x_vec, xsm, a.norm_w, nscale);
        else stage_x_q8<1>(a.x, nb, a.x_vec, xsm, a.norm_w, nscale);
    } else {
        const float nscale = a.norm_w ? cta_rms_scale(a.x, nb * 32, a.norm_eps, dscratch) : 1.f;
        float* xs = reinterpret_cast<float*>(xsm);
        for (int i = threadIdx.x; i < nb * 32; i += kStreamThreads) {
            float v = __ldg(a.x + i);
            if (a.norm_w) v = __fmul_rn(__fmul_rn(v, nscale), __ldg(a.norm_w + i));
            xs[(i >> 5) * kQ8Pitch + (i & 31)] = v;
        }
    }
    if (a.rope_cs && (int)threadIdx.x < a.rope_half) rcs[threadIdx.x] = a.rope_cs[(long long)pos * a.rope_half + threadIdx.x];
    compute_sync();
    pdl_launch_dependents();

    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int item = 0; item < n_items; ++item) {
        const int stage = item % S;
        const uint32_t parity = (uint32_t)((item / S) & 1);
        const int tile = (int)blockIdx.x + (item / nch) * (int)gridDim.x;
        const int chunk = item % nch;
        const Span& sp = a.span[find_span_of(a, tile)];
        const int row0 = (tile - sp.tile0) * RC;
        const int k0 = chunk * KC;
        const int kc = min(KC, nb - k0);
        const bool ok = mbar_wait(&full[stage], parity, a.err);
        if (compute_sync_or(!ok)) return;
        const int tb = (item / nch) & 1;
        // the accumulate epilogue's y[row], fetched while the dot products run
        float yold = 0.f;
        if (a.accumulate && chunk == nch - 1 && sp.epi == kEpiStore && (int)threadIdx.x < RC &&
            row0 + (int)threadIdx.x < sp.rows)
            yold = sp.y[row0 + threadIdx.x];

        const unsigned char* pay = ring + stage * a.stage_bytes;
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(pay + RC * KC * P);
        int sbase[R];
        const unsigned char* prow[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
            const int r = g * R + rr;
            sbase[rr] = nch == 1 ? (int)(((long long)row0 * nb) & 7) + r * nb
                                 : r * SPH + (int)(((long long)(row0 + r) * nb + k0) & 7);
            prow[rr] = pay + r * KC * P;
        }
        float part[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) part[rr] = 0.f;
#pragma unroll 2
        for (int bi = slice; bi < kc; bi += TPG) {
            if (TYPE == 2) {
                const uint4* r4 = reinterpret_cast<const uint4*>(xsm + (k0 + bi) * kQ4Rec);
                const uint4 x0 = r4[0], x1 = r4[1];
                const uint2 xm = *reinterpret_cast<const uint2*>(r4 + 2);
                const float xd = __uint_as_float(xm.x);
#pragma unroll
                for (int rr = 0; rr < R; ++rr) {
                    const float wd = fp16_bits_to_f32(sc[sbase[rr] + bi]);
                    const uint4 w = *reinterpret_cast<const uint4*>(prow[rr] + bi * P);
                    part[rr] = fmaf(wd * xd, small_int_to_f32(q4_block_isum(w, x0, x1, (int)xm.y)), part[rr]);
                }
            } else {
                const ulonglong2* xv2 = reinterpret_cast<const ulonglong2*>(
                    reinterpret_cast<const float*>(xsm) + (k0 + bi) * kQ8Pitch);
                unsigned long long xv[16];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const ulonglong2 t = xv2[k];
                    xv[2 * k] = t.x;
                    xv[2 * k + 1] = t.y;
                }
#pragma unroll
                for (int rr = 0; rr < R; ++rr) {
                    const float wd = fp16_bits_to_f32(sc[sbase[rr] + bi]);
                    const uint4* w4 = reinterpret_cast<const uint4*>(prow[rr] + bi * P);
                    part[rr] = fmaf(wd, q8_block_dot_x2(w4[0], w4[1], xv), part[rr]);
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr) acc[rr] += part[rr];
        // this warp is done with the stage: release it to the copy warp
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (chunk == nch - 1) {
#pragma unroll
            for (int rr = 0; rr < R; ++rr)
#pragma unroll
                for (int o = LPG / 2; o; o >>= 1) acc[rr] += __shfl_xor_sync(0xffffffffu, acc[rr], o);
            // row results -> rowv[] in shared memory
            if (WPG == 1) {
                if (slice == 0) {
#pragma unroll
                    for (int rr = 0; rr < R; ++rr) rowv[tb][g * R + rr] = acc[rr];
                }
            } else if (lane == 0) {
#pragma unroll
                for (int rr = 0; rr < R; ++rr) red[tb][(g * R + rr) * WPG + (warp % WPG)] = acc[rr];
            }
            compute_sync();
            if (WPG > 1 && (int)threadIdx.x < RC) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < WPG; ++w) v += red[tb][threadIdx.x * WPG + w];
                rowv[tb][threadIdx.x] = v;
            }
            if (WPG > 1) compute_sync();
            stream_epilogue(a, sp, row0, RC, rowv[tb], peer_call, pos, rcs, yold);
#pragma unroll
            for (int rr = 0; rr < R; ++rr) acc[rr] = 0.f;
        }
    }
}

// Shared-memory bytes of a streaming launch.
__host__ __device__ constexpr int stream_smem_bytes(int type, int nb, int stages, int stage_bytes) {
    return stream_x_bytes(type, nb) + stages * stage_bytes + 2 * kMaxStages * 8;  // + full and empty barriers
}

// Bytes of one ring stage for RC rows x kc blocks.
__host__ __device__ constexpr int stream_stage_bytes(int type, int rc, int kc) {
    return ((rc * kc * (type == 2 ? 16 : 32) + rc * stream_scale_pitch(kc) * 2 + 16) + 127) & ~127;
}

// Tile plan of a streaming (one-position) launch. Rows per tile: the largest
// of 32, 16, 8, 4, 2 whose tile fits one stage of `stage_target` bytes and
// still gives every SM a tile; rows that do not fit a stage even 2 at a time
// are cut into chunks. forced_rc (2..32, 0: none) imposes a shape instead:
// forced_rc rows, chunks of forced_kc blocks (0 or >= nb: whole rows). The
// ring takes as many stages (<= kMaxStages) as fit `max_smem` with X; smem
// above max_smem means the shape does not fit at all.
struct StreamPlan {
    int rc, kc, nch, stages, stage_bytes, smem;
};
inline StreamPlan plan_stream_tiles(int type, int nb, size_t total_rows, int sms, int stage_target, int max_smem,
                                    int forced_rc, int forced_kc) {
    const int P = type == 2 ? 16 : 32;
    const long long row_bytes = (long long)nb * (P + 2);
    StreamPlan p{};
    if (forced_rc) {
        p.rc = forced_rc;
        p.kc = forced_kc <= 0 || forced_kc >= nb ? nb : forced_kc;
        p.nch = (nb + p.kc - 1) / p.kc;
    } else if (row_bytes * 2 <= stage_target) {
        p.kc = nb;
        p.nch = 1;
        p.rc = 32;
        while (p.rc > 2 && ((long long)p.rc * row_bytes > stage_target ||
                            (long long)((total_rows + p.rc - 1) / p.rc) < sms))
            p.rc /= 2;
    } else {
        p.rc = 2;
        const int nch = (int)((row_bytes * 2 + stage_target - 1) / stage_target);
        p.kc = ((nb + nch - 1) / nch + 7) & ~7;
        p.nch = (nb + p.kc - 1) / p.kc;
    }
    p.stage_bytes = stream_stage_bytes(type, p.rc, p.kc);
    p.stages = kMaxStages;
    p.smem = stream_smem_bytes(type, nb, p.stages, p.stage_bytes);
    while (p.stages > 1 && p.smem > max_smem) {
        --p.stages;
        p.smem = stream_smem_bytes(type, nb, p.stages, p.stage_bytes);
    }
    return p;
}

// ---------------------------------------------------------------------------
// Any number of positions (prefill), CUDA-core path. grid.y tiles the
// positions by T; X comes from global memory (fp32 for Q8_0 weights, the
// pre-quantised Q8_0 scratch for Q4_0 weights).
// ---------------------------------------------------------------------------
template <int TYPE, int R, int T>
__global__ void __launch_bounds__(kThreads) matvec_multipos_kernel(const __grid_constant__ MatvecArgs a) {
    const int lane = threadIdx.x & 31;
    const int nb = a.nb;
    const int t0 = blockIdx.y * T;
    pdl_launch_dependents();
    pdl_wait();
    for (int tile = blockIdx.x * kWarps + (threadIdx.x >> 5); tile < a.n_tiles;
         tile += gridDim.x * kWarps) {
        const int si = find_span(a, tile);
        const Span& sp = a.span[si];
        const int row0 = (tile - sp.tile0) * R;
        float acc[R][T];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < T; ++t) acc[r][t] = 0.f;
        for (int b = lane; b < nb; b += 32) {
            uint4 w[R][2];
            float wdf[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = min(row0 + r, sp.rows - 1);
                const long long i = (long long)row * nb + b;
                if (TYPE == 2) {
                    w[r][0] = ld_weights_u4(sp.qs + i * 16);
                } else {
                    w[r][0] = ld_weights_u4(sp.qs + i * 32);
                    w[r][1] = ld_weights_u4(sp.qs + i * 32 + 16);
                }
                wdf[r] = fp16_bits_to_f32(ld_weights_u16(sp.d + i));
            }
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const int tt = t0 + t;
                if (tt >= a.seq) break;
                if (TYPE == 2) {
                    const uint4* q4 = reinterpret_cast<const uint4*>(a.xq + ((long long)tt * nb + b) * 32);
                    const uint4 x0 = q4[0], x1 = q4[1];
                    const float xd = a.xd[(long long)tt * nb + b];
                    const int xsum = a.xs[(long long)tt * nb + b];
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        acc[r][t] = fmaf(wdf[r] * xd, (float)q4_block_isum(w[r][0], x0, x1, xsum), acc[r][t]);
                } else {
                    const float* xp = a.x + (long long)tt * a.x_stride + (long long)b * 32;
                    float4 xr[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) xr[k] = make_float4(xp[4 * k], xp[4 * k + 1], xp[4 * k + 2], xp[4 * k + 3]);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        acc[r][t] = fmaf(wdf[r], q8_block_dot(w[r][0], w[r][1], xr), acc[r][t]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const int tt = t0 + t;
            if (tt >= a.seq) break;
            float mine = 0.f;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float v = warp_sum(acc[r][t]);
                if (lane == r) mine = v;
            }
            if (lane < R && row0 + lane < sp.rows) {
                float* yp = sp.y + (long long)tt * sp.y_stride + row0 + lane;
                *yp = a.accumulate ? *yp + mine : mine;
            }
        }
    }
}

}  // namespace neon
