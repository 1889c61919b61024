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

namespace neon {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSpans = 8;

// One projection target of a launch: rows [0, rows) of one uploaded tensor.
struct Span {
    const uint8_t* qs;   // payload plane
    const uint16_t* d;   // fp16 scale plane
    float* y;            // output, element (t, r) at y[t*y_stride + r]
    long long y_stride;
    int rows;
    int tile0;           // index of this span's first row tile in the launch
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
    const float id = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
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
        const float id = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
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
__device__ __forceinline__ int q4_block_isum(const uint4 w, const uint4 x0, const uint4 x1, int qsum) {
    int acc = 0;
    acc = __dp4a((int)(w.x & 0x0F0F0F0Fu), (int)x0.x, acc);
    acc = __dp4a((int)(w.y & 0x0F0F0F0Fu), (int)x0.y, acc);
    acc = __dp4a((int)(w.z & 0x0F0F0F0Fu), (int)x0.z, acc);
    acc = __dp4a((int)(w.w & 0x0F0F0F0Fu), (int)x0.w, acc);
    acc = __dp4a((int)((w.x >> 4) & 0x0F0F0F0Fu), (int)x1.x, acc);
    acc = __dp4a((int)((w.y >> 4) & 0x0F0F0F0Fu), (int)x1.y, acc);
    acc = __dp4a((int)((w.z >> 4) & 0x0F0F0F0Fu), (int)x1.z, acc);
    acc = __dp4a((int)((w.w >> 4) & 0x0F0F0F0Fu), (int)x1.w, acc);
    return acc - 8 * qsum;
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
// Q4_0 weights, one position: X quantised to Q8_0 inside every CTA.
// ---------------------------------------------------------------------------

// Shared memory: nb records of 48 bytes (32 quants, fp32 d, int32 sum, pad) --
// the 48-byte pitch keeps a warp's 128-bit reads conflict-free -- followed by a
// staging area of kThreads x 33 floats for X (33-float pitch: one thread reads
// one block without bank conflicts).
constexpr int kQ4Rec = 48;
__host__ __device__ constexpr int q4_seq1_smem_bytes(int nb) {
    return nb * kQ4Rec + kThreads * 33 * 4;
}

template <int R, int U>
__global__ void __launch_bounds__(kThreads) q4_0_seq1_kernel(const __grid_constant__ MatvecArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char* rec = smem;
    float* stage = reinterpret_cast<float*>(smem + a.nb * kQ4Rec);
    const int lane = threadIdx.x & 31;
    const int nb = a.nb;
    const int tile_step = gridDim.x * kWarps;

    pdl_launch_dependents();

    // 1. Fetch the first chunk of this warp's first tile. Weights are never
    //    written by earlier kernels, so this may run before the PDL wait.
    int tile = blockIdx.x * kWarps + (threadIdx.x >> 5);
    uint4 wq[R][U];
    uint16_t wd[R][U];
    int si = 0, row0 = 0;
    auto load_chunk = [&](int c) {
        const Span& sp = a.span[si];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int b = c + u * 32 + lane;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = row0 + r;
                if (b < nb && row < sp.rows) {
                    const long long i = (long long)row * nb + b;
                    wq[r][u] = ld_weights_u4(sp.qs + i * 16);
                    wd[r][u] = ld_weights_u16(sp.d + i);
                } else {
                    wq[r][u] = make_uint4(0, 0, 0, 0);
                    wd[r][u] = 0;
                }
            }
        }
    };
    if (tile < a.n_tiles) {
        si = find_span(a, tile);
        row0 = (tile - a.span[si].tile0) * R;
        load_chunk(0);
    }

    // 2. Quantise X (written by the previous kernel) into shared memory,
    //    kThreads blocks at a time, one block per thread.
    pdl_wait();
    const float* x = a.x;
    for (int c0 = 0; c0 < nb; c0 += kThreads) {
        const int nblk = min(kThreads, nb - c0);
        for (int i = threadIdx.x; i < nblk * 32; i += kThreads)
            stage[(i >> 5) * 33 + (i & 31)] = x[(long long)c0 * 32 + i];
        __syncthreads();
        if ((int)threadIdx.x < nblk) {
            uint32_t q[8];
            float d;
            int s;
            quantize_block_thread(stage + threadIdx.x * 33, q, d, s);
            uint4* r4 = reinterpret_cast<uint4*>(rec + (c0 + threadIdx.x) * kQ4Rec);
            r4[0] = make_uint4(q[0], q[1], q[2], q[3]);
            r4[1] = make_uint4(q[4], q[5], q[6], q[7]);
            r4[2] = make_uint4(__float_as_uint(d), (uint32_t)s, 0u, 0u);
        }
        __syncthreads();
    }

    // 3. Row tiles.
    while (tile < a.n_tiles) {
        const Span& sp = a.span[si];
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.f;
        for (int c = 0;;) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int b = c + u * 32 + lane;
                if (b < nb) {
                    const uint4* r4 = reinterpret_cast<const uint4*>(rec + b * kQ4Rec);
                    const uint4 x0 = r4[0], x1 = r4[1], xm = r4[2];
                    const float xd = __uint_as_float(xm.x);
                    const int xs = (int)xm.y;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int isum = q4_block_isum(wq[r][u], x0, x1, xs);
                        acc[r] = fmaf(fp16_bits_to_f32(wd[r][u]) * xd, (float)isum, acc[r]);
                    }
                }
            }
            c += 32 * U;
            if (c >= nb) break;
            load_chunk(c);
        }
        store_tile<R>(acc, sp.y, row0, sp.rows, lane);
        tile += tile_step;
        if (tile < a.n_tiles) {
            si = find_span(a, tile);
            row0 = (tile - a.span[si].tile0) * R;
            load_chunk(0);
        }
    }
}

// ---------------------------------------------------------------------------
// Q8_0 weights, one position: fp32 X staged in shared memory.
// ---------------------------------------------------------------------------

// X block b at smem float offset b*36 (a 144-byte pitch keeps the warp's
// 128-bit reads conflict-free).
constexpr int kQ8Pitch = 36;
__host__ __device__ constexpr int q8_seq1_smem_bytes(int nb) { return nb * kQ8Pitch * 4; }

template <int R, int U>
__global__ void __launch_bounds__(kThreads) q8_0_seq1_kernel(const __grid_constant__ MatvecArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* xs = reinterpret_cast<float*>(smem);
    const int lane = threadIdx.x & 31;
    const int nb = a.nb;
    const int tile_step = gridDim.x * kWarps;

    pdl_launch_dependents();

    int tile = blockIdx.x * kWarps + (threadIdx.x >> 5);
    uint4 wq[R][U][2];
    uint16_t wd[R][U];
    int si = 0, row0 = 0;
    auto load_chunk = [&](int c) {
        const Span& sp = a.span[si];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int b = c + u * 32 + lane;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = row0 + r;
                if (b < nb && row < sp.rows) {
                    const long long i = (long long)row * nb + b;
                    wq[r][u][0] = ld_weights_u4(sp.qs + i * 32);
                    wq[r][u][1] = ld_weights_u4(sp.qs + i * 32 + 16);
                    wd[r][u] = ld_weights_u16(sp.d + i);
                } else {
                    wq[r][u][0] = make_uint4(0, 0, 0, 0);
                    wq[r][u][1] = make_uint4(0, 0, 0, 0);
                    wd[r][u] = 0;
                }
            }
        }
    };
    if (tile < a.n_tiles) {
        si = find_span(a, tile);
        row0 = (tile - a.span[si].tile0) * R;
        load_chunk(0);
    }

    pdl_wait();
    const float* x = a.x;
    for (int i = threadIdx.x; i < nb * 32; i += kThreads) xs[(i >> 5) * kQ8Pitch + (i & 31)] = x[i];
    __syncthreads();

    while (tile < a.n_tiles) {
        const Span& sp = a.span[si];
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.f;
        for (int c = 0;;) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int b = c + u * 32 + lane;
                if (b < nb) {
                    const float4* xv = reinterpret_cast<const float4*>(xs + b * kQ8Pitch);
                    float4 xr[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) xr[k] = xv[k];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float s = q8_block_dot(wq[r][u][0], wq[r][u][1], xr);
                        acc[r] = fmaf(fp16_bits_to_f32(wd[r][u]), s, acc[r]);
                    }
                }
            }
            c += 32 * U;
            if (c >= nb) break;
            load_chunk(c);
        }
        store_tile<R>(acc, sp.y, row0, sp.rows, lane);
        tile += tile_step;
        if (tile < a.n_tiles) {
            si = find_span(a, tile);
            row0 = (tile - a.span[si].tile0) * R;
            load_chunk(0);
        }
    }
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
            if (lane < R && row0 + lane < sp.rows) sp.y[(long long)tt * sp.y_stride + row0 + lane] = mine;
        }
    }
}

}  // namespace neon
