// neon_dequant.cuh -- the matvec of the remaining GGUF weight types:
// F32, F16, BF16, Q4_1, Q5_0, Q5_1 and the K-quant super-blocks Q4_K, Q5_K,
// Q6_K (sm_100a, CUDA cores).
//
// Reference path: every weight type other than Q4_0 is dequantised a row at a
// time (dequantize_row, rawllm_forward.hpp:301-321, with the block decoders of
// :133-298) and dotted with fp32 X (dot_f32, :446-479), inside
// proj_all_positions (:597-605) and proj_all_positions_multi (:632-726).
// Here the weights are decoded straight from the block bytes in registers,
// never written out as fp32 rows.
//
// Device layout (neon_cuda_upload): the GGUF rows unchanged, each row padded
// to a 16-byte pitch so that every row -- and every chunk of CB blocks, whose
// byte size is a multiple of 16 for every type -- starts on a 16-byte
// boundary. The plain float types are cut into 32-value "blocks" and their
// rows zero-padded to a whole number of them.
//
// Work decomposition: a CTA (8 warps) owns a tile of 8 consecutive rows, one
// row per warp. A warp walks its row a chunk at a time: the chunk's bytes are
// read with coalesced 128-bit loads (two chunks in flight per warp, held in
// registers), parked in the warp's shared-memory buffer, and every lane then
// takes whole 32-value sub-blocks from it (one
// for the 32-value types, two for the K-quants: 8 super-blocks = 64
// sub-blocks a chunk): their integer codes and affine map (dq_codes), and
// the dot product a*sum((code - OFF)*x) + b*sum(x) on packed fp32 pairs
// (dq_code_dot) against X, which the CTA staged once in shared memory (fp32,
// 36-float pitch per 32 values, so the lanes' 128-bit reads of consecutive
// sub-blocks do not collide; the spare float holds the sub-block's sum).
// The float types skip shared memory: each lane multiplies the 16-byte words
// it loaded. A butterfly shuffle finishes each row; the decode-step
// epilogues are the one-position kernel's (stream_epilogue).
//
// Every weight the decoders form equals the reference's bit for bit (dq_sub:
// one exact product -- at most 23 significant bits, fp16 scale x 6-bit
// sub-scale x 6-bit quant -- plus at most one rounded add); the kernel's dot
// product regroups the same sum: per sub-block a*sum((code-OFF)*x) + b*sum(x)
// instead of sum((a*(code-OFF)+b)*x), and its additions run in another order
// than dot_f32's.
#pragma once

#include <string.h>

#include "neon_kernels.cuh"

namespace neon {

// BE values and BB bytes per block; CB blocks per chunk (CB*BB is a multiple
// of 16 for every type).
template <int TYPE> struct DqType;
template <> struct DqType<NEON_GGML_F32> { static constexpr int BE = 32, BB = 128, CB = 32; };
template <> struct DqType<NEON_GGML_F16> { static constexpr int BE = 32, BB = 64, CB = 32; };
template <> struct DqType<NEON_GGML_BF16> { static constexpr int BE = 32, BB = 64, CB = 32; };
template <> struct DqType<NEON_GGML_Q4_1> { static constexpr int BE = 32, BB = 20, CB = 32; };
template <> struct DqType<NEON_GGML_Q5_0> { static constexpr int BE = 32, BB = 22, CB = 32; };
template <> struct DqType<NEON_GGML_Q5_1> { static constexpr int BE = 32, BB = 24, CB = 32; };
template <> struct DqType<NEON_GGML_Q4_K> { static constexpr int BE = 256, BB = 144, CB = 8; };
template <> struct DqType<NEON_GGML_Q5_K> { static constexpr int BE = 256, BB = 176, CB = 8; };
template <> struct DqType<NEON_GGML_Q6_K> { static constexpr int BE = 256, BB = 210, CB = 8; };

template <int TYPE> struct DqShape {
    static constexpr int BE = DqType<TYPE>::BE, BB = DqType<TYPE>::BB, CB = DqType<TYPE>::CB;
    static constexpr int SUBS = BE / 32;                 // 32-value sub-blocks per block
    static constexpr int UNITS = CB * SUBS;              // sub-blocks per chunk: 32 or 64
    static constexpr int UPL = UNITS / 32;               // per lane
    static constexpr int CHUNK = CB * BB;                // bytes per chunk
    static constexpr int WPL = (CHUNK / 16 + 31) / 32;   // 128-bit loads per lane per chunk
    static_assert(CHUNK % 16 == 0, "chunks must stay 16-byte aligned");
};

// Host view of the block geometry of a type: values per block, bytes per
// block, blocks per chunk (0 if the type is not one of this kernel's).
__host__ __device__ inline void dq_geometry(int type, int* be, int* bb, int* cb) {
    switch (type) {
#define NEON_DQ_GEOMETRY(T)    \
    case T:                    \
        *be = DqType<T>::BE;   \
        *bb = DqType<T>::BB;   \
        *cb = DqType<T>::CB;   \
        return;
        NEON_DQ_GEOMETRY(NEON_GGML_F32)
        NEON_DQ_GEOMETRY(NEON_GGML_F16)
        NEON_DQ_GEOMETRY(NEON_GGML_BF16)
        NEON_DQ_GEOMETRY(NEON_GGML_Q4_1)
        NEON_DQ_GEOMETRY(NEON_GGML_Q5_0)
        NEON_DQ_GEOMETRY(NEON_GGML_Q5_1)
        NEON_DQ_GEOMETRY(NEON_GGML_Q4_K)
        NEON_DQ_GEOMETRY(NEON_GGML_Q5_K)
        NEON_DQ_GEOMETRY(NEON_GGML_Q6_K)
#undef NEON_DQ_GEOMETRY
        default:
            *be = *bb = *cb = 0;
    }
}

struct DqArgs {
    StreamArgs s;         // spans (qs = the padded GGUF rows), X, epilogue and fused-collective options
    long long pitch;      // bytes per device row (same for every span: one type, one input dim)
    long long x_stride;   // floats between positions of X
    int cols;             // values per row (X entries read; the float types may be ragged)
    int nu;               // 32-value sub-blocks per row (cols rounded up)
    int nblk;             // blocks per row
    int nch;              // chunks per row
    int seq;              // positions
};

// Shared memory of a launch: X for T positions, then one chunk buffer per warp.
__host__ __device__ constexpr int dq_x_bytes(int T, int nu) { return ((T * nu * kQ8Pitch * 4) + 127) & ~127; }

// The block decoders below are __host__ __device__: the host build of the
// same source is what the CPU tests compare against the oracle.
#ifdef __CUDA_ARCH__
#define NEON_HD_MUL(a, b) __fmul_rn((a), (b))  // never contracted into an FMA
#define NEON_HD_BITS_F32(u) __uint_as_float(u)
#else
#define NEON_HD_MUL(a, b) ((a) * (b))
inline float neon_hd_bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
#define NEON_HD_BITS_F32(u) neon_hd_bits_f32(u)
#endif

__host__ __device__ __forceinline__ uint32_t sh_u16(const unsigned char* p) { return *reinterpret_cast<const uint16_t*>(p); }
__host__ __device__ __forceinline__ uint32_t sh_u32(const unsigned char* p) { return *reinterpret_cast<const uint32_t*>(p); }
// binary16 -> binary32, exact (subnormals included)
__host__ __device__ __forceinline__ float sh_half(const unsigned char* p) {
    return __half2float(__ushort_as_half((unsigned short)sh_u16(p)));
}

// The value of byte i of u minus OFF, exactly. On the device the word
// 0x4B0000vv, read as a float, is 2^23 + v, and one exact subtraction leaves
// v - OFF: no integer-to-float conversion instruction (those issue at a
// fraction of the FMA rate).
template <int OFF>
__host__ __device__ __forceinline__ float byte_val(uint32_t u, int i) {
#ifdef __CUDA_ARCH__
    return __int_as_float(__byte_perm(u, 0x4B000000u, 0x7650 + i)) - (8388608.0f + (float)OFF);
#else
    return (float)((int)((u >> (8 * i)) & 0xFFu) - OFF);
#endif
}

// Bits 0-3 of x to bit 0 of bytes 0-3 (the four shifted copies never overlap).
__host__ __device__ __forceinline__ uint32_t spread4(uint32_t x) { return (x * 0x00204081u) & 0x01010101u; }

// The (scale, min) pair of sub-block s of a Q4_K / Q5_K super-block from its
// 12 packed bytes (get_scale_min_k4, rawllm_forward.hpp:224-233): sub-blocks
// 0-3 use the low six bits of bytes s and s+4; 4-7 take a nibble of byte s+4
// and two high bits from bytes s-4 (scale) and s (min).
__host__ __device__ __forceinline__ void k4_scale_min(const unsigned char* sc, int s, int& scale, int& mn) {
    if (s < 4) {
        scale = sc[s] & 63;
        mn = sc[s + 4] & 63;
    } else {
        scale = (sc[s + 4] & 0x0F) | ((sc[s - 4] >> 6) << 4);
        mn = (sc[s + 4] >> 4) | ((sc[s] >> 6) << 4);
    }
}

// The 32 integer codes of sub-block s of a block type, four per word in
// value order (value 4k + i in byte i of v[k]), and the affine map back to
// weights: value = a * (code - OFF) + b, with a = a0 for values 0-15 and a1
// for 16-31 (they differ only for Q6_K's 16-value scales). Formulas of
// rawllm_forward.hpp, regrouped by sub-block:
//   Q4_1 :164-175  d*q + m             Q5_0 :177-191  d*(q - 16), q = nibble | qh bit << 4
//   Q5_1 :193-208  d*q + m (q as Q5_0)
//   Q4_K :235-253  (d*sc)*q - dmin*mn on nibble (s&1) of bytes 32*(s/2)..
//   Q5_K :255-275  as Q4_K, q += 16 * bit s of qh[l]
//   Q6_K :277-298  (d*sc)*(q - 32); sub-block s = 4h + k: low bytes 64h + 32(k&1)..,
//                  high nibble when k >= 2, 2-bit pair k of qh[32h + l], scales 8h + 2k + l/16
template <int TYPE> struct DqCode {
    static constexpr int OFF = TYPE == NEON_GGML_Q5_0 ? 16 : TYPE == NEON_GGML_Q6_K ? 32 : 0;
    static constexpr bool HAS_B = TYPE == NEON_GGML_Q4_1 || TYPE == NEON_GGML_Q5_1 ||
                                  TYPE == NEON_GGML_Q4_K || TYPE == NEON_GGML_Q5_K;
    uint32_t v[8];
    float a0, a1, b;
};

template <int TYPE>
__host__ __device__ __forceinline__ void dq_codes(const unsigned char* blk, int s, DqCode<TYPE>& c) {
    if constexpr (TYPE == NEON_GGML_Q4_1 || TYPE == NEON_GGML_Q5_1) {
        // 4-byte aligned blocks (20 / 24 bytes)
        constexpr bool five = TYPE == NEON_GGML_Q5_1;
        c.a0 = c.a1 = sh_half(blk);
        c.b = sh_half(blk + 2);
        const uint32_t qh = five ? sh_u32(blk + 4) : 0u;
        const unsigned char* qs = blk + (five ? 8 : 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t q4 = sh_u32(qs + 4 * k);
            uint32_t lo = q4 & 0x0F0F0F0Fu, hi = (q4 >> 4) & 0x0F0F0F0Fu;
            if (five) {
                lo |= spread4((qh >> (4 * k)) & 0xFu) << 4;
                hi |= spread4((qh >> (4 * k + 16)) & 0xFu) << 4;
            }
            c.v[k] = lo;
            c.v[k + 4] = hi;
        }
    } else if constexpr (TYPE == NEON_GGML_Q5_0) {
        // 22-byte blocks: only 2-byte alignment
        c.a0 = c.a1 = sh_half(blk);
        c.b = 0.f;
        const uint32_t qh = sh_u16(blk + 2) | (sh_u16(blk + 4) << 16);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t q4 = sh_u16(blk + 6 + 4 * k) | (sh_u16(blk + 8 + 4 * k) << 16);
            c.v[k] = (q4 & 0x0F0F0F0Fu) | (spread4((qh >> (4 * k)) & 0xFu) << 4);
            c.v[k + 4] = ((q4 >> 4) & 0x0F0F0F0Fu) | (spread4((qh >> (4 * k + 16)) & 0xFu) << 4);
        }
    } else if constexpr (TYPE == NEON_GGML_Q4_K || TYPE == NEON_GGML_Q5_K) {
        // 16-byte aligned super-blocks (144 / 176 bytes)
        constexpr bool five = TYPE == NEON_GGML_Q5_K;
        const float d = sh_half(blk), dmin = sh_half(blk + 2);
        int sc, mn;
        k4_scale_min(blk + 4, s, sc, mn);
        c.a0 = c.a1 = NEON_HD_MUL(d, (float)sc);
        c.b = -NEON_HD_MUL(dmin, (float)mn);
        const unsigned char* q = blk + (five ? 48 : 16) + 32 * (s >> 1);
        const int shift = (s & 1) * 4;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t v = (sh_u32(q + 4 * k) >> shift) & 0x0F0F0F0Fu;
            if (five) v |= ((sh_u32(blk + 16 + 4 * k) >> s) & 0x01010101u) << 4;
            c.v[k] = v;
        }
    } else if constexpr (TYPE == NEON_GGML_Q6_K) {
        // 210-byte super-blocks: only 2-byte alignment
        const int h = s >> 2, k = s & 3;
        const unsigned char* ql = blk + 64 * h + 32 * (k & 1);
        const unsigned char* qh = blk + 128 + 32 * h;
        const signed char* scp = reinterpret_cast<const signed char*>(blk + 192 + 8 * h + 2 * k);
        const float d = sh_half(blk + 208);
        c.a0 = NEON_HD_MUL(d, (float)scp[0]);
        c.a1 = NEON_HD_MUL(d, (float)scp[1]);
        c.b = 0.f;
        const int lshift = (k >> 1) * 4, hshift = 2 * k;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t l4 = sh_u16(ql + 4 * j) | (sh_u16(ql + 4 * j + 2) << 16);
            const uint32_t h4 = sh_u16(qh + 4 * j) | (sh_u16(qh + 4 * j + 2) << 16);
            c.v[j] = ((l4 >> lshift) & 0x0F0F0F0Fu) | (((h4 >> hshift) & 0x03030303u) << 4);
        }
    }
}

// The 32 values of sub-block s of the block at `blk` (shared or global memory,
// aligned as a block of the padded-row layout is): the float types' words, or
// a * (code - OFF) + b of the block types. Each value is the reference's bit
// for bit: a * (code - OFF) is exact, so one fused multiply-add rounds once,
// as the reference's multiply (exact) and add do; types without b multiply.
template <int TYPE>
__host__ __device__ __forceinline__ void dq_sub(const unsigned char* blk, int s, float (&w)[32]) {
    if constexpr (TYPE == NEON_GGML_F32) {
        const float4* p = reinterpret_cast<const float4*>(blk);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 v = p[k];
            w[4 * k] = v.x;
            w[4 * k + 1] = v.y;
            w[4 * k + 2] = v.z;
            w[4 * k + 3] = v.w;
        }
    } else if constexpr (TYPE == NEON_GGML_F16 || TYPE == NEON_GGML_BF16) {
        const uint4* p = reinterpret_cast<const uint4*>(blk);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 v = p[k];
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if constexpr (TYPE == NEON_GGML_F16) {
                    w[8 * k + 2 * i] = __half2float(__ushort_as_half((unsigned short)(u[i] & 0xFFFFu)));
                    w[8 * k + 2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(u[i] >> 16)));
                } else {
                    w[8 * k + 2 * i] = NEON_HD_BITS_F32(u[i] << 16);
                    w[8 * k + 2 * i + 1] = NEON_HD_BITS_F32(u[i] & 0xFFFF0000u);
                }
            }
        }
    } else {
        DqCode<TYPE> c;
        dq_codes<TYPE>(blk, s, c);
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float q = byte_val<DqCode<TYPE>::OFF>(c.v[k], i);
                // no additive term: a plain product, as the reference's (keeps -0)
                w[4 * k + i] = DqCode<TYPE>::HAS_B ? fmaf(k < 4 ? c.a0 : c.a1, q, c.b)
                                                   : NEON_HD_MUL(k < 4 ? c.a0 : c.a1, q);
            }
    }
}

// The dot product of a block-type sub-block with 32 floats of X (shared
// memory, 16-byte aligned), without forming the weights:
//     sum_j (a*(code_j - OFF) + b) * x_j = a * sum_j (code_j - OFF) * x_j + b * xsum
// with xsum = sum_j x_j (staged with X). The inner sum runs on packed fp32
// pairs (two values per fma.rn.f32x2); codes become floats exactly through
// the 2^23 bias. The host build runs the same operations one lane at a time,
// so its results equal the device's bit for bit.
#ifdef __CUDA_ARCH__
#define NEON_PAIR unsigned long long
#define NEON_PAIR_ZERO 0ull
__device__ __forceinline__ NEON_PAIR pair_bias(uint32_t v, int half, float bias) {
    // bytes 2*half, 2*half+1 of v as 2^23 + code, minus the bias 2^23 + OFF
    unsigned long long p;
    if (half == 0)
        asm("{ .reg .b32 lo, hi; prmt.b32 lo, %1, 0x4B000000, 0x7650; prmt.b32 hi, %1, 0x4B000000, 0x7651; "
            "mov.b64 %0, {lo, hi}; }" : "=l"(p) : "r"(v));
    else
        asm("{ .reg .b32 lo, hi; prmt.b32 lo, %1, 0x4B000000, 0x7652; prmt.b32 hi, %1, 0x4B000000, 0x7653; "
            "mov.b64 %0, {lo, hi}; }" : "=l"(p) : "r"(v));
    const uint32_t nb = __float_as_uint(-bias);
    return f32x2_add(p, ((unsigned long long)nb << 32) | nb);
}
__device__ __forceinline__ NEON_PAIR pair_fma(NEON_PAIR a, NEON_PAIR b, NEON_PAIR c) { return f32x2_fma(a, b, c); }
__device__ __forceinline__ float pair_sum(NEON_PAIR p) {
    return __uint_as_float((uint32_t)p) + __uint_as_float((uint32_t)(p >> 32));
}
__device__ __forceinline__ void x_pairs(const float* x, int k, NEON_PAIR& p0, NEON_PAIR& p1) {
    const ulonglong2 t = reinterpret_cast<const ulonglong2*>(x)[k];
    p0 = t.x;
    p1 = t.y;
}
#else
struct NeonPair {
    float lo, hi;
};
#define NEON_PAIR NeonPair
#define NEON_PAIR_ZERO NeonPair{0.f, 0.f}
inline NeonPair pair_bias(uint32_t v, int half, float bias) {
    const float b0 = (float)((v >> (16 * half)) & 0xFFu) + 8388608.0f;  // exact
    const float b1 = (float)((v >> (16 * half + 8)) & 0xFFu) + 8388608.0f;
    return NeonPair{b0 - bias, b1 - bias};
}
inline NeonPair pair_fma(NeonPair a, NeonPair b, NeonPair c) { return NeonPair{fmaf(a.lo, b.lo, c.lo), fmaf(a.hi, b.hi, c.hi)}; }
inline float pair_sum(NeonPair p) { return p.lo + p.hi; }
inline void x_pairs(const float* x, int k, NeonPair& p0, NeonPair& p1) {
    p0 = NeonPair{x[4 * k], x[4 * k + 1]};
    p1 = NeonPair{x[4 * k + 2], x[4 * k + 3]};
}
#endif

template <int TYPE>
__host__ __device__ __forceinline__ float dq_code_dot(const DqCode<TYPE>& c, const float* x, float xsum) {
    constexpr float bias = 8388608.0f + (float)DqCode<TYPE>::OFF;
    NEON_PAIR s0 = NEON_PAIR_ZERO, s1 = NEON_PAIR_ZERO;  // values 0-15, 16-31
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        NEON_PAIR x0, x1;
        x_pairs(x, k, x0, x1);
        if (k < 4) {
            s0 = pair_fma(pair_bias(c.v[k], 0, bias), x0, s0);
            s0 = pair_fma(pair_bias(c.v[k], 1, bias), x1, s0);
        } else {
            s1 = pair_fma(pair_bias(c.v[k], 0, bias), x0, s1);
            s1 = pair_fma(pair_bias(c.v[k], 1, bias), x1, s1);
        }
    }
    if constexpr (TYPE == NEON_GGML_Q6_K) return fmaf(c.a0, pair_sum(s0), NEON_HD_MUL(c.a1, pair_sum(s1)));
    const float dot = NEON_HD_MUL(c.a0, pair_sum(s0) + pair_sum(s1));
    if constexpr (DqCode<TYPE>::HAS_B) return fmaf(c.b, xsum, dot);
    return dot;
}

// T positions per CTA (grid.y tiles the positions); one row per warp.
//
// Every warp holds two chunks of its row in registers: the loads of chunk
// i + 2 go out as soon as chunk i has left its registers -- parked in the
// warp's shared-memory buffer for the block types, consumed in place for the
// float types, whose lanes take the 16-byte words l, l + 32, ... of a chunk
// and so read X without bank conflicts.
template <int TYPE, int T>
__global__ void __launch_bounds__(kThreads) matvec_dq_kernel(const __grid_constant__ DqArgs a) {
    using D = DqShape<TYPE>;
    constexpr bool kFloat = TYPE == NEON_GGML_F32 || TYPE == NEON_GGML_F16 || TYPE == NEON_GGML_BF16;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float rowv[2][T][kWarps];   // by tile parity: a tile's results never wait on the last epilogue
    __shared__ double dscratch[32];
    __shared__ float2 rcs[kMaxRopeHalf];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nu = a.nu, nch = a.nch;
    float* xs = reinterpret_cast<float*>(smem);
    unsigned char* wbuf = smem + dq_x_bytes(T, nu) + warp * D::CHUNK;
    const int p0 = (int)blockIdx.y * T;
    const int npos = min(T, a.seq - p0);
    const int my_tiles =
        (int)blockIdx.x < a.s.n_tiles ? (a.s.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_items = my_tiles * nch;

    // this warp's row of item `item`, its chunk, and the chunk's block count
    auto locate = [&](int item, int& span, int& row0, int& chunk, int& nblk_c) {
        const int tile = (int)blockIdx.x + (item / nch) * (int)gridDim.x;
        span = find_span_of(a.s, tile);
        row0 = (tile - a.s.span[span].tile0) * kWarps;
        chunk = item % nch;
        nblk_c = min(D::CB, a.nblk - chunk * D::CB);
    };
    auto load = [&](uint4 (&buf)[D::WPL], int item) {
        int span, row0, chunk, nblk_c;
        locate(item, span, row0, chunk, nblk_c);
        const int row = row0 + warp;
        if (row >= a.s.span[span].rows) return;
        const unsigned char* src = a.s.span[span].qs + (long long)row * a.pitch + (long long)chunk * D::CHUNK;
        const int words = (nblk_c * D::BB + 15) >> 4;
#pragma unroll
        for (int k = 0; k < D::WPL; ++k) {
            const int wi = lane + 32 * k;
            if (wi < words) buf[k] = ld_weights_u4(src + 16 * wi);
        }
    };
    // weights are never written by an earlier kernel of the stream: the first
    // two chunks' loads go out before the dependency wait
    uint4 bufA[D::WPL], bufB[D::WPL];
    if (n_items > 0) load(bufA, 0);
    if (n_items > 1) load(bufB, 1);
    pdl_wait();

    const unsigned int peer_call =
        a.s.peer_mode ? *reinterpret_cast<volatile const unsigned int*>(a.s.peer.calls) + 1u : 0u;
    const int pos = a.s.d_pos ? *a.s.d_pos : 0;
    if (a.s.rope_cs)
        for (int i = threadIdx.x; i < a.s.rope_half; i += kThreads) rcs[i] = a.s.rope_cs[(long long)pos * a.s.rope_half + i];

    // X of this CTA's positions (rms-normalised first when asked; one position
    // then), zero past `cols`; 128-bit loads, several in flight per thread
    {
        const float nscale = a.s.norm_w ? cta_rms_scale(a.s.x, a.cols, a.s.norm_eps, dscratch) : 1.f;
        for (int t = 0; t < npos; ++t) {
            const float* xp = a.s.x + (long long)(p0 + t) * a.x_stride;
            float* xd = xs + (long long)t * nu * kQ8Pitch;
            if (a.s.x_vec) {
                const int n4 = a.cols >> 2;
#pragma unroll 4
                for (int i4 = threadIdx.x; i4 < n4; i4 += kThreads) {
                    float4 v = __ldg(reinterpret_cast<const float4*>(xp) + i4);
                    if (a.s.norm_w) {
                        const float4 g = __ldg(reinterpret_cast<const float4*>(a.s.norm_w) + i4);
                        v.x = __fmul_rn(__fmul_rn(v.x, nscale), g.x);
                        v.y = __fmul_rn(__fmul_rn(v.y, nscale), g.y);
                        v.z = __fmul_rn(__fmul_rn(v.z, nscale), g.z);
                        v.w = __fmul_rn(__fmul_rn(v.w, nscale), g.w);
                    }
                    const int i = 4 * i4;
                    *reinterpret_cast<float4*>(xd + (i >> 5) * kQ8Pitch + (i & 31)) = v;
                }
                for (int i = 4 * n4 + threadIdx.x; i < nu * 32; i += kThreads) {
                    float v = 0.f;
                    if (i < a.cols) {
                        v = __ldg(xp + i);
                        if (a.s.norm_w) v = __fmul_rn(__fmul_rn(v, nscale), __ldg(a.s.norm_w + i));
                    }
                    xd[(i >> 5) * kQ8Pitch + (i & 31)] = v;
                }
            } else {
#pragma unroll 4
                for (int i = threadIdx.x; i < nu * 32; i += kThreads) {
                    float v = 0.f;
                    if (i < a.cols) {
                        v = __ldg(xp + i);
                        if (a.s.norm_w) v = __fmul_rn(__fmul_rn(v, nscale), __ldg(a.s.norm_w + i));
                    }
                    xd[(i >> 5) * kQ8Pitch + (i & 31)] = v;
                }
            }
        }
    }
    __syncthreads();
    if constexpr (!kFloat && DqCode<TYPE>::HAS_B) {
        // sum of each 32-value sub-block of X, kept in the pitch's spare float
        for (int idx = threadIdx.x; idx < npos * nu; idx += kThreads) {
            float* xu = xs + (long long)idx * kQ8Pitch;
            const float4* x4 = reinterpret_cast<const float4*>(xu);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                const float4 p = x4[k], q = x4[k + 1];
                s0 += (p.x + p.y) + (p.z + p.w);
                s1 += (q.x + q.y) + (q.z + q.w);
            }
            xu[32] = s0 + s1;
        }
        __syncthreads();
    }
    pdl_launch_dependents();

    float acc[T];
#pragma unroll
    for (int t = 0; t < T; ++t) acc[t] = 0.f;
    // the dot products of the item held in `buf`, then `buf` refilled with
    // item + 2; at a row's last chunk, the row's results and their epilogue
    auto consume = [&](uint4 (&buf)[D::WPL], int item) {
        int span, row0, chunk, nblk_c;
        locate(item, span, row0, chunk, nblk_c);
        const Span& sp = a.s.span[span];
        const bool valid = row0 + warp < sp.rows;
        const int words = (nblk_c * D::BB + 15) >> 4;
        if constexpr (kFloat) {
            if (valid) {
#pragma unroll
                for (int k = 0; k < D::WPL; ++k) {
                    const int wi = lane + 32 * k;
                    if (wi >= words) continue;
                    const uint4 v = buf[k];
                    constexpr int VPW = TYPE == NEON_GGML_F32 ? 4 : 8;  // values per 16-byte word
                    const int e = chunk * (D::UNITS * 32) + VPW * wi;
                    float wv[VPW];
                    if constexpr (TYPE == NEON_GGML_F32) {
                        wv[0] = __uint_as_float(v.x);
                        wv[1] = __uint_as_float(v.y);
                        wv[2] = __uint_as_float(v.z);
                        wv[3] = __uint_as_float(v.w);
                    } else {
                        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            if constexpr (TYPE == NEON_GGML_F16) {
                                wv[2 * q] = __half2float(__ushort_as_half((unsigned short)(u[q] & 0xFFFFu)));
                                wv[2 * q + 1] = __half2float(__ushort_as_half((unsigned short)(u[q] >> 16)));
                            } else {
                                wv[2 * q] = __uint_as_float(u[q] << 16);
                                wv[2 * q + 1] = __uint_as_float(u[q] & 0xFFFF0000u);
                            }
                        }
                    }
#pragma unroll
                    for (int t = 0; t < T; ++t) {
                        if (t >= npos) break;
                        const float4* x4 = reinterpret_cast<const float4*>(
                            xs + ((long long)t * nu + (e >> 5)) * kQ8Pitch + (e & 31));
#pragma unroll
                        for (int q = 0; q < VPW / 4; ++q) {
                            const float4 xv = x4[q];
                            acc[t] = fmaf(wv[4 * q], xv.x, acc[t]);
                            acc[t] = fmaf(wv[4 * q + 1], xv.y, acc[t]);
                            acc[t] = fmaf(wv[4 * q + 2], xv.z, acc[t]);
                            acc[t] = fmaf(wv[4 * q + 3], xv.w, acc[t]);
                        }
                    }
                }
            }
            if (item + 2 < n_items) load(buf, item + 2);
        } else {
            // park the chunk in the warp's buffer, start the loads of item + 2, decode
            __syncwarp();
            if (valid) {
#pragma unroll
                for (int k = 0; k < D::WPL; ++k) {
                    const int wi = lane + 32 * k;
                    if (wi < words) reinterpret_cast<uint4*>(wbuf)[wi] = buf[k];
                }
            }
            __syncwarp();
            if (item + 2 < n_items) load(buf, item + 2);
            if (valid) {
#pragma unroll
                for (int j = 0; j < D::UPL; ++j) {
                    const int u = lane + 32 * j;
                    if (u < nblk_c * D::SUBS) {
                        DqCode<TYPE> c;
                        dq_codes<TYPE>(wbuf + (u / D::SUBS) * D::BB, u % D::SUBS, c);
                        const int unit = chunk * D::UNITS + u;
#pragma unroll
                        for (int t = 0; t < T; ++t) {
                            if (t >= npos) break;
                            const float* xu = xs + ((long long)t * nu + unit) * kQ8Pitch;
                            acc[t] += dq_code_dot<TYPE>(c, xu, xu[32]);
                        }
                    }
                }
            }
        }
        if (chunk == nch - 1) {
            const int tb = (item / nch) & 1;
#pragma unroll
            for (int t = 0; t < T; ++t) {
#pragma unroll
                for (int o = 16; o; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
                if (lane == 0) rowv[tb][t][warp] = acc[t];
                acc[t] = 0.f;
            }
            __syncthreads();
            if constexpr (T == 1) {
                // one position: the decode epilogues (plain store at position p0 otherwise)
                Span spo = sp;
                spo.y += (long long)p0 * sp.y_stride;
                float yold = 0.f;
                if (a.s.accumulate && spo.epi == kEpiStore && (int)threadIdx.x < kWarps &&
                    row0 + (int)threadIdx.x < spo.rows)
                    yold = spo.y[row0 + threadIdx.x];
                stream_epilogue(a.s, spo, row0, kWarps, rowv[tb][0], peer_call, pos, rcs, yold);
            } else {
                const int t = threadIdx.x / kWarps, r = threadIdx.x % kWarps;
                const int row = row0 + r;
                if (t < npos && row < sp.rows) {
                    float* y = sp.y + (long long)(p0 + t) * sp.y_stride + row;
                    const float v = rowv[tb][t][r];
                    *y = a.s.accumulate ? *y + v : v;
                }
            }
        }
    };
    for (int item = 0; item < n_items; item += 2) {
        consume(bufA, item);
        if (item + 1 < n_items) consume(bufB, item + 1);
    }
}

// One position on a bulk-copy ring (the streaming kernel's scheme, for every
// dequantised type): a copy warp moves the weights of an item -- the RC rows
// of a tile, one chunk of kcb blocks of each -- into a ring of shared-memory
// stages with cp.async.bulk, one mbarrier per stage counting its bytes, so a
// CTA keeps several items in flight where matvec_dq_kernel keeps two chunks
// per warp in registers, and the compute warps decode straight from the
// stage. Every warp owns RPW rows of a tile: a read of X serves all of them.
//
// Stage layout: row r of the item at r * row_stride; row_stride is the pitch
// when a whole row is one chunk (the tile is then one contiguous copy), else
// kcb * BB. Every copy starts and ends on a 16-byte boundary: the pitch and
// kcb * BB are multiples of 16, and a row's last chunk runs to its pitch.
constexpr int kDqRingMaxStages = 4;

struct DqRingArgs {
    DqArgs d;         // spans of RC-row tiles, X, epilogue options; d.nch chunks per row
    int kcb;          // blocks per chunk
    int row_stride;   // bytes between a stage's rows
    int stages;       // ring depth (<= kDqRingMaxStages)
    int stage_bytes;  // bytes per stage (a multiple of 128)
};

// Tile plan of a ring launch: RC = 8 * rpw rows per tile (two rows per warp
// once every SM has 16-row tiles to take); a row is one chunk when the tile's
// rows fit `stage_target` bytes, else chunks of kcb blocks, kcb a multiple of
// the smallest block count whose bytes are a multiple of 16 (so every copy
// starts and ends 16-byte aligned). pitch: bytes per device row.
struct DqRingPlan {
    int rpw, kcb, nch, row_stride, stage_bytes;
};
inline DqRingPlan plan_dq_ring(int type, int nblk, long long pitch, size_t total_rows, int sms, int stage_target) {
    int be, bb, cb;
    dq_geometry(type, &be, &bb, &cb);
    DqRingPlan p{};
    p.rpw = total_rows >= (size_t)16 * (size_t)sms ? 2 : 1;
    const int rc = kStreamWarps * p.rpw;
    int g = 1;
    while ((g * bb) % 16) ++g;
    p.kcb = nblk;
    p.nch = 1;
    p.row_stride = (int)pitch;
    if (rc * pitch > stage_target) {
        const int k = stage_target / (rc * bb) / g * g;
        p.kcb = k > g ? k : g;
        p.nch = (nblk + p.kcb - 1) / p.kcb;
        if (p.nch == 1) p.kcb = nblk;
        else p.row_stride = p.kcb * bb;
    }
    p.stage_bytes = (rc * p.row_stride + 127) & ~127;
    return p;
}

template <int TYPE, int RPW>
__global__ void __launch_bounds__(kStreamBlock) matvec_dq_ring_kernel(const __grid_constant__ DqRingArgs r) {
    using D = DqShape<TYPE>;
    constexpr bool kFloat = TYPE == NEON_GGML_F32 || TYPE == NEON_GGML_F16 || TYPE == NEON_GGML_BF16;
    constexpr int RC = kStreamWarps * RPW;
    const DqArgs& a = r.d;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float rowv[2][RC];  // by tile parity: a tile's results never wait on the last epilogue
    __shared__ double dscratch[32];
    __shared__ float2 rcs[kMaxRopeHalf];
    __shared__ __align__(8) uint64_t full[kDqRingMaxStages];
    __shared__ __align__(8) uint64_t empty[kDqRingMaxStages];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nu = a.nu, nch = a.nch, S = r.stages, RS = r.row_stride;
    float* xs = reinterpret_cast<float*>(smem);
    unsigned char* ring = smem + dq_x_bytes(1, nu);
    const int my_tiles =
        (int)blockIdx.x < a.s.n_tiles ? (a.s.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_items = my_tiles * nch;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStreamWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kStreamWarps) {
        // Copy warp. Weights are never written by an earlier kernel of the
        // stream: no dependency wait; a stage is refilled as soon as every
        // compute warp has released it.
        pdl_launch_dependents();
        for (int item = 0; item < n_items; ++item) {
            const int stage = item % S;
            if (item >= S && !mbar_wait(&empty[stage], (uint32_t)(((item / S) - 1) & 1), a.s.err)) break;
            const int tile = (int)blockIdx.x + (item / nch) * (int)gridDim.x;
            const int chunk = item % nch;
            const Span& sp = a.s.span[find_span_of(a.s, tile)];
            const int row0 = (tile - sp.tile0) * RC;
            const int nrows = min(RC, sp.rows - row0);
            unsigned char* dst = ring + stage * r.stage_bytes;
            if (nch == 1) {
                const uint32_t bytes = (uint32_t)((long long)nrows * a.pitch);
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[stage], bytes);
                    bulk_g2s(dst, sp.qs + (long long)row0 * a.pitch, bytes, &full[stage]);
                }
                continue;
            }
            const long long off = (long long)chunk * RS;
            const uint32_t cbytes = (uint32_t)min((long long)RS, a.pitch - off);
            if (lane == 0) mbar_arrive_expect_tx(&full[stage], (uint32_t)nrows * cbytes);
            __syncwarp();
            for (int rr = lane; rr < nrows; rr += 32)
                bulk_g2s(dst + rr * RS, sp.qs + (long long)(row0 + rr) * a.pitch + off, cbytes, &full[stage]);
        }
        return;
    }

    pdl_wait();
    const unsigned int peer_call =
        a.s.peer_mode ? *reinterpret_cast<volatile const unsigned int*>(a.s.peer.calls) + 1u : 0u;
    const int pos = a.s.d_pos ? *a.s.d_pos : 0;
    if (a.s.rope_cs)
        for (int i = threadIdx.x; i < a.s.rope_half; i += kStreamThreads)
            rcs[i] = a.s.rope_cs[(long long)pos * a.s.rope_half + i];

    // X (rms-normalised first when asked), zero past `cols`
    {
        const float nscale = a.s.norm_w ? cta_rms_scale(a.s.x, a.cols, a.s.norm_eps, dscratch) : 1.f;
        const float* xp = a.s.x;
        if (a.s.x_vec) {
            const int n4 = a.cols >> 2;
#pragma unroll 4
            for (int i4 = threadIdx.x; i4 < n4; i4 += kStreamThreads) {
                float4 v = __ldg(reinterpret_cast<const float4*>(xp) + i4);
                if (a.s.norm_w) {
                    const float4 g = __ldg(reinterpret_cast<const float4*>(a.s.norm_w) + i4);
                    v.x = __fmul_rn(__fmul_rn(v.x, nscale), g.x);
                    v.y = __fmul_rn(__fmul_rn(v.y, nscale), g.y);
                    v.z = __fmul_rn(__fmul_rn(v.z, nscale), g.z);
                    v.w = __fmul_rn(__fmul_rn(v.w, nscale), g.w);
                }
                const int i = 4 * i4;
                *reinterpret_cast<float4*>(xs + (i >> 5) * kQ8Pitch + (i & 31)) = v;
            }
            for (int i = 4 * n4 + threadIdx.x; i < nu * 32; i += kStreamThreads) {
                float v = 0.f;
                if (i < a.cols) {
                    v = __ldg(xp + i);
                    if (a.s.norm_w) v = __fmul_rn(__fmul_rn(v, nscale), __ldg(a.s.norm_w + i));
                }
                xs[(i >> 5) * kQ8Pitch + (i & 31)] = v;
            }
        } else {
#pragma unroll 4
            for (int i = threadIdx.x; i < nu * 32; i += kStreamThreads) {
                float v = 0.f;
                if (i < a.cols) {
                    v = __ldg(xp + i);
                    if (a.s.norm_w) v = __fmul_rn(__fmul_rn(v, nscale), __ldg(a.s.norm_w + i));
                }
                xs[(i >> 5) * kQ8Pitch + (i & 31)] = v;
            }
        }
    }
    compute_sync();
    if constexpr (!kFloat && DqCode<TYPE>::HAS_B) {
        // sum of each 32-value sub-block of X, kept in the pitch's spare float
        for (int u = threadIdx.x; u < nu; u += kStreamThreads) {
            float* xu = xs + (long long)u * kQ8Pitch;
            const float4* x4 = reinterpret_cast<const float4*>(xu);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                const float4 p = x4[k], q = x4[k + 1];
                s0 += (p.x + p.y) + (p.z + p.w);
                s1 += (q.x + q.y) + (q.z + q.w);
            }
            xu[32] = s0 + s1;
        }
        compute_sync();
    }
    pdl_launch_dependents();

    float acc[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) acc[i] = 0.f;
    for (int item = 0; item < n_items; ++item) {
        const int stage = item % S;
        const uint32_t parity = (uint32_t)((item / S) & 1);
        const int tile = (int)blockIdx.x + (item / nch) * (int)gridDim.x;
        const int chunk = item % nch;
        const Span& sp = a.s.span[find_span_of(a.s, tile)];
        const int row0 = (tile - sp.tile0) * RC;
        const bool ok = mbar_wait(&full[stage], parity, a.s.err);
        if (compute_sync_or(!ok)) return;
        const unsigned char* st = ring + stage * r.stage_bytes;
        const int k0 = chunk * r.kcb;
        const int nblk_c = min(r.kcb, a.nblk - k0);
        bool valid[RPW];
#pragma unroll
        for (int i = 0; i < RPW; ++i) valid[i] = row0 + warp * RPW + i < sp.rows;
        if constexpr (kFloat) {
            // lanes take the 16-byte words l, l + 32, ... of the chunk: X is
            // then read without bank conflicts
            constexpr int VPW = TYPE == NEON_GGML_F32 ? 4 : 8;  // values per word
            const int words = (nblk_c * D::BB) >> 4;
            for (int wi = lane; wi < words; wi += 32) {
                const int e = k0 * 32 + VPW * wi;
                const float4* x4 = reinterpret_cast<const float4*>(xs + (e >> 5) * kQ8Pitch + (e & 31));
                float xv[VPW];
#pragma unroll
                for (int q = 0; q < VPW / 4; ++q) {
                    const float4 t = x4[q];
                    xv[4 * q] = t.x;
                    xv[4 * q + 1] = t.y;
                    xv[4 * q + 2] = t.z;
                    xv[4 * q + 3] = t.w;
                }
#pragma unroll
                for (int i = 0; i < RPW; ++i) {
                    if (!valid[i]) continue;
                    const uint4 v = *reinterpret_cast<const uint4*>(st + (warp * RPW + i) * RS + 16 * wi);
                    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if constexpr (TYPE == NEON_GGML_F32) {
                            acc[i] = fmaf(__uint_as_float(u[q]), xv[q], acc[i]);
                        } else if constexpr (TYPE == NEON_GGML_F16) {
                            acc[i] = fmaf(__half2float(__ushort_as_half((unsigned short)(u[q] & 0xFFFFu))),
                                          xv[2 * q], acc[i]);
                            acc[i] = fmaf(__half2float(__ushort_as_half((unsigned short)(u[q] >> 16))),
                                          xv[2 * q + 1], acc[i]);
                        } else {
                            acc[i] = fmaf(__uint_as_float(u[q] << 16), xv[2 * q], acc[i]);
                            acc[i] = fmaf(__uint_as_float(u[q] & 0xFFFF0000u), xv[2 * q + 1], acc[i]);
                        }
                    }
                }
            }
        } else {
            for (int u = lane; u < nblk_c * D::SUBS; u += 32) {
                const float* xu = xs + (long long)(k0 * D::SUBS + u) * kQ8Pitch;
                const float xsum = DqCode<TYPE>::HAS_B ? xu[32] : 0.f;
#pragma unroll
                for (int i = 0; i < RPW; ++i) {
                    if (!valid[i]) continue;
                    DqCode<TYPE> c;
                    dq_codes<TYPE>(st + (warp * RPW + i) * RS + (u / D::SUBS) * D::BB, u % D::SUBS, c);
                    acc[i] += dq_code_dot<TYPE>(c, xu, xsum);
                }
            }
        }
        // this warp is done with the stage: release it to the copy warp
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (chunk == nch - 1) {
            const int tb = (item / nch) & 1;
#pragma unroll
            for (int i = 0; i < RPW; ++i) {
#pragma unroll
                for (int o = 16; o; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
                if (lane == 0) rowv[tb][warp * RPW + i] = acc[i];
                acc[i] = 0.f;
            }
            compute_sync();
            float yold = 0.f;
            if (a.s.accumulate && sp.epi == kEpiStore && (int)threadIdx.x < RC && row0 + (int)threadIdx.x < sp.rows)
                yold = sp.y[row0 + threadIdx.x];
            stream_epilogue(a.s, sp, row0, RC, rowv[tb], peer_call, pos, rcs, yold);
        }
    }
}

// h[t] = the values of embedding row tokens[t] (transformer_forward's
// embedding lookup, rawllm_forward.hpp:1023-1033, through dequantize_row).
// One thread per 32-value sub-block; an out-of-range id sets bit 1 of *err
// and reads row 0 (the split-layout embed kernel's rule).
template <int TYPE>
__global__ void __launch_bounds__(128) embed_dq_kernel(const unsigned char* __restrict__ rows, long long pitch,
                                                       int n_embd, const int* __restrict__ tokens, int n_vocab,
                                                       float* __restrict__ h, unsigned int* err) {
    using D = DqShape<TYPE>;
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.y;
    int tok = tokens[t];
    if (tok < 0 || tok >= n_vocab) {
        if (threadIdx.x == 0) atomicOr(err, 2u);
        tok = 0;
    }
    float* out = h + (long long)t * n_embd;
    const int nu = (n_embd + 31) / 32;
    for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < nu; u += gridDim.x * blockDim.x) {
        float w[32];
        dq_sub<TYPE>(rows + (long long)tok * pitch + (u / D::SUBS) * D::BB, u % D::SUBS, w);
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (u * 32 + j < n_embd) out[u * 32 + j] = w[j];
    }
}

// n values of one row of `type` as the host holds it (GGUF layout, any
// alignment) into out, decoded on the host with the device decoders'
// arithmetic: the reference's dequantize_row (rawllm_forward.hpp:301-321)
// bit for bit. For the float types any n; for a block type n whole blocks.
// Returns false for another type or a ragged block row.
inline bool dq_row_host(int type, const unsigned char* p, size_t n, float* out) {
    if (type == NEON_GGML_F32) {
        memcpy(out, p, n * 4);
        return true;
    }
    if (type == NEON_GGML_F16 || type == NEON_GGML_BF16) {
        for (size_t i = 0; i < n; ++i) {
            alignas(4) unsigned char h[2];
            memcpy(h, p + 2 * i, 2);
            out[i] = type == NEON_GGML_F16 ? sh_half(h) : NEON_HD_BITS_F32(sh_u16(h) << 16);
        }
        return true;
    }
    const bool split = type == NEON_GGML_Q8_0 || type == NEON_GGML_Q4_0;
    int be = 32, bb = type == NEON_GGML_Q8_0 ? 34 : 18, cb;
    if (!split) dq_geometry(type, &be, &bb, &cb);
    if (be == 0 || n % (size_t)be != 0) return false;
    alignas(16) unsigned char blk[256];  // the largest block, Q6_K, is 210 bytes
    for (size_t b = 0; b < n / be; ++b) {
        memcpy(blk, p + b * bb, bb);
        float* o = out + b * be;
        if (split) {  // dequant_q8_0 / dequant_q4_0 (:143-162): d * q, exact
            const float d = sh_half(blk);
            for (int i = 0; i < 32; ++i) {
                const int q = type == NEON_GGML_Q8_0 ? (int)(int8_t)blk[2 + i]
                                                     : (int)((blk[2 + (i & 15)] >> (i < 16 ? 0 : 4)) & 15) - 8;
                o[i] = NEON_HD_MUL(d, (float)q);
            }
            continue;
        }
        for (int s = 0; s < be / 32; ++s) {
            float w[32];
            switch (type) {
                case NEON_GGML_Q4_1: dq_sub<NEON_GGML_Q4_1>(blk, s, w); break;
                case NEON_GGML_Q5_0: dq_sub<NEON_GGML_Q5_0>(blk, s, w); break;
                case NEON_GGML_Q5_1: dq_sub<NEON_GGML_Q5_1>(blk, s, w); break;
                case NEON_GGML_Q4_K: dq_sub<NEON_GGML_Q4_K>(blk, s, w); break;
                case NEON_GGML_Q5_K: dq_sub<NEON_GGML_Q5_K>(blk, s, w); break;
                case NEON_GGML_Q6_K: dq_sub<NEON_GGML_Q6_K>(blk, s, w); break;
                default: return false;
            }
            memcpy(o + 32 * s, w, sizeof w);
        }
    }
    return true;
}

}  // namespace neon
