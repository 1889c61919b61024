// neon_quant.cuh -- on-load weight quantisation on the device: rows of F32,
// F16 or BF16 values to GGUF blocks (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1) or to
// F16 / BF16.
//
// The reference's runtime never quantises weights; its exporters do, through
// gguf-py (third-party, version 0.19.0 here): export_gguf
// (train_nanity_fixed.py:1162-1169) and nanity_convert.py's quantize_tensor
// (:472-484) both call gguf.quants.quantize, and a .nctr file holds F32
// tensors only (export_nctr, train_nanity_fixed.py:1259-1433). Quantising a
// float tensor at load time with the same published algorithms gives, byte
// for byte, the tensor those exporters would have written with --quant
// Q8_0 / Q4_0 / ... (gguf/quants.py, quantize_blocks of each type):
//   Q8_0  d = amax/127, id = d ? 1/d : 0, q = round-half-away(x*id)
//   Q4_0  m = the value of largest |x| (first such), d = m/-8, id as above,
//         q = clamp(trunc(x*id + 8.5), 0, 15)
//   Q5_0  as Q4_0 with d = m/-16, q = clamp(trunc(x*id + 16.5), 0, 31)
//   Q4_1  d = (max - min)/15, q = clamp(trunc((x - min)*id + 0.5), 0, 15), m = min
//   Q5_1  as Q4_1 with /31 and clamp 31
// all in fp32 with one rounding per operation (numpy float32 arithmetic), the
// scales stored as fp16 rounded to nearest even; F16 is numpy's cast, BF16
// ggml's round-to-nearest-even with NaNs quieted. Inputs are finite (numpy's
// max/argmax treat NaN differently from IEEE max; a weight tensor with NaNs
// has no meaningful quantisation).
//
// The block quantisers are __host__ __device__: the CPU tests run the host
// build against gguf-py's own output.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "neon_cuda.h"

namespace neon {

#ifdef __CUDA_ARCH__
#define NEON_Q_MUL(a, b) __fmul_rn((a), (b))
#define NEON_Q_ADD(a, b) __fadd_rn((a), (b))
#define NEON_Q_SUB(a, b) __fsub_rn((a), (b))
#define NEON_Q_DIV(a, b) __fdiv_rn((a), (b))
#else
#define NEON_Q_MUL(a, b) ((a) * (b))
#define NEON_Q_ADD(a, b) ((a) + (b))
#define NEON_Q_SUB(a, b) ((a) - (b))
#define NEON_Q_DIV(a, b) ((a) / (b))
#endif

// The bits of a float.
__host__ __device__ inline uint32_t q_bits(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t x;
    memcpy(&x, &f, 4);
    return x;
#endif
}

// fp32 -> binary16 bits, round to nearest even (numpy's cast): overflow to
// infinity from 65520 up, subnormals below 2^-14, zero below 2^-25 (2^-25
// itself ties to even, to zero); a NaN keeps its top payload bits, quieted.
// Integer arithmetic only, the same on host and device.
__host__ __device__ inline uint16_t q_f16_bits(float f) {
    const uint32_t x = q_bits(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u)
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u | ((ax >> 13) & 0x3FFu) : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (ax >= 0x38800000u) {
        // normal: rebias the exponent (127 -> 15) and round off 13 mantissa bits
        const uint32_t r = ax - 0x38000000u;
        return (uint16_t)(sign | ((r + 0x0FFFu + ((r >> 13) & 1u)) >> 13));
    }
    if (ax < 0x33000000u) return (uint16_t)sign;
    // subnormal: the value in units of 2^-24, rounded to nearest even
    const uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e;  // 14..24
    const uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    return (uint16_t)(sign | (q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u)));
}

// Little-endian stores of 16 / 32 bits at any byte address.
__host__ __device__ inline void q_put_u16(unsigned char* p, uint32_t v) {
    p[0] = (unsigned char)(v & 0xFFu);
    p[1] = (unsigned char)((v >> 8) & 0xFFu);
}
__host__ __device__ inline void q_put_u32(unsigned char* p, uint32_t v) {
    q_put_u16(p, v & 0xFFFFu);
    q_put_u16(p + 2, v >> 16);
}

// ggml's fp32 -> bf16: quiet a NaN, else round to nearest even on the bits.
__host__ __device__ inline uint16_t q_bf16_bits(float v) {
    const uint32_t n = q_bits(v);
    if ((n & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(((n & 0xffff0000u) | (64u << 16)) >> 16);
    return (uint16_t)(((uint64_t)n + (0x7fffu + ((n >> 16) & 1u))) >> 16);
}

// Value i of a row of a float type (F32, F16, BF16); rows start on an
// element boundary (the device buffers are cudaMalloc'd, rows of whole elements).
__host__ __device__ inline float q_src_value(const unsigned char* row, int src_type, long long i) {
#ifdef __CUDA_ARCH__
    if (src_type == NEON_GGML_F32) return reinterpret_cast<const float*>(row)[i];
    const unsigned short h = reinterpret_cast<const unsigned short*>(row)[i];
    if (src_type == NEON_GGML_F16) return __half2float(__ushort_as_half(h));
    return __uint_as_float((uint32_t)h << 16);
#else
    if (src_type == NEON_GGML_F32) {
        float v;
        memcpy(&v, row + 4 * i, 4);
        return v;
    }
    uint16_t h;
    memcpy(&h, row + 2 * i, 2);
    if (src_type == NEON_GGML_F16) return __half2float(__ushort_as_half(h));
    const uint32_t u = (uint32_t)h << 16;
    float v;
    memcpy(&v, &u, 4);
    return v;
#endif
}

__host__ __device__ inline int q_trunc_clamp(float v, int hi) {
    int q = (int)truncf(v);
    return q < 0 ? 0 : (q > hi ? hi : q);
}

__host__ __device__ inline void q_put_f16(unsigned char* p, float v) { q_put_u16(p, q_f16_bits(v)); }

// One block of 32 values -> the GGUF block of `dst` (18 / 20 / 22 / 24 / 34
// bytes). Returns false for a type this quantiser does not produce.
__host__ __device__ inline bool q_quantize_block(const float* x, int dst, unsigned char* out) {
    if (dst == NEON_GGML_Q8_0) {
        float amax = 0.f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
        const float d = NEON_Q_DIV(amax, 127.f);
        const float id = d == 0.f ? 0.f : NEON_Q_DIV(1.f, d);
        q_put_f16(out, d);
        for (int j = 0; j < 32; ++j) {
            const int q = (int)roundf(NEON_Q_MUL(x[j], id));  // half away from zero, as np_roundf
            out[2 + j] = (unsigned char)(signed char)q;
        }
        return true;
    }
    if (dst == NEON_GGML_Q4_0 || dst == NEON_GGML_Q5_0) {
        const bool five = dst == NEON_GGML_Q5_0;
        int imax = 0;
        float amax = fabsf(x[0]);
        for (int j = 1; j < 32; ++j)
            if (fabsf(x[j]) > amax) {
                amax = fabsf(x[j]);
                imax = j;
            }
        const float d = NEON_Q_DIV(x[imax], five ? -16.f : -8.f);
        const float id = d == 0.f ? 0.f : NEON_Q_DIV(1.f, d);
        int q[32];
        for (int j = 0; j < 32; ++j)
            q[j] = q_trunc_clamp(NEON_Q_ADD(NEON_Q_MUL(x[j], id), five ? 16.5f : 8.5f), five ? 31 : 15);
        q_put_f16(out, d);
        unsigned char* qs = out + (five ? 6 : 2);
        uint32_t qh = 0;
        for (int j = 0; j < 16; ++j) qs[j] = (unsigned char)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
        if (five) {
            for (int j = 0; j < 32; ++j) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
            q_put_u32(out + 2, qh);
        }
        return true;
    }
    if (dst == NEON_GGML_Q4_1 || dst == NEON_GGML_Q5_1) {
        const bool five = dst == NEON_GGML_Q5_1;
        float mx = x[0], mn = x[0];
        for (int j = 1; j < 32; ++j) {
            mx = fmaxf(mx, x[j]);
            mn = fminf(mn, x[j]);
        }
        const float d = NEON_Q_DIV(NEON_Q_SUB(mx, mn), five ? 31.f : 15.f);
        const float id = d == 0.f ? 0.f : NEON_Q_DIV(1.f, d);
        int q[32];
        for (int j = 0; j < 32; ++j)
            q[j] = q_trunc_clamp(NEON_Q_ADD(NEON_Q_MUL(NEON_Q_SUB(x[j], mn), id), 0.5f), five ? 31 : 15);
        q_put_f16(out, d);
        q_put_f16(out + 2, mn);
        unsigned char* qs = out + (five ? 8 : 4);
        for (int j = 0; j < 16; ++j) qs[j] = (unsigned char)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
        if (five) {
            uint32_t qh = 0;
            for (int j = 0; j < 32; ++j) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
            q_put_u32(out + 4, qh);
        }
        return true;
    }
    return false;
}

// Bytes of one quantised block (0 for another type).
__host__ __device__ constexpr int q_block_bytes(int dst) {
    return dst == NEON_GGML_Q8_0 ? 34
           : dst == NEON_GGML_Q4_0 ? 18
           : dst == NEON_GGML_Q4_1 ? 20
           : dst == NEON_GGML_Q5_0 ? 22
           : dst == NEON_GGML_Q5_1 ? 24
                                   : 0;
}

// rows x cols float values (src_row bytes per row) -> GGUF rows of `dst`
// (dst_row bytes per row). Block types: one thread per 32-value block;
// F16 / BF16: one thread per value.
__global__ void quantize_rows_kernel(const unsigned char* __restrict__ src, long long src_row, int src_type,
                                     long long rows, long long cols, int dst, unsigned char* __restrict__ out,
                                     long long dst_row) {
    const bool block = q_block_bytes(dst) != 0;
    const long long per_row = block ? cols / 32 : cols;
    const long long n = rows * per_row;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / per_row, b = i % per_row;
        const unsigned char* row = src + r * src_row;
        unsigned char* orow = out + r * dst_row;
        if (block) {
            float x[32];
            for (int j = 0; j < 32; ++j) x[j] = q_src_value(row, src_type, 32 * b + j);
            q_quantize_block(x, dst, orow + b * q_block_bytes(dst));
        } else {
            const float v = q_src_value(row, src_type, b);
            q_put_u16(orow + 2 * b, dst == NEON_GGML_F16 ? q_f16_bits(v) : q_bf16_bits(v));
        }
    }
}

}  // namespace neon
