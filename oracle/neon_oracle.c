/*
 * neon_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A plain-C restatement of the NEON runtime's CPU hot path for block-quantized
 * matvecs (reference: rawllm_forward.hpp of NANITY-project/NEON-Runtime-Beta-
 * Variation). It exists only so that the tests, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py can check the CUDA kernels against the
 * reference's arithmetic. Nothing in the shipped library links or calls it.
 *
 * Every function cites the reference file:line it restates. The restatement is
 * pinned bit-for-bit against the reference itself (the same header compiled
 * with the reference's own flags into oracle/_ref/, see oracle/Makefile) by
 * tests/test_oracle_pin.py, and against the committed golden vectors in
 * tests/golden/ by tests/test_oracle_golden.py.
 *
 * Floating-point order is restated exactly as the reference's optimised build
 * (g++ -std=c++17 -O3 -mavx2 -mfma) evaluates it:
 *   - dot_q4_0_q8_0: g++ contracts `total += wd * x_d[b] * (float)isum` into
 *     total = fma(wd * x_d[b], (float)isum, total); restated with fmaf.
 *   - dot_f32 (AVX2 + FMA build): eight lane accumulators, acc[l] = fma(a, b,
 *     acc[l]) over i = l (mod 8), then (acc[l] + acc[l+4]) for l < 4 and two
 *     horizontal adds, i.e. ((s0 + s1) + (s2 + s3)); restated with scalars.
 * Build with -ffp-contract=off so the compiler adds no contraction of its own.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>

#define ORACLE_GGML_Q4_0 2
#define ORACLE_GGML_Q8_0 8

/* Exact IEEE binary16 -> binary32, subnormals included.
 * Restates fp16_to_fp32, rawllm_forward.hpp:94-117. */
float oracle_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t ex = (uint32_t)(h >> 10) & 0x1Fu;
    uint32_t mant = (uint32_t)h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (mant == 0) {
            bits = sign << 31;
        } else {
            /* normalise: shift the mantissa up until the implicit bit appears */
            int shift = 0;
            while (!(mant & 0x400u)) { mant <<= 1; ++shift; }
            mant &= 0x3FFu;
            bits = (sign << 31) | ((uint32_t)(127 - 15 - shift + 1) << 23) | (mant << 13);
        }
    } else if (ex == 31) {
        bits = (sign << 31) | 0x7F800000u | (mant << 13);
    } else {
        bits = (sign << 31) | ((ex - 15 + 127) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

static float rd_fp16(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return oracle_fp16_to_fp32(h);
}

/* Row-wise Q8_0 activation quantisation with fp32 scales.
 * Restates quantize_rows_q8_0, rawllm_forward.hpp:360-381:
 *   amax = max |x|, d = amax / 127, id = d > 0 ? 1 / d : 0,
 *   q = clamp((int)lround(x * id), -127, 127).
 * (int) of the long that lroundf returns keeps its low 32 bits, as the
 * reference's (int)std::lround does. */
void oracle_quantize_rows_q8_0(const float* X, size_t x_stride, size_t cols, size_t seq,
                               float* d_out, int8_t* q_out) {
    size_t nb = cols / 32;
    for (size_t t = 0; t < seq; ++t) {
        const float* x = X + t * x_stride;
        for (size_t b = 0; b < nb; ++b) {
            const float* xb = x + b * 32;
            float amax = 0.f;
            for (int j = 0; j < 32; ++j) {
                float a = fabsf(xb[j]);
                amax = (amax < a) ? a : amax; /* std::max(amax, a) */
            }
            float d = amax / 127.0f;
            float id = d > 0.f ? 1.0f / d : 0.f;
            d_out[t * nb + b] = d;
            for (int j = 0; j < 32; ++j) {
                int v = (int)lroundf(xb[j] * id);
                if (v < -127) v = -127;
                if (v > 127) v = 127;
                q_out[t * cols + b * 32 + j] = (int8_t)v;
            }
        }
    }
}

/* Exact integer dot of one Q4_0 block (16 packed bytes: low nibble -> element
 * j, high nibble -> element j + 16, value = nibble - 8) against 32 int8.
 * Restates block_isum_scalar, rawllm_forward.hpp:384-392 (block_isum_avx2,
 * :394-412, returns the same integer). */
int32_t oracle_block_isum(const uint8_t* qs, const int8_t* xq) {
    int32_t isum = 0;
    for (int j = 0; j < 16; ++j) {
        int lo = (qs[j] & 0x0F) - 8;
        int hi = (qs[j] >> 4) - 8;
        isum += lo * (int)xq[j] + hi * (int)xq[j + 16];
    }
    return isum;
}

/* One GGUF Q4_0 row (18-byte blocks: fp16 d, 16 nibble bytes) against one Q8_0
 * activation row. Restates dot_q4_0_q8_0, rawllm_forward.hpp:419-434, with the
 * FMA contraction of the optimised reference build. */
float oracle_dot_q4_0_q8_0(const uint8_t* w, const float* x_d, const int8_t* x_q, size_t cols) {
    size_t nb = cols / 32;
    float total = 0.f;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = w + b * 18;
        float wd = rd_fp16(blk);
        int32_t isum = oracle_block_isum(blk + 2, x_q + b * 32);
        total = fmaf(wd * x_d[b], (float)isum, total);
    }
    return total;
}

/* Q8_0 block dequantisation (34-byte blocks: fp16 d, 32 int8): out = d * q.
 * Restates dequant_q8_0, rawllm_forward.hpp:143-150. */
void oracle_dequant_q8_0(const uint8_t* p, size_t n, float* out) {
    for (size_t b = 0; b < n; b += 32) {
        float d = rd_fp16(p);
        const int8_t* qs = (const int8_t*)(p + 2);
        for (int j = 0; j < 32; ++j) out[b + j] = d * (float)qs[j];
        p += 34;
    }
}

/* Q4_0 block dequantisation: out[j] = d*(lo-8), out[j+16] = d*(hi-8).
 * Restates dequant_q4_0, rawllm_forward.hpp:152-162. */
void oracle_dequant_q4_0(const uint8_t* p, size_t n, float* out) {
    for (size_t b = 0; b < n; b += 32) {
        float d = rd_fp16(p);
        const uint8_t* qs = p + 2;
        for (int j = 0; j < 16; ++j) {
            out[b + j] = d * ((float)(qs[j] & 0xF) - 8.f);
            out[b + j + 16] = d * ((float)(qs[j] >> 4) - 8.f);
        }
        p += 18;
    }
}

/* fp32 dot product in the AVX2+FMA summation order.
 * Restates dot_f32, rawllm_forward.hpp:446-479 (the RAWLLM_AVX2 branch). */
float oracle_dot_f32(const float* a, const float* b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s0 = acc[0] + acc[4], s1 = acc[1] + acc[5];
    float s2 = acc[2] + acc[6], s3 = acc[3] + acc[7];
    float sum = (s0 + s1) + (s2 + s3);
    for (; i < n; ++i) sum += a[i] * b[i];
    return sum;
}

/* Bytes per row of a GGUF tensor. Restates nbytes_for, rawllm_loader.hpp:367-386
 * (Q4_0 and Q8_0 rows only). Returns 0 for other types. */
size_t oracle_row_bytes(int type, size_t cols) {
    if (type == ORACLE_GGML_Q4_0) return cols / 32 * 18;
    if (type == ORACLE_GGML_Q8_0) return cols / 32 * 34;
    return 0;
}

/* Y[t*y_stride + r] = W_r . X_t for r < rows, t < seq, single-threaded.
 * Restates proj_all_positions, rawllm_forward.hpp:522-609: Q4_0 weights take
 * the fused path (X quantised to Q8_0 once, then dot_q4_0_q8_0 per row);
 * Q8_0 weights take dequant_q8_0 + dot_f32 against fp32 X.
 * `scratch` must hold seq*cols/32 floats + seq*cols bytes (Q4_0 only) and
 * `rowbuf` cols floats (Q8_0 only). Returns 0, or -1 on a bad argument
 * (cols not a multiple of 32, unsupported type), where the reference throws. */
int oracle_proj_all_positions(int type, const uint8_t* W, size_t rows, size_t cols,
                              const float* X, size_t x_stride, float* Y, size_t y_stride,
                              size_t seq, float* scratch_d, int8_t* scratch_q, float* rowbuf) {
    if (cols % 32 != 0) return -1;
    size_t row_bytes = oracle_row_bytes(type, cols);
    if (row_bytes == 0) return -1;
    size_t nb = cols / 32;
    if (type == ORACLE_GGML_Q4_0) {
        oracle_quantize_rows_q8_0(X, x_stride, cols, seq, scratch_d, scratch_q);
        for (size_t r = 0; r < rows; ++r)
            for (size_t t = 0; t < seq; ++t)
                Y[t * y_stride + r] = oracle_dot_q4_0_q8_0(W + r * row_bytes, scratch_d + t * nb,
                                                           scratch_q + t * cols, cols);
        return 0;
    }
    for (size_t r = 0; r < rows; ++r) {
        oracle_dequant_q8_0(W + r * row_bytes, cols, rowbuf);
        for (size_t t = 0; t < seq; ++t)
            Y[t * y_stride + r] = oracle_dot_f32(rowbuf, X + t * x_stride, cols);
    }
    return 0;
}
