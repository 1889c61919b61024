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
 * The row loops run under OpenMP when built with -fopenmp: rows are
 * independent, so the results do not depend on the thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>

#define ORACLE_GGML_F32 0
#define ORACLE_GGML_F16 1
#define ORACLE_GGML_Q4_0 2
#define ORACLE_GGML_Q4_1 3
#define ORACLE_GGML_Q5_0 6
#define ORACLE_GGML_Q5_1 7
#define ORACLE_GGML_Q8_0 8
#define ORACLE_GGML_Q4_K 12
#define ORACLE_GGML_Q5_K 13
#define ORACLE_GGML_Q6_K 14
#define ORACLE_GGML_BF16 30

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
/* Test switch: when nonzero, dot_q4_0_q8_0 sums its blocks in reverse order.
 * A legitimate fp32 reordering, used only by tests/test_oracle_decode.py to
 * measure how far a mere summation-order change moves whole-model logits. */
int oracle_reverse_block_order = 0;

float oracle_dot_q4_0_q8_0(const uint8_t* w, const float* x_d, const int8_t* x_q, size_t cols) {
    size_t nb = cols / 32;
    float total = 0.f;
    for (size_t bb = 0; bb < nb; ++bb) {
        size_t b = oracle_reverse_block_order ? nb - 1 - bb : bb;
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

size_t oracle_block_elems(int type);
static size_t block_bytes(int type);

/* bfloat16 -> fp32: the 16 bits become the high half. Restates bf16_to_fp32,
 * rawllm_forward.hpp:119-123. */
float oracle_bf16_to_fp32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* The six-bit (scale, min) pair of sub-block s (0..7) of a Q4_K / Q5_K
 * super-block, from its 12 packed bytes: sub-blocks 0-3 keep their pair in
 * the low six bits of bytes s and s+4; sub-blocks 4-7 take four bits from
 * byte s+4 and their top two bits from the spare high bits of bytes s-4 (scale)
 * and s (min). Restates get_scale_min_k4, rawllm_forward.hpp:224-233. */
static void k4_scale_min(const uint8_t* sc, int s, int* scale, int* min) {
    if (s < 4) {
        *scale = sc[s] & 63;
        *min = sc[s + 4] & 63;
    } else {
        *scale = (sc[s + 4] & 0x0F) | ((sc[s - 4] >> 6) << 4);
        *min = (sc[s + 4] >> 4) | ((sc[s] >> 6) << 4);
    }
}

/* The 32 values of sub-block s of one block of `type` (s = 0 for the 32-value
 * types; 0..7 for the 256-value K-quant super-blocks). Each restates the
 * matching dequantiser of rawllm_forward.hpp, regrouped by sub-block:
 *   Q4_1 :164-175  v = d*q + m,          q = nibble (low: j, high: j+16)
 *   Q5_0 :177-191  v = d*(q - 16),       q = nibble | bit j (or j+16) of qh << 4
 *   Q5_1 :193-208  v = d*q + m,          q as Q5_0
 *   Q4_K :235-253  v = (d*sc)*q - dmin*mn, sub-block s: bytes 32*(s/2).., nibble s&1
 *   Q5_K :255-275  as Q4_K with q += 16 * bit s of qh[l]
 *   Q6_K :277-298  v = (d*sc)*(q - 32), q = nibble | 2-bit pair << 4; sub-block
 *                  s = 4h + k takes low-nibble bytes 64h + 32(k&1).., the high
 *                  nibble when k >= 2, pair k of qh[32h + l], scales 8h + l/16 + 2k
 * Every product d*q here is exact in fp32 (at most 23 significant bits), so
 * evaluating with or without fused multiply-adds gives the same values. */
static void sub_block(int type, const uint8_t* blk, int s, float* out) {
    switch (type) {
        case ORACLE_GGML_Q4_1: {
            const float d = rd_fp16(blk), m = rd_fp16(blk + 2);
            for (int j = 0; j < 16; ++j) {
                out[j] = d * (float)(blk[4 + j] & 0x0F) + m;
                out[j + 16] = d * (float)(blk[4 + j] >> 4) + m;
            }
            return;
        }
        case ORACLE_GGML_Q5_0:
        case ORACLE_GGML_Q5_1: {
            const int has_m = type == ORACLE_GGML_Q5_1;
            const float d = rd_fp16(blk), m = has_m ? rd_fp16(blk + 2) : 0.f;
            uint32_t qh;
            memcpy(&qh, blk + (has_m ? 4 : 2), 4);
            const uint8_t* qs = blk + (has_m ? 8 : 6);
            for (int j = 0; j < 16; ++j) {
                int lo = (qs[j] & 0x0F) | (int)(((qh >> j) & 1u) << 4);
                int hi = (qs[j] >> 4) | (int)(((qh >> (j + 16)) & 1u) << 4);
                if (has_m) {
                    out[j] = d * (float)lo + m;
                    out[j + 16] = d * (float)hi + m;
                } else {
                    out[j] = d * (float)(lo - 16);
                    out[j + 16] = d * (float)(hi - 16);
                }
            }
            return;
        }
        case ORACLE_GGML_Q4_K:
        case ORACLE_GGML_Q5_K: {
            const int five = type == ORACLE_GGML_Q5_K;
            const float d = rd_fp16(blk), dmin = rd_fp16(blk + 2);
            int sc, mn;
            k4_scale_min(blk + 4, s, &sc, &mn);
            const float ds = d * (float)sc, ms = dmin * (float)mn;
            const uint8_t* qh = blk + 16;
            const uint8_t* q = blk + (five ? 48 : 16) + 32 * (s / 2);
            for (int l = 0; l < 32; ++l) {
                int v = (s & 1) ? (q[l] >> 4) : (q[l] & 0x0F);
                if (five && ((qh[l] >> s) & 1)) v += 16;
                out[l] = ds * (float)v - ms;
            }
            return;
        }
        case ORACLE_GGML_Q6_K: {
            const int h = s / 4, k = s % 4;
            const uint8_t* ql = blk + 64 * h + 32 * (k & 1);
            const uint8_t* qh = blk + 128 + 32 * h;
            const int8_t* sc = (const int8_t*)(blk + 192) + 8 * h + 2 * k;
            const float d = rd_fp16(blk + 208);
            for (int l = 0; l < 32; ++l) {
                int lo = k >= 2 ? (ql[l] >> 4) : (ql[l] & 0x0F);
                int q = (lo | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
                out[l] = d * (float)sc[l / 16] * (float)q;
            }
            return;
        }
        default:
            return;
    }
}

/* n values of a row of `type` into out (n whole blocks of the type).
 * Restates dequantize_row, rawllm_forward.hpp:301-321, and the dequantisers it
 * dispatches to (:133-298). Returns -1 for a type the reference does not
 * dequantise there. */
int oracle_dequantize_row(int type, const uint8_t* p, size_t n, float* out) {
    size_t be = oracle_block_elems(type), bb = block_bytes(type);
    if (be == 0) return -1;
    switch (type) {
        case ORACLE_GGML_F32:
            memcpy(out, p, n * 4);
            return 0;
        case ORACLE_GGML_F16:
        case ORACLE_GGML_BF16:
            for (size_t i = 0; i < n; ++i) {
                uint16_t h;
                memcpy(&h, p + 2 * i, 2);
                out[i] = type == ORACLE_GGML_F16 ? oracle_fp16_to_fp32(h) : oracle_bf16_to_fp32(h);
            }
            return 0;
        case ORACLE_GGML_Q8_0: oracle_dequant_q8_0(p, n, out); return 0;
        case ORACLE_GGML_Q4_0: oracle_dequant_q4_0(p, n, out); return 0;
        default:
            for (size_t b = 0; b < n / be; ++b)
                for (int s = 0; s < (int)(be / 32); ++s) sub_block(type, p + b * bb, s, out + b * be + 32 * s);
            return 0;
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
    /* the scalar tail (n not a multiple of 8: plain float rows only), as g++
     * -O3 compiles `sum += a[i] * b[i]`: with four or more left, four products
     * are formed as one vector multiply and added in order; the rest are
     * contracted into FMAs */
    if (n - i >= 4) {
        for (int k = 0; k < 4; ++k, ++i) {
            const float p = a[i] * b[i];
            sum += p;
        }
    }
    for (; i < n; ++i) sum = fmaf(a[i], b[i], sum);
    return sum;
}

/* Elements per block of a weight type: 256 for the K-quants, 1 for the plain
 * float types, 32 for the rest. Restates block_size_for,
 * rawllm_forward.hpp:289-299. Returns 0 for a type the matvec path does not
 * dequantise (rawllm_forward.hpp:301-321 throws for those). */
size_t oracle_block_elems(int type) {
    switch (type) {
        case ORACLE_GGML_F32: case ORACLE_GGML_F16: case ORACLE_GGML_BF16: return 1;
        case ORACLE_GGML_Q4_0: case ORACLE_GGML_Q4_1: case ORACLE_GGML_Q5_0:
        case ORACLE_GGML_Q5_1: case ORACLE_GGML_Q8_0: return 32;
        case ORACLE_GGML_Q4_K: case ORACLE_GGML_Q5_K: case ORACLE_GGML_Q6_K: return 256;
        default: return 0;
    }
}

/* Bytes of one block of a weight type (the GGUF block structs' sizes).
 * Restates nbytes_for, rawllm_loader.hpp:367-386. */
static size_t block_bytes(int type) {
    switch (type) {
        case ORACLE_GGML_F32: return 4;
        case ORACLE_GGML_F16: case ORACLE_GGML_BF16: return 2;
        case ORACLE_GGML_Q4_0: return 18;   /* d, 16 nibble bytes */
        case ORACLE_GGML_Q4_1: return 20;   /* d, m, 16 nibble bytes */
        case ORACLE_GGML_Q5_0: return 22;   /* d, 4 high-bit bytes, 16 nibble bytes */
        case ORACLE_GGML_Q5_1: return 24;   /* d, m, 4 high-bit bytes, 16 nibble bytes */
        case ORACLE_GGML_Q8_0: return 34;   /* d, 32 int8 */
        case ORACLE_GGML_Q4_K: return 144;  /* d, dmin, 12 scale bytes, 128 nibble bytes */
        case ORACLE_GGML_Q5_K: return 176;  /* d, dmin, 12 scale bytes, 32 high-bit bytes, 128 nibble bytes */
        case ORACLE_GGML_Q6_K: return 210;  /* 128 low-nibble bytes, 64 high-pair bytes, 16 int8 scales, d */
        default: return 0;
    }
}

/* Bytes per row of a GGUF tensor (0 for an unsupported type or a row that is
 * not whole blocks). Restates nbytes_for, rawllm_loader.hpp:367-386. */
size_t oracle_row_bytes(int type, size_t cols) {
    size_t be = oracle_block_elems(type);
    if (be == 0 || cols % be != 0) return 0;
    return cols / be * block_bytes(type);
}

/* Y[t*y_stride + r] = W_r . X_t for r < rows, t < seq.
 * Restates proj_all_positions, rawllm_forward.hpp:522-609: Q4_0 weights take
 * the fused path (X quantised to Q8_0 once, then dot_q4_0_q8_0 per row);
 * every other type is dequantised a row at a time (dequantize_row) and dotted
 * with fp32 X (dot_f32).
 * `scratch_d`/`scratch_q` must hold seq*cols/32 floats and seq*cols bytes
 * (Q4_0 only); `rowbuf` is unused (each worker allocates its own row).
 * Returns 0, or -1 on a bad argument (cols not a multiple of the type's block
 * size, a type the reference cannot dequantise), where the reference throws. */
int oracle_proj_all_positions(int type, const uint8_t* W, size_t rows, size_t cols,
                              const float* X, size_t x_stride, float* Y, size_t y_stride,
                              size_t seq, float* scratch_d, int8_t* scratch_q, float* rowbuf) {
    size_t row_bytes = oracle_row_bytes(type, cols);
    if (row_bytes == 0) return -1;
    size_t nb = cols / 32;
    if (type == ORACLE_GGML_Q4_0) {
        oracle_quantize_rows_q8_0(X, x_stride, cols, seq, scratch_d, scratch_q);
#pragma omp parallel for schedule(static)
        for (size_t r = 0; r < rows; ++r)
            for (size_t t = 0; t < seq; ++t)
                Y[t * y_stride + r] = oracle_dot_q4_0_q8_0(W + r * row_bytes, scratch_d + t * nb,
                                                           scratch_q + t * cols, cols);
        return 0;
    }
    (void)rowbuf;
#pragma omp parallel
    {
        float* rb = (float*)malloc(sizeof(float) * cols);
#pragma omp for schedule(static)
        for (size_t r = 0; r < rows; ++r) {
            oracle_dequantize_row(type, W + r * row_bytes, cols, rb);
            for (size_t t = 0; t < seq; ++t)
                Y[t * y_stride + r] = oracle_dot_f32(rb, X + t * x_stride, cols);
        }
        free(rb);
    }
    return 0;
}

/* ======================================================================== */
/* Decode step: restatement of fwd::transformer_forward                      */
/* (rawllm_forward.hpp:987-1236) and the pieces it calls.                    */
/* ======================================================================== */
#include <stdlib.h>

/* Schraudolph exp approximation with the reference's constants; g++ contracts
 * kA * x + kB into one FMA. Restates engine::fast_expf, rawllm_common.hpp:88-100. */
float oracle_fast_expf(float x) {
    if (x < -88.f || x > 88.f) return expf(x);
    const float kA = 12102203.9f;
    const float kB = 1064872507.f;
    int32_t i = (int32_t)fmaf(kA, x, kB);
    float f;
    memcpy(&f, &i, 4);
    return f;
}

/* x / (1 + fast_expf(-x)). Restates fwd::silu, rawllm_forward.hpp:740. */
float oracle_silu(float x) { return x / (1.0f + oracle_fast_expf(-x)); }

/* RMSNorm with a double accumulator (contracted into FMAs by g++).
 * Restates fwd::rms_norm, rawllm_forward.hpp:730-735. */
void oracle_rms_norm(const float* x, const float* w, float* out, size_t n, float eps) {
    double ss = 0.0;
    for (size_t i = 0; i < n; ++i) ss = fma((double)x[i], (double)x[i], ss);
    float scale = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* freqs[i] = base^(-2i/head_dim). Restates fwd::rope_make_freqs, :755-761. */
void oracle_rope_freqs(size_t head_dim, float base, float* out) {
    for (size_t i = 0; i < head_dim / 2; ++i) out[i] = powf(base, -2.0f * (float)i / (float)head_dim);
}

/* Adjacent-pair rotation of every head at position pos.
 * Restates fwd::rope_apply, rawllm_forward.hpp:767-782, with g++'s
 * contraction of x0*c - x1*s and x0*s + x1*c. */
void oracle_rope_apply(float* vec, size_t n_heads, size_t head_dim, size_t rope_half, size_t pos,
                       float rope_scale, const float* freqs) {
    float fpos = (float)pos / rope_scale;
    for (size_t h = 0; h < n_heads; ++h) {
        float* v = vec + h * head_dim;
        for (size_t i = 0; i < rope_half; ++i) {
            float theta = fpos * freqs[i];
            float c = cosf(theta), s = sinf(theta);
            float x0 = v[2 * i], x1 = v[2 * i + 1];
            v[2 * i] = fmaf(x0, c, -(x1 * s));
            v[2 * i + 1] = fmaf(x0, s, x1 * c);
        }
    }
}

/* out[i] += w * v[i] as one FMA per element (AVX2+FMA build).
 * Restates fwd::axpy_f32, rawllm_forward.hpp:485-503. */
void oracle_axpy_f32(float* out, float w, const float* v, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = fmaf(w, v[i], out[i]);
}

enum { R_TOKEN_EMBD = 0, R_OUTPUT_NORM, R_OUTPUT, R_ATTN_NORM, R_ATTN_Q, R_ATTN_K, R_ATTN_V, R_ATTN_OUT,
       R_FFN_NORM, R_FFN_GATE, R_FFN_UP, R_FFN_DOWN };
#define ORACLE_LAYER_ROLES 9 /* R_ATTN_NORM .. R_FFN_DOWN */

typedef struct {
    uint32_t n_vocab, n_embd, n_layer, n_head, n_kv_head, head_dim, n_ff, ctx_len;
    float rope_base, rope_scale;
    uint32_t rope_dim_count;
    float norm_eps;
    uint32_t plain_ffn; /* 1: act = silu(up), no gate (engine::Config::use_swiglu == false) */
} oracle_config_t;

typedef struct {
    uint8_t* data; /* owned copy, NULL if absent */
    int type;
    size_t ne0, ne1;
} oracle_tensor_t;

typedef struct {
    oracle_config_t cfg;
    oracle_tensor_t global[3];  /* token_embd, output_norm, output */
    oracle_tensor_t* layers;    /* n_layer * 9 */
    float *K, *V;               /* [layer][ctx_len][kv_dim] */
    size_t length;
} oracle_model_t;

void* oracle_model_new(const oracle_config_t* cfg) {
    oracle_model_t* m = (oracle_model_t*)calloc(1, sizeof(oracle_model_t));
    m->cfg = *cfg;
    m->layers = (oracle_tensor_t*)calloc((size_t)cfg->n_layer * ORACLE_LAYER_ROLES, sizeof(oracle_tensor_t));
    size_t kv = (size_t)cfg->n_layer * cfg->ctx_len * cfg->n_kv_head * cfg->head_dim;
    m->K = (float*)calloc(kv, sizeof(float));
    m->V = (float*)calloc(kv, sizeof(float));
    return m;
}

void oracle_model_free(void* p) {
    oracle_model_t* m = (oracle_model_t*)p;
    for (int i = 0; i < 3; ++i) free(m->global[i].data);
    for (size_t i = 0; i < (size_t)m->cfg.n_layer * ORACLE_LAYER_ROLES; ++i) free(m->layers[i].data);
    free(m->layers);
    free(m->K);
    free(m->V);
    free(m);
}

int oracle_model_set(void* p, int role, int layer, const uint8_t* bytes, size_t nbytes, int type, size_t ne0,
                     size_t ne1) {
    oracle_model_t* m = (oracle_model_t*)p;
    oracle_tensor_t* t;
    if (role <= R_OUTPUT) {
        t = &m->global[role];
    } else {
        if (layer < 0 || (uint32_t)layer >= m->cfg.n_layer || role > R_FFN_DOWN) return -1;
        t = &m->layers[(size_t)layer * ORACLE_LAYER_ROLES + (role - R_ATTN_NORM)];
    }
    free(t->data);
    if ((role == R_OUTPUT_NORM || role == R_ATTN_NORM || role == R_FFN_NORM) && type != ORACLE_GGML_F32) {
        /* norm weights go through dequant_full (rawllm_forward.hpp:325-328,
         * at :1077, :1161, :1226): any dequantisable type, read as F32 */
        t->data = (uint8_t*)malloc(ne0 * sizeof(float) + 1);
        if (oracle_row_bytes(type, ne0) == 0 || oracle_row_bytes(type, ne0) > nbytes ||
            oracle_dequantize_row(type, bytes, ne0, (float*)t->data) != 0) {
            free(t->data);
            t->data = NULL;
            return -1;
        }
        t->type = ORACLE_GGML_F32;
        t->ne0 = ne0;
        t->ne1 = ne1;
        return 0;
    }
    t->data = (uint8_t*)malloc(nbytes ? nbytes : 1);
    memcpy(t->data, bytes, nbytes);
    t->type = type;
    t->ne0 = ne0;
    t->ne1 = ne1;
    return 0;
}

size_t oracle_model_length(void* p) { return ((oracle_model_t*)p)->length; }

/* fwd::kv_cache_shift (rawllm_forward.hpp:949-969): K rows [keep+discard,
 * length) are rotated by -discard positions (rope_rotate_by_delta, :794-809,
 * cos/sin from libm, g++'s contraction as in rope_apply), then K and V rows
 * move down by `discard`; length shrinks by `discard`. */
void oracle_model_kv_shift(void* p, size_t keep, size_t discard) {
    oracle_model_t* m = (oracle_model_t*)p;
    const oracle_config_t* c = &m->cfg;
    if (discard == 0 || m->length <= keep + discard) return;
    const size_t hd = c->head_dim, n_kv = c->n_kv_head, kv_dim = n_kv * hd;
    const size_t rope_half = c->rope_dim_count ? c->rope_dim_count / 2 : hd / 2;
    const size_t tail = m->length - keep - discard;
    float* freqs = (float*)malloc(sizeof(float) * (hd / 2 + 1));
    oracle_rope_freqs(hd, c->rope_base, freqs);
    const float fdelta = -(float)discard / c->rope_scale;
    for (size_t li = 0; li < c->n_layer; ++li) {
        float* K = m->K + li * c->ctx_len * kv_dim;
        float* V = m->V + li * c->ctx_len * kv_dim;
        for (size_t t = 0; t < tail; ++t) {
            float* row = K + (keep + discard + t) * kv_dim;
            for (size_t h = 0; h < n_kv; ++h) {
                float* v = row + h * hd;
                for (size_t i = 0; i < rope_half; ++i) {
                    float theta = fdelta * freqs[i];
                    float cs = cosf(theta), sn = sinf(theta);
                    float x0 = v[2 * i], x1 = v[2 * i + 1];
                    v[2 * i] = fmaf(x0, cs, -(x1 * sn));
                    v[2 * i + 1] = fmaf(x0, sn, x1 * cs);
                }
            }
        }
        memmove(K + keep * kv_dim, K + (keep + discard) * kv_dim, tail * kv_dim * sizeof(float));
        memmove(V + keep * kv_dim, V + (keep + discard) * kv_dim, tail * kv_dim * sizeof(float));
    }
    m->length = keep + tail;
    free(freqs);
}
void oracle_model_set_length(void* p, size_t n) { ((oracle_model_t*)p)->length = n; }

static const oracle_tensor_t* L_(const oracle_model_t* m, uint32_t li, int role) {
    return &m->layers[(size_t)li * ORACLE_LAYER_ROLES + (role - R_ATTN_NORM)];
}

/* Y (seq x y_stride) = proj of X (seq x x_stride) through a 2-D tensor. */
static int proj(const oracle_tensor_t* W, const float* X, size_t x_stride, float* Y, size_t y_stride, size_t seq) {
    size_t cols = W->ne0, rows = W->ne1;
    float* sd = (float*)malloc(sizeof(float) * (seq * cols / 32 + 1));
    int8_t* sq = (int8_t*)malloc(seq * cols + 1);
    float* rb = (float*)malloc(sizeof(float) * (cols + 1));
    int rc = oracle_proj_all_positions(W->type, W->data, rows, cols, X, x_stride, Y, y_stride, seq, sd, sq, rb);
    free(sd);
    free(sq);
    free(rb);
    return rc;
}

/* fwd::transformer_forward (rawllm_forward.hpp:987-1236): appends `n` new
 * tokens to the KV cache and writes the logits of the last one. */
int oracle_model_forward(void* p, const int32_t* tokens, size_t seq, float* out_logits) {
    oracle_model_t* m = (oracle_model_t*)p;
    const oracle_config_t* c = &m->cfg;
    const size_t n_embd = c->n_embd, n_head = c->n_head, n_kv = c->n_kv_head, hd = c->head_dim, n_ff = c->n_ff;
    const size_t kv_dim = n_kv * hd, q_dim = n_head * hd, base = m->length;
    if (seq == 0 || base + seq > c->ctx_len) return -1;
    const size_t rope_half = c->rope_dim_count ? c->rope_dim_count / 2 : hd / 2;
    float* freqs = (float*)malloc(sizeof(float) * (hd / 2 + 1));
    oracle_rope_freqs(hd, c->rope_base, freqs);

    float* h = (float*)malloc(sizeof(float) * seq * n_embd);
    const oracle_tensor_t* te = &m->global[R_TOKEN_EMBD];
    size_t te_row = oracle_row_bytes(te->type, n_embd);
    for (size_t t = 0; t < seq; ++t) {
        if (tokens[t] < 0 || (size_t)tokens[t] >= te->ne1) return -2;
        const uint8_t* row = te->data + (size_t)tokens[t] * te_row;
        oracle_dequantize_row(te->type, row, n_embd, h + t * n_embd);
    }
    float* normed = (float*)malloc(sizeof(float) * seq * n_embd);
    float* q = (float*)malloc(sizeof(float) * seq * q_dim);
    float* k = (float*)malloc(sizeof(float) * seq * kv_dim);
    float* v = (float*)malloc(sizeof(float) * seq * kv_dim);
    float* att = (float*)malloc(sizeof(float) * seq * q_dim);
    float* pout = (float*)malloc(sizeof(float) * seq * n_embd);
    float* g = (float*)malloc(sizeof(float) * seq * n_ff);
    float* u = (float*)malloc(sizeof(float) * seq * n_ff);
    float* scores = (float*)malloc(sizeof(float) * (base + seq));
    const size_t group = n_head / n_kv;
    const float scale = 1.0f / sqrtf((float)hd);

    for (uint32_t li = 0; li < c->n_layer; ++li) {
        const float* wn = (const float*)L_(m, li, R_ATTN_NORM)->data;
        for (size_t t = 0; t < seq; ++t) oracle_rms_norm(h + t * n_embd, wn, normed + t * n_embd, n_embd, c->norm_eps);
        proj(L_(m, li, R_ATTN_Q), normed, n_embd, q, q_dim, seq);
        proj(L_(m, li, R_ATTN_K), normed, n_embd, k, kv_dim, seq);
        proj(L_(m, li, R_ATTN_V), normed, n_embd, v, kv_dim, seq);
        for (size_t t = 0; t < seq; ++t) {
            oracle_rope_apply(q + t * q_dim, n_head, hd, rope_half, base + t, c->rope_scale, freqs);
            oracle_rope_apply(k + t * kv_dim, n_kv, hd, rope_half, base + t, c->rope_scale, freqs);
        }
        float* Kl = m->K + (size_t)li * c->ctx_len * kv_dim;
        float* Vl = m->V + (size_t)li * c->ctx_len * kv_dim;
        for (size_t t = 0; t < seq; ++t) {
            memcpy(Kl + (base + t) * kv_dim, k + t * kv_dim, kv_dim * sizeof(float));
            memcpy(Vl + (base + t) * kv_dim, v + t * kv_dim, kv_dim * sizeof(float));
        }
        /* causal GQA attention, rawllm_forward.hpp:1115-1151 */
        for (size_t t = 0; t < seq; ++t) {
            for (size_t hh = 0; hh < n_head; ++hh) {
                size_t kvh = hh / group, klen = base + t + 1;
                const float* qv = q + t * q_dim + hh * hd;
                float maxs = -INFINITY;
                for (size_t s = 0; s < klen; ++s) {
                    float dot = oracle_dot_f32(qv, Kl + s * kv_dim + kvh * hd, hd) * scale;
                    scores[s] = dot;
                    if (dot > maxs) maxs = dot;
                }
                float sum = 0.f;
                for (size_t s = 0; s < klen; ++s) {
                    scores[s] = oracle_fast_expf(scores[s] - maxs);
                    sum += scores[s];
                }
                float inv = 1.0f / sum;
                float* o = att + t * q_dim + hh * hd;
                for (size_t i = 0; i < hd; ++i) o[i] = 0.f;
                for (size_t s = 0; s < klen; ++s) oracle_axpy_f32(o, scores[s] * inv, Vl + s * kv_dim + kvh * hd, hd);
            }
        }
        proj(L_(m, li, R_ATTN_OUT), att, q_dim, pout, n_embd, seq);
        for (size_t i = 0; i < seq * n_embd; ++i) h[i] += pout[i];
        const float* wf = (const float*)L_(m, li, R_FFN_NORM)->data;
        for (size_t t = 0; t < seq; ++t) oracle_rms_norm(h + t * n_embd, wf, normed + t * n_embd, n_embd, c->norm_eps);
        /* SwiGLU or the plain SiLU-FFN variant (rawllm_forward.hpp:1167-1190) */
        proj(L_(m, li, R_FFN_UP), normed, n_embd, u, n_ff, seq);
        if (c->plain_ffn) {
            for (size_t i = 0; i < seq * n_ff; ++i) g[i] = oracle_silu(u[i]);
        } else {
            proj(L_(m, li, R_FFN_GATE), normed, n_embd, g, n_ff, seq);
            for (size_t i = 0; i < seq * n_ff; ++i) g[i] = oracle_silu(g[i]) * u[i];
        }
        proj(L_(m, li, R_FFN_DOWN), g, n_ff, pout, n_embd, seq);
        for (size_t i = 0; i < seq * n_embd; ++i) h[i] += pout[i];
    }
    m->length = base + seq;
    float* fin = (float*)malloc(sizeof(float) * n_embd);
    oracle_rms_norm(h + (seq - 1) * n_embd, (const float*)m->global[R_OUTPUT_NORM].data, fin, n_embd, c->norm_eps);
    const oracle_tensor_t* ow = m->global[R_OUTPUT].data ? &m->global[R_OUTPUT] : te;
    proj(ow, fin, n_embd, out_logits, c->n_vocab, 1);
    free(fin); free(freqs); free(h); free(normed); free(q); free(k); free(v); free(att); free(pout); free(g);
    free(u); free(scores);
    return 0;
}

/* K/V rows of one layer for positions [0, n). */
void oracle_model_kv(void* p, int layer, size_t n, float* k, float* v) {
    oracle_model_t* m = (oracle_model_t*)p;
    size_t kvd = (size_t)m->cfg.n_kv_head * m->cfg.head_dim;
    memcpy(k, m->K + (size_t)layer * m->cfg.ctx_len * kvd, n * kvd * sizeof(float));
    memcpy(v, m->V + (size_t)layer * m->cfg.ctx_len * kvd, n * kvd * sizeof(float));
}
