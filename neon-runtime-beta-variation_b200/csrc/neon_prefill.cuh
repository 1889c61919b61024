// neon_prefill.cuh -- a Q4_0 projection of several positions (prefill) on the
// tensor cores, bit-exact with the reference.
//
// Reference: proj_all_positions' Q4_0 path (rawllm_forward.hpp:544-588): X is
// quantised to Q8_0 once per call, then every (row, position) is
// dot_q4_0_q8_0 (:419-434): over the row's 32-value blocks b in order,
//     total = fma(d_w[b] * d_x[b], (float)isum_b, total),   total = 0 first,
// where isum_b = sum_j (q_w[j] - 8) * q_x[j] is an exact integer.
//
// Here isum_b comes from the tensor cores: one mma.sync m16n8k32 (int8 x
// int8 -> int32) is exactly one block (K = 32) for 16 rows x 8 positions,
// with the nibbles widened to q - 8 in registers. Each thread keeps fp32
// accumulators for its (row, position) pairs and applies the block's scales
// in block order with the reference's own fma, so every output equals the
// reference's bit for bit. (The block scales rule out a TMEM-accumulating
// tcgen05 form: each 32-value block needs its own scale product before the
// next is added, and the block-scaled MMA kinds take power-of-two scales.)
//
// Tile: a CTA of 4 warps owns 64 rows x 64 positions; warp w the rows
// 16w..16w+15 and all 64 positions (8 MMA column tiles). The K loop stages
// 4 blocks at a time in shared memory (weights: 16 payload bytes per row and
// block, rows padded to 80 bytes; activations: 32 quants per position and
// block, positions padded to 144 bytes -- both conflict-free for the
// fragment reads), double-buffered through registers: the next chunk's
// global loads are in flight while the current chunk is multiplied.
#pragma once

#include "neon_kernels.cuh"

namespace neon {

constexpr int kMmaRows = 64;  // rows per CTA
constexpr int kMmaPos = 64;   // positions per CTA
constexpr int kMmaKb = 4;     // blocks per staged chunk
constexpr int kMmaWarps = 4;
constexpr int kMmaThreads = kMmaWarps * 32;
constexpr int kMmaWPitch = kMmaKb + 1;      // uint4 per staged weight row (80 bytes)
constexpr int kMmaXPitch = 2 * kMmaKb + 1;  // uint4 per staged position (144 bytes)

struct MmaStage {
    uint4 w[kMmaRows * kMmaWPitch];  // [row][kb]: the block's 16 nibble bytes
    float wd[kMmaRows * kMmaKb];     // [row][kb]: its fp16 scale, as fp32
    uint4 x[kMmaPos * kMmaXPitch];   // [pos][kb][2]: the block's 32 activation quants
    float xd[kMmaPos * kMmaKb];      // [pos][kb]: their fp32 scale
};

// D = A (16x32 s8, row-major) x B (32x8 s8, column-major) + 0x4B400000, int32:
// |A x B| < 2^22 for a Q4_0 x Q8_0 block (32 * 8 * 127), so each D read as a
// float is exactly 1.5 * 2^23 + isum, and isum as a float is one FADD away
// (no int-to-float conversion, which runs at an eighth of the FMA rate).
constexpr int kMmaFloatBias = 0x4B400000;
__device__ __forceinline__ void mma_s8_m16n8k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(kMmaFloatBias), "r"(kMmaFloatBias),
          "r"(kMmaFloatBias), "r"(kMmaFloatBias));
}
__device__ __forceinline__ float mma_isum_f32(int d) { return __int_as_float(d) - 12582912.0f; }

// Positions of a 64-position tile (grid.x) and rows of a 64-row tile (grid.y).
// MatvecArgs as the CUDA-core multi-position kernel takes it, with the span
// tiles counted in 64-row units and xq / xd the call's Q8_0 activations.
__global__ void __launch_bounds__(kMmaThreads) matvec_mma_q4_0_kernel(const __grid_constant__ MatvecArgs a) {
    __shared__ MmaStage st[2];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;  // the MMA fragment coordinates of this lane
    const int nb = a.nb, cols = nb * 32;
    const int tile = blockIdx.y;  // position tiles vary fastest: a row tile's weights stay in L2 for all of them
    const Span& sp = a.span[find_span(a, tile)];
    const int row0 = (tile - sp.tile0) * kMmaRows;
    const int p0 = blockIdx.x * kMmaPos;
    const int nchunks = (nb + kMmaKb - 1) / kMmaKb;

    pdl_launch_dependents();
    pdl_wait();  // the activation quants come from the kernel before

    // this thread's share of a chunk: 2 weight words + 2 scales, 4 activation
    // words + 2 scales
    uint4 rw[2], rx[4];
    float rwd[2], rxd[2];
    auto load = [&](int c) {
        const int b0 = c * kMmaKb;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + kMmaThreads * i;      // [row][kb]
            const int row = idx / kMmaKb, kb = idx % kMmaKb;
            const int gr = row0 + row, gb = b0 + kb;
            const bool ok = gr < sp.rows && gb < nb;
            const long long e = (long long)gr * nb + gb;
            rw[i] = ok ? ld_weights_u4(sp.qs + e * 16) : make_uint4(0, 0, 0, 0);
            rwd[i] = ok ? fp16_bits_to_f32(ld_weights_u16(sp.d + e)) : 0.f;
            const int gp = p0 + idx / kMmaKb;           // [pos][kb] for the scales
            rxd[i] = (gp < a.seq && gb < nb) ? a.xd[(long long)gp * nb + gb] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = tid + kMmaThreads * i;      // [pos][kb][half]
            const int pos = idx / (2 * kMmaKb), piece = idx % (2 * kMmaKb);
            const int gp = p0 + pos, gb = b0 + piece / 2;
            rx[i] = (gp < a.seq && gb < nb)
                        ? *reinterpret_cast<const uint4*>(a.xq + (long long)gp * cols + (long long)gb * 32 + (piece & 1) * 16)
                        : make_uint4(0, 0, 0, 0);
        }
    };
    auto store = [&](MmaStage& s) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + kMmaThreads * i;
            const int row = idx / kMmaKb, kb = idx % kMmaKb;
            s.w[row * kMmaWPitch + kb] = rw[i];
            s.wd[idx] = rwd[i];
            s.xd[idx] = rxd[i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = tid + kMmaThreads * i;
            const int pos = idx / (2 * kMmaKb), piece = idx % (2 * kMmaKb);
            s.x[pos * kMmaXPitch + piece] = rx[i];
        }
    };

    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;

    load(0);
    store(st[0]);
    __syncthreads();
    const int wr = warp * 16;  // this warp's first row in the tile
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) load(c + 1);
        const MmaStage& s = st[c & 1];
        const int kbn = min(kMmaKb, nb - c * kMmaKb);
        for (int kb = 0; kb < kbn; ++kb) {
            // A: rows wr+g and wr+g+8, values 4t..4t+3 (low nibbles of bytes
            // 4t..4t+3) and 16+4t.. (their high nibbles), widened to q - 8
            const uint32_t ug = reinterpret_cast<const uint32_t*>(&s.w[(wr + g) * kMmaWPitch + kb])[t];
            const uint32_t ug8 = reinterpret_cast<const uint32_t*>(&s.w[(wr + g + 8) * kMmaWPitch + kb])[t];
            const uint32_t a0 = __vsub4(ug & 0x0F0F0F0Fu, 0x08080808u);
            const uint32_t a1 = __vsub4(ug8 & 0x0F0F0F0Fu, 0x08080808u);
            const uint32_t a2 = __vsub4((ug >> 4) & 0x0F0F0F0Fu, 0x08080808u);
            const uint32_t a3 = __vsub4((ug8 >> 4) & 0x0F0F0F0Fu, 0x08080808u);
            const float wdg = s.wd[(wr + g) * kMmaKb + kb], wdg8 = s.wd[(wr + g + 8) * kMmaKb + kb];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                // B: position 8j+g, values 4t..4t+3 and 16+4t..16+4t+3
                const uint32_t* xp = reinterpret_cast<const uint32_t*>(&s.x[(8 * j + g) * kMmaXPitch + 2 * kb]);
                int d[4];
                mma_s8_m16n8k32(d, a0, a1, a2, a3, xp[t], xp[4 + t]);
                // D: rows g, g+8 x positions 8j+2t, 8j+2t+1; the reference's
                // block step total = fma(d_w * d_x, (float)isum, total)
                const float xd0 = s.xd[(8 * j + 2 * t) * kMmaKb + kb];
                const float xd1 = s.xd[(8 * j + 2 * t + 1) * kMmaKb + kb];
                acc[j][0] = fmaf(__fmul_rn(wdg, xd0), mma_isum_f32(d[0]), acc[j][0]);
                acc[j][1] = fmaf(__fmul_rn(wdg, xd1), mma_isum_f32(d[1]), acc[j][1]);
                acc[j][2] = fmaf(__fmul_rn(wdg8, xd0), mma_isum_f32(d[2]), acc[j][2]);
                acc[j][3] = fmaf(__fmul_rn(wdg8, xd1), mma_isum_f32(d[3]), acc[j][3]);
            }
        }
        if (c + 1 < nchunks) store(st[(c + 1) & 1]);
        __syncthreads();
    }

#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int gr = row0 + wr + g + (e >= 2 ? 8 : 0);
            const int gp = p0 + 8 * j + 2 * t + (e & 1);
            if (gr < sp.rows && gp < a.seq) {
                float* y = sp.y + (long long)gp * sp.y_stride + gr;
                *y = a.accumulate ? *y + acc[j][e] : acc[j][e];
            }
        }
}

// ---------------------------------------------------------------------------
// Q8_0 weights, several positions, on the tensor cores.
//
// Reference: for Q8_0 weights proj_all_positions dequantises each row
// (dequant_q8_0, rawllm_forward.hpp:143-150: w = d * q) and takes dot_f32 with
// fp32 X (:446-479, :597-605) -- no activation quantisation. Here, per block,
//     S_b = sum_j q_j * x_j,   acc = fma(d_b, S_b, acc)   (blocks in order),
// with S_b from TF32 MMAs (mma.sync m16n8k8): the int8 quants are exact in
// TF32, and X is split into x_hi = tf32(x) and x_lo = tf32(x - x_hi), so
// q*x_hi + q*x_lo carries x to within 2^-21 relative -- fp32 accuracy, with
// the additions in another order than dot_f32's (not bit-exact).
//
// Tile as the Q4_0 kernel: 4 warps x 16 rows, 64 positions (8 column tiles
// of 8), 2 blocks per staged chunk: weights 32 quants per row and block (rows
// padded to 80 bytes), X fp32 32 values per position and block (positions
// padded to 272 bytes) -- conflict-free for the fragment reads.
// ---------------------------------------------------------------------------
constexpr int kMma8Kb = 2;                   // blocks per staged chunk
constexpr int kMma8WPitch = 2 * kMma8Kb + 1; // uint4 per staged weight row (80 bytes)
constexpr int kMma8XPitch = 8 * kMma8Kb + 1; // float4 per staged position (272 bytes)

struct Mma8Stage {
    uint4 w[kMmaRows * kMma8WPitch];     // [row][kb][2]: the block's 32 int8 quants
    float wd[kMmaRows * kMma8Kb];        // [row][kb]: its fp16 scale, as fp32
    float4 x[kMmaPos * kMma8XPitch];     // [pos][kb][8]: the block's 32 fp32 activations
};

__device__ __forceinline__ uint32_t to_tf32(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return r;
}

// D += A (16x8 tf32, row-major) x B (8x8 tf32, column-major), fp32.
__device__ __forceinline__ void mma_tf32_m16n8k8(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kMmaThreads) matvec_mma_q8_0_kernel(const __grid_constant__ MatvecArgs a) {
    __shared__ Mma8Stage st[2];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nb = a.nb;
    const int tile = blockIdx.y;  // position tiles vary fastest: a row tile's weights stay in L2 for all of them
    const Span& sp = a.span[find_span(a, tile)];
    const int row0 = (tile - sp.tile0) * kMmaRows;
    const int p0 = blockIdx.x * kMmaPos;
    const int nchunks = (nb + kMma8Kb - 1) / kMma8Kb;

    pdl_launch_dependents();
    pdl_wait();  // X comes from the kernel before

    // a thread's share of a chunk: 2 weight words, 1 scale, 8 activation float4
    uint4 rw[2];
    float rwd;
    float4 rx[8];
    auto load = [&](int c) {
        const int b0 = c * kMma8Kb;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + kMmaThreads * i;  // [row][kb][half]
            const int row = idx / (2 * kMma8Kb), piece = idx % (2 * kMma8Kb);
            const int gr = row0 + row, gb = b0 + piece / 2;
            rw[i] = (gr < sp.rows && gb < nb)
                        ? ld_weights_u4(sp.qs + ((long long)gr * nb + gb) * 32 + (piece & 1) * 16)
                        : make_uint4(0, 0, 0, 0);
        }
        {
            const int row = tid / kMma8Kb, kb = tid % kMma8Kb;  // [row][kb], 128 of them
            const int gr = row0 + row, gb = b0 + kb;
            rwd = (gr < sp.rows && gb < nb) ? fp16_bits_to_f32(ld_weights_u16(sp.d + (long long)gr * nb + gb)) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = tid + kMmaThreads * i;  // [pos][kb][8 float4]
            const int pos = idx / (8 * kMma8Kb), piece = idx % (8 * kMma8Kb);
            const int gp = p0 + pos, gb = b0 + piece / 8;
            const float* xp = a.x + (long long)gp * a.x_stride + (long long)gb * 32 + (piece & 7) * 4;
            rx[i] = (gp < a.seq && gb < nb) ? make_float4(xp[0], xp[1], xp[2], xp[3]) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store = [&](Mma8Stage& s) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + kMmaThreads * i;
            const int row = idx / (2 * kMma8Kb), piece = idx % (2 * kMma8Kb);
            s.w[row * kMma8WPitch + piece] = rw[i];
        }
        s.wd[tid] = rwd;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = tid + kMmaThreads * i;
            const int pos = idx / (8 * kMma8Kb), piece = idx % (8 * kMma8Kb);
            s.x[pos * kMma8XPitch + piece] = rx[i];
        }
    };

    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;

    load(0);
    store(st[0]);
    __syncthreads();
    const int wr = warp * 16;
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) load(c + 1);
        const Mma8Stage& s = st[c & 1];
        const int kbn = min(kMma8Kb, nb - c * kMma8Kb);
        for (int kb = 0; kb < kbn; ++kb) {
            const signed char* qg = reinterpret_cast<const signed char*>(&s.w[(wr + g) * kMma8WPitch + 2 * kb]);
            const signed char* qg8 = reinterpret_cast<const signed char*>(&s.w[(wr + g + 8) * kMma8WPitch + 2 * kb]);
            const float dg = s.wd[(wr + g) * kMma8Kb + kb], dg8 = s.wd[(wr + g + 8) * kMma8Kb + kb];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float* xs = reinterpret_cast<const float*>(&s.x[(8 * j + g) * kMma8XPitch + 8 * kb]);
                float sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    // A: rows g, g+8, values 8ks+t and 8ks+t+4 (exact in TF32)
                    const uint32_t a0 = __float_as_uint((float)qg[8 * ks + t]);
                    const uint32_t a1 = __float_as_uint((float)qg8[8 * ks + t]);
                    const uint32_t a2 = __float_as_uint((float)qg[8 * ks + t + 4]);
                    const uint32_t a3 = __float_as_uint((float)qg8[8 * ks + t + 4]);
                    // B: position 8j+g, values 8ks+t and 8ks+t+4, as x_hi + x_lo
                    const float x0 = xs[8 * ks + t], x1 = xs[8 * ks + t + 4];
                    const uint32_t h0 = to_tf32(x0), h1 = to_tf32(x1);
                    const uint32_t l0 = to_tf32(x0 - __uint_as_float(h0)), l1 = to_tf32(x1 - __uint_as_float(h1));
                    mma_tf32_m16n8k8(sb, a0, a1, a2, a3, h0, h1);
                    mma_tf32_m16n8k8(sb, a0, a1, a2, a3, l0, l1);
                }
                // D: rows g, g+8 x positions 8j+2t, 8j+2t+1
                acc[j][0] = fmaf(dg, sb[0], acc[j][0]);
                acc[j][1] = fmaf(dg, sb[1], acc[j][1]);
                acc[j][2] = fmaf(dg8, sb[2], acc[j][2]);
                acc[j][3] = fmaf(dg8, sb[3], acc[j][3]);
            }
        }
        if (c + 1 < nchunks) store(st[(c + 1) & 1]);
        __syncthreads();
    }

#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int gr = row0 + wr + g + (e >= 2 ? 8 : 0);
            const int gp = p0 + 8 * j + 2 * t + (e & 1);
            if (gr < sp.rows && gp < a.seq) {
                float* y = sp.y + (long long)gp * sp.y_stride + gr;
                *y = a.accumulate ? *y + acc[j][e] : acc[j][e];
            }
        }
}

}  // namespace neon
