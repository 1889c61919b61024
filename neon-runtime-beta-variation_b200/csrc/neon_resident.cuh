// neon_resident.cuh -- one-position Q4_0 / Q8_0 matvec whose weights are in
// shared memory before the launch's dependency wait.
//
// Reference path: the same as matvec_stream_kernel -- proj_all_positions'
// Q4_0 x Q8_0 block dot (dot_q4_0_q8_0, rawllm_forward.hpp:419-434, X
// quantised by quantize_rows_q8_0, :360-381) and its Q8_0 dequant + fp32 dot
// (:597-605) -- and every epilogue of the decode step.
//
// Why a second one-position kernel. A decode-sized projection (the 4096x4096
// configuration moves 9.5 MB, 64 KB per SM) is short next to the fixed cost
// of a launch: the dependency wait after the previous kernel, the X staging,
// the tail. The streaming kernel fills an SM's shared memory with one CTA's
// ring, so the next launch's CTAs only become resident when this launch's
// leave, and every launch pays the full HBM latency of its first bytes after
// the previous launch has ended. Here a CTA owns a contiguous range of rows
// small enough that its whole share fits in shared memory next to the shares
// of the following launches:
//   1. at CTA start, one thread issues ONE bulk copy per span piece for the
//      payload and one for the scales (weights are never written by earlier
//      kernels, so this happens before the dependency wait);
//   2. after the wait the CTA stages X (Q4_0: bit-exact Q8_0 records, RMSNorm
//      folded as in the streaming kernel; Q8_0: fp32) and lets the next
//      launch start: its CTAs become resident beside this one and start their
//      own copies, so the weight stream of launch N+1 runs while launch N
//      computes and N+1 waits (triggering before the X loads made them queue
//      behind the next launch's weight traffic);
//   3. the CTA waits for its weights (already there in steady state),
//      computes and runs the epilogues.
// The host sizes the CTAs (matvec_resident_plan) so that two launches fit on
// an SM at once; larger matrices take the streaming kernel.
//
// Work mapping: TPG threads per row group, G = 256 / TPG groups; thread
// (g, s) owns the CTA's local rows g, g + G, g + 2G, ... (at most
// kResRowsPerThread) and the blocks s, s + TPG, ... of each: one
// shared-memory read of an X block serves all its rows. A row's partial sums
// meet by shuffles (and, for TPG > 32, through shared memory). For a given
// TPG a row's sum is formed the same way whatever CTA owns it.
//
// Shared memory: X (the streaming kernel's layout), then the payload of the
// CTA's rows (local row lr at lr * nb * P), then the scale windows (a
// 16-byte-aligned window per span piece, as the streaming kernel copies
// them), then one mbarrier.
#pragma once

#include "neon_kernels.cuh"

namespace neon {

constexpr int kResRowsPerThread = 8;
constexpr int kResMaxSegs = kMaxSpans;

// Most rows a CTA of TPG threads per row group can own.
__host__ __device__ constexpr int res_max_rows(int tpg) { return (kStreamThreads / tpg) * kResRowsPerThread; }

// Threads per row group for rows of nb blocks: the largest power of two <= nb,
// between 16 and 256.
__host__ __device__ constexpr int res_tpg(int nb) {
    return nb >= 256 ? 256 : nb >= 128 ? 128 : nb >= 64 ? 64 : nb >= 32 ? 32 : 16;
}

struct ResLayout {
    int pay, sc, bar, total;  // byte offsets in dynamic shared memory (X at 0)
};
__host__ __device__ inline ResLayout res_layout(int type, int nb, int rpc) {
    const int P = type == 2 ? 16 : 32;
    ResLayout L;
    L.pay = stream_x_bytes(type, nb);
    L.sc = L.pay + ((rpc * nb * P + 127) & ~127);
    // each piece's window: its rows' scales plus at most 15 halfs of alignment
    const int sc_halfs = rpc * nb + 16 * kResMaxSegs;
    L.bar = L.sc + ((sc_halfs * 2 + 127) & ~127);
    L.total = L.bar + 16;
    return L;
}

// First row of each of n spans of rows[i] rows in a resident launch: every
// span starts at an even row, so a pair epilogue's rows (2i, 2i+1) never
// straddle two CTAs (CTAs own an even number of rows). Returns the rows of
// the launch (the last span's end).
__host__ __device__ inline long long res_span_starts(const long long* rows, int n, int* tile0) {
    long long v = 0;
    for (int i = 0; i < n; ++i) {
        v = (v + 1) & ~1LL;
        tile0[i] = (int)v;
        v += rows[i];
    }
    return v;
}

// A CTA's piece of one span: local rows [lr0, lr0 + n) are rows
// [row0, row0 + n) of span `span`; the scale of local row lr, block b sits at
// halfs sb + lr * nb + b of the scale area.
struct ResSeg {
    int lr0, n, span, row0, sb;
};

// The pieces of the CTA whose rows are [v0, v0 + nloc) (spans sorted by
// their first row, tile0) and the bytes of their copies; returns the count.
__host__ __device__ inline int res_segments(const Span* span, int n_spans, int v0, int nloc, int nb, int P,
                                            ResSeg* seg, uint32_t* bytes) {
    int n = 0, wofs = 0;
    uint32_t b = 0;
    for (int s = 0; s < n_spans; ++s) {
        const int lo = v0 > span[s].tile0 ? v0 : span[s].tile0;
        const int end = span[s].tile0 + span[s].rows;
        const int hi = v0 + nloc < end ? v0 + nloc : end;
        if (lo >= hi) continue;
        const int cnt = hi - lo;
        const int off = (int)(((long long)(lo - span[s].tile0) * nb) & 7);
        const int win = (off + cnt * nb + 7) & ~7;
        b += (uint32_t)cnt * (uint32_t)nb * (uint32_t)P + 2u * (uint32_t)win;
        seg[n].lr0 = lo - v0;
        seg[n].n = cnt;
        seg[n].span = s;
        seg[n].row0 = lo - span[s].tile0;
        seg[n].sb = wofs + off - (lo - v0) * nb;
        wofs += win;
        ++n;
    }
    *bytes = b;
    return n;
}

// The two copies of a piece: payload bytes from byte (row0 * nb * P) of the
// span's payload plane to byte (lr0 * nb * P) of the payload area; scales, a
// 16-byte-aligned window, from half (row0 * nb - off) of the span's scale
// plane to half sc_dst_half of the scale area.
struct ResCopy {
    long long pay_src, pay_dst, sc_src_half, sc_dst_half;
    uint32_t pay_bytes, sc_bytes;
};
__host__ __device__ inline ResCopy res_copy(const ResSeg& g, int nb, int P) {
    ResCopy c;
    const long long e = (long long)g.row0 * nb;
    const int off = (int)(e & 7);
    const int win = (off + g.n * nb + 7) & ~7;
    c.pay_src = e * P;
    c.pay_dst = (long long)g.lr0 * nb * P;
    c.pay_bytes = (uint32_t)g.n * (uint32_t)nb * (uint32_t)P;
    c.sc_src_half = e - off;
    c.sc_dst_half = (long long)g.sb + (long long)g.lr0 * nb - off;
    c.sc_bytes = 2u * (uint32_t)win;
    return c;
}

template <int TYPE, int TPG>
__global__ void __launch_bounds__(kStreamThreads, 4) matvec_resident_kernel(const __grid_constant__ StreamArgs a) {
    constexpr int P = TYPE == 2 ? 16 : 32;
    constexpr int G = kStreamThreads / TPG;
    constexpr int WPG = TPG >= 32 ? TPG / 32 : 1;
    constexpr int LPG = TPG >= 32 ? 32 : TPG;
    constexpr int MAXR = kResRowsPerThread;
    constexpr int MAXROWS = G * MAXR;
    static_assert(MAXR == 8 && LPG >= 8, "the row butterfly takes 8 rows per thread and 8 or more lanes per group");
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float rowres[MAXROWS];
    __shared__ float red[WPG > 1 ? MAXROWS * WPG : 1];
    __shared__ int rowsb[MAXROWS];  // scale index of (local row, block 0); 0 for span padding
    __shared__ ResSeg seg[kResMaxSegs];
    __shared__ int n_seg;
    __shared__ float2 rcs[kMaxRopeHalf];
    __shared__ double dscratch[32];

    const int nb = a.nb;
    const ResLayout L = res_layout(TYPE, nb, a.rpc);
    unsigned char* xsm = smem;
    unsigned char* pay = smem + L.pay;
    uint16_t* sc = reinterpret_cast<uint16_t*>(smem + L.sc);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    const int tid = threadIdx.x, lane = tid & 31;
    const int v0 = (int)blockIdx.x * a.rpc;
    const int nloc = min(a.rpc, a.n_vrows - v0);

    // the CTA's piece of every span, and the bytes of their copies
    uint32_t bytes = 0;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        n_seg = res_segments(a.span, a.n_spans, v0, nloc, nb, P, seg, &bytes);
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, bytes);
        for (int k = 0; k < n_seg; ++k) {
            const Span& sp = a.span[seg[k].span];
            const ResCopy c = res_copy(seg[k], nb, P);
            bulk_g2s(pay + c.pay_dst, sp.qs + c.pay_src, c.pay_bytes, bar);
            bulk_g2s(sc + c.sc_dst_half, sp.d + c.sc_src_half, c.sc_bytes, bar);
        }
    }
    // Everything that depends on the launch's parameters only, before the
    // wait: each local row's scale index, and this thread's epilogue piece
    // (thread tid runs the epilogue of local row tid).
    int eseg = -1;
    if (tid < MAXROWS) {
        int sbv = 0;
        for (int k = 0; k < n_seg; ++k)
            if (tid >= seg[k].lr0 && tid < seg[k].lr0 + seg[k].n) {
                sbv = seg[k].sb + tid * nb;
                eseg = k;
            }
        rowsb[tid] = sbv;
    }
    const float* yold_p = nullptr;  // the accumulate epilogue's y[row]
    if (eseg >= 0) {
        const Span& sp = a.span[seg[eseg].span];
        if (a.accumulate && sp.epi == kEpiStore) yold_p = sp.y + seg[eseg].row0 + tid - seg[eseg].lr0;
    }
    const bool rope_row = a.rope_cs && tid < a.rope_half;
    pdl_wait();

    // what the kernel before may have written: the position, the collective's
    // call count and y[row]; loaded now, used after the X staging
    const unsigned int peer_call =
        a.peer_mode ? *reinterpret_cast<volatile const unsigned int*>(a.peer.calls) + 1u : 0u;
    const int pos = a.d_pos ? *a.d_pos : 0;
    const float yold = yold_p ? *yold_p : 0.f;

    // X, staged once per CTA (normalised first when asked)
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
        for (int i = tid; i < nb * 32; i += kStreamThreads) {
            float v = __ldg(a.x + i);
            if (a.norm_w) v = __fmul_rn(__fmul_rn(v, nscale), __ldg(a.norm_w + i));
            xs[(i >> 5) * kQ8Pitch + (i & 31)] = v;
        }
    }
    // X is read: the next launch's CTAs may take their places now and start
    // their copies (earlier, their weight traffic would delay these X loads)
    pdl_launch_dependents();
    const bool ok = mbar_wait(bar, 0, a.err);
    if (__syncthreads_or(!ok)) return;  // also: X, the RoPE row and rowsb are in place

    // Dot products, all MAXR rows of the thread without branches (a row past
    // nloc repeats the last row; its sum is not stored), so the compiler
    // interleaves the rows' independent chains.
    // the position's RoPE row: loaded here, in shared memory before the epilogue
    float2 rope_v = make_float2(0.f, 0.f);
    if (rope_row) rope_v = a.rope_cs[(long long)pos * a.rope_half + tid];
    const int g = tid / TPG, s = tid % TPG;
    int wofs[MAXR], sofs[MAXR];
#pragma unroll
    for (int i = 0; i < MAXR; ++i) {
        const int lr = min(g + i * G, nloc - 1);
        wofs[i] = lr * nb;
        sofs[i] = rowsb[lr];
    }
    float part[MAXR];
#pragma unroll
    for (int i = 0; i < MAXR; ++i) part[i] = 0.f;
    for (int b = s; b < nb; b += TPG) {
        if (TYPE == 2) {
            const uint4* r4 = reinterpret_cast<const uint4*>(xsm + b * kQ4Rec);
            const uint4 x0 = r4[0], x1 = r4[1];
            const uint2 xm = *reinterpret_cast<const uint2*>(r4 + 2);
            const float xd = __uint_as_float(xm.x);
            const int bias = 0x4B400000 - 128 * (int)xm.y;
#pragma unroll
            for (int i = 0; i < MAXR; ++i) {
                const float wd = fp16_bits_to_f32(sc[sofs[i] + b]);
                const uint4 w = *reinterpret_cast<const uint4*>(pay + (size_t)(wofs[i] + b) * P);
                part[i] = fmaf(wd * xd, q4_block_dot16(w, x0, x1, bias), part[i]);
            }
        } else {
            const ulonglong2* xv2 =
                reinterpret_cast<const ulonglong2*>(reinterpret_cast<const float*>(xsm) + b * kQ8Pitch);
            unsigned long long xv[16];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const ulonglong2 t = xv2[k];
                xv[2 * k] = t.x;
                xv[2 * k + 1] = t.y;
            }
#pragma unroll
            for (int i = 0; i < MAXR; ++i) {
                const float wd = fp16_bits_to_f32(sc[sofs[i] + b]);
                const uint4* w4 = reinterpret_cast<const uint4*>(pay + (size_t)(wofs[i] + b) * P);
                part[i] = fmaf(wd, q8_block_dot_x2(w4[0], w4[1], xv), part[i]);
            }
        }
    }
    // Row sums over the group's LPG lanes by a transposing butterfly: three
    // exchange steps each hand half of the remaining rows to the partner lane
    // (8 -> 4 -> 2 -> 1 rows per lane), then plain steps finish the one row a
    // lane keeps -- 9 shuffles for 8 rows instead of 40. Every row's sum is the
    // same tree over the same lanes, whatever its place in the CTA.
    float v4[4], v2[2];
    const bool h4 = lane & (LPG / 2), h2 = lane & (LPG / 4), h1 = lane & (LPG / 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float r = __shfl_xor_sync(0xffffffffu, h4 ? part[j] : part[j + 4], LPG / 2);
        v4[j] = (h4 ? part[j + 4] : part[j]) + r;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float r = __shfl_xor_sync(0xffffffffu, h2 ? v4[j] : v4[j + 2], LPG / 4);
        v2[j] = (h2 ? v4[j + 2] : v4[j]) + r;
    }
    float v1;
    {
        const float r = __shfl_xor_sync(0xffffffffu, h1 ? v2[0] : v2[1], LPG / 8);
        v1 = (h1 ? v2[1] : v2[0]) + r;
    }
#pragma unroll
    for (int o = LPG / 16; o; o >>= 1) v1 += __shfl_xor_sync(0xffffffffu, v1, o);
    {
        const int ri = (h4 ? 4 : 0) + (h2 ? 2 : 0) + (h1 ? 1 : 0);
        const int lr = g + ri * G;
        if ((lane & (LPG / 8 - 1)) == 0 && lr < nloc) {
            if (WPG == 1) rowres[lr] = v1;
            else red[lr * WPG + (s >> 5)] = v1;
        }
    }
    if (rope_row) rcs[tid] = rope_v;
    __syncthreads();
    if (WPG > 1 && tid < nloc) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < WPG; ++w) v += red[tid * WPG + w];
        rowres[tid] = v;
    }
    if (WPG > 1) __syncthreads();
    if (eseg >= 0)
        stream_epilogue(a, a.span[seg[eseg].span], seg[eseg].row0, seg[eseg].n, rowres + seg[eseg].lr0, peer_call,
                        pos, rcs, yold, tid - seg[eseg].lr0);
}

// Launch shape of a resident launch over n_vrows rows of nb blocks: rows per
// CTA (even) and grid; false when the rows do not fit the kernel (too many
// per CTA) or two launches' CTAs would not fit one SM's shared memory.
struct ResPlan {
    int tpg, rpc, grid, smem;
};
inline bool matvec_resident_plan(int type, int nb, int n_vrows, int sms, int ctas_per_sm, int smem_per_sm,
                                 ResPlan* p) {
    if (n_vrows <= 0 || nb <= 0 || ctas_per_sm <= 0 || sms <= 0) return false;
    for (int k = ctas_per_sm; k <= 8 * ctas_per_sm; k *= 2) {
        int rpc = (n_vrows + k * sms - 1) / (k * sms);
        rpc = (rpc + 1) & ~1;
        // fewer threads per row group hold more rows per CTA
        int tpg = res_tpg(nb);
        while (rpc > res_max_rows(tpg) && tpg > 16) tpg /= 2;
        if (rpc > res_max_rows(tpg)) continue;
        const ResLayout L = res_layout(type, nb, rpc);
        const int grid = (n_vrows + rpc - 1) / rpc;
        const int per_sm = (grid + sms - 1) / sms;  // this launch's CTAs on the busiest SM
        // two launches side by side (+1 KB the hardware reserves per CTA, + static shared memory)
        if (2 * per_sm * (L.total + 1024 + 2048) > smem_per_sm) return false;
        p->tpg = tpg;
        p->rpc = rpc;
        p->grid = grid;
        p->smem = L.total;
        return true;
    }
    return false;
}

}  // namespace neon
