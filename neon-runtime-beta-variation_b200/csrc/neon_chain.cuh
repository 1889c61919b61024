// Decode projection chain: the one-position Q4_0 projections that run between
// two attention launches of the decode step -- attn_output (+= residual),
// ffn gate/up (RMSNorm folded, SwiGLU or SiLU), ffn_down (+= residual) and the
// next layer's Q/K/V (RMSNorm folded, RoPE, K/V cache rows) -- as the phases of
// ONE launch instead of four (neon_cuda_set_decode_chain).
//
// Each phase is exactly a matvec_stream_kernel<Q4_0, RC, R> launch (same tile
// plan, X staging, dot products and epilogues, so the results are the same
// bits); what changes is between the phases:
//  - the copy warp walks every phase's items without stopping: weights never
//    depend on the phases, so the next phase's tiles stream into the ring
//    while the CTA waits for the others to finish the current one;
//  - phases are separated by a grid barrier (an arrival counter in global
//    memory, acquire polls bounded in time) instead of a kernel boundary;
//  - X and the residual are written inside the launch by other CTAs, so they
//    are read through L2 (ld.global.cg), never the non-coherent path.
// Every CTA of the grid must be resident at once for the barriers: the host
// sizes the grid to the CTAs the SMs hold (one wave), and a barrier that
// waits longer than its bound records bit 4 of the error word, raises the
// abort word and returns, so every other CTA leaves too.
//
// Tensor parallel (fused collectives): attn_output and ffn_down store their
// partial rows as LL words into every rank's slot (the streaming kernel's
// kEpiPeer epilogue), and an LL-reduce phase -- comm_ll_reduce_kernel's work,
// each CTA a slice of the vector -- adds the ranks' words into the residual
// before the next projection reads it; a layer is then 6 phases in one launch
// instead of 7 launches. The launch reads the communicator's count of
// completed LL collectives once, numbers its own (count + 1, + 2), and the
// last CTA to leave records the new count.
#pragma once

#include "neon_kernels.cuh"

namespace neon {

constexpr int kChainMaxPhases = 6;
constexpr int kChainMaxSpans = 3;   // Q, K, V
constexpr int kChainMaxStages = 8;

struct ChainPhase {
    Span span[kChainMaxSpans];
    const float* x;          // the phase's input, one position
    const float* norm_w;     // non-null: X = rms_norm(X, norm_w, norm_eps) first
    const float2* rope_cs;   // kEpiRope spans: (cos, sin) [position][rope_half]
    float norm_eps;
    int n_spans, n_tiles;
    int nb, kc, nch, rc;     // blocks per row, blocks per chunk, chunks per row, rows per tile
    int x_vec;               // x is 16-byte aligned
    int accumulate;          // kEpiStore spans: y += result
    int rope_half, head_dim;
    int ll_reduce;           // 1: an LL-reduce phase (h[i] += the ranks' words, i < n); no projection
    float* h;                //   its residual
    int n;                   //   and length
    int peer_k;              // LL collective of a kEpiPeer or LL-reduce phase: count + 1 + peer_k
};

struct ChainArgs {
    ChainPhase ph[kChainMaxPhases];
    const int* d_pos;        // the token's position
    unsigned int* err;       // device error word: bit 0 a ring wait, bit 4 a grid barrier timed out
    unsigned int* sync;      // [0] barrier arrivals, [1] departures, [2] abort; zero between launches
    int n_phases;
    int has_peer;            // tensor parallel: `peer` is the communicator's LL set
    int n_peer;              // LL collectives of the launch
    PeerSet peer;
    unsigned long long barrier_ns;  // bound of a grid-barrier wait
    int stages;              // ring depth
    int slot_bytes;          // bytes per ring slot: the largest phase's stream_stage_bytes
    int x_bytes;             // X region: the largest phase's stream_x_bytes
};

// Ring of a chain launch: a slot holds the largest phase's stage, the X
// region the largest phase's X; `max_stages` is how many slots fit beside X in
// max_smem (0: the chain does not fit). nb[i], rows[i]: phase i's blocks per
// row and rows (all targets); projection phases only.
struct ChainRing {
    int slot_bytes, x_bytes, max_stages;
};
inline ChainRing plan_chain_ring(const int* nb, const size_t* rows, int n, int sms, int stage_target, int max_smem,
                                 int forced_rc, int forced_kc) {
    ChainRing r{0, 0, 0};
    for (int i = 0; i < n; ++i) {
        const StreamPlan p = plan_stream_tiles(2, nb[i], rows[i], sms, stage_target, max_smem, forced_rc, forced_kc);
        if (p.stage_bytes > r.slot_bytes) r.slot_bytes = p.stage_bytes;
        const int xb = stream_x_bytes(2, nb[i]);
        if (xb > r.x_bytes) r.x_bytes = xb;
    }
    while (r.max_stages < kChainMaxStages && r.x_bytes + (r.max_stages + 1) * r.slot_bytes <= max_smem) ++r.max_stages;
    return r;
}

__device__ __forceinline__ int chain_span_of(const ChainPhase& p, int tile) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kChainMaxSpans; ++i)
        if (i < p.n_spans && p.span[i].tile0 <= tile) s = i;
    return s;
}

__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier number `k` (1, 2, ...) of the launch, for the compute warps:
// every CTA's writes before it are visible to every CTA after it. False (the
// same in every thread of the CTA) when the wait gave up or another CTA did.
__device__ __forceinline__ bool chain_barrier(const ChainArgs& c, int k) {
    compute_sync();  // this CTA's epilogue stores are done
    bool ok = true;
    if (threadIdx.x == 0) {
        const unsigned int target = (unsigned int)k * gridDim.x;
        __threadfence();
        atomicAdd(&c.sync[0], 1u);
        const uint64_t t0 = globaltimer_ns();
        for (;;) {
            if (ld_acquire_gpu_u32(&c.sync[0]) >= target) break;
            if (ld_acquire_gpu_u32(&c.sync[2]) != 0u) {
                ok = false;
                break;
            }
            if (globaltimer_ns() - t0 > c.barrier_ns) {
                atomicOr(c.err, 16u);
                atomicExch(&c.sync[2], 1u);
                ok = false;
                break;
            }
        }
        __threadfence();
    }
    return !compute_sync_or(!ok);
}

// matvec_stream_kernel's epilogues for the chain's phases; kEpiPeer stores LL
// collective `call`.
__device__ __forceinline__ void chain_epilogue(const ChainArgs& c, const ChainPhase& P, const Span& sp, int row0,
                                               int RC, const float* rowv, int pos, const float2* rcs, float yold,
                                               unsigned int call) {
    const int t = threadIdx.x;
    if (t >= RC) return;
    const int row = row0 + t;
    if (row >= sp.rows) return;
    const float v = rowv[t];
    switch (sp.epi) {
        case kEpiStore:
            sp.y[row] = P.accumulate ? yold + v : v;
            break;
        case kEpiAtPos:
            sp.y[(long long)pos * sp.pos_stride + row] = v;
            break;
        case kEpiRope: {
            float* dst = sp.y + (long long)pos * sp.pos_stride;
            if (t & 1) break;
            const float x0 = v, x1 = rowv[t + 1];
            const int i = (row % P.head_dim) / 2;
            if (i < P.rope_half) {
                const float2 cs = rcs[i];
                dst[row] = __fmaf_rn(x0, cs.x, -__fmul_rn(x1, cs.y));
                dst[row + 1] = __fmaf_rn(x0, cs.y, __fmul_rn(x1, cs.x));
            } else {
                dst[row] = x0;
                dst[row + 1] = x1;
            }
            break;
        }
        case kEpiSwiglu:
            if (!(t & 1)) sp.y[row / 2] = __fmul_rn(silu_dev(v), rowv[t + 1]);
            break;
        case kEpiSilu:
            sp.y[row] = silu_dev(v);
            break;
        case kEpiPeer: {
            // this rank's partial row sum, as an LL word, into its slot on every rank (NVLink stores)
            const long long off = ll_slot_off(c.peer.world, (int)(call & 1u), c.peer.rank) / 8 + row;
            const unsigned long long w = ll_pack(v, call);
            for (int p = 0; p < c.peer.world; ++p)
                st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(c.peer.base[p]) + off, w);
            break;
        }
        default:
            break;
    }
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64_chain(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// An LL-reduce phase (comm_ll_reduce_kernel's arithmetic): h[i] = h[i] +
// (slot_0[i] + slot_1[i] + ...) in rank order for this CTA's elements, every
// word polled until it carries `call`, each poll bounded by the
// communicator's timeout (bit 0 of its error word, then no more waits).
__device__ __forceinline__ void chain_ll_reduce(const ChainArgs& c, const ChainPhase& P, unsigned int call,
                                                volatile int* skip) {
    const PeerSet& p = c.peer;
    const unsigned long long* slots =
        reinterpret_cast<const unsigned long long*>(p.base[p.rank] + ll_slot_off(p.world, (int)(call & 1u), 0));
    for (int i = blockIdx.x * kStreamThreads + threadIdx.x; i < P.n; i += gridDim.x * kStreamThreads) {
        float s = 0.f;
        // four ranks' words in flight at a time (registers: the kernel shares
        // them with the projections' phases)
        for (int r0 = 0; r0 < p.world; r0 += 4) {
            unsigned long long w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (r0 + k < p.world) w[k] = ld_relaxed_sys_u64_chain(slots + (long long)(r0 + k) * kCommFusedFloats + i);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int r = r0 + k;
                if (r >= p.world) break;
                const unsigned long long* a = slots + (long long)r * kCommFusedFloats + i;
                if ((unsigned int)(w[k] >> 32) != call && !*skip) {
                    const unsigned long long t0 = globaltimer_ns();
                    for (;;) {
                        w[k] = ld_relaxed_sys_u64_chain(a);
                        if ((unsigned int)(w[k] >> 32) == call || *skip) break;
                        if (globaltimer_ns() - t0 > p.timeout_ns) {
                            atomicOr(p.err, 1u);
                            *skip = 1;
                            break;
                        }
                        __nanosleep(32);
                    }
                }
                const float v = __uint_as_float((unsigned int)w[k]);
                s = r ? s + v : v;
            }
        }
        P.h[i] = __ldcg(P.h + i) + s;
    }
}

// The compute warps' items of one phase (matvec_stream_kernel<Q4_0, RC, R>'s
// item loop); g: the CTA's running item count over all phases (ring slot and
// phase parity). False when a ring wait gave up.
template <int RC, int R>
__device__ __forceinline__ bool chain_consume(const ChainArgs& c, const ChainPhase& P, int n_items, int& g,
                                              const unsigned char* xsm, const unsigned char* ring, uint64_t* full,
                                              uint64_t* empty, float (*red)[128], float (*rowv)[32], int pos,
                                              const float2* rcs, unsigned int call) {
    constexpr int P16 = 16;
    constexpr int G = RC / R;
    constexpr int TPG = kStreamThreads / G;
    constexpr int WPG = TPG >= 32 ? TPG / 32 : 1;
    constexpr int LPG = TPG >= 32 ? 32 : TPG;
    static_assert(RC % R == 0 && kStreamThreads % G == 0 && RC * WPG <= 128 && RC <= 32, "bad tile shape");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gi = TPG >= 32 ? warp / WPG : warp * (32 / TPG) + lane / TPG;
    const int slice = TPG >= 32 ? (warp % WPG) * 32 + lane : lane % TPG;
    const int nb = P.nb, KC = P.kc, nch = P.nch, S = c.stages;
    const int SPH = stream_scale_pitch(KC);
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int it = 0; it < n_items; ++it, ++g) {
        const int stage = g % S;
        const uint32_t parity = (uint32_t)((g / S) & 1);
        const int tile = (int)blockIdx.x + (it / nch) * (int)gridDim.x;
        const int chunk = it % nch;
        const Span& sp = P.span[chain_span_of(P, tile)];
        const int row0 = (tile - sp.tile0) * RC;
        const int k0 = chunk * KC;
        const int kc = min(KC, nb - k0);
        const bool ok = mbar_wait(&full[stage], parity, c.err);
        if (compute_sync_or(!ok)) return false;
        const int tb = (it / nch) & 1;
        // the accumulate epilogue's y[row] (written earlier in this launch: through L2)
        float yold = 0.f;
        if (P.accumulate && chunk == nch - 1 && sp.epi == kEpiStore && (int)threadIdx.x < RC &&
            row0 + (int)threadIdx.x < sp.rows)
            yold = __ldcg(sp.y + row0 + threadIdx.x);

        const unsigned char* pay = ring + stage * c.slot_bytes;
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(pay + RC * KC * P16);
        int sbase[R];
        const unsigned char* prow[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
            const int r = gi * R + rr;
            sbase[rr] = nch == 1 ? (int)(((long long)row0 * nb) & 7) + r * nb
                                 : r * SPH + (int)(((long long)(row0 + r) * nb + k0) & 7);
            prow[rr] = pay + r * KC * P16;
        }
        float part[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) part[rr] = 0.f;
#pragma unroll 2
        for (int bi = slice; bi < kc; bi += TPG) {
            const uint4* r4 = reinterpret_cast<const uint4*>(xsm + (k0 + bi) * kQ4Rec);
            const uint4 x0 = r4[0], x1 = r4[1];
            const uint2 xm = *reinterpret_cast<const uint2*>(r4 + 2);
            const float xd = __uint_as_float(xm.x);
#pragma unroll
            for (int rr = 0; rr < R; ++rr) {
                const float wd = fp16_bits_to_f32(sc[sbase[rr] + bi]);
                const uint4 w = *reinterpret_cast<const uint4*>(prow[rr] + bi * P16);
                part[rr] = fmaf(wd * xd, small_int_to_f32(q4_block_isum(w, x0, x1, (int)xm.y)), part[rr]);
            }
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr) acc[rr] += part[rr];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (chunk == nch - 1) {
#pragma unroll
            for (int rr = 0; rr < R; ++rr)
#pragma unroll
                for (int o = LPG / 2; o; o >>= 1) acc[rr] += __shfl_xor_sync(0xffffffffu, acc[rr], o);
            if (WPG == 1) {
                if (slice == 0) {
#pragma unroll
                    for (int rr = 0; rr < R; ++rr) rowv[tb][gi * R + rr] = acc[rr];
                }
            } else if (lane == 0) {
#pragma unroll
                for (int rr = 0; rr < R; ++rr) red[tb][(gi * R + rr) * WPG + (warp % WPG)] = acc[rr];
            }
            compute_sync();
            if (WPG > 1 && (int)threadIdx.x < RC) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < WPG; ++w) v += red[tb][threadIdx.x * WPG + w];
                rowv[tb][threadIdx.x] = v;
            }
            if (WPG > 1) compute_sync();
            chain_epilogue(c, P, sp, row0, RC, rowv[tb], pos, rcs, yold, call);
#pragma unroll
            for (int rr = 0; rr < R; ++rr) acc[rr] = 0.f;
        }
    }
    return true;
}

// Q4_0 only (the phases' X is staged as Q8_0 records, as the streaming kernel
// does for Q4_0 weights). Block: kStreamWarps compute warps + one copy warp.
__global__ void __launch_bounds__(kStreamBlock) matvec_chain_kernel(const __grid_constant__ ChainArgs c) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float red[2][128];
    __shared__ float rowv[2][32];
    __shared__ float2 rcs[kMaxRopeHalf];
    __shared__ double dscratch[32];
    __shared__ __align__(8) uint64_t full[kChainMaxStages];
    __shared__ __align__(8) uint64_t empty[kChainMaxStages];
    const int S = c.stages;
    unsigned char* xsm = smem;
    unsigned char* ring = smem + c.x_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto items_of = [&](const ChainPhase& P) {
        if (P.ll_reduce) return 0;
        const int my_tiles =
            (int)blockIdx.x < P.n_tiles ? (P.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        return my_tiles * P.nch;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStreamWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kStreamWarps) {
        // Copy warp: every phase's items in order, a slot refilled as soon as
        // the compute warps release it; never waits for a phase.
        pdl_launch_dependents();
        int g = 0;
        for (int p = 0; p < c.n_phases; ++p) {
            const ChainPhase& P = c.ph[p];
            const int n_items = items_of(P);
            const int RC = P.rc, KC = P.kc, nb = P.nb, nch = P.nch;
            const int SPH = stream_scale_pitch(KC);
            for (int it = 0; it < n_items; ++it, ++g) {
                const int stage = g % S;
                if (g >= S && !mbar_wait(&empty[stage], (uint32_t)(((g / S) - 1) & 1), c.err)) return;
                const int tile = (int)blockIdx.x + (it / nch) * (int)gridDim.x;
                const int chunk = it % nch;
                const Span& sp = P.span[chain_span_of(P, tile)];
                const int row0 = (tile - sp.tile0) * RC;
                const int k0 = chunk * KC;
                const int kc = min(KC, nb - k0);
                const int nrows = min(RC, sp.rows - row0);
                unsigned char* pay = ring + stage * c.slot_bytes;
                uint16_t* sc = reinterpret_cast<uint16_t*>(pay + RC * KC * 16);
                if (nch == 1) {
                    const long long e = (long long)row0 * nb;
                    const int off = (int)(e & 7);
                    const uint32_t pbytes = (uint32_t)(nrows * nb * 16);
                    const uint32_t sbytes = 2u * (uint32_t)((off + nrows * nb + 7) & ~7);
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&full[stage], pbytes + sbytes);
                        bulk_g2s(pay, sp.qs + e * 16, pbytes, &full[stage]);
                        bulk_g2s(sc, sp.d + (e - off), sbytes, &full[stage]);
                    }
                    continue;
                }
                uint32_t bytes = 0;
                for (int r = lane; r < nrows; r += 32) {
                    const long long e = (long long)(row0 + r) * nb + k0;
                    const int off = (int)(e & 7);
                    bytes += (uint32_t)(kc * 16) + 2u * (uint32_t)((off + kc + 7) & ~7);
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
                if (lane == 0) mbar_arrive_expect_tx(&full[stage], bytes);
                __syncwarp();
                for (int r = lane; r < nrows; r += 32) {
                    const long long e = (long long)(row0 + r) * nb + k0;
                    const int off = (int)(e & 7);
                    bulk_g2s(pay + r * KC * 16, sp.qs + e * 16, (uint32_t)(kc * 16), &full[stage]);
                    bulk_g2s(sc + r * SPH, sp.d + (e - off), 2u * (uint32_t)((off + kc + 7) & ~7), &full[stage]);
                }
            }
        }
        return;
    }

    // compute warps
    __shared__ int s_skip;
    pdl_wait();
    const int pos = c.d_pos ? *c.d_pos : 0;
    // the communicator's count of completed LL collectives, before any CTA of
    // this launch can have recorded a new one (that happens after the last
    // barrier)
    const unsigned int call0 = c.has_peer ? *reinterpret_cast<volatile const unsigned int*>(c.peer.calls) : 0u;
    if (threadIdx.x == 0) s_skip = c.has_peer && *reinterpret_cast<volatile unsigned int*>(c.peer.err) != 0u;
    compute_sync();
    int g = 0;
    for (int p = 0; p < c.n_phases; ++p) {
        const ChainPhase& P = c.ph[p];
        if (p > 0 && !chain_barrier(c, p)) return;
        const unsigned int call = call0 + 1u + (unsigned int)P.peer_k;
        if (P.ll_reduce) {
            chain_ll_reduce(c, P, call, &s_skip);
            continue;
        }
        if (P.rope_cs && (int)threadIdx.x < P.rope_half) prefetch_l1(P.rope_cs + (long long)pos * P.rope_half + threadIdx.x);
        const int nb = P.nb;
        const int tpb = kStreamThreads / nb;
        if (P.norm_w && tpb >= 1) {
            if (tpb >= 4) stage_x_q8_norm<4, true>(P.x, nb, P.x_vec, xsm, P.norm_w, P.norm_eps, dscratch);
            else if (tpb >= 2) stage_x_q8_norm<2, true>(P.x, nb, P.x_vec, xsm, P.norm_w, P.norm_eps, dscratch);
            else stage_x_q8_norm<1, true>(P.x, nb, P.x_vec, xsm, P.norm_w, P.norm_eps, dscratch);
        } else {
            const float nscale = P.norm_w ? cta_rms_scale<true>(P.x, nb * 32, P.norm_eps, dscratch) : 1.f;
            if (tpb >= 4) stage_x_q8<4, true>(P.x, nb, P.x_vec, xsm, P.norm_w, nscale);
            else if (tpb >= 2) stage_x_q8<2, true>(P.x, nb, P.x_vec, xsm, P.norm_w, nscale);
            else stage_x_q8<1, true>(P.x, nb, P.x_vec, xsm, P.norm_w, nscale);
        }
        if (P.rope_cs && (int)threadIdx.x < P.rope_half)
            rcs[threadIdx.x] = P.rope_cs[(long long)pos * P.rope_half + threadIdx.x];
        compute_sync();
        if (p == 0) pdl_launch_dependents();
        const int n_items = items_of(P);
        bool ok = true;
        switch (P.rc) {  // R per RC: matvec_stream_kernel's Q4_0 instantiations
            case 2: ok = chain_consume<2, 2>(c, P, n_items, g, xsm, ring, full, empty, red, rowv, pos, rcs, call); break;
            case 4: ok = chain_consume<4, 2>(c, P, n_items, g, xsm, ring, full, empty, red, rowv, pos, rcs, call); break;
            case 8: ok = chain_consume<8, 2>(c, P, n_items, g, xsm, ring, full, empty, red, rowv, pos, rcs, call); break;
            case 16: ok = chain_consume<16, 4>(c, P, n_items, g, xsm, ring, full, empty, red, rowv, pos, rcs, call); break;
            default: ok = chain_consume<32, 4>(c, P, n_items, g, xsm, ring, full, empty, red, rowv, pos, rcs, call); break;
        }
        if (!ok) {
            if (threadIdx.x == 0) atomicExch(&c.sync[2], 1u);
            return;
        }
    }
    // Every CTA has passed its last barrier once all have departed: the last
    // to depart zeroes the counters for the next launch and records the LL
    // collectives of this one as completed.
    if (c.n_phases > 1) {
        compute_sync();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(&c.sync[1], 1u) == gridDim.x - 1) {
                atomicExch(&c.sync[0], 0u);
                atomicExch(&c.sync[1], 0u);
                if (c.has_peer) *c.peer.calls = call0 + (unsigned int)c.n_peer;
            }
        }
    }
}

}  // namespace neon
