// Shared-memory layout and work split of the decode attention kernel
// (attn_decode_kernel in neon_decode.cu), host and device: the host sizes the
// launch with it, the kernel places its regions and picks its rows with it,
// and the CPU tests check it (nvcc builds every file that includes it).
#pragma once

constexpr int kAttnThreads = 256;         // threads per CTA
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxGroup = 8;          // query heads per KV head
constexpr int kAttnMaxCluster = 16;       // CTAs per KV head at most (a cluster)
constexpr int kAttnBoxRows = 32;          // cache rows per TMA tensor copy
constexpr int kAttnMinScores = 256;       // score rows a CTA holds at least
constexpr int kAttnMaxRound = 256;        // rows of one round (a TMA box dimension is at most 256)
constexpr int kAttnSmemTwo = 112 * 1024;  // dynamic shared memory of two CTAs per SM
constexpr int kAttnSmemMax = 200 * 1024;  // dynamic shared memory a CTA may take

// Query heads per KV head rounded up to a power of two (the kernel's template
// argument; the padding heads have zero query rows).
__host__ __device__ inline int attn_group_pad(int group) {
    return group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8;
}

// Floats per row of a dim block: the widest TMA swizzle span (128, 64 or 32
// bytes) that divides the head dim; 0 when none does (head_dim % 8 != 0).
__host__ __device__ inline int attn_block_width(int hd) {
    return hd % 32 == 0 ? 32 : hd % 16 == 0 ? 16 : hd % 8 == 0 ? 8 : 0;
}

// Cache rows of one CTA of a cluster of cs at context length L: the context
// over the cluster in whole 32-row boxes, at least min_rows (a multiple of
// 32). The first ceil(L / rows) CTAs have rows; n_act <= cs always.
__host__ __device__ inline int attn_rows_per_cta(int L, int cs, int min_rows) {
    int c = (L + cs - 1) / cs;
    c = (c + kAttnBoxRows - 1) / kAttnBoxRows * kAttnBoxRows;
    return c < min_rows ? min_rows : c;
}

struct AttnSmem {  // offsets (floats) into the dynamic shared memory
    int k, v, ps, sc, q, red, wm, wl, cmax, lsum, bar, total;
};

// k / v: the two slots, each one round of the CTA's K or V rows, [hd/bw dim
// blocks][round rows][bw floats], each dim block as its TMA boxes land
// (swizzled 16-byte chunks), 1024-byte aligned; ps: the round's partial dot
// products [hd/bw][round rows][gp], at the end the CTA's o [gp][hd] (hd * gp
// floats at most: the round holds a box of 32 rows); sc: the scores, then p, of all the CTA's
// rows [score rows][gp]; q: the group's query rows [gp][hd]; red: the warps'
// p*v sums [warps][gp][hd] (overlays slot 0 when it fits: slot 0 is read only
// before); wm / wl: the warps' maxima and sums [warps][gp]; cmax: the
// cluster's maxima [cs][gp] (written by the other CTAs); lsum: the CTA's l
// [gp]; bar: five mbarriers (slot 0, slot 1, the maxima, the peers' partials
// in CTA 0, CTA 0's release in the peers).
__host__ __device__ inline AttnSmem attn_smem_layout(int hd, int gp, int bw, int round_rows, int score_rows, int cs) {
    auto up4 = [](int v) { return (v + 3) & ~3; };
    AttnSmem l;
    l.k = 0;
    l.v = l.k + round_rows * hd;  // round_rows % 32 == 0 and hd % 8 == 0: a multiple of 1024 bytes
    l.ps = l.v + round_rows * hd;
    l.sc = up4(l.ps + (hd / bw) * round_rows * gp);
    l.q = up4(l.sc + score_rows * gp);
    int end = up4(l.q + gp * hd);
    const int red = kAttnWarps * gp * hd;
    if (red <= round_rows * hd) {
        l.red = l.k;
    } else {
        l.red = end;
        end = up4(end + red);
    }
    l.wm = end;
    l.wl = up4(l.wm + kAttnWarps * gp);
    l.cmax = up4(l.wl + kAttnWarps * gp);
    l.lsum = up4(l.cmax + cs * gp);
    l.bar = up4(l.lsum + gp);  // 16-byte aligned
    l.total = l.bar + 10;      // five 8-byte mbarriers
    return l;
}

struct AttnPlan {
    int gp, cs, round_rows, score_rows, smem_bytes;
};

// The split of a model's decode attention, fixed when the model is created:
// a cluster of cs CTAs per KV head, the smallest power of two (at most
// cs_max) whose share of ctx is at most share_rows rows; a CTA's scores for
// up to score_rows rows (its largest share, at least kAttnMinScores); its K
// and V rows in rounds of round_rows: its largest share (at most
// kAttnMaxRound), lowered until the
// CTA fits kAttnSmemTwo (two CTAs per SM, so that the device holds the
// clusters of every KV head at once), else kAttnSmemMax. False when no
// split fits.
inline bool attn_plan(int ctx, int group, int hd, int cs_max, int share_rows, AttnPlan* p) {
    auto up32 = [](int v) { return (v + kAttnBoxRows - 1) / kAttnBoxRows * kAttnBoxRows; };
    p->gp = attn_group_pad(group);
    p->cs = 1;
    while (p->cs < cs_max && up32((ctx + p->cs - 1) / p->cs) > share_rows) p->cs *= 2;
    const int share = up32((ctx + p->cs - 1) / p->cs);
    p->score_rows = share > kAttnMinScores ? share : kAttnMinScores;
    auto fit = [&](int rr, int limit) {
        p->round_rows = rr;
        p->smem_bytes = 4 * attn_smem_layout(hd, p->gp, attn_block_width(hd), rr, p->score_rows, p->cs).total;
        return p->smem_bytes <= limit;
    };
    if (attn_block_width(hd) == 0) return false;
    for (int limit : {kAttnSmemTwo, kAttnSmemMax})
        for (int r = share < kAttnMaxRound ? share : kAttnMaxRound; r >= kAttnBoxRows; r -= kAttnBoxRows)
            if (fit(r, limit)) return true;
    return false;
}
