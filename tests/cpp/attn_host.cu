// Host build of the decode attention's layout and split (neon_attn_layout.h).
#include "neon_attn_layout.h"

// out = {k, v, ps, sc, q, red, wm, wl, cmax, lsum, bar, total} in floats.
extern "C" void attn_host_layout(int hd, int gp, int bw, int round_rows, int score_rows, int cs, int* out) {
    const AttnSmem l = attn_smem_layout(hd, gp, bw, round_rows, score_rows, cs);
    const int v[12] = {l.k, l.v, l.ps, l.sc, l.q, l.red, l.wm, l.wl, l.cmax, l.lsum, l.bar, l.total};
    for (int i = 0; i < 12; ++i) out[i] = v[i];
}

// out = {gp, cs, round_rows, score_rows, smem_bytes}; returns attn_plan's verdict.
extern "C" int attn_host_plan(int ctx, int group, int hd, int cs_max, int max_round_rows, int* out) {
    AttnPlan p{};
    const bool ok = attn_plan(ctx, group, hd, cs_max, max_round_rows, &p);
    const int v[5] = {p.gp, p.cs, p.round_rows, p.score_rows, p.smem_bytes};
    for (int i = 0; i < 5; ++i) out[i] = v[i];
    return ok ? 1 : 0;
}

extern "C" int attn_host_rows(int L, int cs, int min_rows) { return attn_rows_per_cta(L, cs, min_rows); }

