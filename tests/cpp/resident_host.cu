// Host build of the resident kernel's launch arithmetic (neon_resident.cuh):
// its plan, shared-memory layout, the span pieces a CTA copies and the two
// copies of each piece -- the same functions the kernel and its launcher run.
#include <stddef.h>

#include "neon_resident.cuh"

// out = {ok, tpg, rpc, grid, smem}
extern "C" void resident_host_plan(int type, int nb, int n_vrows, int sms, int ctas_per_sm, int smem_per_sm,
                                   int* out) {
    neon::ResPlan p{};
    out[0] = neon::matvec_resident_plan(type, nb, n_vrows, sms, ctas_per_sm, smem_per_sm, &p) ? 1 : 0;
    out[1] = p.tpg;
    out[2] = p.rpc;
    out[3] = p.grid;
    out[4] = p.smem;
}

// out = {pay, sc, bar, total, x bytes, most rows per CTA for tpg}
extern "C" void resident_host_layout(int type, int nb, int rpc, int tpg, int* out) {
    const neon::ResLayout L = neon::res_layout(type, nb, rpc);
    out[0] = L.pay;
    out[1] = L.sc;
    out[2] = L.bar;
    out[3] = L.total;
    out[4] = neon::stream_x_bytes(type, nb);
    out[5] = neon::res_max_rows(tpg);
}

// Span starts for n spans of rows[i] rows: tile0[i]; returns the launch's rows.
extern "C" long long resident_host_starts(const long long* rows, int n, int* tile0) {
    return neon::res_span_starts(rows, n, tile0);
}

// The pieces of the CTA owning rows [v0, v0 + nloc): seg_out[5*k..] =
// {lr0, n, span, row0, sb}; copies_out[6*k..] = {pay_src, pay_dst, pay_bytes,
// sc_src_half, sc_dst_half, sc_bytes}; *bytes = the mbarrier's byte count.
extern "C" int resident_host_pieces(const int* tile0, const int* rows, int n_spans, int v0, int nloc, int nb, int P,
                                    int* seg_out, long long* copies_out, unsigned int* bytes) {
    neon::Span span[neon::kMaxSpans] = {};
    for (int i = 0; i < n_spans; ++i) {
        span[i].tile0 = tile0[i];
        span[i].rows = rows[i];
    }
    neon::ResSeg seg[neon::kResMaxSegs];
    uint32_t b = 0;
    const int n = neon::res_segments(span, n_spans, v0, nloc, nb, P, seg, &b);
    for (int k = 0; k < n; ++k) {
        const int s[5] = {seg[k].lr0, seg[k].n, seg[k].span, seg[k].row0, seg[k].sb};
        for (int j = 0; j < 5; ++j) seg_out[5 * k + j] = s[j];
        const neon::ResCopy c = neon::res_copy(seg[k], nb, P);
        const long long v[6] = {c.pay_src, c.pay_dst, c.pay_bytes, c.sc_src_half, c.sc_dst_half, c.sc_bytes};
        for (int j = 0; j < 6; ++j) copies_out[6 * k + j] = v[j];
    }
    *bytes = b;
    return n;
}
