// Shared-memory layout of the decode attention kernel (attn_decode_kernel in
// neon_decode.cu), host and device: the host sizes the launch with it, the
// kernel places its regions with it, and the CPU tests check it (nvcc
// builds every file that includes it).
#pragma once

constexpr int kAttnThreads = 256;          // threads per CTA
constexpr int kAttnMaxGroup = 8;           // query heads per KV head
constexpr int kAttnMaxCluster = 16;        // CTAs per KV head at most (a cluster)
constexpr int kAttnSub = 64;               // cache rows per ring slot
constexpr int kAttnBox = 16;               // cache rows per TMA tensor copy (a slot is up to 4 boxes)
constexpr int kAttnMaxSlots = 8;
constexpr int kAttnSmemMax = 200 * 1024;   // dynamic shared memory a slot count may take

struct AttnSmem {  // offsets (floats) into the dynamic shared memory; slots: ring depth
    int q, sc, ring, co, csum, cmax, bar, total, slots;
};

// q: the group's query rows [group][hd]; sc: scores [group][chunk_max]; ring:
// `slots` slots of kAttnSub cache rows of hd floats, 128-byte aligned for the
// TMA copies (later the per-part partial sums, and in CTA 0 the cluster's
// partials); csum / cmax: the cluster's per-head sums and maxima; bar: one
// mbarrier per slot.
__host__ __device__ inline AttnSmem attn_smem_layout(int group, int hd, int chunk_max, int cs, int slots) {
    auto up4 = [](int v) { return (v + 3) & ~3; };  // float4-aligned regions
    auto mx = [](int a, int b) { return a > b ? a : b; };
    auto up32 = [](int v) { return (v + 31) & ~31; };  // 128-byte-aligned regions
    const int pitch = hd;
    const int parts = kAttnThreads / (hd / 4);
    AttnSmem l;
    l.q = 0;
    l.sc = up4(l.q + group * hd);
    l.ring = up32(l.sc + group * chunk_max);
    l.slots = slots;
    const int ring = mx(slots * kAttnSub * pitch, mx(parts * group * hd, cs * group * hd));
    l.co = l.ring;
    l.csum = up4(l.ring + ring);
    l.cmax = up4(l.csum + cs * kAttnMaxGroup);
    l.bar = up4(l.cmax + cs * kAttnMaxGroup);
    l.total = l.bar + 2 * slots;  // 8-byte mbarriers
    return l;
}
