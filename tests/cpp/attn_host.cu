// Host build of the decode attention's shared-memory layout (neon_attn_layout.h).
#include "neon_attn_layout.h"

// out = {q, sc, ring, co, csum, cmax, bar, total} in floats.
extern "C" void attn_host_layout(int group, int hd, int chunk_max, int cs, int slots, int* out) {
    const AttnSmem l = attn_smem_layout(group, hd, chunk_max, cs, slots);
    const int v[8] = {l.q, l.sc, l.ring, l.co, l.csum, l.cmax, l.bar, l.total};
    for (int i = 0; i < 8; ++i) out[i] = v[i];
}
