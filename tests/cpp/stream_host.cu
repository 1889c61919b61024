// Host build of the streaming kernel's tile planner (neon_kernels.cuh): the
// CPU tests emulate the kernel's copies and reads on the plans it returns.
#include <stddef.h>

#include "neon_kernels.cuh"

// out = {rc, kc, nch, stages, stage_bytes, smem}; also the scale pitch and X bytes.
extern "C" void stream_host_plan(int type, int nb, size_t total_rows, int sms, int stage_target, int max_smem,
                                 int forced_rc, int forced_kc, int* out) {
    const neon::StreamPlan p =
        neon::plan_stream_tiles(type, nb, total_rows, sms, stage_target, max_smem, forced_rc, forced_kc);
    out[0] = p.rc;
    out[1] = p.kc;
    out[2] = p.nch;
    out[3] = p.stages;
    out[4] = p.stage_bytes;
    out[5] = p.smem;
    out[6] = neon::stream_scale_pitch(p.kc);
    out[7] = neon::stream_x_bytes(type, nb);
}
