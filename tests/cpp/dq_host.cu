// Host build of the device block decoders (neon_dequant.cuh's dq_sub is
// __host__ __device__): the CPU tests decode padded device rows with the very
// source the kernels run and compare the values with the oracle.
#include <stdint.h>

#include "neon_dequant.cuh"

namespace {
template <int TYPE>
void decode_row(const unsigned char* row, int nu, float* out) {
    using D = neon::DqShape<TYPE>;
    for (int u = 0; u < nu; ++u) {
        float w[32];
        neon::dq_sub<TYPE>(row + (u / D::SUBS) * D::BB, u % D::SUBS, w);
        for (int j = 0; j < 32; ++j) out[32 * u + j] = w[j];
    }
}
template <int TYPE>
void dot_row(const unsigned char* row, int nu, const float* x, float* out) {
    using D = neon::DqShape<TYPE>;
    for (int u = 0; u < nu; ++u) {
        neon::DqCode<TYPE> c;
        neon::dq_codes<TYPE>(row + (u / D::SUBS) * D::BB, u % D::SUBS, c);
        float xsum = 0.f;
        for (int j = 0; j < 32; ++j) xsum += x[32 * u + j];
        out[u] = neon::dq_code_dot<TYPE>(c, x + 32 * u, xsum);
    }
}
}  // namespace

// Per 32-value sub-block of one padded device row, the kernel's dot product
// with x (nu * 32 floats), computed without forming the weights (the packed
// code sums, emulated lane by lane). Block types only; -1 otherwise.
extern "C" int dq_host_code_dots(int type, const unsigned char* row, int nu, const float* x, float* out) {
    switch (type) {
        case NEON_GGML_Q4_1: dot_row<NEON_GGML_Q4_1>(row, nu, x, out); return 0;
        case NEON_GGML_Q5_0: dot_row<NEON_GGML_Q5_0>(row, nu, x, out); return 0;
        case NEON_GGML_Q5_1: dot_row<NEON_GGML_Q5_1>(row, nu, x, out); return 0;
        case NEON_GGML_Q4_K: dot_row<NEON_GGML_Q4_K>(row, nu, x, out); return 0;
        case NEON_GGML_Q5_K: dot_row<NEON_GGML_Q5_K>(row, nu, x, out); return 0;
        case NEON_GGML_Q6_K: dot_row<NEON_GGML_Q6_K>(row, nu, x, out); return 0;
        default: return -1;
    }
}

// nu 32-value sub-blocks of one padded device row -> out (nu * 32 floats).
// Returns -1 for a type the dequantising kernel does not take.
extern "C" int dq_host_decode_row(int type, const unsigned char* row, int nu, float* out) {
    switch (type) {
        case NEON_GGML_F32: decode_row<NEON_GGML_F32>(row, nu, out); return 0;
        case NEON_GGML_F16: decode_row<NEON_GGML_F16>(row, nu, out); return 0;
        case NEON_GGML_BF16: decode_row<NEON_GGML_BF16>(row, nu, out); return 0;
        case NEON_GGML_Q4_1: decode_row<NEON_GGML_Q4_1>(row, nu, out); return 0;
        case NEON_GGML_Q5_0: decode_row<NEON_GGML_Q5_0>(row, nu, out); return 0;
        case NEON_GGML_Q5_1: decode_row<NEON_GGML_Q5_1>(row, nu, out); return 0;
        case NEON_GGML_Q4_K: decode_row<NEON_GGML_Q4_K>(row, nu, out); return 0;
        case NEON_GGML_Q5_K: decode_row<NEON_GGML_Q5_K>(row, nu, out); return 0;
        case NEON_GGML_Q6_K: decode_row<NEON_GGML_Q6_K>(row, nu, out); return 0;
        default: return -1;
    }
}

// The block geometry the upload and the launcher use (values and bytes per
// block, blocks per chunk).
extern "C" void dq_host_geometry(int type, int* be, int* bb, int* cb) { neon::dq_geometry(type, be, bb, cb); }

// n values of one host row of `type` (GGUF layout, any alignment) -> out, by
// neon::dq_row_host, the decoder the engine runs on norm weights at load time.
extern "C" int dq_host_row(int type, const unsigned char* p, size_t n, float* out) {
    return neon::dq_row_host(type, p, n, out) ? 0 : -1;
}

// The ring kernel's tile plan (neon::plan_dq_ring): out = {rpw, kcb, nch,
// row_stride, stage_bytes}.
extern "C" void dq_host_ring_plan(int type, int nblk, long long pitch, size_t total_rows, int sms,
                                  int stage_target, int* out) {
    const neon::DqRingPlan p = neon::plan_dq_ring(type, nblk, pitch, total_rows, sms, stage_target);
    out[0] = p.rpw;
    out[1] = p.kcb;
    out[2] = p.nch;
    out[3] = p.row_stride;
    out[4] = p.stage_bytes;
}
