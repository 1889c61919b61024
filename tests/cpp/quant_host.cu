// Host build of the on-load quantiser's block code (neon_quant.cuh is
// __host__ __device__): the CPU tests compare its bytes with gguf-py's.
#include <stdint.h>

#include "neon_quant.cuh"

// rows x cols float values (src_type bytes) -> GGUF rows of dst_type, the loop
// quantize_rows_kernel runs, one block (or value) at a time. Returns -1 for a
// pair the quantiser does not take.
extern "C" int q_host_quantize_rows(const unsigned char* src, int src_type, long long rows, long long cols,
                                    int dst, unsigned char* out) {
    const bool block = neon::q_block_bytes(dst) != 0;
    if (!block && dst != NEON_GGML_F16 && dst != NEON_GGML_BF16) return -1;
    if (src_type != NEON_GGML_F32 && src_type != NEON_GGML_F16 && src_type != NEON_GGML_BF16) return -1;
    const long long esz = src_type == NEON_GGML_F32 ? 4 : 2;
    const long long dst_row = block ? cols / 32 * neon::q_block_bytes(dst) : cols * 2;
    for (long long r = 0; r < rows; ++r) {
        const unsigned char* row = src + r * cols * esz;
        unsigned char* orow = out + r * dst_row;
        if (block) {
            for (long long b = 0; b < cols / 32; ++b) {
                float x[32];
                for (int j = 0; j < 32; ++j) x[j] = neon::q_src_value(row, src_type, 32 * b + j);
                neon::q_quantize_block(x, dst, orow + b * neon::q_block_bytes(dst));
            }
        } else {
            for (long long i = 0; i < cols; ++i) {
                const float v = neon::q_src_value(row, src_type, i);
                neon::q_put_u16(orow + 2 * i, dst == NEON_GGML_F16 ? neon::q_f16_bits(v) : neon::q_bf16_bits(v));
            }
        }
    }
    return 0;
}

// fp32 -> binary16 bits of n values (the quantiser's own conversion).
extern "C" void q_host_f16_bits(const float* x, long long n, uint16_t* out) {
    for (long long i = 0; i < n; ++i) out[i] = neon::q_f16_bits(x[i]);
}
