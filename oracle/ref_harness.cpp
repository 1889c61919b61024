// ref_harness.cpp -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
//
// A C-ABI shim around the reference's OWN CPU implementation of the quantized
// matvec path. It #includes rawllm_forward.hpp from the reference tree at
// compile time (oracle/Makefile passes -I to that tree) and is built with the
// reference's own compiler flags (nanity.html:2504-2510: g++ -std=c++17 -O3
// -mavx2 -mfma -lpthread) into oracle/_ref/libneon_ref.so. No reference source
// is copied into this repository; the built library is git-ignored.
//
// It is used (a) to pin the C restatement in oracle/neon_oracle.c bit-for-bit,
// (b) to generate the golden vectors in tests/golden/, and (c) as the timed
// CPU baseline ("kind": "reference") in bench.py, with the reference's
// util::ThreadPool at the host's core count.
#include "rawllm_forward.hpp"

#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

int fail(const std::exception& e) {
    g_err = e.what();
    return -1;
}

loader::TensorInfo make_tensor(const uint8_t* bytes, int type, size_t rows, size_t cols,
                               const char* name) {
    loader::TensorInfo t;
    t.name = name ? name : "w";
    t.shape = {(uint64_t)cols, (uint64_t)rows};
    t.type = static_cast<loader::GGMLType>(type);
    t.file_offset = 0;
    t.nbytes = loader::GGUFLoader::bytes_for_type(t.type, cols) * rows;
    t.data_ptr = bytes;
    return t;
}

}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

int ref_has_avx2(void) {
#if defined(RAWLLM_AVX2)
    return 1;
#else
    return 0;
#endif
}

// util::ThreadPool (rawllm_util.hpp:24-101), kept alive across calls so that
// timing does not include thread start-up.
void* ref_pool_new(int n_threads) { return new util::ThreadPool(n_threads); }
void ref_pool_free(void* pool) { delete static_cast<util::ThreadPool*>(pool); }
int ref_pool_size(void* pool) { return static_cast<util::ThreadPool*>(pool)->size(); }

float ref_fp16_to_fp32(uint16_t h) { return fwd::fp16_to_fp32(h); }

// fwd::quantize_rows_q8_0, rawllm_forward.hpp:360-381.
void ref_quantize_rows_q8_0(const float* X, size_t x_stride, size_t cols, size_t seq,
                            float* d_out, int8_t* q_out) {
    fwd::quantize_rows_q8_0(X, x_stride, cols, seq, d_out, q_out);
}

// block_isum_avx2 (AVX2 build) / block_isum_scalar, rawllm_forward.hpp:384-412.
int32_t ref_block_isum(const uint8_t* qs, const int8_t* xq) {
#if defined(RAWLLM_AVX2)
    return fwd::detail_q4_0_fused::block_isum_avx2(qs, xq);
#else
    return fwd::detail_q4_0_fused::block_isum_scalar(qs, xq);
#endif
}

int32_t ref_block_isum_scalar(const uint8_t* qs, const int8_t* xq) {
    return fwd::detail_q4_0_fused::block_isum_scalar(qs, xq);
}

// fwd::dot_q4_0_q8_0, rawllm_forward.hpp:419-434.
float ref_dot_q4_0_q8_0(const uint8_t* w, const float* x_d, const int8_t* x_q, size_t cols) {
    return fwd::dot_q4_0_q8_0(w, x_d, x_q, cols);
}

// fwd::dot_f32, rawllm_forward.hpp:446-479.
float ref_dot_f32(const float* a, const float* b, size_t n) { return fwd::dot_f32(a, b, n); }

// fwd::dequantize_row, rawllm_forward.hpp:301-321.
int ref_dequantize_row(int type, const uint8_t* p, size_t n, float* out) {
    try {
        fwd::dequantize_row(static_cast<loader::GGMLType>(type), p, n, out);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// fwd::proj_all_positions, rawllm_forward.hpp:522-609, on one in-memory tensor.
int ref_proj_all_positions(void* pool, const uint8_t* W, int type, size_t rows, size_t cols,
                           const float* X, size_t x_stride, float* Y, size_t y_stride,
                           size_t seq) {
    try {
        loader::TensorInfo t = make_tensor(W, type, rows, cols, "w");
        fwd::proj_all_positions(t, X, x_stride, Y, y_stride, seq,
                                *static_cast<util::ThreadPool*>(pool));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// fwd::proj_all_positions_multi, rawllm_forward.hpp:632-726.
int ref_proj_all_positions_multi(void* pool, size_t n_targets, const uint8_t* const* Ws,
                                 const int* types, const size_t* rows, const size_t* cols,
                                 float* const* Ys, const size_t* y_strides, const float* X,
                                 size_t x_stride, size_t seq) {
    try {
        std::vector<loader::TensorInfo> ts;
        ts.reserve(n_targets);
        for (size_t i = 0; i < n_targets; ++i)
            ts.push_back(make_tensor(Ws[i], types[i], rows[i], cols[i], "w"));
        std::vector<fwd::ProjTarget> targets;
        for (size_t i = 0; i < n_targets; ++i) targets.push_back({&ts[i], Ys[i], y_strides[i]});
        fwd::proj_all_positions_multi(targets, X, x_stride, seq,
                                      *static_cast<util::ThreadPool*>(pool));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

}  // extern "C"
