// neon_internal.h -- declarations shared by the library's translation units;
// nothing here is exported from libneon_cuda.so.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "neon_cuda.h"

// A device-resident weight tensor (or tensor-parallel shard) in the split
// layout: payload plane rows x nb x P bytes, then fp16 scales rows x nb.
struct neon_tensor {
    int device;
    int type;
    size_t rows, cols, nb;
    uint8_t* base;  // single allocation: payload plane, then scale plane
    uint8_t* qs;
    uint16_t* d;
    size_t bytes;
};

namespace neon_internal {

// Decode-step options of a one-position matvec launch (seq == 1 only):
// RMSNorm of X folded into the X staging, and per-target epilogues (the
// kEpi* values of neon_kernels.cuh: plain store, RoPE pairs stored at the
// position's cache row, store at the position's cache row, SwiGLU pairs).
struct MatvecExt {
    const float* norm_w = nullptr;
    float norm_eps = 0.f;
    const int* d_pos = nullptr;
    const float2* rope_cs = nullptr;
    int rope_half = 0;
    int head_dim = 0;
    const int* epi = nullptr;               // per target; null: plain store
    const long long* pos_stride = nullptr;  // per target
};

// neon_cuda_matvec_multi on `st`, with y += result when `accumulate`.
int matvec(const neon_proj_target_t* targets, size_t n, const float* dX, size_t x_stride, size_t seq,
           cudaStream_t st, int accumulate, const MatvecExt* ext = nullptr);
int error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);
int launched(int n);  // count kernels launched outside the matvec path
bool pdl_enabled();
int device_sms(int device);
int check_device_error(int device);
}  // namespace neon_internal
