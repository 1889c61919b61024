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
// neon_cuda_matvec_multi on `st`, with y += result when `accumulate`.
int matvec(const neon_proj_target_t* targets, size_t n, const float* dX, size_t x_stride, size_t seq,
           cudaStream_t st, int accumulate);
int error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);
int launched(int n);  // count kernels launched outside the matvec path
bool pdl_enabled();
int device_sms(int device);
int check_device_error(int device);
}  // namespace neon_internal
