// neon_proj_cuda.hpp -- C++ drop-in for NEON's matvec operator surface over the
// CUDA C ABI (include/neon_cuda.h).
//
// The NEON runtime calls, for every projection of transformer_forward():
//   fwd::proj_all_positions(const loader::TensorInfo& W, const float* X,
//       size_t x_stride, float* Y, size_t y_stride, size_t seq,
//       util::ThreadPool& pool)                         rawllm_forward.hpp:522-525
//   fwd::proj_all_positions_multi(const std::vector<ProjTarget>& targets,
//       const float* X, size_t x_stride, size_t seq,
//       util::ThreadPool& pool)                         rawllm_forward.hpp:632-634
// neon_cuda::proj_all_positions[_multi] below take the same arguments with the
// same meaning (host X and Y, blocking, std::runtime_error on a bad argument
// with the reference's wording) and run the projection on the GPU. They are
// templates over the tensor-handle and pool types, so the header depends on
// no reference header: any type with the public fields of loader::TensorInfo
// (name, shape, type, data_ptr; rawllm_loader.hpp:34-41) works, and the pool
// argument is accepted and ignored (the GPU grid replaces the CPU pool).
//
// Weights are uploaded to HBM the first time a TensorInfo is seen (or all at
// once with upload_model(), the load-time hook of ModelWeights::build /
// get_engine_state, rawllm_forward.hpp:847, NEON-3.cpp:558-562) and are kept
// in a side table keyed by the TensorInfo's address for the process lifetime.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "neon_cuda.h"

namespace neon_cuda {

inline void check(int rc) {
    if (rc != NEON_OK) throw std::runtime_error(neon_cuda_last_error());
}

// Bytes of one GGUF row, as loader::GGUFLoader::bytes_for_type
// (rawllm_loader.hpp:367-386) gives them for the types this backend runs.
inline size_t row_bytes(int ggml_type, size_t cols) {
    if (ggml_type == NEON_GGML_Q4_0) return cols / 32 * 18;
    if (ggml_type == NEON_GGML_Q8_0) return cols / 32 * 34;
    return 0;
}

// Side table TensorInfo address -> device tensor.
class TensorTable {
public:
    ~TensorTable() { clear(); }

    template <class TensorInfoT>
    neon_tensor_t get(const TensorInfoT& W) {
        std::lock_guard<std::mutex> lk(mu_);
        auto it = map_.find(static_cast<const void*>(&W));
        if (it != map_.end()) return it->second;
        check_shape(W);
        const size_t cols = (size_t)W.shape[0], rows = (size_t)W.shape[1];
        neon_tensor_t h = nullptr;
        check(neon_cuda_upload(W.data_ptr, static_cast<int>(W.type), rows, cols, NEON_SHARD_NONE, 0, 1, &h));
        map_.emplace(static_cast<const void*>(&W), h);
        return h;
    }

    void clear() {
        std::lock_guard<std::mutex> lk(mu_);
        for (auto& kv : map_) neon_cuda_free(kv.second);
        map_.clear();
    }

    size_t size() const { return map_.size(); }

    // The reference's argument checks (rawllm_forward.hpp:527-534).
    template <class TensorInfoT>
    static void check_shape(const TensorInfoT& W) {
        if (W.shape.size() < 2)
            throw std::runtime_error("forward(): expected a 2D weight tensor: " + W.name);
        const size_t cols = (size_t)W.shape[0];
        const int t = static_cast<int>(W.type);
        const size_t bs = (t == NEON_GGML_F32 || t == NEON_GGML_F16 || t == 30) ? 1
                          : (t >= 12 && t <= 14)                                 ? 256
                                                                                 : 32;
        if (cols % bs != 0)
            throw std::runtime_error("forward(): " + W.name + " input dim (" + std::to_string(cols) +
                                     ") isn't a multiple of its quant block size (" + std::to_string(bs) +
                                     ") — can't dequantize safely.");
    }

private:
    std::mutex mu_;
    std::unordered_map<const void*, neon_tensor_t> map_;
};

inline TensorTable& tensors() {
    static TensorTable t;
    return t;
}

// Upload every 2-D Q4_0/Q8_0 tensor of a loader (GGUFLoader or NCTRLoader:
// anything with a `.tensors` vector of TensorInfo) once, at load time.
template <class LoaderT>
size_t upload_model(const LoaderT& loader) {
    size_t n = 0;
    for (const auto& t : loader.tensors) {
        const int ty = static_cast<int>(t.type);
        if (t.shape.size() == 2 && (ty == NEON_GGML_Q4_0 || ty == NEON_GGML_Q8_0)) {
            tensors().get(t);
            ++n;
        }
    }
    return n;
}

// fwd::proj_all_positions on the GPU (rawllm_forward.hpp:522-609).
template <class TensorInfoT, class PoolT>
void proj_all_positions(const TensorInfoT& W, const float* X, size_t x_stride, float* Y, size_t y_stride,
                        size_t seq, PoolT& /*pool*/) {
    neon_tensor_t h = tensors().get(W);
    check(neon_cuda_proj_all_positions(h, X, x_stride, Y, y_stride, seq));
}

// fwd::proj_all_positions_multi on the GPU (rawllm_forward.hpp:632-726).
// ProjTargetT has the public fields of fwd::ProjTarget: W (TensorInfo*), Y, y_stride.
template <class ProjTargetT, class PoolT>
void proj_all_positions_multi(const std::vector<ProjTargetT>& targets, const float* X, size_t x_stride,
                              size_t seq, PoolT& /*pool*/) {
    std::vector<neon_proj_target_t> t;
    t.reserve(targets.size());
    for (const auto& tg : targets) t.push_back({tensors().get(*tg.W), tg.Y, tg.y_stride});
    check(neon_cuda_proj_all_positions_multi(t.data(), t.size(), X, x_stride, seq));
}

}  // namespace neon_cuda
