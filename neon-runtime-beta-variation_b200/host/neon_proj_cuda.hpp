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
// (rawllm_loader.hpp:367-386) gives them for the types this backend runs
// (0 for any other type).
inline size_t row_bytes(int ggml_type, size_t cols) {
    switch (ggml_type) {
        case NEON_GGML_F32: return cols * 4;
        case NEON_GGML_F16: case NEON_GGML_BF16: return cols * 2;
        case NEON_GGML_Q4_0: return cols / 32 * 18;
        case NEON_GGML_Q4_1: return cols / 32 * 20;
        case NEON_GGML_Q5_0: return cols / 32 * 22;
        case NEON_GGML_Q5_1: return cols / 32 * 24;
        case NEON_GGML_Q8_0: return cols / 32 * 34;
        case NEON_GGML_Q4_K: return cols / 256 * 144;
        case NEON_GGML_Q5_K: return cols / 256 * 176;
        case NEON_GGML_Q6_K: return cols / 256 * 210;
        default: return 0;
    }
}

// A 2-D weight type the backend multiplies (the eleven dequantize_row decodes,
// rawllm_forward.hpp:301-321).
inline bool runs_type(int ggml_type) { return row_bytes(ggml_type, 256) != 0; }

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

// Upload every 2-D weight tensor of a loader (GGUFLoader or NCTRLoader:
// anything with a `.tensors` vector of TensorInfo) once, at load time.
template <class LoaderT>
size_t upload_model(const LoaderT& loader) {
    size_t n = 0;
    for (const auto& t : loader.tensors) {
        const int ty = static_cast<int>(t.type);
        if (t.shape.size() == 2 && runs_type(ty)) {
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

// ---------------------------------------------------------------------------
// The decode step on the device (neon_cuda_model_*): replaces get_engine_state's
// ModelWeights + KVCache and the transformer_forward calls of run_generation
// (NEON-3.cpp:535-564, 676-759).
// ---------------------------------------------------------------------------

// engine::Config (rawllm_common.hpp:113-145) -> the C config. The KV cache
// holds cfg.kv_window positions when it is set, as get_engine_state sizes it
// (NEON-3.cpp:560), else cfg.ctx_len.
template <class ConfigT>
neon_model_config_t model_config(const ConfigT& c) {
    neon_model_config_t m{};
    m.n_vocab = c.n_vocab;
    m.n_embd = c.n_embd;
    m.n_layer = c.n_layer;
    m.n_head = c.n_head;
    m.n_kv_head = c.n_kv_head;
    m.head_dim = c.head_dim;
    m.n_ff = c.n_ff;
    m.ctx_len = c.kv_window ? c.kv_window : c.ctx_len;
    m.rope_base = c.rope_base;
    m.rope_scale = c.rope_scale;
    m.rope_dim_count = c.rope_dim_count;
    m.norm_eps = c.norm_eps;
    m.plain_ffn = c.use_swiglu ? 0u : 1u;
    return m;
}

// GGUF tensor name -> (NEON_ROLE_*, layer), for the names ModelWeights::build
// looks up (rawllm_forward.hpp:847-866); false for any other tensor.
inline bool tensor_role(const std::string& name, int* role, int* layer) {
    static const struct { const char* name; int role; } globals[] = {
        {"token_embd.weight", NEON_ROLE_TOKEN_EMBD}, {"output_norm.weight", NEON_ROLE_OUTPUT_NORM},
        {"output.weight", NEON_ROLE_OUTPUT}};
    static const struct { const char* suffix; int role; } per_layer[] = {
        {"attn_norm.weight", NEON_ROLE_ATTN_NORM}, {"attn_q.weight", NEON_ROLE_ATTN_Q},
        {"attn_k.weight", NEON_ROLE_ATTN_K},       {"attn_v.weight", NEON_ROLE_ATTN_V},
        {"attn_output.weight", NEON_ROLE_ATTN_OUT}, {"ffn_norm.weight", NEON_ROLE_FFN_NORM},
        {"ffn_gate.weight", NEON_ROLE_FFN_GATE},   {"ffn_up.weight", NEON_ROLE_FFN_UP},
        {"ffn_down.weight", NEON_ROLE_FFN_DOWN}};
    for (const auto& g : globals)
        if (name == g.name) {
            *role = g.role;
            *layer = -1;
            return true;
        }
    if (name.compare(0, 4, "blk.") != 0) return false;
    const size_t dot = name.find('.', 4);
    if (dot == std::string::npos || dot == 4) return false;
    int li = 0;
    for (size_t i = 4; i < dot; ++i) {
        if (name[i] < '0' || name[i] > '9') return false;
        li = li * 10 + (name[i] - '0');
    }
    const std::string rest = name.substr(dot + 1);
    for (const auto& p : per_layer)
        if (rest == p.suffix) {
            *role = p.role;
            *layer = li;
            return true;
        }
    return false;
}

// A decoder on the current device, or this rank's share of one split over the
// ranks of `comm` (every rank passes the whole loader; each keeps its shard).
class Decoder {
public:
    // `quantize_to` (a NEON_GGML_* type, -1 for none): float weight tensors --
    // a loader::NCTRLoader's, F32/F16 GGUF tensors -- are quantised on load to
    // that type, as the exporters' gguf-py would have written them.
    template <class ConfigT, class LoaderT>
    Decoder(const ConfigT& cfg, const LoaderT& loader, neon_comm_t comm = nullptr, int quantize_to = -1) {
        const neon_model_config_t c = model_config(cfg);
        check(neon_cuda_model_create_tp(&c, comm, &m_));
        try {
            if (quantize_to >= 0) check(neon_cuda_model_set_quantize(m_, quantize_to));
            for (const auto& t : loader.tensors) {
                int role = 0, layer = -1;
                if (!tensor_role(t.name, &role, &layer)) continue;
                if (role == NEON_ROLE_FFN_GATE && c.plain_ffn) continue;
                const size_t ne0 = (size_t)t.shape[0], ne1 = t.shape.size() > 1 ? (size_t)t.shape[1] : 0;
                check(neon_cuda_model_set_tensor(m_, role, layer, t.data_ptr, t.nbytes, static_cast<int>(t.type), ne0,
                                                 ne1));
            }
        } catch (...) {
            neon_cuda_model_free(m_);
            throw;
        }
    }
    ~Decoder() { neon_cuda_model_free(m_); }
    Decoder(const Decoder&) = delete;
    Decoder& operator=(const Decoder&) = delete;

    // fwd::transformer_forward: append `tokens` at positions length.., return
    // the logits of the last one.
    std::vector<float> forward(const std::vector<int32_t>& tokens, size_t n_vocab) {
        std::vector<float> logits(n_vocab);
        check(neon_cuda_model_forward(m_, tokens.data(), tokens.size(), logits.data()));
        return logits;
    }
    // run_generation's greedy loop: the prompt, then up to max_new tokens,
    // stopping before eos_id.
    std::vector<int32_t> generate(const std::vector<int32_t>& prompt, size_t max_new, int32_t eos_id) {
        std::vector<int32_t> out(max_new ? max_new : 1);
        size_t n = 0;
        check(neon_cuda_model_generate(m_, prompt.data(), prompt.size(), max_new, eos_id, out.data(), &n));
        out.resize(n);
        return out;
    }
    size_t length() const {
        size_t n = 0;
        check(neon_cuda_model_length(m_, &n));
        return n;
    }
    // KVCache::length rewind (run_generation's prefix reuse, NEON-3.cpp:690-703)
    void set_length(size_t n) { check(neon_cuda_model_set_length(m_, n)); }
    // fwd::kv_cache_shift: ensure_cache_room's slide of the window (NEON-3.cpp:590-630)
    void kv_shift(size_t keep, size_t discard) { check(neon_cuda_model_kv_shift(m_, keep, discard)); }
    neon_model_t handle() const { return m_; }

private:
    neon_model_t m_ = nullptr;
};

}  // namespace neon_cuda
