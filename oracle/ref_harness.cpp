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

// ---------------------------------------------------------------------------
// Decode step: the reference's own transformer_forward (rawllm_forward.hpp:
// 987-1236) on a model held in memory. Tensor roles and their numbering match
// include/neon_cuda.h's NEON_ROLE_* values.
// ---------------------------------------------------------------------------
namespace {

enum Role { TOKEN_EMBD = 0, OUTPUT_NORM = 1, OUTPUT = 2, ATTN_NORM = 3, ATTN_Q = 4, ATTN_K = 5, ATTN_V = 6,
            ATTN_OUT = 7, FFN_NORM = 8, FFN_GATE = 9, FFN_UP = 10, FFN_DOWN = 11 };

struct RefModel {
    engine::Config cfg;
    std::vector<std::vector<uint8_t>> blobs;           // owned tensor bytes
    std::vector<std::unique_ptr<loader::TensorInfo>> tensors;
    fwd::ModelWeights mw;
    fwd::KVCache cache;
};

}  // namespace

extern "C" {

typedef struct {
    uint32_t n_vocab, n_embd, n_layer, n_head, n_kv_head, head_dim, n_ff, ctx_len;
    float rope_base, rope_scale;
    uint32_t rope_dim_count;
    float norm_eps;
    uint32_t plain_ffn;
} ref_config_t;

void* ref_model_new(const ref_config_t* c) {
    auto* m = new RefModel();
    m->cfg.n_vocab = c->n_vocab;
    m->cfg.n_embd = c->n_embd;
    m->cfg.n_layer = c->n_layer;
    m->cfg.n_head = c->n_head;
    m->cfg.n_kv_head = c->n_kv_head;
    m->cfg.head_dim = c->head_dim;
    m->cfg.n_ff = c->n_ff;
    m->cfg.ctx_len = c->ctx_len;
    m->cfg.kv_window = c->ctx_len;
    m->cfg.rope_base = c->rope_base;
    m->cfg.rope_scale = c->rope_scale;
    m->cfg.rope_dim_count = c->rope_dim_count;
    m->cfg.norm_eps = c->norm_eps;
    m->cfg.use_swiglu = c->plain_ffn == 0;
    m->mw.layers.resize(c->n_layer);
    m->cache = fwd::KVCache(c->n_layer, (size_t)c->n_kv_head * c->head_dim, c->ctx_len);
    return m;
}

void ref_model_free(void* p) { delete static_cast<RefModel*>(p); }

// Copies `nbytes` of tensor data; shape is GGUF ne (ne1 == 0 for a 1-D tensor).
int ref_model_set(void* p, int role, int layer, const uint8_t* bytes, size_t nbytes, int type, size_t ne0,
                  size_t ne1) {
    auto* m = static_cast<RefModel*>(p);
    m->blobs.emplace_back(bytes, bytes + nbytes);
    auto t = std::make_unique<loader::TensorInfo>();
    t->name = "role" + std::to_string(role) + "." + std::to_string(layer);
    t->shape = ne1 ? std::vector<uint64_t>{ne0, ne1} : std::vector<uint64_t>{ne0};
    t->type = static_cast<loader::GGMLType>(type);
    t->nbytes = nbytes;
    t->data_ptr = m->blobs.back().data();
    const loader::TensorInfo* tp = t.get();
    m->tensors.push_back(std::move(t));
    if (role <= OUTPUT) {
        if (role == TOKEN_EMBD) m->mw.token_embd = tp;
        if (role == OUTPUT_NORM) m->mw.output_norm = tp;
        if (role == OUTPUT) m->mw.output = tp;
        return 0;
    }
    if (layer < 0 || (size_t)layer >= m->mw.layers.size()) return -1;
    auto& L = m->mw.layers[layer];
    switch (role) {
        case ATTN_NORM: L.attn_norm = tp; break;
        case ATTN_Q: L.attn_q = tp; break;
        case ATTN_K: L.attn_k = tp; break;
        case ATTN_V: L.attn_v = tp; break;
        case ATTN_OUT: L.attn_out = tp; break;
        case FFN_NORM: L.ffn_norm = tp; break;
        case FFN_GATE: L.ffn_gate = tp; break;
        case FFN_UP: L.ffn_up = tp; break;
        case FFN_DOWN: L.ffn_down = tp; break;
        default: return -1;
    }
    return 0;
}

// fwd::transformer_forward on `n` new tokens; logits of the last one.
int ref_model_forward(void* p, void* pool, const int32_t* tokens, size_t n, float* logits) {
    auto* m = static_cast<RefModel*>(p);
    try {
        std::vector<int32_t> t(tokens, tokens + n);
        fwd::transformer_forward(m->cfg, m->mw, t, m->cache, logits, *static_cast<util::ThreadPool*>(pool));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

size_t ref_model_length(void* p) { return static_cast<RefModel*>(p)->cache.length; }
void ref_model_set_length(void* p, size_t len) { static_cast<RefModel*>(p)->cache.length = len; }

// fwd::kv_cache_shift (rawllm_forward.hpp:949-969) on the model's cache, with
// the freqs ensure_cache_room builds (NEON-3.cpp:618-624).
void ref_model_kv_shift(void* p, size_t keep, size_t discard) {
    auto* m = static_cast<RefModel*>(p);
    const auto& c = m->cfg;
    const std::vector<float> freqs = fwd::rope_make_freqs(c.head_dim, c.rope_base);
    const size_t rope_half = c.rope_dim_count ? c.rope_dim_count / 2 : c.head_dim / 2;
    fwd::kv_cache_shift(m->cache, keep, discard, c.n_kv_head, c.head_dim, rope_half, c.rope_scale, freqs.data());
}

// K/V cache rows of one layer (kv_dim floats each) for positions [0, n).
void ref_model_kv(void* p, int layer, size_t n, float* k, float* v) {
    auto* m = static_cast<RefModel*>(p);
    const size_t kvd = m->cache.kv_dim;
    std::memcpy(k, m->cache.k_row(layer, 0), n * kvd * sizeof(float));
    std::memcpy(v, m->cache.v_row(layer, 0), n * kvd * sizeof(float));
}

// Building blocks, exposed for pinning the C restatement.
float ref_fast_expf(float x) { return engine::fast_expf(x); }
float ref_silu(float x) { return fwd::silu(x); }
void ref_rms_norm(const float* x, const float* w, float* out, size_t n, float eps) { fwd::rms_norm(x, w, out, n, eps); }
void ref_rope_freqs(size_t head_dim, float base, float* out) {
    auto f = fwd::rope_make_freqs(head_dim, base);
    std::memcpy(out, f.data(), f.size() * sizeof(float));
}
void ref_rope_apply(float* vec, size_t n_heads, size_t head_dim, size_t rope_half, size_t pos, float rope_scale,
                    const float* freqs) {
    fwd::rope_apply(vec, n_heads, head_dim, rope_half, pos, rope_scale, freqs);
}
void ref_axpy_f32(float* out, float w, const float* v, size_t n) { fwd::axpy_f32(out, w, v, n); }

}  // extern "C"

// ---------------------------------------------------------------------------
// The reference's .nctr reader, loader::NCTRLoader (rawllm_nctr_loader.hpp),
// behind a C ABI: open, validate_config, and the positional tensor table, so
// the tests can check that the package's reader sees the same tensors, the
// same configuration and the same errors.
// ---------------------------------------------------------------------------
#include "rawllm_nctr_loader.hpp"

extern "C" {

// NCTRLoader::open (rawllm_nctr_loader.hpp:87-137); null and ref_last_error() on a throw.
void* ref_nctr_open(const char* path) {
    auto* l = new loader::NCTRLoader();
    try {
        l->open(path);
        return l;
    } catch (const std::exception& e) {
        delete l;
        fail(e);
        return nullptr;
    }
}

void ref_nctr_free(void* h) { delete static_cast<loader::NCTRLoader*>(h); }

size_t ref_nctr_count(void* h) { return static_cast<loader::NCTRLoader*>(h)->tensors.size(); }

// Tensor i: its name (into name, cap bytes), GGUF shape (ne0, ne1; ne1 = 0 for
// 1-D), type, absolute file offset and byte count.
int ref_nctr_tensor(void* h, size_t i, char* name, size_t cap, uint64_t* ne0, uint64_t* ne1, int* type,
                    uint64_t* offset, uint64_t* nbytes) {
    const auto& t = static_cast<loader::NCTRLoader*>(h)->tensors.at(i);
    std::snprintf(name, cap, "%s", t.name.c_str());
    *ne0 = t.shape.size() > 0 ? t.shape[0] : 0;
    *ne1 = t.shape.size() > 1 ? t.shape[1] : 0;
    *type = static_cast<int>(t.type);
    *offset = t.file_offset;
    *nbytes = t.nbytes;
    return 0;
}

// NCTRLoader::validate_config (:146-184) into a ref_config_t (ctx_len = the
// resulting kv_window; plain_ffn = !use_swiglu); -1 on a throw.
int ref_nctr_config(void* h, ref_config_t* c, uint32_t* header_ctx_len, int* bos, int* eos, size_t* n_tokens) {
    try {
        engine::Config cfg;
        static_cast<loader::NCTRLoader*>(h)->validate_config(cfg);
        c->n_vocab = cfg.n_vocab;
        c->n_embd = cfg.n_embd;
        c->n_layer = cfg.n_layer;
        c->n_head = cfg.n_head;
        c->n_kv_head = cfg.n_kv_head;
        c->head_dim = cfg.head_dim;
        c->n_ff = cfg.n_ff;
        c->ctx_len = cfg.kv_window;
        c->rope_base = cfg.rope_base;
        c->rope_scale = cfg.rope_scale;
        c->rope_dim_count = cfg.rope_dim_count;
        c->norm_eps = cfg.norm_eps;
        c->plain_ffn = cfg.use_swiglu ? 0 : 1;
        *header_ctx_len = cfg.ctx_len;
        const auto& tm = static_cast<loader::NCTRLoader*>(h)->tok_meta;
        *bos = tm.bos_id;
        *eos = tm.eos_id;
        *n_tokens = tm.tokens.size();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The reference's GGUF reader, loader::GGUFLoader (rawllm_loader.hpp:84-330),
// behind the same C ABI as the .nctr one.
// ---------------------------------------------------------------------------
extern "C" {

void* ref_gguf_open(const char* path) {
    auto* l = new loader::GGUFLoader();
    try {
        l->open(path);
        return l;
    } catch (const std::exception& e) {
        delete l;
        fail(e);
        return nullptr;
    }
}

void ref_gguf_free(void* h) { delete static_cast<loader::GGUFLoader*>(h); }

size_t ref_gguf_count(void* h) { return static_cast<loader::GGUFLoader*>(h)->tensors.size(); }

// Tensor i: name, GGUF shape (ne0, ne1), type, the distance of its data from
// tensor 0's data (bytes), and its byte count.
int ref_gguf_tensor(void* h, size_t i, char* name, size_t cap, uint64_t* ne0, uint64_t* ne1, int* type,
                    int64_t* rel_offset, uint64_t* nbytes) {
    auto* l = static_cast<loader::GGUFLoader*>(h);
    const auto& t = l->tensors.at(i);
    std::snprintf(name, cap, "%s", t.name.c_str());
    *ne0 = t.shape.size() > 0 ? t.shape[0] : 0;
    *ne1 = t.shape.size() > 1 ? t.shape[1] : 0;
    *type = static_cast<int>(t.type);
    *rel_offset = (int64_t)(t.data_ptr - l->tensors.at(0).data_ptr);
    *nbytes = t.nbytes;
    return 0;
}

// validate_config into a ref_config_t (ctx_len = kv_window); -1 on a throw.
int ref_gguf_config(void* h, ref_config_t* c, uint32_t* header_ctx_len, int* bos, int* eos) {
    try {
        engine::Config cfg;
        auto* l = static_cast<loader::GGUFLoader*>(h);
        l->validate_config(cfg);
        c->n_vocab = cfg.n_vocab;
        c->n_embd = cfg.n_embd;
        c->n_layer = cfg.n_layer;
        c->n_head = cfg.n_head;
        c->n_kv_head = cfg.n_kv_head;
        c->head_dim = cfg.head_dim;
        c->n_ff = cfg.n_ff;
        c->ctx_len = cfg.kv_window;
        c->rope_base = cfg.rope_base;
        c->rope_scale = cfg.rope_scale;
        c->rope_dim_count = cfg.rope_dim_count;
        c->norm_eps = cfg.norm_eps;
        c->plain_ffn = cfg.use_swiglu ? 0 : 1;
        *header_ctx_len = cfg.ctx_len;
        *bos = l->tok_meta.bos_id;
        *eos = l->tok_meta.eos_id;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

}  // extern "C"
