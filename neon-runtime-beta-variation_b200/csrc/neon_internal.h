// neon_internal.h -- declarations shared by the library's translation units;
// nothing here is exported from libneon_cuda.so.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "neon_cuda.h"

// A device-resident weight tensor (or tensor-parallel shard). Q4_0 / Q8_0 use
// the split layout: payload plane rows x nb x P bytes, then fp16 scales
// rows x nb (pitch 0). The other types keep the GGUF rows, each padded to a
// 16-byte pitch (d null; nb counts 32-value sub-blocks, cols rounded up).
struct neon_tensor {
    int device;
    int type;
    size_t rows, cols, nb;
    uint8_t* base;  // single allocation: payload plane, then scale plane
    uint8_t* qs;
    uint16_t* d;
    size_t bytes;
    size_t pitch;   // bytes per row of the padded-row layout; 0 for the split layout
};

// Tensor-parallel communicator: one per rank (process, device). Every rank
// owns a buffer in its own HBM, exported with CUDA IPC and opened by all
// peers; collectives push data into the peers' buffers with plain P2P stores.
// Two protocols share the buffer:
//  - bulk (comm kernel, any size): data, then a system-scope fence and a
//    released epoch flag per slice; readers acquire the flag, then the data;
//  - low latency ("LL", decode-sized vectors): every 8-byte word carries a
//    value and the call number that wrote it, so no fence or flag is needed --
//    a reader polls a word until the number is the one it expects (one 8-byte
//    store is single-copy atomic, so value and number arrive together).
constexpr int kCommMaxRanks = 8;
constexpr int kCommSlices = 32;         // CTAs of the bulk all-reduce kernel (one flag each)
constexpr int kCommFusedFloats = 65536; // LL slot: one position's vector (n_embd), at most

struct CommPeers {  // passed to kernels by value
    unsigned char* base[kCommMaxRanks];  // each rank's buffer, mapped here (own: base[rank])
    int rank, world;
    long long max_floats;                // capacity of one bulk receive slot, in floats
};

// Buffer layout (bytes from base):
//   bulk slots  [parity][src][max_floats] f32
//   bulk flags  [src][slice] u32
//   LL slots    [parity][src][kCommFusedFloats] u64   (comm_ll_off)
//   LL keys     [parity][src][2] u64                  (argmax exchange)
__host__ __device__ inline long long comm_recv_off(const CommPeers& c, int parity, int src) {
    return ((long long)parity * c.world + src) * c.max_floats * 4;
}
__host__ __device__ inline long long comm_flags_off(const CommPeers& c) { return 2LL * c.world * c.max_floats * 4; }
__host__ __device__ inline long long comm_ll_off(const CommPeers& c) {
    return (comm_flags_off(c) + (long long)kCommMaxRanks * kCommSlices * 4 + 255) & ~255LL;
}
// offsets inside the LL region
__host__ __device__ inline long long ll_slot_off(int world, int parity, int src) {
    return ((long long)parity * world + src) * kCommFusedFloats * 8;
}
__host__ __device__ inline long long ll_keys_off(int world) { return 2LL * world * kCommFusedFloats * 8; }
__host__ __device__ inline long long comm_bytes(const CommPeers& c) {
    return comm_ll_off(c) + ll_keys_off(c.world) + 2LL * kCommMaxRanks * 2 * 8 + 256;
}

// An LL word: the value's bits, and the call number in the high half.
__host__ __device__ inline unsigned long long ll_pack(float v, unsigned int call) {
    union { float f; unsigned int u; } b;
    b.f = v;
    return ((unsigned long long)call << 32) | b.u;
}

// What a matvec launch needs to produce a fused (LL) all-reduce: the
// column-split projection (attn_output / ffn_down of one position) stores
// each row as an LL word into slot [parity][rank] of every rank; the
// communicator's LL reduce kernel then polls the words of all ranks' slots
// and adds slot_0 + slot_1 + ... (the bulk kernel's order, bit for bit) into
// the residual, and records the call as completed.
struct PeerSet {
    unsigned char* base[kCommMaxRanks];  // every rank's LL region (this process's mappings)
    unsigned int* calls;                 // this rank's count of completed LL collectives (device)
    unsigned int* counter;               // last-CTA election of the reduce kernel (device)
    unsigned int* err;                   // the communicator's error word
    unsigned long long timeout_ns;
    int rank, world;
};

struct neon_comm_impl {
    int device = 0;
    CommPeers peers{};
    unsigned char* local = nullptr;        // this rank's buffer
    unsigned int* epochs = nullptr;        // device: per-slice call counts, then the key-exchange count,
                                           // the fused collectives' count and their last-CTA counter
    unsigned int* err = nullptr;           // device error word: bit 0 = a peer wait timed out
    unsigned long long timeout_ns = 4000000000ull;  // bound of every wait on a peer
    bool connected = false;
    bool opened_ipc = false;               // peers' buffers were opened with CUDA IPC
    std::string ipc_handle;                // cudaIpcMemHandle_t bytes
};
struct neon_comm : neon_comm_impl {};  // the public handle type (neon_comm_t)

namespace neon_internal {

// out[i] (+)= sum over ranks, in rank order, of in[i] for i < n, on stream `st`.
int comm_allreduce(neon_comm_impl* c, const float* in, float* out, long long n, int add, cudaStream_t st);
// out[n*r/world .. n*(r+1)/world) = rank r's `in` (its shard of the n rows), for every r.
int comm_allgather(neon_comm_impl* c, const float* in, float* out, long long n, cudaStream_t st);
// Greedy-sampling exchange: every rank's argmax key (*key, the packed
// (value, index) of argmax_kernel) is compared; the winner's index becomes
// *d_tok and out[*d_step]; *d_step += 1, *d_pos += advance, *key = 0.
int comm_argmax(neon_comm_impl* c, unsigned long long* key, int* d_tok, int* out, int* d_step, int* d_pos,
                int advance, cudaStream_t st);
// The fused-collective view of a connected communicator.
PeerSet comm_peer_set(neon_comm_impl* c);
// Completes a fused all-reduce a producing matvec started: h[i] += slot_0[i]
// + slot_1[i] + ... for i < n, waiting (bounded) for every rank's words.
// wait_producer false: no dependency wait (the LL words are the
// synchronisation; worth it when the producer is a long launch)
int comm_ll_reduce(neon_comm_impl* c, float* h, long long n, cudaStream_t st, bool wait_producer = true);
// Completes a fused all-gather the producing row-shard matvecs started:
// y[i] = the gather slot's word i for i < n, waiting (bounded) for each.
int comm_ll_gather(neon_comm_impl* c, float* y, long long n, cudaStream_t st);
bool fused_collectives();
// neon_cuda_set_prefill_mma: prompt passes on the tensor-core kernels.
bool prefill_mma();

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
    // produce a fused collective (one target, one position) instead of
    // storing Y: 1 (all-reduce) the rows go as LL words to this rank's slot on
    // every rank; 2 (all-gather) each row r goes as an LL word to position
    // gather_row0 + r of the gather slot on every rank
    int peer_mode = 0;
    long long gather_row0 = 0;
    PeerSet peer{};
    // set to true when the call ran on the streaming kernel (a long launch,
    // whose tail a following LL reduce may overlap); left alone otherwise
    bool* launched_stream = nullptr;
};

// neon_cuda_matvec_multi on `st`, with y += result when `accumulate`.
int matvec(const neon_proj_target_t* targets, size_t n, const float* dX, size_t x_stride, size_t seq,
           cudaStream_t st, int accumulate, const MatvecExt* ext = nullptr);

int error(int code, const std::string& msg);
// Bytes of one GGUF row of `type` with `cols` values (0: unsupported type, or
// cols not a multiple of the type's block size). rawllm_loader.hpp:367-386.
size_t gguf_row_bytes(int type, size_t cols);
// Values per block of `type` (block_size_for, rawllm_forward.hpp:289-299); 0 if unsupported.
size_t gguf_block_elems(int type);
// n values of a host row of `type`, decoded bit for bit as the reference's
// dequantize_row does (rawllm_forward.hpp:301-321); false if n or the type
// does not fit.
bool dequantize_row_host(int type, const uint8_t* p, size_t n, float* out);
// h[t] = row toks[t] of a padded-row (non Q4_0/Q8_0) embedding, decoded; a
// token id out of range sets bit 1 of *err. seq rows of n_embd floats.
int embed_rows(const neon_tensor* E, const int* toks, int seq, int n_embd, int n_vocab, float* h, unsigned int* err,
               cudaStream_t st);
int cuda_error(cudaError_t e, const char* what);
int launched(int n);  // count kernels launched outside the matvec path
bool pdl_enabled();
int device_sms(int device);
int check_device_error(int device);
}  // namespace neon_internal
