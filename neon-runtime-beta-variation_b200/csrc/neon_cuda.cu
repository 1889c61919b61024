// neon_cuda.cu -- C ABI of the sm_100a quantized matvec backend (see
// include/neon_cuda.h for the contract of every entry point).
#include "neon_cuda.h"
#include "neon_internal.h"
#include "neon_kernels.cuh"
#include "neon_dequant.cuh"
#include "neon_quant.cuh"
#include "neon_prefill.cuh"
#include "neon_resident.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

using namespace neon;

namespace {

constexpr int kMaxDevices = 64;
// Rows per warp tile and positions per CTA of the multi-position kernel.
constexpr int kMpR = 2, kMpT = 4;
// Shared memory a streaming launch may use, and the target bytes of one ring
// stage (weights of one item).
constexpr int kMaxSmem = 220 * 1024;
constexpr int kStageTarget = 40 * 1024;
// Stage target of the streaming (one-position Q4_0 / Q8_0) kernel's tiles:
// a tile sweep on B200 put the best tile at 64-80 KB on every large shape
// (e.g. Q4_0 28672x8192: 16-row tiles; Q8_0 4096x14336: 4-row tiles).
constexpr int kStreamStageTarget = 80 * 1024;
// Resident streaming CTAs per SM the grid is sized for.
constexpr int kStreamCtasPerSm = 4;

thread_local std::string g_err;
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_pdl{1};
std::atomic<int> g_prefill_mma{1};  // neon_cuda_set_prefill_mma
std::atomic<int> g_dq_ring{-1};     // neon_cuda_set_dq_ring: 1 on, 0 off, -1 the types it is faster for
std::atomic<int> g_tile_rc{0}, g_tile_kc{0};  // neon_cuda_set_stream_tiles (0: the planner's choice)
std::atomic<int> g_resident{1};  // neon_cuda_set_resident: CTAs per SM of a resident launch (0: off)

struct DeviceState {
    bool ready = false;
    int sms = 0;
    int smem_per_sm = 0;  // shared memory of one SM (bytes)
    unsigned int* err = nullptr;  // device error word (g_neon_device_err on this device)
    unsigned int* err_host = nullptr;  // pinned copy of the error word, read back by the host-buffer calls
    std::mutex mu;
    // scratch of multi-position Q4_0 calls (activation quants)
    int8_t* xq = nullptr;
    float* xd = nullptr;
    int* xs = nullptr;
    size_t scratch_cols = 0;  // capacity in seq*cols elements
    // staging of the host-buffer calls
    cudaStream_t stream = nullptr;
    float* dx = nullptr;
    float* dy = nullptr;
    size_t dx_cap = 0, dy_cap = 0;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_init_mu;
}  // namespace

// Device-side error word: bit 0 = a bounded wait in a kernel timed out.
static __device__ unsigned int g_neon_device_err;

namespace {

int set_err(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

int cuda_err(cudaError_t e, const char* what) {
    return set_err(NEON_ERR_CUDA, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}
// NEON_OK for cudaSuccess, else the error as cuda_err reports it.
int cuda_check(cudaError_t e, const char* what) { return e == cudaSuccess ? NEON_OK : cuda_err(e, what); }

#define NEON_CUDA_TRY(call)                                      \
    do {                                                         \
        cudaError_t _e = (call);                                 \
        if (_e != cudaSuccess) return cuda_err(_e, #call);       \
    } while (0)

size_t payload_bytes(int type) { return type == NEON_GGML_Q4_0 ? 16 : 32; }
size_t gguf_block_bytes(int type) { return type == NEON_GGML_Q4_0 ? 18 : 34; }
bool split_type(int type) { return type == NEON_GGML_Q4_0 || type == NEON_GGML_Q8_0; }
// The types of the dequantising kernel (padded-row layout).
bool dq_type(int type) {
    int be, bb, cb;
    dq_geometry(type, &be, &bb, &cb);
    return be != 0;
}
bool supported_type(int type) { return split_type(type) || dq_type(type); }

// Values per GGUF block (block_size_for, rawllm_forward.hpp:289-299) and
// bytes per GGUF row (nbytes_for, rawllm_loader.hpp:367-386); 0 if unsupported.
size_t block_elems_of(int type) {
    if (split_type(type)) return 32;
    if (type == NEON_GGML_F32 || type == NEON_GGML_F16 || type == NEON_GGML_BF16) return 1;
    int be, bb, cb;
    dq_geometry(type, &be, &bb, &cb);
    return (size_t)be;
}
size_t row_bytes_of(int type, size_t cols) {
    const size_t be = block_elems_of(type);
    if (be == 0 || cols % be != 0) return 0;
    if (split_type(type)) return cols / 32 * gguf_block_bytes(type);
    if (type == NEON_GGML_F32) return cols * 4;
    if (type == NEON_GGML_F16 || type == NEON_GGML_BF16) return cols * 2;
    int e, bb, cb;
    dq_geometry(type, &e, &bb, &cb);
    return cols / be * (size_t)bb;
}

// Runs `fn` with `device` current, restoring the caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != device) ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

using StreamKernel = void (*)(StreamArgs);
StreamKernel stream_kernel(int type, int rc);
using DqKernel = void (*)(DqArgs);
DqKernel dq_kernel(int type, int T);
using DqRingKernel = void (*)(DqRingArgs);
DqRingKernel dq_ring_kernel(int type, int rpw);
StreamKernel resident_kernel(int type, int tpg);
constexpr int kResTpgs[] = {16, 32, 64, 128, 256};
constexpr int kDqTypes[] = {NEON_GGML_F32, NEON_GGML_F16, NEON_GGML_BF16, NEON_GGML_Q4_1, NEON_GGML_Q5_0,
                            NEON_GGML_Q5_1, NEON_GGML_Q4_K, NEON_GGML_Q5_K, NEON_GGML_Q6_K};

template <typename Kern>
int ensure_smem(Kern k, int bytes) {
    if (bytes > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return cuda_err(e, "cudaFuncSetAttribute");
    }
    return NEON_OK;
}

int init_device(int device) {
    if (device < 0 || device >= kMaxDevices) return set_err(NEON_ERR_INVALID, "device index out of range");
    DeviceState& st = g_dev[device];
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (st.ready) return NEON_OK;
    int n = 0;
    NEON_CUDA_TRY(cudaGetDeviceCount(&n));
    if (device >= n) return set_err(NEON_ERR_INVALID, "device " + std::to_string(device) + " not present");
    DeviceGuard g(device);
    if (!g.ok) return set_err(NEON_ERR_CUDA, "cudaSetDevice failed");
    cudaDeviceProp p;
    NEON_CUDA_TRY(cudaGetDeviceProperties(&p, device));
    if (p.major < 10)
        return set_err(NEON_ERR_UNSUPPORTED, std::string("device ") + p.name +
                                                 " is not sm_100-class; this library is built for sm_100a only");
    st.sms = p.multiProcessorCount;
    st.smem_per_sm = (int)p.sharedMemPerMultiprocessor;
    NEON_CUDA_TRY(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking));
    int rc = NEON_OK;
    for (int t : {NEON_GGML_Q4_0, NEON_GGML_Q8_0})
        for (int r : {2, 4, 8, 16, 32}) rc = rc ? rc : ensure_smem(stream_kernel(t, r), kMaxSmem);
    for (int t : {NEON_GGML_Q4_0, NEON_GGML_Q8_0})
        for (int tpg : kResTpgs) rc = rc ? rc : ensure_smem(resident_kernel(t, tpg), kMaxSmem);
    for (int t : kDqTypes)
        for (int T : {1, 2, 4}) rc = rc ? rc : ensure_smem(dq_kernel(t, T), kMaxSmem);
    for (int t : kDqTypes)
        for (int rpw : {1, 2}) rc = rc ? rc : ensure_smem(dq_ring_kernel(t, rpw), kMaxSmem);
    if (rc) return rc;
    void* err = nullptr;
    NEON_CUDA_TRY(cudaGetSymbolAddress(&err, g_neon_device_err));
    st.err = static_cast<unsigned int*>(err);
    void* eh = nullptr;
    NEON_CUDA_TRY(cudaHostAlloc(&eh, sizeof(unsigned int), cudaHostAllocPortable));
    st.err_host = static_cast<unsigned int*>(eh);
    *st.err_host = 0;
    st.ready = true;
    return NEON_OK;
}

int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
    return init_device(*dev);
}

template <typename... KArgs, typename... Args>
int launch_n(void (*kern)(KArgs...), dim3 grid, int threads, size_t smem, cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (g_pdl.load(std::memory_order_relaxed)) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_err(e, "cudaLaunchKernelEx");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return NEON_OK;
}

template <typename... KArgs, typename... Args>
int launch(void (*kern)(KArgs...), dim3 grid, size_t smem, cudaStream_t st, Args&&... args) {
    return launch_n(kern, grid, kThreads, smem, st, std::forward<Args>(args)...);
}

// Tile plan of a streaming (one-position) launch: plan_stream_tiles with
// this library's stage target, shared-memory budget and tile override.
StreamPlan plan_stream(int type, int nb, size_t total_rows, int sms) {
    return plan_stream_tiles(type, nb, total_rows, sms, kStreamStageTarget, kMaxSmem,
                             g_tile_rc.load(std::memory_order_relaxed), g_tile_kc.load(std::memory_order_relaxed));
}

// The streaming kernel instantiation for (type, rows per tile).
StreamKernel stream_kernel(int type, int rc) {
    // R rows per thread: each shared-memory read of an X block serves R rows
    // (shared-memory bandwidth, not HBM, limits R = 1 on large matrices);
    // 4 for tall tiles, 2 for the 8-row tiles of long rows (measured best)
    if (type == NEON_GGML_Q4_0) {
        switch (rc) {
            case 2: return matvec_stream_kernel<NEON_GGML_Q4_0, 2, 2>;
            case 4: return matvec_stream_kernel<NEON_GGML_Q4_0, 4, 2>;
            case 8: return matvec_stream_kernel<NEON_GGML_Q4_0, 8, 2>;
            case 16: return matvec_stream_kernel<NEON_GGML_Q4_0, 16, 4>;
            default: return matvec_stream_kernel<NEON_GGML_Q4_0, 32, 4>;
        }
    }
    switch (rc) {
        case 2: return matvec_stream_kernel<NEON_GGML_Q8_0, 2, 2>;
        case 4: return matvec_stream_kernel<NEON_GGML_Q8_0, 4, 2>;
        case 8: return matvec_stream_kernel<NEON_GGML_Q8_0, 8, 2>;
        case 16: return matvec_stream_kernel<NEON_GGML_Q8_0, 16, 2>;
        default: return matvec_stream_kernel<NEON_GGML_Q8_0, 32, 2>;
    }
}

// Resident CTAs per SM of a streaming kernel instantiation at `smem` bytes.
int stream_occupancy(int type, int rc, int smem) {
    static std::mutex mu;
    static std::vector<std::pair<long long, int>> cache;
    const long long key = ((long long)type << 40) | ((long long)rc << 32) | (unsigned)smem;
    std::lock_guard<std::mutex> lk(mu);
    for (auto& kv : cache)
        if (kv.first == key) return kv.second;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, stream_kernel(type, rc), kStreamBlock, smem) !=
        cudaSuccess)
        occ = 1;
    occ = std::max(1, occ);
    cache.emplace_back(key, occ);
    return occ;
}

// The resident kernel instantiation for (type, threads per row group).
StreamKernel resident_kernel(int type, int tpg) {
    if (type == NEON_GGML_Q4_0) {
        switch (tpg) {
            case 16: return matvec_resident_kernel<NEON_GGML_Q4_0, 16>;
            case 32: return matvec_resident_kernel<NEON_GGML_Q4_0, 32>;
            case 64: return matvec_resident_kernel<NEON_GGML_Q4_0, 64>;
            case 128: return matvec_resident_kernel<NEON_GGML_Q4_0, 128>;
            default: return matvec_resident_kernel<NEON_GGML_Q4_0, 256>;
        }
    }
    switch (tpg) {
        case 16: return matvec_resident_kernel<NEON_GGML_Q8_0, 16>;
        case 32: return matvec_resident_kernel<NEON_GGML_Q8_0, 32>;
        case 64: return matvec_resident_kernel<NEON_GGML_Q8_0, 64>;
        case 128: return matvec_resident_kernel<NEON_GGML_Q8_0, 128>;
        default: return matvec_resident_kernel<NEON_GGML_Q8_0, 256>;
    }
}

// One-position targets whose weights fit the resident kernel (all targets in
// one launch): launched, NEON_OK; 1 when the plan does not apply (nothing
// launched); an error code otherwise.
int launch_resident(const std::vector<const neon_proj_target_t*>& t, int type, int nb, const float* dX,
                    cudaStream_t st, DeviceState& ds, int accumulate, const neon_proj_target_t* base,
                    const neon_internal::MatvecExt* ext) {
    const int k = g_resident.load(std::memory_order_relaxed);
    if (k <= 0 || t.empty() || t.size() > (size_t)kMaxSpans || g_tile_rc.load(std::memory_order_relaxed)) return 1;
    StreamArgs a;
    std::memset(&a, 0, sizeof(a));
    long long rows[kMaxSpans];
    int tile0[kMaxSpans];
    for (size_t i = 0; i < t.size(); ++i) rows[i] = (long long)t[i]->W->rows;
    const long long vrows = res_span_starts(rows, (int)t.size(), tile0);
    if (vrows > (1LL << 30)) return 1;
    ResPlan p;
    if (!matvec_resident_plan(type, nb, (int)vrows, ds.sms, k, ds.smem_per_sm, &p)) return 1;
    for (size_t i = 0; i < t.size(); ++i) {
        const neon_proj_target_t* tg = t[i];
        Span& s = a.span[i];
        s.qs = tg->W->qs;
        s.d = tg->W->d;
        s.y = tg->Y;
        s.y_stride = (long long)tg->y_stride;
        s.rows = (int)tg->W->rows;
        s.tile0 = tile0[i];
        if (ext && ext->epi) {
            const size_t j = (size_t)(tg - base);
            s.epi = ext->epi[j];
            s.pos_stride = ext->pos_stride ? ext->pos_stride[j] : 0;
        }
        if (ext && ext->peer_mode == 1) s.epi = kEpiPeer;
        if (ext && ext->peer_mode == 2) {
            s.epi = kEpiGather;
            s.pos_stride = ext->gather_row0;
        }
    }
    a.x = dX;
    a.err = ds.err;
    if (ext) {
        a.norm_w = ext->norm_w;
        a.norm_eps = ext->norm_eps;
        a.d_pos = ext->d_pos;
        a.rope_cs = ext->rope_cs;
        a.rope_half = ext->rope_half;
        a.head_dim = ext->head_dim;
        a.peer_mode = ext->peer_mode;
        if (ext->peer_mode) a.peer = ext->peer;
    }
    a.x_vec = (reinterpret_cast<uintptr_t>(dX) % 16) == 0;
    a.accumulate = accumulate;
    a.n_spans = (int)t.size();
    a.nb = nb;
    a.rpc = p.rpc;
    a.n_vrows = (int)vrows;
    return launch_n(resident_kernel(type, p.tpg), dim3(p.grid), kStreamThreads, p.smem, st, a);
}

int launch_stream(const std::vector<const neon_proj_target_t*>& t, int type, int nb, const float* dX,
                  cudaStream_t st, DeviceState& ds, int accumulate, const neon_proj_target_t* base,
                  const neon_internal::MatvecExt* ext) {
    {
        const int rrc = launch_resident(t, type, nb, dX, st, ds, accumulate, base, ext);
        if (rrc != 1) return rrc;
    }
    size_t total_rows = 0;
    for (auto* tg : t) total_rows += tg->W->rows;
    const StreamPlan p = plan_stream(type, nb, total_rows, ds.sms);
    if (p.smem > kMaxSmem)
        return set_err(NEON_ERR_UNSUPPORTED, "input dim " + std::to_string((size_t)nb * 32) +
                                                 " is too large for the one-position kernel's shared memory");
    const int rc_rows = p.rc;
    size_t start = 0;
    while (start < t.size()) {
        StreamArgs a;
        std::memset(&a, 0, sizeof(a));
        size_t n = std::min(t.size() - start, (size_t)kMaxSpans);
        int tiles = 0;
        for (size_t i = 0; i < n; ++i) {
            const neon_proj_target_t* tg = t[start + i];
            Span& s = a.span[i];
            s.qs = tg->W->qs;
            s.d = tg->W->d;
            s.y = tg->Y;
            s.y_stride = (long long)tg->y_stride;
            s.rows = (int)tg->W->rows;
            s.tile0 = tiles;
            tiles += (int)((tg->W->rows + rc_rows - 1) / rc_rows);
            if (ext && ext->epi) {
                const size_t k = (size_t)(tg - base);
                s.epi = ext->epi[k];
                s.pos_stride = ext->pos_stride ? ext->pos_stride[k] : 0;
            }
            if (ext && ext->peer_mode == 1) s.epi = kEpiPeer;
        if (ext && ext->peer_mode == 2) {
            s.epi = kEpiGather;
            s.pos_stride = ext->gather_row0;
        }
        }
        a.x = dX;
        a.err = ds.err;
        if (ext) {
            a.norm_w = ext->norm_w;
            a.norm_eps = ext->norm_eps;
            a.d_pos = ext->d_pos;
            a.rope_cs = ext->rope_cs;
            a.rope_half = ext->rope_half;
            a.head_dim = ext->head_dim;
            a.peer_mode = ext->peer_mode;
            if (ext->peer_mode) a.peer = ext->peer;
        }
        a.n_spans = (int)n;
        a.n_tiles = tiles;
        a.nb = nb;
        a.kc = p.kc;
        a.nch = p.nch;
        a.stage_bytes = p.stage_bytes;
        a.x_vec = (reinterpret_cast<uintptr_t>(dX) % 16) == 0;
        a.accumulate = accumulate;
        // Pick the ring depth that keeps the most weight bytes in flight per
        // SM (resident CTAs x stages x stage bytes), then size the grid to what
        // is resident: a CTA that starts late repays the X staging.
        int best_stages = 1, best_occ = 1;
        long long best_bytes = -1;
        for (int st_n = 1; st_n <= p.stages; ++st_n) {
            const int sm_bytes = stream_smem_bytes(type, nb, st_n, p.stage_bytes);
            const int occ = std::min(stream_occupancy(type, p.rc, sm_bytes), kStreamCtasPerSm);
            const long long inflight = (long long)occ * st_n * p.stage_bytes;
            if (inflight >= best_bytes) {
                best_bytes = inflight;
                best_stages = st_n;
                best_occ = occ;
            }
        }
        const int grid = std::min(tiles, ds.sms * best_occ);
        const int per_cta_items = ((tiles + grid - 1) / grid) * p.nch;
        a.stages = std::max(1, std::min(best_stages, per_cta_items));
        const int smem = stream_smem_bytes(type, nb, a.stages, p.stage_bytes);
        int rc = launch_n(stream_kernel(type, p.rc), dim3(grid), kStreamBlock, smem, st, a);
        if (rc) return rc;
        if (ext && ext->launched_stream) *ext->launched_stream = true;
        start += n;
    }
    return NEON_OK;
}

// The dequantising kernel instantiation for (type, positions per CTA).
DqKernel dq_kernel(int type, int T) {
#define NEON_DQ_CASE(TY)                                               \
    case TY:                                                           \
        return T >= 4 ? matvec_dq_kernel<TY, 4>                        \
                      : (T == 2 ? matvec_dq_kernel<TY, 2> : matvec_dq_kernel<TY, 1>);
    switch (type) {
        NEON_DQ_CASE(NEON_GGML_F32)
        NEON_DQ_CASE(NEON_GGML_F16)
        NEON_DQ_CASE(NEON_GGML_BF16)
        NEON_DQ_CASE(NEON_GGML_Q4_1)
        NEON_DQ_CASE(NEON_GGML_Q5_0)
        NEON_DQ_CASE(NEON_GGML_Q5_1)
        NEON_DQ_CASE(NEON_GGML_Q4_K)
        NEON_DQ_CASE(NEON_GGML_Q5_K)
        NEON_DQ_CASE(NEON_GGML_Q6_K)
        default: return nullptr;
    }
#undef NEON_DQ_CASE
}

// The ring kernel instantiation for (type, rows per warp).
DqRingKernel dq_ring_kernel(int type, int rpw) {
#define NEON_DQ_RING_CASE(TY) \
    case TY:                  \
        return rpw >= 2 ? matvec_dq_ring_kernel<TY, 2> : matvec_dq_ring_kernel<TY, 1>;
    switch (type) {
        NEON_DQ_RING_CASE(NEON_GGML_F32)
        NEON_DQ_RING_CASE(NEON_GGML_F16)
        NEON_DQ_RING_CASE(NEON_GGML_BF16)
        NEON_DQ_RING_CASE(NEON_GGML_Q4_1)
        NEON_DQ_RING_CASE(NEON_GGML_Q5_0)
        NEON_DQ_RING_CASE(NEON_GGML_Q5_1)
        NEON_DQ_RING_CASE(NEON_GGML_Q4_K)
        NEON_DQ_RING_CASE(NEON_GGML_Q5_K)
        NEON_DQ_RING_CASE(NEON_GGML_Q6_K)
        default: return nullptr;
    }
#undef NEON_DQ_RING_CASE
}

int dq_ring_occupancy(int type, int rpw, int smem) {
    static std::mutex mu;
    static std::vector<std::pair<long long, int>> cache;
    const long long key = ((long long)type << 40) | ((long long)rpw << 32) | (unsigned)smem;
    std::lock_guard<std::mutex> lk(mu);
    for (auto& kv : cache)
        if (kv.first == key) return kv.second;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, dq_ring_kernel(type, rpw), kStreamBlock, smem) !=
        cudaSuccess)
        occ = 1;
    occ = std::max(1, occ);
    cache.emplace_back(key, occ);
    return occ;
}

// One launch group of a dequantising type at one position on the ring
// kernel; returns 1 (nothing launched) when X and one stage do not fit.
int launch_dq_ring(const std::vector<const neon_proj_target_t*>& t, int type, size_t cols, const float* dX,
                   cudaStream_t st, DeviceState& ds, int accumulate, const neon_proj_target_t* base,
                   const neon_internal::MatvecExt* ext) {
    int be, bb, cb;
    dq_geometry(type, &be, &bb, &cb);
    const int nu = (int)((cols + 31) / 32);
    const int nblk = nu / (be / 32);
    const long long pitch = (long long)t[0]->W->pitch;
    size_t total_rows = 0;
    for (const auto* tg : t) total_rows += tg->W->rows;
    const DqRingPlan p = plan_dq_ring(type, nblk, pitch, total_rows, ds.sms, kStageTarget);
    const int rc_rows = kStreamWarps * p.rpw;
    const int xb = dq_x_bytes(1, nu);
    if (xb + p.stage_bytes > kMaxSmem) return 1;
    size_t start = 0;
    while (start < t.size()) {
        DqRingArgs r;
        std::memset(&r, 0, sizeof(r));
        DqArgs& a = r.d;
        size_t n = std::min(t.size() - start, (size_t)kMaxSpans);
        int tiles = 0;
        for (size_t i = 0; i < n; ++i) {
            const neon_proj_target_t* tg = t[start + i];
            Span& sp = a.s.span[i];
            sp.qs = tg->W->qs;
            sp.d = nullptr;
            sp.y = tg->Y;
            sp.y_stride = (long long)tg->y_stride;
            sp.rows = (int)tg->W->rows;
            sp.tile0 = tiles;
            tiles += (int)((tg->W->rows + rc_rows - 1) / rc_rows);
            if (ext && ext->epi) {
                const size_t k = (size_t)(tg - base);
                sp.epi = ext->epi[k];
                sp.pos_stride = ext->pos_stride ? ext->pos_stride[k] : 0;
            }
            if (ext && ext->peer_mode == 1) sp.epi = kEpiPeer;
            if (ext && ext->peer_mode == 2) {
                sp.epi = kEpiGather;
                sp.pos_stride = ext->gather_row0;
            }
        }
        a.s.x = dX;
        a.s.err = ds.err;
        a.s.n_spans = (int)n;
        a.s.n_tiles = tiles;
        a.s.accumulate = accumulate;
        if (ext) {
            a.s.norm_w = ext->norm_w;
            a.s.norm_eps = ext->norm_eps;
            a.s.d_pos = ext->d_pos;
            a.s.rope_cs = ext->rope_cs;
            a.s.rope_half = ext->rope_half;
            a.s.head_dim = ext->head_dim;
            a.s.peer_mode = ext->peer_mode;
            if (ext->peer_mode) a.s.peer = ext->peer;
        }
        a.s.x_vec = (reinterpret_cast<uintptr_t>(dX) % 16) == 0 &&
                    (!a.s.norm_w || (reinterpret_cast<uintptr_t>(a.s.norm_w) % 16) == 0);
        a.pitch = pitch;
        a.x_stride = (long long)cols;
        a.cols = (int)cols;
        a.nu = nu;
        a.nblk = nblk;
        a.nch = p.nch;
        a.seq = 1;
        r.kcb = p.kcb;
        r.row_stride = p.row_stride;
        r.stage_bytes = p.stage_bytes;
        // the ring depth that keeps the most weight bytes in flight per SM
        int best_stages = 1, best_occ = 1;
        long long best_bytes = -1;
        for (int st_n = 1; st_n <= kDqRingMaxStages; ++st_n) {
            const int sm_bytes = xb + st_n * p.stage_bytes;
            if (sm_bytes > kMaxSmem) break;
            const int occ = std::min(dq_ring_occupancy(type, p.rpw, sm_bytes), kStreamCtasPerSm);
            const long long inflight = (long long)occ * st_n * p.stage_bytes;
            if (inflight >= best_bytes) {
                best_bytes = inflight;
                best_stages = st_n;
                best_occ = occ;
            }
        }
        const int grid = std::min(tiles, ds.sms * best_occ);
        const int per_cta_items = ((tiles + grid - 1) / grid) * p.nch;
        r.stages = std::max(1, std::min(best_stages, per_cta_items));
        const int smem = xb + r.stages * p.stage_bytes;
        int rc = launch_n(dq_ring_kernel(type, p.rpw), dim3(grid), kStreamBlock, smem, st, r);
        if (rc) return rc;
        start += n;
    }
    return NEON_OK;
}

int dq_occupancy(int type, int T, int smem) {
    static std::mutex mu;
    static std::vector<std::pair<long long, int>> cache;
    const long long key = ((long long)type << 40) | ((long long)T << 32) | (unsigned)smem;
    std::lock_guard<std::mutex> lk(mu);
    for (auto& kv : cache)
        if (kv.first == key) return kv.second;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, dq_kernel(type, T), kThreads, smem) != cudaSuccess)
        occ = 1;
    occ = std::max(1, occ);
    cache.emplace_back(key, occ);
    return occ;
}

// One launch group of a dequantising type: tiles of 8 rows, T positions per
// CTA (grid.y over the positions), X of those positions in shared memory.
int launch_dq(const std::vector<const neon_proj_target_t*>& t, int type, size_t cols, const float* dX,
              size_t x_stride, size_t seq, cudaStream_t st, DeviceState& ds, int accumulate,
              const neon_proj_target_t* base, const neon_internal::MatvecExt* ext) {
    // the ring by default only where it measured faster on B200 (4096x4096,
    // one position: Q4_1 1402 vs 1221 GB/s, F16 3252 vs 2714, BF16 3291 vs
    // 2831); the K-quants, Q5_0/Q5_1 and F32 ran slower on it
    const int ring = g_dq_ring.load(std::memory_order_relaxed);
    const bool ring_type = type == NEON_GGML_Q4_1 || type == NEON_GGML_F16 || type == NEON_GGML_BF16;
    if (seq == 1 && (ring == 1 || (ring < 0 && ring_type))) {
        const int rc = launch_dq_ring(t, type, cols, dX, st, ds, accumulate, base, ext);
        if (rc != 1) return rc;  // 1: X does not fit beside a stage; the register-buffer kernel below
    }
    int be, bb, cb;
    dq_geometry(type, &be, &bb, &cb);
    const int nu = (int)((cols + 31) / 32);
    const int nblk = nu / (be / 32);
    const int chunk = cb * bb;
    int T = 1;
    if (seq >= 4 && dq_x_bytes(4, nu) + kWarps * chunk <= kMaxSmem) T = 4;
    else if (seq >= 2 && dq_x_bytes(2, nu) + kWarps * chunk <= kMaxSmem) T = 2;
    const int smem = dq_x_bytes(T, nu) + kWarps * chunk;
    if (smem > kMaxSmem)
        return set_err(NEON_ERR_UNSUPPORTED, "input dim " + std::to_string(cols) +
                                                 " is too large for the dequantising kernel's shared memory");
    if ((seq + T - 1) / T > 65535) return set_err(NEON_ERR_UNSUPPORTED, "too many positions in one call");
    size_t start = 0;
    while (start < t.size()) {
        DqArgs a;
        std::memset(&a, 0, sizeof(a));
        size_t n = std::min(t.size() - start, (size_t)kMaxSpans);
        int tiles = 0;
        for (size_t i = 0; i < n; ++i) {
            const neon_proj_target_t* tg = t[start + i];
            Span& sp = a.s.span[i];
            sp.qs = tg->W->qs;
            sp.d = nullptr;
            sp.y = tg->Y;
            sp.y_stride = (long long)tg->y_stride;
            sp.rows = (int)tg->W->rows;
            sp.tile0 = tiles;
            tiles += (int)((tg->W->rows + kWarps - 1) / kWarps);
            if (ext && ext->epi) {
                const size_t k = (size_t)(tg - base);
                sp.epi = ext->epi[k];
                sp.pos_stride = ext->pos_stride ? ext->pos_stride[k] : 0;
            }
            if (ext && ext->peer_mode == 1) sp.epi = kEpiPeer;
            if (ext && ext->peer_mode == 2) {
                sp.epi = kEpiGather;
                sp.pos_stride = ext->gather_row0;
            }
        }
        a.s.x = dX;
        a.s.err = ds.err;
        a.s.n_spans = (int)n;
        a.s.n_tiles = tiles;
        a.s.accumulate = accumulate;
        if (ext) {
            a.s.norm_w = ext->norm_w;
            a.s.norm_eps = ext->norm_eps;
            a.s.d_pos = ext->d_pos;
            a.s.rope_cs = ext->rope_cs;
            a.s.rope_half = ext->rope_half;
            a.s.head_dim = ext->head_dim;
            a.s.peer_mode = ext->peer_mode;
            if (ext->peer_mode) a.s.peer = ext->peer;
        }
        // 128-bit X staging: X, every position's row and the norm weights 16-byte aligned
        a.s.x_vec = (reinterpret_cast<uintptr_t>(dX) % 16) == 0 && (seq == 1 || x_stride % 4 == 0) &&
                    (!a.s.norm_w || (reinterpret_cast<uintptr_t>(a.s.norm_w) % 16) == 0);
        a.pitch = (long long)t[start]->W->pitch;
        a.x_stride = (long long)x_stride;
        a.cols = (int)cols;
        a.nu = nu;
        a.nblk = nblk;
        a.nch = (nblk + cb - 1) / cb;
        a.seq = (int)seq;
        const int occ = dq_occupancy(type, T, smem);
        const int grid = std::min(tiles, ds.sms * occ);
        int rc = launch_n(dq_kernel(type, T), dim3(grid, (unsigned)((seq + T - 1) / T)), kThreads, smem, st, a);
        if (rc) return rc;
        start += n;
    }
    return NEON_OK;
}

// Reads (and clears) the device error word after the stream has drained.
int check_device_err(int device) {
    if (device < 0 || device >= kMaxDevices || !g_dev[device].ready) return NEON_OK;
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_neon_device_err, sizeof(v));
    if (e != cudaSuccess) return cuda_err(e, "cudaMemcpyFromSymbol");
    if (v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_neon_device_err, &zero, sizeof(zero));
        return set_err(NEON_ERR_CUDA, "a device-side wait timed out (shared-memory copy never completed)");
    }
    return NEON_OK;
}

int grow(void** p, size_t* cap, size_t need) {
    if (*cap >= need) return NEON_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(p, need);
    if (e != cudaSuccess) {
        *p = nullptr;
        return set_err(NEON_ERR_NOMEM, std::string("cudaMalloc of library scratch failed: ") + cudaGetErrorString(e));
    }
    *cap = need;
    return NEON_OK;
}

// Device scratch for seq*cols Q8_0 activations (quants, scales, sums).
int ensure_act_scratch(DeviceState& st, size_t n) {
    if (st.scratch_cols >= n) return NEON_OK;
    if (st.xq) cudaFree(st.xq);
    if (st.xd) cudaFree(st.xd);
    if (st.xs) cudaFree(st.xs);
    st.xq = nullptr; st.xd = nullptr; st.xs = nullptr; st.scratch_cols = 0;
    size_t nblk = n / 32 + 1;
    if (cudaMalloc(&st.xq, n) != cudaSuccess || cudaMalloc(&st.xd, nblk * 4) != cudaSuccess ||
        cudaMalloc(&st.xs, nblk * 4) != cudaSuccess)
        return set_err(NEON_ERR_NOMEM, "cudaMalloc of activation scratch failed");
    st.scratch_cols = n;
    return NEON_OK;
}

int validate_tensor(neon_tensor_t W) {
    if (!W) return set_err(NEON_ERR_INVALID, "null tensor handle");
    if (!supported_type(W->type)) return set_err(NEON_ERR_UNSUPPORTED, "tensor type not supported");
    return NEON_OK;
}

// One group of targets that share type and input dim -> one launch.
struct Group {
    int type;
    size_t cols;
    std::vector<const neon_proj_target_t*> t;
};

int launch_group(const Group& g, const float* dX, size_t x_stride, size_t seq, cudaStream_t st,
                 DeviceState& ds, int accumulate, const neon_proj_target_t* base,
                 const neon_internal::MatvecExt* ext) {
    if (dq_type(g.type)) {
        if (seq > 1 && ext) return set_err(NEON_ERR_UNSUPPORTED, "fused norm / epilogues need one position");
        return launch_dq(g.t, g.type, g.cols, dX, x_stride, seq, st, ds, accumulate, base, ext);
    }
    const int nb = (int)(g.cols / 32);
    const bool q4 = g.type == NEON_GGML_Q4_0;
    if (seq == 1) return launch_stream(g.t, g.type, nb, dX, st, ds, accumulate, base, ext);
    if (ext) return set_err(NEON_ERR_UNSUPPORTED, "fused norm / epilogues need one position");
    if (g_prefill_mma.load(std::memory_order_relaxed)) {
        // tensor-core tiles of 64 rows x 64 positions: Q4_0 over the Q8_0
        // activations (int8 MMA), Q8_0 over fp32 X (TF32 MMA)
        size_t start = 0;
        while (start < g.t.size()) {
            MatvecArgs a;
            std::memset(&a, 0, sizeof(a));
            a.nb = nb;
            a.seq = (int)seq;
            a.x = dX;
            a.x_stride = (long long)x_stride;
            a.xq = q4 ? ds.xq : nullptr;
            a.xd = q4 ? ds.xd : nullptr;
            a.xs = q4 ? ds.xs : nullptr;
            a.accumulate = accumulate;
            int tiles = 0;
            size_t n = std::min(g.t.size() - start, (size_t)kMaxSpans);
            for (size_t i = 0; i < n; ++i) {
                const neon_proj_target_t* tg = g.t[start + i];
                Span& s = a.span[i];
                s.qs = tg->W->qs;
                s.d = tg->W->d;
                s.y = tg->Y;
                s.y_stride = (long long)tg->y_stride;
                s.rows = (int)tg->W->rows;
                s.tile0 = tiles;
                tiles += (int)((tg->W->rows + kMmaRows - 1) / kMmaRows);
            }
            a.n_spans = (int)n;
            a.n_tiles = tiles;
            if (tiles > 65535) return set_err(NEON_ERR_UNSUPPORTED, "more than 65535 row tiles in one prefill launch");
            // position tiles along x, so that the CTAs of one row tile run together and read its weights once
            const dim3 grid((unsigned)((seq + kMmaPos - 1) / kMmaPos), tiles);
            int rc = launch_n(q4 ? matvec_mma_q4_0_kernel : matvec_mma_q8_0_kernel, grid, kMmaThreads, 0, st, a);
            if (rc) return rc;
            start += n;
        }
        return NEON_OK;
    }
    size_t start = 0;
    while (start < g.t.size()) {
        MatvecArgs a;
        std::memset(&a, 0, sizeof(a));
        a.x = dX;
        a.x_stride = (long long)x_stride;
        a.nb = nb;
        a.seq = (int)seq;
        int tiles = 0;
        size_t n = std::min(g.t.size() - start, (size_t)kMaxSpans);
        for (size_t i = 0; i < n; ++i) {
            const neon_proj_target_t* tg = g.t[start + i];
            Span& s = a.span[i];
            s.qs = tg->W->qs;
            s.d = tg->W->d;
            s.y = tg->Y;
            s.y_stride = (long long)tg->y_stride;
            s.rows = (int)tg->W->rows;
            s.tile0 = tiles;
            tiles += (int)((tg->W->rows + kMpR - 1) / kMpR);
        }
        a.n_spans = (int)n;
        a.n_tiles = tiles;
        a.accumulate = accumulate;
        if (q4) {
            a.xq = ds.xq;
            a.xd = ds.xd;
            a.xs = ds.xs;
        }
        int ctas = (tiles + kWarps - 1) / kWarps;
        ctas = std::min(ctas, ds.sms * 4);
        dim3 grid(ctas, (unsigned)((seq + kMpT - 1) / kMpT));
        int rc = q4 ? launch(matvec_multipos_kernel<NEON_GGML_Q4_0, kMpR, kMpT>, grid, 0, st, a)
                    : launch(matvec_multipos_kernel<NEON_GGML_Q8_0, kMpR, kMpT>, grid, 0, st, a);
        if (rc) return rc;
        start += n;
    }
    return NEON_OK;
}

// Shared body of neon_cuda_matvec[_multi] on device buffers.
int matvec_targets(const neon_proj_target_t* targets, size_t n_targets, const float* dX,
                   size_t x_stride, size_t seq, void* stream, int accumulate = 0,
                   const neon_internal::MatvecExt* ext = nullptr) {
    if (n_targets == 0 || seq == 0) return NEON_OK;
    if (!targets || !dX) return set_err(NEON_ERR_INVALID, "null targets or X");
    int device = targets[0].W ? targets[0].W->device : -1;
    std::vector<Group> groups;
    size_t q4_cols = 0;
    for (size_t i = 0; i < n_targets; ++i) {
        const neon_proj_target_t& tg = targets[i];
        int rc = validate_tensor(tg.W);
        if (rc) return rc;
        if (!tg.Y) return set_err(NEON_ERR_INVALID, "null output pointer");
        if (tg.W->device != device)
            return set_err(NEON_ERR_INVALID, "targets of one call live on different devices");
        if (seq > 1 && tg.y_stride < tg.W->rows)
            return set_err(NEON_ERR_INVALID, "y_stride smaller than the tensor's rows");
        if (tg.W->type == NEON_GGML_Q4_0) {
            if (q4_cols != 0 && q4_cols != tg.W->cols)
                return set_err(NEON_ERR_INVALID,
                               "forward(): proj_all_positions_multi() got Q4_0 targets with mismatched input dims (" +
                                   std::to_string(q4_cols) + " vs " + std::to_string(tg.W->cols) +
                                   ") in one call -- the shared Q8_0 activation buffer assumes all fused Q4_0 "
                                   "targets share `cols`");
            q4_cols = tg.W->cols;
        }
        Group* g = nullptr;
        for (auto& gg : groups)
            if (gg.type == tg.W->type && gg.cols == tg.W->cols) g = &gg;
        if (!g) {
            groups.push_back(Group{tg.W->type, tg.W->cols, {}});
            g = &groups.back();
        }
        g->t.push_back(&tg);
    }
    DeviceGuard guard(device);
    if (!guard.ok) return set_err(NEON_ERR_CUDA, "cudaSetDevice failed");
    int rc = init_device(device);
    if (rc) return rc;
    DeviceState& ds = g_dev[device];
    cudaStream_t st = (cudaStream_t)stream;
    if (seq > 1 && q4_cols) {
        // Quantise X once for every Q4_0 target (quantize_rows_q8_0 on the
        // calling thread in the reference, rawllm_forward.hpp:544-552).
        rc = ensure_act_scratch(ds, seq * q4_cols);
        if (rc) return rc;
        const int nb = (int)(q4_cols / 32);
        long long blocks = (long long)nb * (long long)seq;
        int ctas = (int)std::min<long long>((blocks + kWarps - 1) / kWarps, (long long)ds.sms * 8);
        rc = launch(quantize_q8_0_kernel, dim3(ctas), 0, st, dX, (long long)x_stride, nb, (int)seq, ds.xq,
                    ds.xd, ds.xs);
        if (rc) return rc;
    }
    // Targets of different (type, cols) groups -- a Q4_K_M-style model's Q4_K
    // Q/K with a Q6_K V -- take one launch per group; every launch folds the
    // same norm into its own X staging and applies each target's own epilogue
    // (ext->epi / pos_stride are indexed by the target's place in `targets`).
    if (ext && ext->rope_cs && (ext->rope_half < 0 || ext->rope_half > kMaxRopeHalf))
        return set_err(NEON_ERR_UNSUPPORTED, "RoPE epilogue: rope dimension above 256");
    if (ext && ext->peer_mode) {
        if (seq != 1 || (ext->peer_mode != 1 && ext->peer_mode != 2) || n_targets != 1 || ext->peer.world < 1 ||
            ext->peer.world > kCommMaxRanks || ext->gather_row0 < 0)
            return set_err(NEON_ERR_INVALID, "fused collective: bad launch options");
        if ((size_t)ext->gather_row0 + targets[0].W->rows > (size_t)kCommFusedFloats)
            return set_err(NEON_ERR_UNSUPPORTED, "fused collective: vector longer than its slot");
    }
    for (const Group& g : groups) {
        rc = launch_group(g, dX, x_stride, seq, st, ds, accumulate, targets, ext);
        if (rc) return rc;
    }
    return NEON_OK;
}

}  // namespace

// Library-internal (not exported): the matvec launcher with the accumulate
// epilogue, and the error helpers, for the decode engine (neon_decode.cu).
namespace neon_internal {
int matvec(const neon_proj_target_t* targets, size_t n, const float* dX, size_t x_stride, size_t seq,
           cudaStream_t st, int accumulate, const MatvecExt* ext) {
    return matvec_targets(targets, n, dX, x_stride, seq, (void*)st, accumulate, ext);
}
int error(int code, const std::string& msg) { return set_err(code, msg); }
size_t gguf_row_bytes(int type, size_t cols) { return row_bytes_of(type, cols); }
int embed_rows(const neon_tensor* E, const int* toks, int seq, int n_embd, int n_vocab, float* h, unsigned int* err,
               cudaStream_t st) {
    using EmbedKernel = void (*)(const unsigned char*, long long, int, const int*, int, float*, unsigned int*);
    EmbedKernel k = nullptr;
    switch (E->type) {
        case NEON_GGML_F32: k = embed_dq_kernel<NEON_GGML_F32>; break;
        case NEON_GGML_F16: k = embed_dq_kernel<NEON_GGML_F16>; break;
        case NEON_GGML_BF16: k = embed_dq_kernel<NEON_GGML_BF16>; break;
        case NEON_GGML_Q4_1: k = embed_dq_kernel<NEON_GGML_Q4_1>; break;
        case NEON_GGML_Q5_0: k = embed_dq_kernel<NEON_GGML_Q5_0>; break;
        case NEON_GGML_Q5_1: k = embed_dq_kernel<NEON_GGML_Q5_1>; break;
        case NEON_GGML_Q4_K: k = embed_dq_kernel<NEON_GGML_Q4_K>; break;
        case NEON_GGML_Q5_K: k = embed_dq_kernel<NEON_GGML_Q5_K>; break;
        case NEON_GGML_Q6_K: k = embed_dq_kernel<NEON_GGML_Q6_K>; break;
        default: return set_err(NEON_ERR_UNSUPPORTED, "embedding type not supported");
    }
    const int nu = (n_embd + 31) / 32;
    return launch_n(k, dim3((nu + 127) / 128, seq), 128, 0, st, (const unsigned char*)E->qs, (long long)E->pitch,
                    n_embd, toks, n_vocab, h, err);
}
size_t gguf_block_elems(int type) { return block_elems_of(type); }
bool dequantize_row_host(int type, const uint8_t* p, size_t n, float* out) {
    return row_bytes_of(type, n) != 0 && dq_row_host(type, p, n, out);
}
int cuda_error(cudaError_t e, const char* what) { return cuda_err(e, what); }
int launched(int n) {
    g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed);
    return NEON_OK;
}
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }
bool prefill_mma() { return g_prefill_mma.load(std::memory_order_relaxed) != 0; }

int device_sms(int device) {
    int rc = init_device(device);
    return rc ? -1 : g_dev[device].sms;
}
int check_device_error(int device) { return check_device_err(device); }
}  // namespace neon_internal

extern "C" {

const char* neon_cuda_last_error(void) { return g_err.c_str(); }

const char* neon_cuda_version(void) { return "0.1.0"; }

int neon_cuda_device_count(int* count) {
    if (!count) return set_err(NEON_ERR_INVALID, "null count");
    cudaError_t e = cudaGetDeviceCount(count);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        *count = 0;
        cudaGetLastError();
        return NEON_OK;
    }
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDeviceCount");
    return NEON_OK;
}

int neon_cuda_init(int device) {
    int rc = init_device(device);
    if (rc) return rc;
    NEON_CUDA_TRY(cudaSetDevice(device));
    return NEON_OK;
}

int neon_cuda_set_prefill_mma(int enabled) {
    g_prefill_mma.store(enabled ? 1 : 0);
    return NEON_OK;
}

int neon_cuda_set_dq_ring(int enabled) {
    g_dq_ring.store(enabled < 0 ? -1 : enabled ? 1 : 0);
    return NEON_OK;
}

int neon_cuda_set_stream_tiles(int rows_per_tile, int blocks_per_chunk) {
    if (rows_per_tile != 0 && rows_per_tile != 2 && rows_per_tile != 4 && rows_per_tile != 8 && rows_per_tile != 16 &&
        rows_per_tile != 32)
        return set_err(NEON_ERR_INVALID, "rows per tile must be 0 (the planner's choice), 2, 4, 8, 16 or 32");
    if (blocks_per_chunk < 0) return set_err(NEON_ERR_INVALID, "blocks per chunk must be >= 0");
    g_tile_kc.store(blocks_per_chunk);
    g_tile_rc.store(rows_per_tile);
    return NEON_OK;
}

int neon_cuda_set_resident(int ctas_per_sm) {
    if (ctas_per_sm < 0 || ctas_per_sm > 8) return set_err(NEON_ERR_INVALID, "CTAs per SM must be 0 (off) .. 8");
    g_resident.store(ctas_per_sm);
    return NEON_OK;
}

int neon_cuda_set_pdl(int enabled) {
    g_pdl.store(enabled ? 1 : 0);
    return NEON_OK;
}

uint64_t neon_cuda_launch_count(void) { return g_launches.load(); }

}  // extern "C"

namespace {
// Upload of a dequantising type: the GGUF rows (or the kept shard of them)
// copied unchanged into rows of a 16-byte pitch, the padding zeroed. One 2-D
// copy straight from the caller's bytes; no repack kernel.
int upload_rows(const uint8_t* host_bytes, bool on_device, int type, size_t rows, size_t cols, int shard_mode,
                int shard_index, int shard_count, neon_tensor_t* out) {
    int be, bb, cb;
    dq_geometry(type, &be, &bb, &cb);
    const size_t src_row = row_bytes_of(type, cols);
    const size_t nu = (cols + 31) / 32;
    const size_t nblk = nu / (size_t)(be / 32);
    if (rows > (size_t)INT32_MAX / 2 || nu > (size_t)INT32_MAX / 64) return set_err(NEON_ERR_INVALID, "tensor too large");
    size_t r0 = 0, r1 = rows, b0 = 0, b1 = nblk;
    if (shard_mode != NEON_SHARD_NONE) {
        if (shard_count <= 0 || shard_index < 0 || shard_index >= shard_count)
            return set_err(NEON_ERR_INVALID, "bad shard index/count");
        if (shard_mode == NEON_SHARD_ROWS) {
            r0 = rows * (size_t)shard_index / (size_t)shard_count;
            r1 = rows * (size_t)(shard_index + 1) / (size_t)shard_count;
        } else if (shard_mode == NEON_SHARD_COLS) {
            if (cols % (size_t)be != 0)
                return set_err(NEON_ERR_UNSUPPORTED, "column split of a float tensor whose rows are not whole 32-value blocks");
            b0 = nblk * (size_t)shard_index / (size_t)shard_count;
            b1 = nblk * (size_t)(shard_index + 1) / (size_t)shard_count;
        } else {
            return set_err(NEON_ERR_INVALID, "unknown shard mode");
        }
        if (r1 <= r0 || b1 <= b0) return set_err(NEON_ERR_INVALID, "empty shard");
    }
    int device = 0;
    int rc = current_device(&device);
    if (rc) return rc;
    const bool col_split = shard_mode == NEON_SHARD_COLS;
    const size_t lrows = r1 - r0, lnb = b1 - b0;
    const size_t lcols = col_split ? lnb * (size_t)be : cols;
    const size_t pitch = (lnb * (size_t)bb + 15) & ~(size_t)15;
    const size_t width = col_split ? lnb * (size_t)bb : src_row;
    const size_t total = lrows * pitch;

    neon_tensor* t = new neon_tensor();
    t->device = device;
    t->type = type;
    t->rows = lrows;
    t->cols = lcols;
    t->nb = (lcols + 31) / 32;
    t->bytes = total;
    t->pitch = pitch;
    cudaError_t e = cudaMalloc(&t->base, total);
    if (e != cudaSuccess) {
        delete t;
        return set_err(NEON_ERR_NOMEM, std::string("cudaMalloc of weights failed: ") + cudaGetErrorString(e));
    }
    t->qs = t->base;
    t->d = nullptr;
    cudaStream_t st = g_dev[device].stream;
    e = cudaMemsetAsync(t->base, 0, total, st);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(t->base, pitch, host_bytes + r0 * src_row + b0 * (size_t)bb, src_row, width, lrows,
                              on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        cudaFree(t->base);
        delete t;
        return cuda_err(e, "weight upload");
    }
    *out = t;
    return NEON_OK;
}
}  // namespace

extern "C" {

}  // extern "C"

namespace {
// The upload of neon_cuda_upload, from host bytes or (on_device) from GGUF
// bytes already in this device's memory (the on-load quantiser's output).
int upload_impl(const uint8_t* host_bytes, bool on_device, int ggml_type, size_t rows, size_t cols, int shard_mode,
                int shard_index, int shard_count, neon_tensor_t* out) {
    if (!out) return set_err(NEON_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (!host_bytes) return set_err(NEON_ERR_INVALID, "null weight bytes");
    if (!supported_type(ggml_type))
        return set_err(NEON_ERR_UNSUPPORTED, "quant type " + std::to_string(ggml_type) +
                                                 " is not supported by the CUDA backend (the eleven types "
                                                 "dequantize_row decodes are)");
    if (rows == 0 || cols == 0) return set_err(NEON_ERR_INVALID, "empty tensor");
    const size_t bs = block_elems_of(ggml_type);
    if (cols % bs != 0)
        return set_err(NEON_ERR_INVALID, "forward(): input dim (" + std::to_string(cols) +
                                             ") isn't a multiple of its quant block size (" + std::to_string(bs) +
                                             ") -- can't dequantize safely.");
    if (dq_type(ggml_type))
        return upload_rows(host_bytes, on_device, ggml_type, rows, cols, shard_mode, shard_index, shard_count, out);
    if (rows > (size_t)INT32_MAX / 2 || cols / 32 > (size_t)INT32_MAX / 64)
        return set_err(NEON_ERR_INVALID, "tensor too large");
    size_t nb = cols / 32;
    size_t r0 = 0, r1 = rows, b0 = 0, b1 = nb;
    if (shard_mode != NEON_SHARD_NONE) {
        if (shard_count <= 0 || shard_index < 0 || shard_index >= shard_count)
            return set_err(NEON_ERR_INVALID, "bad shard index/count");
        if (shard_mode == NEON_SHARD_ROWS) {
            r0 = rows * (size_t)shard_index / (size_t)shard_count;
            r1 = rows * (size_t)(shard_index + 1) / (size_t)shard_count;
        } else if (shard_mode == NEON_SHARD_COLS) {
            b0 = nb * (size_t)shard_index / (size_t)shard_count;
            b1 = nb * (size_t)(shard_index + 1) / (size_t)shard_count;
        } else {
            return set_err(NEON_ERR_INVALID, "unknown shard mode");
        }
        if (r1 <= r0 || b1 <= b0) return set_err(NEON_ERR_INVALID, "empty shard");
    }
    int device = 0;
    int rc = current_device(&device);
    if (rc) return rc;
    const size_t P = payload_bytes(ggml_type);
    const size_t src_row = nb * gguf_block_bytes(ggml_type);
    const size_t lrows = r1 - r0, lnb = b1 - b0;
    const size_t qs_bytes = lrows * lnb * P;
    const size_t d_off = (qs_bytes + 255) / 256 * 256;
    const size_t total = d_off + lrows * lnb * 2 + 16;  // tail: aligned scale windows

    neon_tensor* t = new neon_tensor();
    t->device = device;
    t->type = ggml_type;
    t->rows = lrows;
    t->cols = lnb * 32;
    t->nb = lnb;
    t->bytes = total;
    cudaError_t e = cudaMalloc(&t->base, total);
    if (e != cudaSuccess) {
        delete t;
        return set_err(NEON_ERR_NOMEM, std::string("cudaMalloc of weights failed: ") + cudaGetErrorString(e));
    }
    t->qs = t->base;
    t->d = reinterpret_cast<uint16_t*>(t->base + d_off);

    // Stage the GGUF rows in chunks of <= 256 MiB and repack them on the device
    // (device-resident bytes are repacked in place, in one pass).
    const size_t chunk_rows = on_device ? lrows : std::max<size_t>(1, (256u << 20) / src_row);
    uint8_t* tmp = nullptr;
    if (!on_device) {
        size_t tmp_bytes = std::min(lrows, chunk_rows) * src_row;
        e = cudaMalloc(&tmp, tmp_bytes);
        if (e != cudaSuccess) {
            cudaFree(t->base);
            delete t;
            return set_err(NEON_ERR_NOMEM, "cudaMalloc of the upload staging buffer failed");
        }
    }
    cudaStream_t st = g_dev[device].stream;
    for (size_t c = 0; c < lrows; c += chunk_rows) {
        size_t nr = std::min(chunk_rows, lrows - c);
        const uint8_t* src = host_bytes + (r0 + c) * src_row;
        if (!on_device) {
            e = cudaMemcpyAsync(tmp, src, nr * src_row, cudaMemcpyHostToDevice, st);
            if (e != cudaSuccess) break;
            src = tmp;
        }
        long long n = (long long)nr * (long long)lnb;
        int grid = (int)std::min<long long>((n + 255) / 256, 65535LL * 8);
        repack_kernel<<<grid, 256, 0, st>>>(src, (long long)src_row, (int)nr, (int)b0, (int)lnb, (int)P,
                                            t->qs + c * lnb * P, t->d + c * lnb);
        g_launches.fetch_add(1, std::memory_order_relaxed);
        e = cudaGetLastError();
        if (e != cudaSuccess) break;
        e = cudaStreamSynchronize(st);  // tmp is reused by the next chunk
        if (e != cudaSuccess) break;
    }
    cudaFree(tmp);
    if (e != cudaSuccess) {
        cudaFree(t->base);
        delete t;
        return cuda_err(e, "weight upload");
    }
    *out = t;
    return NEON_OK;
}

// On-load quantisation: `dst` is a type the quantiser produces from float rows.
bool quantizable(int src, int dst) {
    const bool float_src = src == NEON_GGML_F32 || src == NEON_GGML_F16 || src == NEON_GGML_BF16;
    return float_src && (q_block_bytes(dst) != 0 || dst == NEON_GGML_F16 || dst == NEON_GGML_BF16);
}

int check_quantize_args(int src_type, size_t rows, size_t cols, int dst_type) {
    if (!quantizable(src_type, dst_type))
        return set_err(NEON_ERR_UNSUPPORTED, "on-load quantisation takes F32/F16/BF16 rows to Q8_0, Q4_0, Q4_1, "
                                             "Q5_0, Q5_1, F16 or BF16 (got " + std::to_string(src_type) + " -> " +
                                                 std::to_string(dst_type) + ")");
    if (rows == 0 || cols == 0) return set_err(NEON_ERR_INVALID, "empty tensor");
    if (q_block_bytes(dst_type) && cols % 32 != 0)
        return set_err(NEON_ERR_INVALID, "input dim (" + std::to_string(cols) +
                                             ") isn't a multiple of the quantised type's block size (32)");
    return NEON_OK;
}

int launch_quantize(const void* d_src, int src_type, size_t rows, size_t cols, int dst_type, void* d_dst,
                    cudaStream_t st, int sms) {
    const long long per_row = q_block_bytes(dst_type) ? (long long)cols / 32 : (long long)cols;
    const long long n = (long long)rows * per_row;
    const int grid = (int)std::min<long long>((n + 255) / 256, (long long)sms * 16);
    quantize_rows_kernel<<<grid, 256, 0, st>>>(static_cast<const unsigned char*>(d_src),
                                               (long long)row_bytes_of(src_type, cols), src_type, (long long)rows,
                                               (long long)cols, dst_type, static_cast<unsigned char*>(d_dst),
                                               (long long)row_bytes_of(dst_type, cols));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cuda_check(cudaGetLastError(), "quantize_rows_kernel");
}

// Host float rows -> device GGUF rows of dst_type (caller frees *d_out).
int quantize_to_device(const void* host_src, int src_type, size_t rows, size_t cols, int dst_type, uint8_t** d_out) {
    *d_out = nullptr;
    int device = 0;
    int rc = current_device(&device);
    if (rc) return rc;
    const size_t in_bytes = rows * row_bytes_of(src_type, cols), out_bytes = rows * row_bytes_of(dst_type, cols);
    void* d_src = nullptr;
    uint8_t* d_dst = nullptr;
    if (cudaMalloc(&d_src, in_bytes) != cudaSuccess || cudaMalloc(&d_dst, out_bytes) != cudaSuccess) {
        cudaFree(d_src);
        cudaFree(d_dst);
        return set_err(NEON_ERR_NOMEM, "cudaMalloc of the quantisation buffers failed");
    }
    cudaStream_t st = g_dev[device].stream;
    cudaError_t e = cudaMemcpyAsync(d_src, host_src, in_bytes, cudaMemcpyHostToDevice, st);
    rc = e == cudaSuccess ? launch_quantize(d_src, src_type, rows, cols, dst_type, d_dst, st, g_dev[device].sms)
                          : cuda_err(e, "quantisation input copy");
    if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "quantisation");
    cudaFree(d_src);
    if (rc) {
        cudaFree(d_dst);
        return rc;
    }
    *d_out = d_dst;
    return NEON_OK;
}
}  // namespace

extern "C" {

int neon_cuda_upload(const uint8_t* host_bytes, int ggml_type, size_t rows, size_t cols, int shard_mode,
                     int shard_index, int shard_count, neon_tensor_t* out) {
    return upload_impl(host_bytes, false, ggml_type, rows, cols, shard_mode, shard_index, shard_count, out);
}

int neon_cuda_quantize_rows(const void* d_src, int src_type, size_t rows, size_t cols, int dst_type, void* d_dst,
                            void* stream) {
    if (!d_src || !d_dst) return set_err(NEON_ERR_INVALID, "null buffer");
    int rc = check_quantize_args(src_type, rows, cols, dst_type);
    if (rc) return rc;
    int device = 0;
    rc = current_device(&device);
    if (rc) return rc;
    return launch_quantize(d_src, src_type, rows, cols, dst_type, d_dst, (cudaStream_t)stream, g_dev[device].sms);
}

int neon_cuda_quantize_host(const void* host_src, int src_type, size_t rows, size_t cols, int dst_type,
                            void* host_dst) {
    if (!host_src || !host_dst) return set_err(NEON_ERR_INVALID, "null buffer");
    int rc = check_quantize_args(src_type, rows, cols, dst_type);
    if (rc) return rc;
    uint8_t* d = nullptr;
    rc = quantize_to_device(host_src, src_type, rows, cols, dst_type, &d);
    if (rc) return rc;
    cudaError_t e = cudaMemcpy(host_dst, d, rows * row_bytes_of(dst_type, cols), cudaMemcpyDeviceToHost);
    cudaFree(d);
    return cuda_check(e, "quantisation output copy");
}

int neon_cuda_upload_quantized(const void* host_src, int src_type, size_t rows, size_t cols, int dst_type,
                               int shard_mode, int shard_index, int shard_count, neon_tensor_t* out) {
    if (!out) return set_err(NEON_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (!host_src) return set_err(NEON_ERR_INVALID, "null weight bytes");
    int rc = check_quantize_args(src_type, rows, cols, dst_type);
    if (rc) return rc;
    // a row shard is quantised alone; a column shard is cut from the quantised rows
    size_t r0 = 0, r1 = rows;
    if (shard_mode == NEON_SHARD_ROWS) {
        if (shard_count <= 0 || shard_index < 0 || shard_index >= shard_count)
            return set_err(NEON_ERR_INVALID, "bad shard index/count");
        r0 = rows * (size_t)shard_index / (size_t)shard_count;
        r1 = rows * (size_t)(shard_index + 1) / (size_t)shard_count;
        if (r1 <= r0) return set_err(NEON_ERR_INVALID, "empty shard");
    }
    uint8_t* d = nullptr;
    rc = quantize_to_device(static_cast<const uint8_t*>(host_src) + r0 * row_bytes_of(src_type, cols), src_type,
                            r1 - r0, cols, dst_type, &d);
    if (rc) return rc;
    rc = upload_impl(d, true, dst_type, r1 - r0, cols, shard_mode == NEON_SHARD_ROWS ? NEON_SHARD_NONE : shard_mode,
                     shard_index, shard_count, out);
    cudaFree(d);
    return rc;
}

int neon_cuda_tensor_info(neon_tensor_t W, size_t* rows, size_t* cols, int* ggml_type, size_t* device_bytes) {
    if (!W) return set_err(NEON_ERR_INVALID, "null tensor handle");
    if (rows) *rows = W->rows;
    if (cols) *cols = W->cols;
    if (ggml_type) *ggml_type = W->type;
    if (device_bytes) *device_bytes = W->bytes;
    return NEON_OK;
}

int neon_cuda_free(neon_tensor_t W) {
    if (!W) return NEON_OK;
    DeviceGuard g(W->device);
    cudaError_t e = cudaFree(W->base);
    delete W;
    if (e != cudaSuccess) return cuda_err(e, "cudaFree");
    return NEON_OK;
}

int neon_cuda_quantize_q8_0(const float* dX, size_t x_stride, size_t cols, size_t seq, float* d_out,
                            int8_t* q_out, void* stream) {
    if (seq == 0 || cols == 0) return NEON_OK;
    if (!dX || !d_out || !q_out) return set_err(NEON_ERR_INVALID, "null pointer");
    if (cols % 32 != 0) return set_err(NEON_ERR_INVALID, "cols is not a multiple of 32");
    int device = 0;
    int rc = current_device(&device);
    if (rc) return rc;
    const int nb = (int)(cols / 32);
    long long blocks = (long long)nb * (long long)seq;
    int ctas = (int)std::min<long long>((blocks + kWarps - 1) / kWarps, (long long)g_dev[device].sms * 8);
    return launch(quantize_q8_0_kernel, dim3(ctas), 0, (cudaStream_t)stream, dX, (long long)x_stride, nb,
                  (int)seq, q_out, d_out, (int*)nullptr);
}

int neon_cuda_matvec(neon_tensor_t W, const float* dX, size_t x_stride, float* dY, size_t y_stride, size_t seq,
                     void* stream) {
    neon_proj_target_t t{W, dY, y_stride};
    return matvec_targets(&t, 1, dX, x_stride, seq, stream);
}

int neon_cuda_matvec_multi(const neon_proj_target_t* targets, size_t n_targets, const float* dX, size_t x_stride,
                           size_t seq, void* stream) {
    return matvec_targets(targets, n_targets, dX, x_stride, seq, stream);
}

int neon_cuda_proj_all_positions_multi(const neon_proj_target_t* targets, size_t n_targets, const float* hX,
                                       size_t x_stride, size_t seq) {
    if (n_targets == 0 || seq == 0) return NEON_OK;
    if (!targets || !hX) return set_err(NEON_ERR_INVALID, "null targets or X");
    int rc = validate_tensor(targets[0].W);
    if (rc) return rc;
    const int device = targets[0].W->device;
    rc = init_device(device);
    if (rc) return rc;
    DeviceState& ds = g_dev[device];
    std::lock_guard<std::mutex> lk(ds.mu);
    DeviceGuard guard(device);
    size_t x_elems = (seq - 1) * x_stride + targets[0].W->cols;
    for (size_t i = 0; i < n_targets; ++i)
        if (targets[i].W) x_elems = std::max(x_elems, (seq - 1) * x_stride + targets[i].W->cols);
    std::vector<size_t> y_off(n_targets), y_len(n_targets);
    size_t y_total = 0;
    for (size_t i = 0; i < n_targets; ++i) {
        rc = validate_tensor(targets[i].W);
        if (rc) return rc;
        size_t ys = seq > 1 ? targets[i].y_stride : targets[i].W->rows;
        y_len[i] = (seq - 1) * ys + targets[i].W->rows;
        y_off[i] = y_total;
        y_total += (y_len[i] + 63) / 64 * 64;
    }
    rc = grow((void**)&ds.dx, &ds.dx_cap, x_elems * 4);
    if (rc) return rc;
    rc = grow((void**)&ds.dy, &ds.dy_cap, y_total * 4);
    if (rc) return rc;
    cudaStream_t st = ds.stream;
    NEON_CUDA_TRY(cudaMemcpyAsync(ds.dx, hX, x_elems * 4, cudaMemcpyHostToDevice, st));
    std::vector<neon_proj_target_t> dt(targets, targets + n_targets);
    for (size_t i = 0; i < n_targets; ++i) {
        dt[i].Y = ds.dy + y_off[i];
        dt[i].y_stride = seq > 1 ? targets[i].y_stride : targets[i].W->rows;
        if (seq > 1 && targets[i].y_stride > targets[i].W->rows) {
            // Positions between rows and y_stride keep the caller's values.
            NEON_CUDA_TRY(cudaMemcpyAsync(dt[i].Y, targets[i].Y, y_len[i] * 4, cudaMemcpyHostToDevice, st));
        }
    }
    rc = matvec_targets(dt.data(), n_targets, ds.dx, x_stride, seq, st);
    if (rc) return rc;
    for (size_t i = 0; i < n_targets; ++i)
        NEON_CUDA_TRY(cudaMemcpyAsync(targets[i].Y, dt[i].Y, y_len[i] * 4, cudaMemcpyDeviceToHost, st));
    // the device error word comes back with Y: one synchronisation for both
    NEON_CUDA_TRY(cudaMemcpyAsync(ds.err_host, ds.err, sizeof(unsigned int), cudaMemcpyDeviceToHost, st));
    NEON_CUDA_TRY(cudaStreamSynchronize(st));
    if (*ds.err_host) {
        *ds.err_host = 0;
        return check_device_err(device);  // clears the device word and reports the timeout
    }
    return NEON_OK;
}

int neon_cuda_proj_all_positions(neon_tensor_t W, const float* hX, size_t x_stride, float* hY, size_t y_stride,
                                 size_t seq) {
    neon_proj_target_t t{W, hY, y_stride};
    return neon_cuda_proj_all_positions_multi(&t, 1, hX, x_stride, seq);
}

int neon_cuda_sync(void* stream) {
    NEON_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    int device = 0;
    NEON_CUDA_TRY(cudaGetDevice(&device));
    return check_device_err(device);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of the multi-position Q4_0 matvec.
//
// neon_cuda_matvec quantises X into library scratch that it cudaMalloc's on
// first use. Some callers cannot let a library allocate device memory: an
// inference server that reserves all of HBM for its own weight and KV-cache
// pools at start-up (a lazy cudaMalloc then fails, or breaks its budget), a
// process whose framework caching allocator already holds the free memory, or
// a latency-critical loop that cannot take cudaMalloc's implicit device-wide
// synchronisation. neon_cuda_matvec_q4_0_noalloc runs the same two kernels
// (quantize_q8_0_kernel, then matvec_multipos_kernel) with their scratch in
// the fixed array below instead: it calls no cudaMalloc, cudaFree or other
// allocating routine.
//
// The array is part of the library's device image, so every GPU that loads
// the library holds its 1.25 MiB until the process exits. Its device address
// is looked up once per device, on the first call made with that device's
// tensor (cudaGetSymbolAddress with the device current); make that first call
// before any stream capture. All calls share the one array: two calls whose
// kernels overlap on the GPU (different streams, or different host threads)
// race on it, so callers must order them. The quantiser writes every byte the
// matvec then reads, so nothing has to be cleared between calls, and the
// array keeps the last call's contents.
// ---------------------------------------------------------------------------

namespace {
constexpr size_t kNoAllocMaxElems = size_t(1) << 20;           // seq * cols limit
constexpr size_t kNoAllocQBytes = kNoAllocMaxElems;              // int8 quants
constexpr size_t kNoAllocDBytes = kNoAllocMaxElems / 32 * 4;     // fp32 block scales
constexpr size_t kNoAllocSBytes = kNoAllocMaxElems / 32 * 4;     // int32 block sums
constexpr size_t kNoAllocBytes = kNoAllocQBytes + kNoAllocDBytes + kNoAllocSBytes;
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_base[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
int noalloc_scratch(int device, unsigned char** base) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_base[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_err(e, "cudaGetSymbolAddress");
        g_noalloc_base[device] = static_cast<unsigned char*>(p);
    }
    *base = g_noalloc_base[device];
    return NEON_OK;
}
}  // namespace

extern "C" int neon_cuda_matvec_q4_0_noalloc(neon_tensor_t W, const float* dX, size_t x_stride, float* dY,
                                             size_t y_stride, size_t seq, void* stream) {
    int vrc = validate_tensor(W);
    if (vrc) return vrc;
    if (W->type != NEON_GGML_Q4_0)
        return set_err(NEON_ERR_UNSUPPORTED, "neon_cuda_matvec_q4_0_noalloc runs Q4_0 tensors only");
    if (W->device < 0 || W->device >= kMaxDevices) return set_err(NEON_ERR_INVALID, "device index out of range");
    if (W->cols == 0 || W->rows == 0) return set_err(NEON_ERR_INVALID, "empty tensor");
    if (seq == 0) return NEON_OK;
    if (!dX || !dY) return set_err(NEON_ERR_INVALID, "null X or Y");
    if (seq > 1 && y_stride < W->rows) return set_err(NEON_ERR_INVALID, "y_stride smaller than the tensor's rows");
    if (seq > kNoAllocMaxElems / W->cols)
        return set_err(NEON_ERR_INVALID, "seq*cols = " + std::to_string(seq) + "*" + std::to_string(W->cols) +
                                             " exceeds the allocation-free limit of " +
                                             std::to_string(kNoAllocMaxElems) + " activation elements");
    DeviceGuard guard(W->device);
    if (!guard.ok) return set_err(NEON_ERR_CUDA, "cudaSetDevice failed");
    unsigned char* base = nullptr;
    int rc = noalloc_scratch(W->device, &base);
    if (rc) return rc;
    int sms = 0;
    NEON_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, W->device));
    int8_t* xq = reinterpret_cast<int8_t*>(base);
    float* xd = reinterpret_cast<float*>(base + kNoAllocQBytes);
    int* xs = reinterpret_cast<int*>(base + kNoAllocQBytes + kNoAllocDBytes);
    cudaStream_t st = (cudaStream_t)stream;
    const int nb = (int)W->nb;
    const long long blocks = (long long)nb * (long long)seq;
    int qctas = (int)std::min<long long>((blocks + kWarps - 1) / kWarps, (long long)sms * 8);
    rc = launch(quantize_q8_0_kernel, dim3(qctas), 0, st, dX, (long long)x_stride, nb, (int)seq, xq, xd, xs);
    if (rc) return rc;
    MatvecArgs a;
    std::memset(&a, 0, sizeof(a));
    a.span[0].qs = W->qs;
    a.span[0].d = W->d;
    a.span[0].y = dY;
    a.span[0].y_stride = (long long)(seq > 1 ? y_stride : W->rows);
    a.span[0].rows = (int)W->rows;
    a.span[0].tile0 = 0;
    a.n_spans = 1;
    a.n_tiles = (int)((W->rows + kMpR - 1) / kMpR);
    a.nb = nb;
    a.seq = (int)seq;
    a.x = dX;
    a.x_stride = (long long)x_stride;
    a.xq = xq;
    a.xd = xd;
    a.xs = xs;
    int ctas = std::min((a.n_tiles + kWarps - 1) / kWarps, sms * 4);
    dim3 grid(ctas, (unsigned)((seq + kMpT - 1) / kMpT));
    return launch(matvec_multipos_kernel<NEON_GGML_Q4_0, kMpR, kMpT>, grid, 0, st, a);
}
