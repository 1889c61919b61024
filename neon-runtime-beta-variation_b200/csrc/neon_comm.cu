// neon_comm.cu -- tensor-parallel communicator of the decode step: one-shot
// collectives over peer memory (NVLink / NVSwitch), one rank per GPU.
//
// Reference counterpart: rocm::MultiGpuCtx::all_reduce_sum (rawllm_rocm.hpp:
// 531-562), an in-place fp32 sum across devices that the reference declares
// but never wires into transformer_forward. Here the all-reduce runs after the
// column-split attn_output and ffn_down projections of every layer, the
// all-gather assembles vocabulary-split logits, and the argmax exchange picks
// the greedy token of a vocabulary-split lm_head.
//
// Protocol of one all-reduce over `world` ranks (comm_reduce_kernel; CTA s of
// the fixed kCommSlices-CTA grid handles slice s of the vector):
//   1. push: rank r stores its slice into receive slot [parity][r] of every
//      rank's buffer (plain P2P stores through the peer mapping);
//   2. publish: after a system-scope fence, r release-stores the call's epoch
//      into flag [r][s] of every rank;
//   3. wait: r acquire-polls flags [src][s] of its own buffer until every
//      source has published this epoch -- bounded by the communicator's
//      timeout, after which it sets bit 0 of the error word and returns; a
//      communicator whose error word is set skips all later calls;
//   4. reduce: out[i] (+)= slot[0][i] + slot[1][i] + ... in rank order, so the
//      replicated residual stream stays bit-identical on every rank.
// Every call runs all kCommSlices CTAs, so all slices share the call count as
// their epoch and the two parity halves alternate per call. That suffices: a
// rank enters call e+2 (writing parity e&1 again) only after every peer has
// published call e+1, which each peer does only after it finished reading
// call e.
//
// Ranks must never be emulated as several launches on one GPU: the waits of
// one launch would need the other to run concurrently, which nothing
// guarantees. A communicator whose peers are buffers on the same device is
// only for a single rank's tests (its waits then run out and report it).
#include "neon_cuda.h"
#include "neon_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <string>

using neon_internal::cuda_error;
using neon_internal::error;

namespace {
constexpr int kEpochWords = kCommSlices + 3;  // slices, key exchange, fused calls, fused counter
std::atomic<int> g_fused{1};
}  // namespace

namespace {

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void pdl_wait_c() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_c() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Wait until flag *f has reached `epoch` (wrap-safe); false after `timeout` ns.
__device__ bool wait_flag(const unsigned int* f, unsigned int epoch, unsigned long long timeout) {
    if ((int)(ld_acquire_sys(f) - epoch) >= 0) return true;
    const unsigned long long t0 = gtimer();
    while ((int)(ld_acquire_sys(f) - epoch) < 0) {
        if (gtimer() - t0 > timeout) return false;
        __nanosleep(64);
    }
    return true;
}

// Slice [i0, i1) of an n-element vector for CTA `s` of kCommSlices (4-aligned starts).
__device__ __forceinline__ void slice_range(long long n, int s, long long& i0, long long& i1) {
    const long long per = ((n + kCommSlices - 1) / kCommSlices + 3) & ~3LL;
    i0 = min((long long)s * per, n);
    i1 = min(i0 + per, n);
}

// mode 0: all-reduce of n floats (out (+)= sum); mode 1: all-gather, rank r
// contributing rows [n*r/world, n*(r+1)/world) of out from `in`.
__global__ void __launch_bounds__(256) comm_reduce_kernel(CommPeers c, const float* __restrict__ in,
                                                          float* __restrict__ out, long long n, int add, int mode,
                                                          int vec, unsigned int* __restrict__ epochs,
                                                          unsigned int* __restrict__ err,
                                                          unsigned long long timeout) {
    __shared__ int s_bad;
    pdl_wait_c();
    pdl_trigger_c();
    const int slice = blockIdx.x;
    if (threadIdx.x == 0) s_bad = *reinterpret_cast<volatile unsigned int*>(err) != 0u;
    __syncthreads();
    if (s_bad) return;  // an earlier wait gave up: the communicator is broken
    const unsigned int epoch = epochs[slice] + 1u;
    const int parity = (int)(epoch & 1u);
    // 1. push
    long long my_n = n;
    if (mode == 1) my_n = n * (c.rank + 1) / c.world - n * c.rank / c.world;
    long long i0, i1;
    slice_range(my_n, slice, i0, i1);
    if (vec) {
        const long long v1 = i0 + ((i1 - i0) & ~3LL);
        for (long long i = i0 + 4 * threadIdx.x; i < v1; i += 4 * blockDim.x) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(in + i));
            for (int p = 0; p < c.world; ++p)
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(c.base[p] + comm_recv_off(c, parity, c.rank)) + i) = v;
        }
        for (long long i = v1 + threadIdx.x; i < i1; i += blockDim.x) {
            const float v = __ldcg(in + i);
            for (int p = 0; p < c.world; ++p)
                reinterpret_cast<float*>(c.base[p] + comm_recv_off(c, parity, c.rank))[i] = v;
        }
    } else {
        for (long long i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
            const float v = __ldcg(in + i);
            for (int p = 0; p < c.world; ++p)
                reinterpret_cast<float*>(c.base[p] + comm_recv_off(c, parity, c.rank))[i] = v;
        }
    }
    __threadfence_system();
    __syncthreads();
    // 2. publish, 3. wait
    if ((int)threadIdx.x < c.world) {
        unsigned int* f = reinterpret_cast<unsigned int*>(c.base[threadIdx.x] + comm_flags_off(c)) +
                          c.rank * kCommSlices + slice;
        st_release_sys(f, epoch);
    }
    __syncthreads();
    if ((int)threadIdx.x < c.world) {
        const unsigned int* f = reinterpret_cast<const unsigned int*>(c.base[c.rank] + comm_flags_off(c)) +
                                threadIdx.x * kCommSlices + slice;
        if (!wait_flag(f, epoch, timeout)) {
            atomicOr(err, 1u);
            s_bad = 1;
        }
    }
    __syncthreads();
    if (s_bad) return;
    // 4. reduce / gather from this rank's own buffer
    const unsigned char* mine = c.base[c.rank];
    if (mode == 0) {
        if (vec) {
            const long long v1 = i0 + ((i1 - i0) & ~3LL);
            for (long long i = i0 + 4 * threadIdx.x; i < v1; i += 4 * blockDim.x) {
                float4 s = __ldcg(reinterpret_cast<const float4*>(
                    reinterpret_cast<const float*>(mine + comm_recv_off(c, parity, 0)) + i));
                for (int src = 1; src < c.world; ++src) {
                    const float4 v = __ldcg(reinterpret_cast<const float4*>(
                        reinterpret_cast<const float*>(mine + comm_recv_off(c, parity, src)) + i));
                    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
                }
                float4* o = reinterpret_cast<float4*>(out + i);
                if (add) {
                    const float4 h = *o;
                    s.x = h.x + s.x; s.y = h.y + s.y; s.z = h.z + s.z; s.w = h.w + s.w;
                }
                *o = s;
            }
            for (long long i = v1 + threadIdx.x; i < i1; i += blockDim.x) {
                float s = 0.f;
                for (int src = 0; src < c.world; ++src)
                    s = src ? s + __ldcg(reinterpret_cast<const float*>(mine + comm_recv_off(c, parity, src)) + i)
                            : __ldcg(reinterpret_cast<const float*>(mine + comm_recv_off(c, parity, src)) + i);
                out[i] = add ? out[i] + s : s;
            }
        } else {
            for (long long i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
                float s = 0.f;
                for (int src = 0; src < c.world; ++src)
                    s = src ? s + __ldcg(reinterpret_cast<const float*>(mine + comm_recv_off(c, parity, src)) + i)
                            : __ldcg(reinterpret_cast<const float*>(mine + comm_recv_off(c, parity, src)) + i);
                out[i] = add ? out[i] + s : s;
            }
        }
    } else {
        for (int src = 0; src < c.world; ++src) {
            const long long off = n * src / c.world;
            const long long len = n * (src + 1) / c.world - off;
            long long j0, j1;
            slice_range(len, slice, j0, j1);
            const float* slot = reinterpret_cast<const float*>(mine + comm_recv_off(c, parity, src));
            for (long long i = j0 + threadIdx.x; i < j1; i += blockDim.x) out[off + i] = __ldcg(slot + i);
        }
    }
    if (threadIdx.x == 0) epochs[slice] = epoch;
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64c(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_sys_u64c(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// One warp, LL words: lane p stores this rank's argmax key -- its high and
// low halves as two words tagged with the exchange number -- into slot
// [parity][rank] of rank p, and lane src polls (bounded) slot [parity][src]
// of this rank. The largest key wins (argmax_kernel's packing: the larger
// value, among equal values the lower global index).
__global__ void comm_argmax_kernel(CommPeers c, unsigned long long* key, int* d_tok, int* out, int* d_step, int* d_pos,
                                   int advance, unsigned int* __restrict__ epochs, unsigned int* __restrict__ err,
                                   unsigned long long timeout) {
    pdl_wait_c();
    pdl_trigger_c();
    const int lane = threadIdx.x;
    if (*reinterpret_cast<volatile unsigned int*>(err) != 0u) return;
    const unsigned int epoch = epochs[kCommSlices] + 1u;
    const int parity = (int)(epoch & 1u);
    const unsigned long long mine = __ldcg(key);
    const long long keys = comm_ll_off(c) + ll_keys_off(c.world);
    if (lane < c.world) {
        unsigned long long* dst =
            reinterpret_cast<unsigned long long*>(c.base[lane] + keys) + 2 * (parity * kCommMaxRanks + c.rank);
        st_relaxed_sys_u64c(dst, ((unsigned long long)epoch << 32) | (mine >> 32));
        st_relaxed_sys_u64c(dst + 1, ((unsigned long long)epoch << 32) | (mine & 0xFFFFFFFFull));
    }
    bool ok = true;
    unsigned long long k = 0ull;
    if (lane < c.world) {
        const unsigned long long* src =
            reinterpret_cast<const unsigned long long*>(c.base[c.rank] + keys) + 2 * (parity * kCommMaxRanks + lane);
        unsigned long long hi = ld_relaxed_sys_u64c(src), lo = ld_relaxed_sys_u64c(src + 1);
        if ((unsigned int)(hi >> 32) != epoch || (unsigned int)(lo >> 32) != epoch) {
            const unsigned long long t0 = gtimer();
            for (;;) {
                hi = ld_relaxed_sys_u64c(src);
                lo = ld_relaxed_sys_u64c(src + 1);
                if ((unsigned int)(hi >> 32) == epoch && (unsigned int)(lo >> 32) == epoch) break;
                if (gtimer() - t0 > timeout) {
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
        }
        k = (hi << 32) | (lo & 0xFFFFFFFFull);
    }
    if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) atomicOr(err, 1u);
        return;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
        k = other > k ? other : k;
    }
    if (lane == 0) {
        const int tok = k ? (int)(0xFFFFFFFFu - (unsigned int)(k & 0xFFFFFFFFull)) : 0;  // all NaN: element 0
        *d_tok = tok;
        out[*d_step] = tok;
        *d_step += 1;
        if (advance) *d_pos += 1;
        *key = 0ull;
        epochs[kCommSlices] = epoch;
    }
}

// Bounded poll of one LL word until it carries `call`.
__device__ __noinline__ unsigned long long ll_wait_word(const unsigned long long* a, unsigned int call, unsigned int* err,
                                                        unsigned long long timeout, volatile int* skip) {
    const unsigned long long t0 = gtimer();
    for (;;) {
        const unsigned long long w = ld_relaxed_sys_u64c(a);
        if ((unsigned int)(w >> 32) == call || *skip) return w;
        if (gtimer() - t0 > timeout) {
            atomicOr(err, 1u);
            *skip = 1;
            return w;
        }
        __nanosleep(32);
    }
}

// Second half of a fused all-reduce (the producing matvec stored this rank's
// partial rows as LL words in every rank's slot): h[i] += slot_0[i] +
// slot_1[i] + ... in rank order, one thread per element; all of a thread's
// loads are issued before any wait. The last CTA records the call as
// completed (every CTA read the count before it counted itself in).
// wait_producer 0 skips the dependency wait, so that the polls overlap a long
// producer's tail: the words carry their call number, so polling them is the
// synchronisation; h and the call count were written by kernels that
// completed before the producer's own dependency wait returned, and a
// producer stages its input before it stores a word, so when every word has
// arrived nothing of the producer's reads is left for later writers. The
// kernel after this one waits for it as usual.
__global__ void __launch_bounds__(256) comm_ll_reduce_kernel(PeerSet p, float* __restrict__ h, int n,
                                                             int wait_producer) {
    __shared__ int s_skip;
    if (wait_producer) pdl_wait_c();
    pdl_trigger_c();
    if (threadIdx.x == 0) s_skip = *reinterpret_cast<volatile unsigned int*>(p.err) != 0u;
    __syncthreads();
    const unsigned int call = *reinterpret_cast<volatile const unsigned int*>(p.calls) + 1u;
    const unsigned long long* slots =
        reinterpret_cast<const unsigned long long*>(p.base[p.rank] + ll_slot_off(p.world, (int)(call & 1u), 0));
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        unsigned long long w[kCommMaxRanks];
#pragma unroll
        for (int r = 0; r < kCommMaxRanks; ++r)
            if (r < p.world) w[r] = ld_relaxed_sys_u64c(slots + (long long)r * kCommFusedFloats + i);
        float s = 0.f;
#pragma unroll
        for (int r = 0; r < kCommMaxRanks; ++r) {
            if (r < p.world) {
                if ((unsigned int)(w[r] >> 32) != call)
                    w[r] = ll_wait_word(slots + (long long)r * kCommFusedFloats + i, call, p.err, p.timeout_ns, &s_skip);
                const float v = __uint_as_float((unsigned int)w[r]);
                s = r ? s + v : v;
            }
        }
        h[i] = h[i] + s;
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(p.counter, 1u) == gridDim.x - 1) {
        *p.counter = 0u;
        *p.calls = call;
    }
}

// Second half of a fused all-gather (each rank's row-shard matvec stored its
// rows as LL words at their places in the gather slot of every rank): y[i] =
// the value of word i of this rank's gather slot, for i < n, waiting
// (bounded) until the word carries this call; all of a thread's loads are
// issued before any wait. The last CTA records the call as completed.
__global__ void __launch_bounds__(256) comm_ll_gather_kernel(PeerSet p, float* __restrict__ y, int n) {
    __shared__ int s_skip;
    pdl_wait_c();
    pdl_trigger_c();
    if (threadIdx.x == 0) s_skip = *reinterpret_cast<volatile unsigned int*>(p.err) != 0u;
    __syncthreads();
    const unsigned int call = *reinterpret_cast<volatile const unsigned int*>(p.calls) + 1u;
    const unsigned long long* slot =
        reinterpret_cast<const unsigned long long*>(p.base[p.rank] + ll_slot_off(p.world, (int)(call & 1u), 0));
    constexpr int kPer = 4;
    for (int i0 = blockIdx.x * blockDim.x * kPer + threadIdx.x; i0 < n; i0 += gridDim.x * blockDim.x * kPer) {
        unsigned long long w[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = i0 + k * blockDim.x;
            if (i < n) w[k] = ld_relaxed_sys_u64c(slot + i);
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = i0 + k * blockDim.x;
            if (i < n) {
                if ((unsigned int)(w[k] >> 32) != call) w[k] = ll_wait_word(slot + i, call, p.err, p.timeout_ns, &s_skip);
                y[i] = __uint_as_float((unsigned int)w[k]);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(p.counter, 1u) == gridDim.x - 1) {
        *p.counter = 0u;
        *p.calls = call;
    }
}

template <typename... KArgs, typename... Args>
int launch_comm(void (*kern)(KArgs...), int grid, int threads, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (neon_internal::pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    if (e != cudaSuccess) return cuda_error(e, "cudaLaunchKernelEx(communicator)");
    return neon_internal::launched(1);
}

}  // namespace

namespace neon_internal {

int comm_allreduce(neon_comm_impl* c, const float* in, float* out, long long n, int add, cudaStream_t st) {
    if (!c || !c->connected) return error(NEON_ERR_INVALID, "communicator not connected");
    if (n <= 0) return NEON_OK;
    if (n > c->peers.max_floats) return error(NEON_ERR_INVALID, "all-reduce larger than the communicator's buffer");
    const int vec = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
    return launch_comm(comm_reduce_kernel, kCommSlices, 256, st, c->peers, in, out, n, add, 0, vec, c->epochs, c->err,
                       c->timeout_ns);
}

int comm_allgather(neon_comm_impl* c, const float* in, float* out, long long n, cudaStream_t st) {
    if (!c || !c->connected) return error(NEON_ERR_INVALID, "communicator not connected");
    if (n <= 0) return NEON_OK;
    if ((n + c->peers.world - 1) / c->peers.world > c->peers.max_floats)
        return error(NEON_ERR_INVALID, "all-gather shard larger than the communicator's buffer");
    const int vec = ((reinterpret_cast<uintptr_t>(in)) & 15u) == 0;
    return launch_comm(comm_reduce_kernel, kCommSlices, 256, st, c->peers, in, out, n, 0, 1, vec, c->epochs, c->err,
                       c->timeout_ns);
}

PeerSet comm_peer_set(neon_comm_impl* c) {
    PeerSet p{};
    for (int r = 0; r < c->peers.world; ++r) p.base[r] = c->peers.base[r] + comm_ll_off(c->peers);
    p.calls = c->epochs + kCommSlices + 1;
    p.counter = c->epochs + kCommSlices + 2;
    p.err = c->err;
    p.timeout_ns = c->timeout_ns;
    p.rank = c->peers.rank;
    p.world = c->peers.world;
    return p;
}

bool fused_collectives() { return g_fused.load(std::memory_order_relaxed) != 0; }

int comm_ll_reduce(neon_comm_impl* c, float* h, long long n, cudaStream_t st, bool wait_producer) {
    if (!c || !c->connected) return error(NEON_ERR_INVALID, "communicator not connected");
    if (n <= 0 || n > kCommFusedFloats) return error(NEON_ERR_INVALID, "fused all-reduce: bad length");
    const int grid = (int)std::min<long long>((n + 255) / 256, 148);
    return launch_comm(comm_ll_reduce_kernel, grid, 256, st, comm_peer_set(c), h, (int)n, wait_producer ? 1 : 0);
}

int comm_ll_gather(neon_comm_impl* c, float* y, long long n, cudaStream_t st) {
    if (!c || !c->connected) return error(NEON_ERR_INVALID, "communicator not connected");
    if (n <= 0 || n > kCommFusedFloats) return error(NEON_ERR_INVALID, "fused all-gather: bad length");
    const int grid = (int)std::min<long long>((n + 1023) / 1024, 148);
    return launch_comm(comm_ll_gather_kernel, grid, 256, st, comm_peer_set(c), y, (int)n);
}

int comm_argmax(neon_comm_impl* c, unsigned long long* key, int* d_tok, int* out, int* d_step, int* d_pos, int advance,
                cudaStream_t st) {
    if (!c || !c->connected) return error(NEON_ERR_INVALID, "communicator not connected");
    return launch_comm(comm_argmax_kernel, 1, 32, st, c->peers, key, d_tok, out, d_step, d_pos, advance, c->epochs,
                       c->err, c->timeout_ns);
}

}  // namespace neon_internal

extern "C" {

int neon_cuda_comm_create(int rank, int world, size_t max_floats, neon_comm_t* out) {
    if (!out) return error(NEON_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (world < 1 || world > kCommMaxRanks || rank < 0 || rank >= world)
        return error(NEON_ERR_INVALID, "rank/world out of range (world at most 8)");
    if (max_floats == 0) return error(NEON_ERR_INVALID, "empty communicator buffer");
    auto* c = new neon_comm();
    cudaGetDevice(&c->device);
    c->peers.rank = rank;
    c->peers.world = world;
    c->peers.max_floats = (long long)((max_floats + 63) / 64 * 64);
    const long long bytes = comm_bytes(c->peers);
    cudaError_t e = cudaMalloc(&c->local, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMemset(c->local, 0, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMalloc(&c->epochs, sizeof(unsigned int) * kEpochWords);
    if (e == cudaSuccess) e = cudaMemset(c->epochs, 0, sizeof(unsigned int) * kEpochWords);
    if (e == cudaSuccess) e = cudaMalloc(&c->err, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof(unsigned int));
    cudaIpcMemHandle_t h;
    std::memset(&h, 0, sizeof(h));
    if (e == cudaSuccess && world > 1) e = cudaIpcGetMemHandle(&h, c->local);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        const int rc = cuda_error(e, "communicator allocation");
        neon_cuda_comm_free(c);
        return rc;
    }
    c->ipc_handle.assign(reinterpret_cast<const char*>(&h), sizeof(h));
    c->peers.base[rank] = c->local;
    if (world == 1) c->connected = true;
    *out = c;
    return NEON_OK;
}

int neon_cuda_comm_ipc_handle(neon_comm_t c, void* handle_out, size_t* handle_bytes) {
    if (!c || !handle_bytes) return error(NEON_ERR_INVALID, "null argument");
    if (handle_out && *handle_bytes < sizeof(cudaIpcMemHandle_t))
        return error(NEON_ERR_INVALID, "handle buffer too small");
    *handle_bytes = sizeof(cudaIpcMemHandle_t);
    if (handle_out) std::memcpy(handle_out, c->ipc_handle.data(), sizeof(cudaIpcMemHandle_t));
    return NEON_OK;
}

int neon_cuda_comm_connect(neon_comm_t c, const void* all_handles, size_t handle_bytes) {
    if (!c || !all_handles) return error(NEON_ERR_INVALID, "null argument");
    if (handle_bytes != sizeof(cudaIpcMemHandle_t)) return error(NEON_ERR_INVALID, "wrong IPC handle size");
    if (c->connected) return NEON_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    int rc = NEON_OK;
    for (int p = 0; p < c->peers.world && !rc; ++p) {
        if (p == c->peers.rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(all_handles) + (size_t)p * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            rc = cuda_error(e, "cudaIpcOpenMemHandle");
            break;
        }
        c->peers.base[p] = static_cast<unsigned char*>(ptr);
    }
    if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
    if (rc) return rc;
    c->opened_ipc = true;
    c->connected = true;
    return NEON_OK;
}

int neon_cuda_comm_connect_local(neon_comm_t* comms, int n) {
    if (!comms || n < 1 || n > kCommMaxRanks) return error(NEON_ERR_INVALID, "bad communicator list");
    for (int i = 0; i < n; ++i) {
        if (!comms[i] || comms[i]->peers.world != n || comms[i]->peers.rank != i)
            return error(NEON_ERR_INVALID, "communicator i must be rank i of a world of n");
        if (comms[i]->connected && n > 1) return error(NEON_ERR_INVALID, "communicator already connected");
    }
    int prev = -1;
    cudaGetDevice(&prev);
    for (int i = 0; i < n; ++i) {
        for (int p = 0; p < n; ++p) {
            if (comms[p]->device != comms[i]->device) {
                cudaSetDevice(comms[i]->device);
                cudaError_t e = cudaDeviceEnablePeerAccess(comms[p]->device, 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
                else if (e != cudaSuccess) {
                    if (prev >= 0) cudaSetDevice(prev);
                    return cuda_error(e, "cudaDeviceEnablePeerAccess");
                }
            }
            comms[i]->peers.base[p] = comms[p]->local;
        }
        comms[i]->connected = true;
    }
    if (prev >= 0) cudaSetDevice(prev);
    return NEON_OK;
}

int neon_cuda_comm_set_timeout(neon_comm_t c, double seconds) {
    if (!c || !(seconds > 0.0) || seconds > 3600.0) return error(NEON_ERR_INVALID, "timeout must be in (0, 3600] s");
    c->timeout_ns = (unsigned long long)(seconds * 1e9);
    return NEON_OK;
}

int neon_cuda_set_fused_collectives(int enabled) {
    g_fused.store(enabled ? 1 : 0);
    return NEON_OK;
}

int neon_cuda_comm_allreduce(neon_comm_t c, const float* dIn, float* dOut, size_t n, int add, void* stream) {
    if (!c || !dIn || !dOut) return error(NEON_ERR_INVALID, "null argument");
    return neon_internal::comm_allreduce(c, dIn, dOut, (long long)n, add, (cudaStream_t)stream);
}

int neon_cuda_matvec_allgather(neon_comm_t c, neon_tensor_t W, const float* dX, float* dY, size_t n_total,
                               size_t row0, void* stream) {
    if (!c || !W || !dX || !dY) return error(NEON_ERR_INVALID, "null argument");
    if (!c->connected) return error(NEON_ERR_INVALID, "communicator not connected");
    if (W->device != c->device) return error(NEON_ERR_INVALID, "the shard and the communicator live on different devices");
    if (n_total == 0 || n_total > (size_t)kCommFusedFloats || row0 + W->rows > n_total)
        return error(NEON_ERR_INVALID, "all-gather matvec: rows [row0, row0 + shard rows) must lie in [0, n_total), "
                                       "n_total <= " + std::to_string(kCommFusedFloats));
    const neon_proj_target_t t{W, dY, W->rows};
    neon_internal::MatvecExt ext;
    ext.peer_mode = 2;
    ext.gather_row0 = (long long)row0;
    ext.peer = neon_internal::comm_peer_set(c);
    const cudaStream_t st = (cudaStream_t)stream;
    int rc = neon_internal::matvec(&t, 1, dX, W->cols, 1, st, 0, &ext);
    if (!rc) rc = neon_internal::comm_ll_gather(c, dY, (long long)n_total, st);
    return rc;
}

int neon_cuda_comm_check(neon_comm_t c) {
    if (!c) return error(NEON_ERR_INVALID, "null communicator");
    unsigned int v = 0;
    cudaError_t e = cudaMemcpy(&v, c->err, sizeof(v), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemcpy");
    if (v) return error(NEON_ERR_CUDA, "a collective gave up waiting for a peer rank; the communicator must be recreated");
    return NEON_OK;
}

int neon_cuda_comm_free(neon_comm_t c) {
    if (!c) return NEON_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    if (c->opened_ipc)
        for (int p = 0; p < c->peers.world; ++p)
            if (p != c->peers.rank && c->peers.base[p]) cudaIpcCloseMemHandle(c->peers.base[p]);
    if (c->local) cudaFree(c->local);
    if (c->epochs) cudaFree(c->epochs);
    if (c->err) cudaFree(c->err);
    if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
    delete c;
    return NEON_OK;
}

}  // extern "C"
