// One-shot all-reduce of float32 vectors over NVLink peer memory, for the
// row-parallel projections of tensor parallelism (the partial outputs of o_proj
// and down_proj, a few KB to a few hundred KB per call).
//
// Every rank owns a region (cudaMalloc, shared with the other ranks through
// CUDA IPC handles): two staging buffers of cap floats (used alternately by
// consecutive calls), a signal pad of kArBlocks x kArMaxRanks epoch words and
// kArBlocks epoch counters. A call with epoch e (one more than the previous
// call's) runs kArBlocks blocks, each on its slice of the vector; block c:
//   1. copies its slice of the local vector into staging buffer e & 1 of its
//      own region;
//   2. publishes e in slot (c, rank) of every rank's signal pad (release, system
//      scope) and waits until every slot (c, q) of its own pad holds e
//      (acquire, system scope; a bounded poll that records error 1 and leaves
//      the data as it was when it gives up);
//   3. sums the slice of every rank's staging buffer in rank order 0..W-1 (so
//      every rank computes bit-identical results) into the local vector.
// A rank reuses a staging buffer two calls later, after it has seen every
// rank's flag of the call in between, which each rank publishes only after
// it has finished reading the buffer: no second barrier is needed.
// No multicast objects and no collective library calls are involved.
#include <cuda_runtime.h>

#include <cstring>

#include "cdq.h"

namespace {

constexpr int kArBlocks = CDQ_AR_BLOCKS;
constexpr int kArMaxRanks = CDQ_AR_MAX_RANKS;
constexpr int kArThreads = 512;
constexpr uint32_t kArSpinLimit = 1u << 24;  // default polls of a flag before a wait gives up

__device__ int g_ar_error;
uint32_t g_ar_spin_limit = kArSpinLimit;  // process-wide, set by cdq_ar_set_spin_limit

struct ArArgs {
    float* stage[kArMaxRanks];     // each rank's staging buffers (2 x cap floats)
    uint32_t* pad[kArMaxRanks];    // each rank's signal pad [block][source rank]
    uint32_t* epoch;               // this rank's epoch counters [block]
    int64_t cap;
    int world, rank;
    uint32_t spin_limit;
};

// Region layout: staging 2 * cap floats | pad kArBlocks * kArMaxRanks words | epochs kArBlocks words
inline int64_t stage_bytes(int64_t cap) { return (2 * cap * 4 + 255) / 256 * 256; }
inline int64_t region_bytes(int64_t cap) {
    return stage_bytes(cap) + (int64_t)kArBlocks * kArMaxRanks * 4 + (int64_t)kArBlocks * 4;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float ld_relaxed_sys(const float* p) {
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kArThreads) ar_kernel(const ArArgs a, float* __restrict__ data, int64_t n) {
    __shared__ uint32_t s_epoch;
    __shared__ int s_ok;
    const int c = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) {
        s_epoch = *reinterpret_cast<volatile uint32_t*>(a.epoch + c) + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t e = s_epoch;
    const int64_t slice = (n + gridDim.x - 1) / gridDim.x;
    const int64_t lo = (int64_t)c * slice, hi = lo + slice < n ? lo + slice : n;
    const int64_t par = (int64_t)(e & 1u) * a.cap;
    float* mine = a.stage[a.rank] + par;
    for (int64_t i = lo + tid; i < hi; i += kArThreads) mine[i] = data[i];
    __syncthreads();
    if (tid < a.world) {
        __threadfence_system();
        st_release_sys(a.pad[tid] + c * kArMaxRanks + a.rank, e);
        const uint32_t* flag = a.pad[a.rank] + c * kArMaxRanks + tid;
        uint32_t spin = 0;
        while ((int32_t)(ld_acquire_sys(flag) - e) < 0) {
            if (++spin >= a.spin_limit) {
                s_ok = 0;
                atomicExch(&g_ar_error, 1);
                break;
            }
        }
    }
    __syncthreads();
    if (!s_ok) return;  // a peer never arrived: the data keeps this rank's partial
    for (int64_t i = lo + tid; i < hi; i += kArThreads) {
        float s = 0.f;
        for (int q = 0; q < a.world; ++q) s += ld_relaxed_sys(a.stage[q] + par + i);
        data[i] = s;
    }
    __syncthreads();
    if (tid == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch + c) = e;
}

}  // namespace

namespace cdq {
cudaError_t ar_read_error(int* out) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_ar_error, sizeof v);
    if (e != cudaSuccess) return e;
    *out = v;
    return cudaSuccess;
}
}  // namespace cdq

extern "C" {

cdq_status cdq_ar_create(int64_t cap, void** region, cdq_ipc_handle* handle) {
    if (cap < 1 || cap > ((int64_t)1 << 30) || !region || !handle) return CDQ_ERR_ARG;
    void* p = nullptr;
    if (cudaMalloc(&p, (size_t)region_bytes(cap)) != cudaSuccess) return CDQ_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, (size_t)region_bytes(cap)) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return CDQ_ERR_CUDA;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(handle->bytes), "handle size");
    std::memset(handle->bytes, 0, sizeof handle->bytes);
    std::memcpy(handle->bytes, &h, sizeof h);
    *region = p;
    return CDQ_OK;
}

cdq_status cdq_ar_open(const cdq_ipc_handle* handle, void** peer_region) {
    if (!handle || !peer_region) return CDQ_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof h);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return CDQ_ERR_CUDA;
    *peer_region = p;
    return CDQ_OK;
}

cdq_status cdq_ar_close(void* peer_region) {
    if (!peer_region) return CDQ_ERR_ARG;
    return cudaIpcCloseMemHandle(peer_region) == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

cdq_status cdq_ar_destroy(void* region) {
    if (!region) return CDQ_ERR_ARG;
    return cudaFree(region) == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

cdq_status cdq_allreduce_f32(void* const* regions, int32_t world, int32_t rank, int64_t cap, float* data,
                             int64_t n, void* stream) {
    if (!regions || world < 1 || world > kArMaxRanks || rank < 0 || rank >= world || cap < 1 || !data ||
        n < 0 || n > cap)
        return CDQ_ERR_ARG;
    if (n == 0) return CDQ_OK;
    ArArgs a;
    std::memset(&a, 0, sizeof a);
    for (int q = 0; q < world; ++q) {
        if (!regions[q]) return CDQ_ERR_ARG;
        uint8_t* base = static_cast<uint8_t*>(regions[q]);
        a.stage[q] = reinterpret_cast<float*>(base);
        a.pad[q] = reinterpret_cast<uint32_t*>(base + stage_bytes(cap));
    }
    a.epoch = a.pad[rank] + kArBlocks * kArMaxRanks;
    a.cap = cap;
    a.world = world;
    a.rank = rank;
    a.spin_limit = g_ar_spin_limit;
    // always kArBlocks blocks: the blocks' epochs advance together, so one call
    // uses one staging parity throughout, whatever slice a block covers
    ar_kernel<<<kArBlocks, kArThreads, 0, (cudaStream_t)stream>>>(a, data, n);
    return cudaGetLastError() == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

cdq_status cdq_ar_error(int32_t* code) {
    if (!code) return CDQ_ERR_ARG;
    int v = 0;
    if (cdq::ar_read_error(&v) != cudaSuccess) return CDQ_ERR_CUDA;
    *code = v;
    return CDQ_OK;
}

cdq_status cdq_ar_clear_error(void) {
    const int zero = 0;
    return cudaMemcpyToSymbol(g_ar_error, &zero, sizeof zero) == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

cdq_status cdq_ar_set_spin_limit(int64_t polls) {
    if (polls < 1 || polls > (int64_t)UINT32_MAX) return CDQ_ERR_ARG;
    g_ar_spin_limit = (uint32_t)polls;
    return CDQ_OK;
}

}  // extern "C"
