// Fused dequant-GEMV for the CDQ-LRR device pack, batch M <= 8 (CUDA cores).
//
// y[m, row] = sum_col w_hat[row, col] * x[m, col] (+ bias[row]) where
// w_hat = bf16(LATTICE[q] * sigma) is rebuilt in registers from the packed
// tiles and never written to memory (the reference materialises w_hat and
// calls F.linear: code/cdq_lrr_qwen05.py:188-198, code/cdq_loader.py:53-58).
//
// Work decomposition. A work item is (job, row block rb of 32 rows, residual
// group g of up to 32 tile columns); one warp processes one item with lane l
// owning row 32*rb + l, so every load of the pack is a coalesced 512-byte
// (plus 128-byte) sweep and the activations are warp-uniform broadcast loads.
// Items of all jobs of a launch are spread over the grid's warps.
//
// Dequantisation. Each pair of neighbouring weights has one pair code
// (26-state: 10 bits, 27 x 27 codes including the zero-valued residual slot;
// 16-state: one byte). A shared-memory table maps the pair code to the bf16
// pair (LATTICE[a], LATTICE[b]); every lane owns a private copy of the table
// in its own bank, so the 32 lookups of a warp never conflict. One bf16x2
// multiply by (sigma, sigma) then yields the two exact w_hat values (a single
// rounding of the exact product, which is what torch's bf16 multiply does),
// and two mixed-precision FMAs (bf16 x bf16 + fp32) accumulate in fp32.
//
// Residuals. Residual positions carry the zero symbol in the codes; their
// bf16 values come from the item's CSR bucket (one per lane) and are added as
// value * x[col] in the same warp after the tile sweep.
//
// Split K. When a row has more than one residual group the warp writes its
// partial sums to a per-group slot of the workspace and bumps the row block's
// arrival counter; the warp that arrives last adds the slots in group order
// (deterministic), applies bias, stores y and resets the counter to zero.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "cdq.h"
#include "cdq_common.cuh"
#include "cdq_internal.cuh"

namespace cdq {

__constant__ uint16_t c_lat26[27];
__constant__ uint16_t c_lat16[16];

namespace {

template <int NS>
struct PackTraits;
template <>
struct PackTraits<26> {
    static constexpr int kWords = 5;
    static constexpr int kPairs = kPairs26;
};
template <>
struct PackTraits<16> {
    static constexpr int kWords = 4;
    static constexpr int kPairs = kPairs16;
};

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint32_t ldg_nc(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ldg_nc4(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
// Activations: read by every lane of a warp (broadcast), cached in L1.
__device__ __forceinline__ uint4 ldg_x4(const uint16_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// acc0 += lo(w2) * lo(x2), acc1 += hi(w2) * hi(x2), single rounding in fp32.
__device__ __forceinline__ void fma_pair(float& acc0, float& acc1, uint32_t w2, uint32_t x2) {
    asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
        "mov.b32 {wl, wh}, %2;\n\t"
        "mov.b32 {xl, xh}, %3;\n\t"
        "fma.rn.f32.bf16 %0, wl, xl, %0;\n\t"
        "fma.rn.f32.bf16 %1, wh, xh, %1;\n\t}"
        : "+f"(acc0), "+f"(acc1)
        : "r"(w2), "r"(x2));
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Pair code j of a tile from its code words.
template <int NS, int J>
__device__ __forceinline__ uint32_t pair_code(const uint32_t (&w)[5]) {
    if constexpr (NS == 26) {
        constexpr int bit = 10 * J, wd = bit / 32, off = bit % 32;
        if constexpr (off <= 22) {
            return (w[wd] >> off) & 0x3FFu;
        } else {
            return __funnelshift_r(w[wd], w[wd + 1], off) & 0x3FFu;
        }
    } else {
        return (w[J / 4] >> (8 * (J % 4))) & 0xFFu;
    }
}

template <int NS, int M, int Q>
__device__ __forceinline__ void tile_quarter(const uint32_t (&w)[5], const uint32_t* tab,
                                             uint32_t ss, const uint4 (&xv)[M],
                                             float (&acc)[M][2]) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        uint32_t code;
        switch (jj) {  // J must be a compile-time constant
            case 0: code = pair_code<NS, Q * 4 + 0>(w); break;
            case 1: code = pair_code<NS, Q * 4 + 1>(w); break;
            case 2: code = pair_code<NS, Q * 4 + 2>(w); break;
            default: code = pair_code<NS, Q * 4 + 3>(w); break;
        }
        uint32_t pair = tab[code * 32];
        uint32_t wp = bmul2(pair, ss);
#pragma unroll
        for (int m = 0; m < M; ++m) fma_pair(acc[m][0], acc[m][1], wp, word_of(xv[m], jj));
    }
}

template <int NS, int M>
__device__ __forceinline__ void tile_dot(const uint32_t (&w)[5], const uint32_t* tab, uint32_t ss,
                                         const uint16_t* xcol, int64_t cols, float (&acc)[M][2]) {
    uint4 xv[M];
#pragma unroll
    for (int m = 0; m < M; ++m) xv[m] = ldg_x4(xcol + m * cols + 0);
    tile_quarter<NS, M, 0>(w, tab, ss, xv, acc);
#pragma unroll
    for (int m = 0; m < M; ++m) xv[m] = ldg_x4(xcol + m * cols + 8);
    tile_quarter<NS, M, 1>(w, tab, ss, xv, acc);
#pragma unroll
    for (int m = 0; m < M; ++m) xv[m] = ldg_x4(xcol + m * cols + 16);
    tile_quarter<NS, M, 2>(w, tab, ss, xv, acc);
#pragma unroll
    for (int m = 0; m < M; ++m) xv[m] = ldg_x4(xcol + m * cols + 24);
    tile_quarter<NS, M, 3>(w, tab, ss, xv, acc);
}

__device__ __forceinline__ void store_out(const GemvJob& J, int m, int row, float v) {
    if (J.bias) v += bf16_to_f32(J.bias[row]);
    if (J.out_f32) {
        reinterpret_cast<float*>(J.y)[(int64_t)m * J.rows + row] = v;
    } else {
        reinterpret_cast<uint16_t*>(J.y)[(int64_t)m * J.rows + row] =
            __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
}

template <int NS, int M, int MAXJ>
__global__ void __launch_bounds__(kThreads, 2)
gemv_kernel(const __grid_constant__ GemvBatch<MAXJ> batch) {
    using T = PackTraits<NS>;
    extern __shared__ __align__(16) uint32_t smem[];
    uint32_t* sig2 = smem + T::kPairs * 32;

    // Lane-private pair table and the (sigma, sigma) table of every fp8 code.
    for (int i = threadIdx.x; i < T::kPairs * 32; i += blockDim.x) {
        int p = i >> 5;
        uint32_t lo, hi;
        if constexpr (NS == 26) {
            lo = c_lat26[p / 27];
            hi = c_lat26[p % 27];
        } else {
            lo = c_lat16[p & 15];
            hi = c_lat16[p >> 4];
        }
        smem[i] = lo | (hi << 16);
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        uint32_t s = fp8_to_bf16((uint8_t)i);
        sig2[i] = s | (s << 16);
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const uint32_t* tab = smem + lane;
    const int64_t warp0 = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int64_t nwarps = (int64_t)gridDim.x * kWarps;

    for (int64_t item = warp0; item < batch.total_items; item += nwarps) {
        int j = 0;
        if constexpr (MAXJ > 1) {
            int lo = 0, hi = batch.n - 1;
            while (lo < hi) {  // last job with item_begin <= item
                int mid = (lo + hi + 1) >> 1;
                if (batch.jobs[mid].item_begin <= item) lo = mid; else hi = mid - 1;
            }
            j = lo;
        }
        const GemvJob& J = batch.jobs[j];
        const int64_t local = item - J.item_begin;
        const int rb = (int)(local / J.kg), g = (int)(local % J.kg);
        const int row = rb * 32 + lane;
        const int c0 = g * kGroupTiles;
        const int c1 = min(c0 + kGroupTiles, J.kt);

        float acc[M][2];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m][0] = acc[m][1] = 0.f;

        const uint32_t* cbase = J.codes + ((int64_t)rb * J.kt) * (T::kWords * 32);
        const uint32_t* sbase = reinterpret_cast<const uint32_t*>(J.scales) + (int64_t)rb * J.kt4 * 32;

        for (int c = c0; c < c1; c += 4) {
            const uint32_t sw = ldg_nc(sbase + (c >> 2) * 32 + lane);
            uint32_t w[4][5];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if (c + t < c1) {
                    const uint32_t* cw = cbase + (int64_t)(c + t) * (T::kWords * 32);
                    uint4 v = ldg_nc4(reinterpret_cast<const uint4*>(cw) + lane);
                    w[t][0] = v.x;
                    w[t][1] = v.y;
                    w[t][2] = v.z;
                    w[t][3] = v.w;
                    w[t][4] = (T::kWords == 5) ? ldg_nc(cw + 128 + lane) : 0u;
                }
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if (c + t < c1) {
                    const uint32_t ss = sig2[(sw >> (8 * t)) & 0xFFu];
                    tile_dot<NS, M>(w[t], tab, ss, J.x + (int64_t)(c + t) * 32, J.cols, acc);
                }
            }
        }

        // residuals of this lane's row within the group
        const int64_t bidx = ((int64_t)rb * J.kg + g) * 32 + lane;
        const uint32_t e0 = J.res_ptr[bidx], e1 = J.res_ptr[bidx + 1];
        for (uint32_t e = e0; e < e1; ++e) {
            const uint32_t ent = J.res_ent[e];
            const float v = bf16_to_f32((uint16_t)(ent & 0xFFFFu));
            const int col = (int)(ent >> 16);
            if (col >= J.cols) continue;  // only a corrupted pack has one
#pragma unroll
            for (int m = 0; m < M; ++m)
                acc[m][0] = fmaf(v, bf16_to_f32(J.x[(int64_t)m * J.cols + col]), acc[m][0]);
        }

        if (J.kg == 1) {
            if (row < J.rows) {
#pragma unroll
                for (int m = 0; m < M; ++m) store_out(J, m, row, acc[m][0] + acc[m][1]);
            }
        } else {
            const int64_t rpad = (int64_t)J.rb * 32;
            // partial sums of this group: slot [m][g][row]
#pragma unroll
            for (int m = 0; m < M; ++m)
                J.partial[((int64_t)m * J.kg + g) * rpad + row] = acc[m][0] + acc[m][1];
            __threadfence();
            __syncwarp();
            uint32_t last = 0;
            if (lane == 0) last = (atomicAdd(&J.counters[rb], 1u) == (uint32_t)(J.kg - 1));
            last = __shfl_sync(0xFFFFFFFFu, last, 0);
            if (last) {
                __threadfence();
                if (row < J.rows) {
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        float s = 0.f;
                        for (int gg = 0; gg < J.kg; ++gg)
                            s += __ldcg(&J.partial[((int64_t)m * J.kg + gg) * rpad + row]);
                        store_out(J, m, row, s);
                    }
                }
                __syncwarp();
                if (lane == 0) atomicExch(&J.counters[rb], 0u);
            }
        }
    }
}

template <int NS, int M, int MAXJ>
cudaError_t launch_one(const GemvBatch<MAXJ>& b, cudaStream_t stream, int num_sms) {
    using T = PackTraits<NS>;
    const size_t smem = (size_t)T::kPairs * 32 * 4 + 256 * 4;
    auto kern = gemv_kernel<NS, M, MAXJ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int per_sm = NS == 26 ? 2 : 3;
    int64_t want = (b.total_items + kWarps - 1) / kWarps;
    int grid = (int)std::min<int64_t>(want, (int64_t)num_sms * per_sm);
    if (grid < 1) grid = 1;
    kern<<<grid, kThreads, smem, stream>>>(b);
    return cudaGetLastError();
}

template <int MAXJ>
cudaError_t dispatch(const GemvBatch<MAXJ>& b, int ns, int m, cudaStream_t s, int sms) {
#define CDQ_M_CASE(MM)                                                  \
    case MM:                                                            \
        return ns == 26 ? launch_one<26, MM, MAXJ>(b, s, sms) : launch_one<16, MM, MAXJ>(b, s, sms);
    switch (m) {
        CDQ_M_CASE(1)
        CDQ_M_CASE(2)
        CDQ_M_CASE(3)
        CDQ_M_CASE(4)
        CDQ_M_CASE(5)
        CDQ_M_CASE(6)
        CDQ_M_CASE(7)
        CDQ_M_CASE(8)
        default:
            return cudaErrorInvalidValue;
    }
#undef CDQ_M_CASE
}

}  // namespace

cudaError_t upload_lattices() {
    uint16_t l27[27];
    for (int i = 0; i < 26; ++i) l27[i] = kLattice26[i];
    l27[26] = 0;  // residual slot contributes zero
    cudaError_t e = cudaMemcpyToSymbol(c_lat26, l27, sizeof l27);
    if (e != cudaSuccess) return e;
    return cudaMemcpyToSymbol(c_lat16, kLattice16, sizeof kLattice16);
}

cudaError_t gemv_launch_single(const GemvBatch<1>& b, int ns, int m, cudaStream_t s, int sms) {
    return dispatch<1>(b, ns, m, s, sms);
}
cudaError_t gemv_launch_grouped(const GemvBatch<kMaxJobs>& b, int ns, int m, cudaStream_t s,
                                int sms) {
    return dispatch<kMaxJobs>(b, ns, m, s, sms);
}

}  // namespace cdq

// ---------------------------------------------------------------------------
// cdq_linear_noalloc: the fused linear for callers that cannot allocate device
// memory. Its split-K scratch (per-group partial sums and per-row-block arrival
// counters, the same layout as cdq_linear's workspace) lives in the file-scope
// array below, which every GPU that loads this library holds until the process
// exits. Host code never touches the array by name: the array's host-side
// symbol is only a stand-in, so set-up asks the runtime for its device address
// once per device (with that device current) and passes that address on.
// ---------------------------------------------------------------------------
#include <mutex>

#define CDQ_NOALLOC_SCRATCH_BYTES ((size_t)4 << 20)  // 4 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[CDQ_NOALLOC_SCRATCH_BYTES];

namespace cdq {
namespace {

constexpr size_t kNoAllocScratchBytes = CDQ_NOALLOC_SCRATCH_BYTES;

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[128] = {};
int g_noalloc_sms[128] = {};

// Once per device: lattice tables, SM count and the scratch's device address.
cdq_status noalloc_setup(void** scratch, int* sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return CDQ_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        if (upload_lattices() != cudaSuccess) return CDQ_ERR_CUDA;
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return CDQ_ERR_CUDA;
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
            return CDQ_ERR_CUDA;
        g_noalloc_sms[dev] = n;
        g_noalloc_ptr[dev] = p;
    }
    *scratch = g_noalloc_ptr[dev];
    *sms = g_noalloc_sms[dev];
    return CDQ_OK;
}

inline int64_t al256(int64_t b) { return (b + 255) / 256 * 256; }

}  // namespace
}  // namespace cdq

extern "C" cdq_status cdq_linear_noalloc(const cdq_packed* w, const uint16_t* x, int64_t m,
                                         uint16_t* y, const uint16_t* bias, void* stream) {
    using namespace cdq;
    if (!w) return CDQ_ERR_ARG;
    if (w->n_states != 26 && w->n_states != 16) return CDQ_ERR_STATES;
    if (w->rows <= 0 || w->cols <= 0 || w->cols % 32 || w->cols > CDQ_MAX_COLS) return CDQ_ERR_SHAPE;
    if (!w->codes || !w->scales || !w->res_ptr || (w->n_res > 0 && !w->res_ent)) return CDQ_ERR_ARG;
    if (m < 1 || m > CDQ_MAX_BATCH || !x || !y) return CDQ_ERR_ARG;
    if ((uintptr_t)w->codes % 16 || (uintptr_t)w->scales % 4 || (uintptr_t)w->res_ptr % 4 ||
        (uintptr_t)x % 16 || (uintptr_t)y % 2 || (bias && (uintptr_t)bias % 2))
        return CDQ_ERR_ARG;
    const Geometry g = geometry(w->rows, w->cols, w->n_states);
    const int64_t slots = al256(m * g.kg * g.rb * 32 * 4);
    const int64_t need = slots + al256(g.rb * 4);
    if (g.kg > 1 && need > (int64_t)kNoAllocScratchBytes) return CDQ_ERR_WORKSPACE;

    void* scratch = nullptr;
    int sms = 0;
    cdq_status st = noalloc_setup(&scratch, &sms);
    if (st) return st;

    GemvBatch<1> b;
    b.n = 1;
    b.pad_ = 0;
    GemvJob& J = b.jobs[0];
    J.codes = w->codes;
    J.scales = w->scales;
    J.res_ptr = w->res_ptr;
    J.res_ent = w->res_ent;
    J.x = x;
    J.y = y;
    J.bias = bias;
    J.rows = w->rows;
    J.cols = w->cols;
    J.rb = (int32_t)g.rb;
    J.kt = (int32_t)g.kt;
    J.kt4 = (int32_t)g.kt4;
    J.kg = (int32_t)g.kg;
    J.out_f32 = 0;
    J.pad_ = 0;
    J.item_begin = 0;
    J.partial = nullptr;
    J.counters = nullptr;
    cudaStream_t s = (cudaStream_t)stream;
    if (g.kg > 1) {
        unsigned char* base = static_cast<unsigned char*>(scratch);
        J.partial = reinterpret_cast<float*>(base);
        J.counters = reinterpret_cast<uint32_t*>(base + slots);
        // the array keeps the previous call's contents: the arrival counters
        // must start at zero (the partial slots are written before they are read)
        if (cudaMemsetAsync(J.counters, 0, (size_t)g.rb * 4, s) != cudaSuccess) return CDQ_ERR_CUDA;
    }
    b.total_items = (int64_t)J.rb * J.kg;
    return gemv_launch_single(b, w->n_states, (int)m, s, sms) == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}
