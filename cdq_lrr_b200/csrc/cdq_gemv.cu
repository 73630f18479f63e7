// Fused dequant linear for the CDQ-LRR device pack: the shared decode pieces
// (bulk-copy ring, pair tables, unit decode into mma.sync), the wide streaming
// pass for batches 9 to 64 and its fix-up pass, and the launchers of every
// path (batches up to 8: cdq_stream.cuh; tcgen05 tile path: cdq_tile.cuh).
//
// y[m, row] = sum_col w_hat[row, col] * x[m, col] (+ bias[row]) where
// w_hat = bf16(LATTICE[q] * sigma) is rebuilt in registers from the packed
// tiles and never written to memory (the reference materialises w_hat and
// calls F.linear: code/cdq_lrr_qwen05.py:188-198, code/cdq_loader.py:53-58).
//
// Memory pipeline (both streaming kernels). Each warp streams its quads
// (2688 or 2176 contiguous bytes; the last quad of a row block may be
// shorter) into a private two-slot ring in shared memory with bulk copies
// (cp.async.bulk, completion counted on one mbarrier per slot), so two quads
// are in flight per warp while it decodes the previous one; lane 0 issues the
// copy of the warp's next quad as soon as a slot is consumed.
//
// Dequantisation. Lane l = 4g + c reads from the slot exactly the 16 pair
// codes of its m16n8k16 A fragments (rows g and g+8 of the block over 16
// contiguous columns of the unit). A shared-memory table maps a pair code to
// the bf16 pair (LATTICE[a], LATTICE[b]); every lane owns a private copy of
// the table in its own bank, so the 32 lookups of a warp never conflict.
// One bf16x2 multiply by (sigma, sigma) then yields the exact w_hat pair (a
// single rounding of the exact product, as torch's bf16 multiply), which is
// the A operand of a tensor-core mma (bf16 inputs, fp32 accumulators); the
// activations form the B operand (batch = the mma's N dimension). Residual
// positions carry the zero symbol; their bf16 values enter through the
// residual pre-pass (cdq_stream.cuh), whose per-group sums are added to the
// mma sums group by group.
//
// Arithmetic of one output (every streaming path, any batch, any grouping):
//     y = sum over the row's residual groups, in group order and starting
//         from zero, of (mma sum of the group + residual sum of the group),
//         + bias, rounded once.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "cdq.h"
#include "cdq_common.cuh"
#include "cdq_decode_math.cuh"
#include "cdq_internal.cuh"

namespace cdq {

__constant__ uint16_t c_lat26[27];
__constant__ uint16_t c_lat16[16];
__device__ int g_gemv_error;

namespace {

template <int NS>
struct PackTraits;
template <>
struct PackTraits<26> {
    static constexpr int kPairs = kPairs26;
    static constexpr int kUnit = 672;
    static constexpr int kSigOff = 640;  // code bytes per unit
};
template <>
struct PackTraits<16> {
    static constexpr int kPairs = kPairs16;
    static constexpr int kUnit = 544;
    static constexpr int kSigOff = 512;
};

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kSlots = 2;                 // quads in flight per warp
constexpr uint32_t kSmemBytes = 232448;   // 227 KB window
constexpr uint32_t kSpinLimit = 1u << 22; // mbarrier polls before a wait gives up

// Shared-memory map in absolute shared-window addresses (the dynamic window
// starts within the first 1 KB, which the system reserves):
//   [1K, 32K)           rings of warps 0 .. kLowWarps-1
//   [32K, 128K)         26-state pair table: code p at entry p ^ 0x300 (128 B
//                       entries, so the entry address is ((code << 7) & mask)
//                       ^ lane_base: one lop3); 16-state table in [64K, 128K)
//                       (256 B entries: the code byte is address byte 1)
//   [61K, 64K)          (unused by both tables) first work item of every job
//                       (binary-search keys), the scale table (fp8 code b ->
//                       (sigma, sigma) at 4b) and one mbarrier per (warp, slot)
//   [128K, ...)         rings of warps kLowWarps .. kWarps-1
// A ring is kSlots slots; a slot holds one quad (its units' bytes as stored).
constexpr uint32_t kLowStage = 1024;
constexpr int kLowWarps = 4;
constexpr uint32_t kLat26Xor = 0x300u << 7;
constexpr uint32_t kLat16Base = 64u << 10;
constexpr uint32_t kBeginAddr = 61u << 10;
constexpr uint32_t kSigAddr = 62u << 10;
constexpr uint32_t kBarAddr = 63u << 10;
constexpr uint32_t kHighStage = 128u << 10;

template <int NS>
struct SlotTraits {
    static constexpr uint32_t kQuadBytes = 4 * PackTraits<NS>::kUnit;
    static constexpr uint32_t kRing = kSlots * kQuadBytes;
    static constexpr uint32_t kTop = kHighStage + (kWarps - kLowWarps) * kRing;
};
static_assert(kLowStage + kLowWarps * SlotTraits<26>::kRing <= (32u << 10), "low rings overlap the table");
static_assert(SlotTraits<26>::kTop <= 232448, "rings exceed the window");
static_assert(kBeginAddr >= (473u << 7) && kBeginAddr + 4 * kMaxJobs <= kSigAddr &&
                  kSigAddr + 1024 <= kBarAddr && kBarAddr + kWarps * kSlots * 8 <= (512u << 7),
              "keys, scale table and barriers must sit in the 26-state table's unused entries 473..511");

template <int NS>
__device__ __forceinline__ uint32_t slot_base(int warp) {
    constexpr uint32_t kRing = SlotTraits<NS>::kRing;
    return warp < kLowWarps ? kLowStage + warp * kRing : kHighStage + (warp - kLowWarps) * kRing;
}

// activations: reused by every row block of the job, so cached in L1
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

// Table lookups: the tables are written before the block barrier and only
// read afterwards, so these loads carry no ordering constraints.
__device__ __forceinline__ uint32_t lds(uint32_t addr) {
    uint32_t v;
    asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
// Slot reads: ordered after the mbarrier wait that published the data.
__device__ __forceinline__ uint4 lds_slot4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint2 lds_slot2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t lds_slot(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t lds_slot_u16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// ---- bulk copies into a slot (one mbarrier per slot, arrival count 1) ----
__device__ __forceinline__ void mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
// Arms a slot's mbarrier for `bytes` of copies (the slot's previous contents
// were read through the generic proxy, hence the proxy fence).
__device__ __forceinline__ void slot_arm(uint32_t bar, uint32_t bytes) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// Waits for the phase of the given parity; false after kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t spin = 0; spin < kSpinLimit; ++spin) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// D (16 x 8, fp32) += A (16 x 16, bf16, row) * B (16 x 8, bf16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory address of slot Q's table entry for this lane.
//   26 states: ((code << 7) & mask) ^ lane_base, the code cut from the 160-bit stream
//   16 states: address byte 1 = the code byte, bytes 0 and 2 from lane_base
template <int NS, int Q>
__device__ __forceinline__ uint32_t slot_addr(const uint32_t (&w)[5], uint32_t lane_base) {
    if constexpr (NS == 26) {
        constexpr int bit = 10 * Q;
        constexpr uint32_t mask = 0x3FFu << 7;
        if constexpr (bit < 7) {
            return ((w[0] << (7 - bit)) & mask) ^ lane_base;
        } else {
            constexpr int b7 = bit - 7, wd = b7 / 32, s = b7 % 32;
            if constexpr (s + 17 <= 32 || wd + 1 >= 5) {
                return ((w[wd] >> s) & mask) ^ lane_base;
            } else {
                return (__funnelshift_r(w[wd], w[wd + 1], s) & mask) ^ lane_base;
            }
        }
    } else {
        return prmt(w[Q >> 2], lane_base, 0x7604u | ((Q & 3) << 4));
    }
}

template <int NS, int Q>
__device__ __forceinline__ uint32_t what_pair(const uint32_t (&w)[5], uint32_t lane_base, uint32_t ss) {
    return bmul2(lds(slot_addr<NS, Q>(w, lane_base)), ss);
}

// One unit: 16 rows x 64 columns, four m16n8k16 mmas over the k16 slices.
// w4 = fifth code word (26 states); sw = scale half-word at bits SH.. of sw
// (fp8 code of row g, then row g + 8).
template <int NS, int SH>
__device__ __forceinline__ void unit_mma(const uint4& a, uint32_t w4, uint32_t sw, const uint4& xa,
                                         const uint4& xb, uint32_t lane_base, uint32_t sig_base,
                                         float (&d)[4]) {
    const uint32_t w[5] = {a.x, a.y, a.z, a.w, w4};
    const uint32_t lo = SH <= 2 ? (sw << (2 - SH)) : (sw >> (SH - 2));
    const uint32_t hi = sw >> (SH + 6);
    const uint32_t ss0 = lds((lo & 0x3FCu) | sig_base);  // (sigma, sigma) of row g
    const uint32_t ss1 = lds((hi & 0x3FCu) | sig_base);  // row g + 8
    mma16816(d, what_pair<NS, 0>(w, lane_base, ss0), what_pair<NS, 1>(w, lane_base, ss1),
             what_pair<NS, 2>(w, lane_base, ss0), what_pair<NS, 3>(w, lane_base, ss1), xa.x, xa.y);
    mma16816(d, what_pair<NS, 4>(w, lane_base, ss0), what_pair<NS, 5>(w, lane_base, ss1),
             what_pair<NS, 6>(w, lane_base, ss0), what_pair<NS, 7>(w, lane_base, ss1), xa.z, xa.w);
    mma16816(d, what_pair<NS, 8>(w, lane_base, ss0), what_pair<NS, 9>(w, lane_base, ss1),
             what_pair<NS, 10>(w, lane_base, ss0), what_pair<NS, 11>(w, lane_base, ss1), xb.x, xb.y);
    mma16816(d, what_pair<NS, 12>(w, lane_base, ss0), what_pair<NS, 13>(w, lane_base, ss1),
             what_pair<NS, 14>(w, lane_base, ss0), what_pair<NS, 15>(w, lane_base, ss1), xb.z, xb.w);
}

// One unit for batches above 8: the unit's 16 w_hat pair registers are built
// once and multiply NT n-tiles of 8 batch rows each (activations from global
// memory: row 8t + g of n-tile t, clamped to the last batch row; rows past it
// only feed output columns that are never stored). zero_x: the phantom tile's
// lanes take zero activations.
template <int NS, int SH, int NT>
__device__ __forceinline__ void unit_mma_wide(const uint4& a, uint32_t w4, uint32_t sw, const uint16_t* xu,
                                              int64_t cols, int g, int m, bool zero_x, uint32_t lane_base,
                                              uint32_t sig_base, float (&d)[NT][4]) {
    const uint32_t w[5] = {a.x, a.y, a.z, a.w, w4};
    const uint32_t lo = SH <= 2 ? (sw << (2 - SH)) : (sw >> (SH - 2));
    const uint32_t hi = sw >> (SH + 6);
    const uint32_t ss0 = lds((lo & 0x3FCu) | sig_base);
    const uint32_t ss1 = lds((hi & 0x3FCu) | sig_base);
    const uint32_t A[16] = {
        what_pair<NS, 0>(w, lane_base, ss0),  what_pair<NS, 1>(w, lane_base, ss1),
        what_pair<NS, 2>(w, lane_base, ss0),  what_pair<NS, 3>(w, lane_base, ss1),
        what_pair<NS, 4>(w, lane_base, ss0),  what_pair<NS, 5>(w, lane_base, ss1),
        what_pair<NS, 6>(w, lane_base, ss0),  what_pair<NS, 7>(w, lane_base, ss1),
        what_pair<NS, 8>(w, lane_base, ss0),  what_pair<NS, 9>(w, lane_base, ss1),
        what_pair<NS, 10>(w, lane_base, ss0), what_pair<NS, 11>(w, lane_base, ss1),
        what_pair<NS, 12>(w, lane_base, ss0), what_pair<NS, 13>(w, lane_base, ss1),
        what_pair<NS, 14>(w, lane_base, ss0), what_pair<NS, 15>(w, lane_base, ss1)};
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (8 * t < m) {
            uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
            if (!zero_x) {
                const uint16_t* xr = xu + (int64_t)min(8 * t + g, m - 1) * cols;
                xa = ldg_x4(xr);
                xb = ldg_x4(xr + 8);
            }
            mma16816(d[t], A[0], A[1], A[2], A[3], xa.x, xa.y);
            mma16816(d[t], A[4], A[5], A[6], A[7], xa.z, xa.w);
            mma16816(d[t], A[8], A[9], A[10], A[11], xb.x, xb.y);
            mma16816(d[t], A[12], A[13], A[14], A[15], xb.z, xb.w);
        }
    }
}

__device__ __forceinline__ void store_out(const GemvJob& J, int n, int row, float v) {
    if (J.bias) v += bf16_to_f32(J.bias[row]);
    if (J.out_f32) {
        reinterpret_cast<float*>(J.y)[(int64_t)n * J.rows + row] = v;
    } else {
        reinterpret_cast<uint16_t*>(J.y)[(int64_t)n * J.rows + row] =
            __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
}

// Where a work item lives: its job, row block, residual group and units.
struct ItemInfo {
    int job, b16, grp, cp0, n_units;
};

template <int MAXJ>
__device__ __forceinline__ ItemInfo item_info(const GemvBatch<MAXJ>& batch, int64_t item) {
    ItemInfo I;
    int j = 0;
    if constexpr (MAXJ > 1) {
        int lo = 0, hi = batch.n - 1;
        while (lo < hi) {  // last job with item_begin <= item (keys in shared memory)
            const int mid = (lo + hi + 1) >> 1;
            if ((int64_t)(int32_t)lds(kBeginAddr + 4 * mid) <= item) lo = mid; else hi = mid - 1;
        }
        j = lo;
    }
    const GemvJob& J = batch.jobs[j];
    const int local = (int)(item - J.item_begin);
    I.job = j;
    I.b16 = local / J.kg;
    I.grp = local - I.b16 * J.kg;
    I.cp0 = I.grp * kGroupPairs;
    I.n_units = min(I.cp0 + kGroupPairs, J.kp) - I.cp0;
    return I;
}

// The wide streaming pass (batches 9 to 64): each unit is decoded once into
// w_hat pair registers that multiply NT n-tiles of 8 batch rows (activations
// from the L1 cache). Items are (job, 16-row block, residual group), dealt
// round-robin to the warps of the grid; each item's sums, added over the
// group's residual sums from the pre-pass, are written to the workspace and
// the fix-up pass adds the groups.
template <int NS, int M, int MAXJ>
__global__ void __launch_bounds__(kThreads, 1)
wide_kernel(const __grid_constant__ GemvBatch<MAXJ> batch) {
    static_assert(M > 8, "batches up to 8 take the stream kernel");
    using Tr = PackTraits<NS>;
    using Sl = SlotTraits<NS>;
    constexpr uint32_t kU = Tr::kUnit;
    constexpr uint32_t kQuad = Sl::kQuadBytes;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
    if (s0 > kLowStage || s0 + kSmemBytes < Sl::kTop) {
        if (threadIdx.x == 0) atomicExch(&g_gemv_error, 1);
        return;
    }
    uint8_t* const base = smem - s0;  // generic pointer of shared address 0
    for (int i = threadIdx.x; i < Tr::kPairs * 32; i += blockDim.x) {
        const uint32_t p = (uint32_t)i >> 5, l = (uint32_t)i & 31;
        uint32_t lo, hi, addr;
        if constexpr (NS == 26) {
            lo = c_lat26[p / 27];
            hi = c_lat26[p % 27];
            addr = ((p << 7) ^ kLat26Xor) + 4 * l;
        } else {
            lo = c_lat16[p & 15];
            hi = c_lat16[p >> 4];
            addr = kLat16Base + (p << 8) + 4 * l;
        }
        *reinterpret_cast<uint32_t*>(base + addr) = lo | (hi << 16);
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        const uint32_t s = fp8_to_bf16((uint8_t)i);
        *reinterpret_cast<uint32_t*>(base + kSigAddr + 4 * i) = s | (s << 16);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    if constexpr (MAXJ > 1) {  // warp-uniform reads of the launch record
        for (int i = warp; i < batch.n; i += kWarps) {
            const int32_t v = (int32_t)batch.jobs[i].item_begin;
            if (lane == 0) *reinterpret_cast<int32_t*>(base + kBeginAddr + 4 * i) = v;
        }
    }
    const uint32_t ring = slot_base<NS>(warp);
    const uint32_t bars = kBarAddr + warp * kSlots * 8;
    if (lane == 0) {
        for (int k = 0; k < kSlots; ++k) mbar_init(bars + 8 * k);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const uint32_t lane_base = NS == 26 ? (kLat26Xor | (4u * lane)) : (kLat16Base + 4u * lane);
    const uint32_t sig_base = kSigAddr;
    const int64_t total = batch.total_items;
    const int64_t stride = (int64_t)gridDim.x * kWarps;
    const int64_t first = (int64_t)blockIdx.x * kWarps + warp;
    constexpr int NT = (M + 7) / 8;  // n-tiles of 8 batch rows
    const int m_rt = batch.m;        // batch rows of this launch

    // Producer cursor (lane 0 issues; every lane keeps the same values): the
    // next quad of this warp's stream of items.
    int64_t p_item = first;
    int p_q = 0, p_nq = 0, p_units = 0;
    const uint8_t* p_base = nullptr;
    uint32_t p_slot = 0;
    auto p_load = [&]() {
        if (p_item < total) {
            const ItemInfo I = item_info(batch, p_item);
            const GemvJob& J = batch.jobs[I.job];
            p_base = J.units + ((int64_t)I.b16 * J.kp + I.cp0) * kU;
            p_units = I.n_units;
            p_nq = (I.n_units + 3) >> 2;
            p_q = 0;
        }
    };
    auto produce = [&]() {
        if (p_item >= total) return;
        const int left = p_units - 4 * p_q;
        const int u = left < 4 ? left : 4;
        const uint32_t bytes = (uint32_t)u * kU;
        if (lane == 0) {
            const uint32_t bar = bars + 8 * p_slot;
            slot_arm(bar, bytes);
            bulk_copy(ring + p_slot * kQuad, p_base + (int64_t)p_q * kQuad, bytes, bar);
        }
        p_slot ^= 1u;
        if (++p_q == p_nq) {
            p_item += stride;
            p_load();
        }
    };
    p_load();
    produce();
    produce();

    uint32_t c_slot = 0, c_phase = 0;
    bool failed = false;
    for (int64_t item = first; item < total && !failed; item += stride) {
        const ItemInfo I = item_info(batch, item);
        const GemvJob& J = batch.jobs[I.job];
        const int n_units = I.n_units, nq = (n_units + 3) >> 2;
        // a phantom second tile (odd tile count) sits in the row's last unit
        const int phantom_u = (J.kt & 1) && I.cp0 + n_units == J.kp ? n_units - 1 : -1;
        const uint16_t* xw = J.x + 64 * I.cp0 + 16 * c;  // batch row 0
        float d[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t) d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0.f;
        // unit i of quad q (the phantom tile's lanes take zero activations)
        auto run_unit = [&](const uint4& A, uint32_t w4, uint32_t sw, bool hi_half, int unit) {
            const bool zx = unit == phantom_u && c >= 2;
            if (hi_half) unit_mma_wide<NS, 16, NT>(A, w4, sw, xw + 64 * unit, J.cols, g, m_rt, zx, lane_base, sig_base, d);
            else unit_mma_wide<NS, 0, NT>(A, w4, sw, xw + 64 * unit, J.cols, g, m_rt, zx, lane_base, sig_base, d);
        };
        for (int q = 0; q < nq; ++q) {
            if (!mbar_wait(bars + 8 * c_slot, c_phase)) {
                failed = true;
                break;
            }
            const uint32_t slot = ring + c_slot * kQuad;
            const int uq = min(4, n_units - 4 * q);
            uint4 A[4];
            uint4 W;
            uint2 S;
            if (uq == 4) {
#pragma unroll
                for (int i = 0; i < 4; ++i) A[i] = lds_slot4(slot + 512 * i + 16 * lane);
                W = NS == 26 ? lds_slot4(slot + 2048 + 16 * lane) : make_uint4(0u, 0u, 0u, 0u);
                S = lds_slot2(slot + 4 * Tr::kSigOff + 8 * (lane >> 1));
            } else {
                // a short last quad (1..3 units, compact)
                uint32_t w4[3] = {0u, 0u, 0u}, h[3] = {0u, 0u, 0u};
#pragma unroll
                for (int i = 0; i < 3; ++i) {
                    A[i] = make_uint4(0u, 0u, 0u, 0u);
                    if (i < uq) {
                        A[i] = lds_slot4(slot + 512 * i + 16 * lane);
                        if constexpr (NS == 26) w4[i] = lds_slot(slot + 512 * uq + 4 * (uq * lane + i));
                        h[i] = lds_slot_u16(slot + Tr::kSigOff * uq + 2 * (uq * (lane >> 1) + i));
                    }
                }
                A[3] = make_uint4(0u, 0u, 0u, 0u);
                W = make_uint4(w4[0], w4[1], w4[2], 0u);
                S = make_uint2(h[0] | (h[1] << 16), h[2]);
            }
            // one register of every slot read: each read has landed before the slot is reused
            uint32_t dep = W.x ^ W.y ^ W.z ^ S.x ^ S.y ^ A[0].x ^ A[1].x ^ A[2].x ^ A[3].x;
            asm volatile("" ::"r"(dep));
            __syncwarp();
            produce();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (i < uq) {
                    const uint32_t w4 = i == 0 ? W.x : i == 1 ? W.y : i == 2 ? W.z : W.w;
                    run_unit(A[i], w4, i < 2 ? S.x : S.y, (i & 1) != 0, 4 * q + i);
                }
            }
            c_slot ^= 1u;
            c_phase ^= c_slot == 0 ? 1u : 0u;
        }
        if (failed) break;
        // this group's sums of rows g and g + 8 (batch columns 8t + 2c, 8t + 2c + 1),
        // added over the group's residual sums from the pre-pass: the group's value
        const int64_t rpad = (int64_t)J.r16 * 16;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int n0 = 8 * t + 2 * c;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t row = I.b16 * 16 + g + 8 * h;
                if (n0 < m_rt) {
                    float* p = J.partial + ((int64_t)n0 * J.kg + I.grp) * rpad + row;
                    *p = d[t][2 * h] + __ldcg(p);
                }
                if (n0 + 1 < m_rt) {
                    float* p = J.partial + ((int64_t)(n0 + 1) * J.kg + I.grp) * rpad + row;
                    *p = d[t][2 * h + 1] + __ldcg(p);
                }
            }
        }
    }
    if (failed) {
        // a copy that never landed: record it, give the copies still in
        // flight a bounded chance to land, and leave
        if (lane == 0) atomicExch(&g_gemv_error, 2);
        for (int k = 0; k < kSlots; ++k) {
            (void)mbar_wait(bars + 8 * c_slot, c_phase);
            c_slot ^= 1u;
            c_phase ^= c_slot == 0 ? 1u : 0u;
        }
    }
}

// Fix-up pass of the wide (batch > 8) streaming kernel: y[m, row] = sum over
// the row's residual groups, in group order and starting from zero, of the
// group's value (its mma sum plus its residual sum from the pre-pass), + bias,
// rounded once to bf16 (or stored as float32): the arithmetic of the batch
// <= 8 kernel, so a row's result does not depend on the batch it is computed
// in. One thread per (job, padded row, batch row); grid row y is job y.
constexpr int kFixThreads = 256;

template <int MAXJ>
__global__ void __launch_bounds__(kFixThreads) fixup_kernel(const __grid_constant__ GemvBatch<MAXJ> batch) {
    // block -> job: rb_begin holds each job's first block (uniform search of the launch record)
    int j = 0;
    if constexpr (MAXJ > 1) {
        int lo = 0, hi = batch.n - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (batch.jobs[mid].rb_begin <= (int)blockIdx.x) lo = mid; else hi = mid - 1;
        }
        j = lo;
    }
    const GemvJob& J = batch.jobs[j];
    const int64_t rpad = (int64_t)J.r16 * 16;
    const int64_t i = ((int64_t)blockIdx.x - J.rb_begin) * kFixThreads + threadIdx.x;
    if (i >= rpad * batch.m) return;
    const int n = (int)(i / rpad), row = (int)(i - n * rpad);
    if (row >= J.rows) return;
    const int kg = J.kg;
    const float* p = J.partial + (int64_t)n * kg * rpad + row;
    float s = 0.f;
    for (int k = 0; k < kg; ++k) s += __ldcg(p + (int64_t)k * rpad);
    store_out(J, n, row, s);
}

#include "cdq_tile.cuh"
#include "cdq_stream.cuh"
#include "cdq_step.cuh"

// The fix-up pass over every job (one thread per padded row and batch row).
template <int MAXJ>
cudaError_t launch_fixup(const GemvBatch<MAXJ>& b, int m, cudaStream_t stream) {
    GemvBatch<MAXJ> fb = b;
    int64_t blocks = 0;
    for (int j = 0; j < b.n; ++j) {
        fb.jobs[j].rb_begin = (int32_t)blocks;
        blocks += ((int64_t)b.jobs[j].r16 * 16 * m + kFixThreads - 1) / kFixThreads;
    }
    if (blocks >= INT32_MAX) return cudaErrorInvalidValue;
    fb.m = m;
    fixup_kernel<MAXJ><<<(int)std::max<int64_t>(blocks, 1), kFixThreads, 0, stream>>>(fb);
    return cudaGetLastError();
}

template <int NS, int M, int MAXJ>
cudaError_t launch_one(const GemvBatch<MAXJ>& b, cudaStream_t stream, int num_sms) {
    auto kern = wide_kernel<NS, M, MAXJ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    const int64_t want = (b.total_items + kWarps - 1) / kWarps;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, num_sms));
    // at most one item per warp of the grid (the projections of a decode step):
    // finishing single-group rows in the streaming pass saves the fix-up
    // launch; larger launches keep the two passes (the rows' residual tail
    // would stall warps that have more items to stream)
    GemvBatch<MAXJ> sb = b;
    e = stream::launch_res(b, b.m, stream);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, kSmemBytes, stream>>>(sb);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_fixup(b, b.m, stream);
}

// The tile path: a launch that lays out the activations (once per distinct x
// of the call, in the workspace of the first job that reads it), then the
// tile kernel, one persistent CTA per SM, jobs dealt heaviest (most units per
// row) first.
template <int NS, int NB, int MAXJ>
cudaError_t launch_tile(const GemvBatch<MAXJ>& b, cudaStream_t stream, int num_sms) {
    GemvBatch<MAXJ> tb = b;
    int order[MAXJ];
    for (int j = 0; j < b.n; ++j) order[j] = j;
    std::stable_sort(order, order + b.n, [&](int a, int c) { return b.jobs[a].kp > b.jobs[c].kp; });
    for (int j = 0; j < b.n; ++j) tb.jobs[j] = b.jobs[order[j]];
    int64_t items = 0;
    int prep_blocks = 0;
    for (int j = 0; j < tb.n; ++j) {
        GemvJob& J = tb.jobs[j];
        J.item_begin = items;
        items += (J.r16 + 7) / 8;
        // the activations are prepared once per (x, cols): later jobs reuse them
        J.reserved0 = 1;
        J.reserved_ptr = J.partial;
        for (int i = 0; i < j; ++i) {
            if (tb.jobs[i].x == J.x && tb.jobs[i].cols == J.cols && tb.jobs[i].reserved0) {
                J.reserved0 = 0;
                J.reserved_ptr = tb.jobs[i].reserved_ptr;
                break;
            }
        }
        J.rb_begin = prep_blocks;
        if (J.reserved0) prep_blocks += (J.kp + 3) / 4;
    }
    if (items >= INT32_MAX) return cudaErrorInvalidValue;
    tb.total_items = items;
    tile::x_prep_kernel<NB, MAXJ><<<std::max(prep_blocks, 1), 256, 0, stream>>>(tb);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    auto kern = tile::tile_kernel<NS, NB, MAXJ>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, num_sms));
    kern<<<grid, tile::kThreads, kSmemBytes, stream>>>(tb);
    return cudaGetLastError();
}

int g_tile_min_batch = 16;  // batches from this size on take the tcgen05 tile path

// The tile path needs enough 128-row tiles to occupy most SMs.
template <int MAXJ>
bool tile_fits(const GemvBatch<MAXJ>& b, int sms) {
    int64_t tiles = 0;
    for (int j = 0; j < b.n; ++j) tiles += (b.jobs[j].r16 + 7) / 8;
    return 2 * tiles >= sms;
}

template <int MAXJ>
cudaError_t dispatch(const GemvBatch<MAXJ>& b, int ns, int m, cudaStream_t s, int sms, bool allow_tile) {
    if (allow_tile && m >= g_tile_min_batch && m <= 64 && tile_fits(b, sms)) {
        if (m <= 16) return ns == 26 ? launch_tile<26, 16, MAXJ>(b, s, sms) : launch_tile<16, 16, MAXJ>(b, s, sms);
        if (m <= 32) return ns == 26 ? launch_tile<26, 32, MAXJ>(b, s, sms) : launch_tile<16, 32, MAXJ>(b, s, sms);
        return ns == 26 ? launch_tile<26, 64, MAXJ>(b, s, sms) : launch_tile<16, 64, MAXJ>(b, s, sms);
    }
#define CDQ_M_CASE(MM)                                                                      \
    case MM:                                                                                \
        return ns == 26 ? stream::launch<26, MM, MAXJ>(b, s, sms) : stream::launch<16, MM, MAXJ>(b, s, sms);
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
            break;
    }
#undef CDQ_M_CASE
    // wider batches: n-tiles of 8 rows, the batch size itself read from the launch record
    if (m <= 16) return ns == 26 ? launch_one<26, 16, MAXJ>(b, s, sms) : launch_one<16, 16, MAXJ>(b, s, sms);
    if (m <= 32) return ns == 26 ? launch_one<26, 32, MAXJ>(b, s, sms) : launch_one<16, 32, MAXJ>(b, s, sms);
    if (m <= 64) return ns == 26 ? launch_one<26, 64, MAXJ>(b, s, sms) : launch_one<16, 64, MAXJ>(b, s, sms);
    return cudaErrorInvalidValue;
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

cudaError_t gemv_launch_single(const GemvBatch<1>& b, int ns, int m, cudaStream_t s, int sms,
                               bool allow_tile) {
    return dispatch<1>(b, ns, m, s, sms, allow_tile);
}
cudaError_t gemv_launch_grouped(const GemvBatch<kMaxJobs>& b, int ns, int m, cudaStream_t s,
                                int sms) {
    return dispatch<kMaxJobs>(b, ns, m, s, sms, true);
}

void gemv_set_tile_min_batch(int m) { g_tile_min_batch = m; }

bool step_smem_layout(StepParams& p) {
    constexpr uint32_t top = stream::Ring<26>::kTop > stream::Ring<16>::kTop ? stream::Ring<26>::kTop
                                                                              : stream::Ring<16>::kTop;
    auto up16 = [](uint64_t a) { return (a + 15) / 16 * 16; };
    const uint64_t xs = up16(top);
    const uint64_t xf = up16(xs + 2ull * (uint64_t)std::max(std::max(p.hidden, p.inter), p.heads * dm::kHd));
    const uint64_t scr = up16(xf + 4ull * (uint64_t)p.hidden);
    const uint64_t sc = up16(scr + step::kScrBytes);
    const uint64_t end = up16(sc + 4ull * (uint64_t)p.max_len);
    if (end > kSmemBytes) return false;
    p.xs_addr = (uint32_t)xs;
    p.xf_addr = (uint32_t)xf;
    p.scr_addr = (uint32_t)scr;
    p.sc_addr = (uint32_t)sc;
    // the rest of the window stages residual data: a quarter bounds, the rest entries
    const uint64_t words = (kSmemBytes - end) / 4;
    p.rst_addr = (uint32_t)end;
    p.rst_bnd_cap = (int32_t)(words / 4);
    p.rst_ent_cap = (int32_t)(words - words / 4);
    return true;
}

// One cooperative launch (every CTA resident, one per SM) of the persistent
// decode step.
cudaError_t step_launch(const StepParams* dev_params, int ns, int sms, cudaStream_t s) {
    auto kern = ns == 26 ? step::decode_step_kernel<26> : step::decode_step_kernel<16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, stream::kSThreads, kSmemBytes);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sms);
    cfg.blockDim = dim3(stream::kSThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, dev_params);
}

cudaError_t gemv_read_error(int* out) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof v);
    if (e != cudaSuccess) return e;
    *out = v;
    return cudaSuccess;
}

}  // namespace cdq

// ---------------------------------------------------------------------------
// cdq_linear_noalloc: the fused linear for callers that cannot allocate device
// memory. Its scratch (one arrival counter per row block, then the per-group
// sums, the same layout as cdq_linear's workspace) lives in the file-scope
// array below, which every GPU that loads this library holds until the process
// exits. The array starts zeroed and every completed call leaves its counters
// at zero again. Host code never touches the array by name: the array's
// host-side symbol is only a stand-in, so set-up asks the runtime for its
// device address once per device (with that device current) and passes that
// address on. The address is cached per device ordinal, so it does not survive
// a cudaDeviceReset of that device.
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

}  // namespace
}  // namespace cdq

extern "C" cdq_status cdq_linear_noalloc(const cdq_packed* w, const uint16_t* x, int64_t m,
                                         uint16_t* y, const uint16_t* bias, void* stream) {
    using namespace cdq;
    if (!w) return CDQ_ERR_ARG;
    if (w->n_states != 26 && w->n_states != 16) return CDQ_ERR_STATES;
    if (w->rows <= 0 || w->cols <= 0 || w->cols % 32 || w->cols > CDQ_MAX_COLS) return CDQ_ERR_SHAPE;
    if (!w->units || !w->res_ptr || (w->n_res > 0 && !w->res_ent)) return CDQ_ERR_ARG;
    if (m < 1 || m > CDQ_MAX_BATCH || !x || !y) return CDQ_ERR_ARG;
    if ((uintptr_t)w->units % 16 || (uintptr_t)w->res_ptr % 4 || (uintptr_t)x % 16 ||
        (uintptr_t)y % 2 || (bias && (uintptr_t)bias % 2))
        return CDQ_ERR_ARG;
    const Geometry g = geometry(w->rows, w->cols, w->n_states);
    if (gemv_partial_bytes(g, m) > (int64_t)kNoAllocScratchBytes) return CDQ_ERR_WORKSPACE;

    void* scratch = nullptr;
    int sms = 0;
    cdq_status st = noalloc_setup(&scratch, &sms);
    if (st) return st;

    GemvBatch<1> b;
    b.n = 1;
    GemvJob& J = b.jobs[0];
    J.units = w->units;
    J.res_ptr = w->res_ptr;
    J.res_ent = w->res_ent;
    J.x = x;
    J.y = y;
    J.bias = bias;
    J.rows = w->rows;
    J.cols = w->cols;
    J.r16 = (int32_t)g.r16;
    J.kt = (int32_t)g.kt;
    J.kp = (int32_t)g.kp;
    J.kg = (int32_t)g.kg;
    J.out_f32 = 0;
    J.n_res = (uint32_t)w->n_res;
    J.item_begin = 0;
    J.unit_begin = 0;
    J.rb_begin = 0;
    J.reserved0 = 0;
    J.reserved_ptr = nullptr;
    // counters first (zero), then the sums: each sum is written before it is read
    J.counters = static_cast<uint32_t*>(scratch);
    J.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + gemv_counter_bytes(g));
    b.total_items = (int64_t)J.r16 * J.kg;
    b.m = (int32_t)m;
    // the streaming paths only: the scratch holds counters and group sums, no prepared activations
    return gemv_launch_single(b, w->n_states, (int)m, (cudaStream_t)stream, sms, false) == cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}
