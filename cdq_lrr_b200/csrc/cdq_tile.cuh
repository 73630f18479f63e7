// tcgen05 tile path of the fused dequant linear (included by cdq_gemv.cu inside
// its anonymous namespace; it shares the pack traits, the shared-memory
// tables, the bulk-copy helpers and the decode helpers of the streaming pass).
//
// y[m, row] = sum_col w_hat[row, col] * x[m, col]: the weight rows are the
// M = 128 side of a tcgen05.mma (kind::f16, bf16 inputs, fp32 accumulators in
// tensor memory), the batch is its N side (16, 32 or 64), K runs along the
// packed columns.
//
// Work item: a 128-row tile (8 row blocks of 16) of one job over all of K.
// Items are dealt round-robin to the CTAs of a persistent grid (one CTA per
// SM), heaviest jobs first. A small launch before the tile kernel lays out
// each distinct activation matrix of the call once in the workspace: the
// B-operand stage of every quad (K-major, no swizzle, 8 x 16-byte core
// matrices, columns permuted within every 64-column unit to the A operand's
// column order) and x^T (the batch of one column contiguous). Per CTA:
//   warps 0..7   decode: warp w streams the quads of row block 2(w%4) + w/4 of
//                the tile through its private bulk-copy ring and rebuilds
//                w_hat exactly (pair table lookup, one bf16x2 multiply by
//                (sigma, sigma)); the 16 pair registers of a unit go to tensor
//                memory with one tcgen05.st.16x256b.x4, which puts lane
//                l = 4g + c's pairs at rows g and g + 8 of the A operand,
//                columns 8r + 2c + j for pair (r, j) of the lane's 16
//                contiguous columns 16c + 4r + 2j.
//   warp 8       lane 0 issues the mmas (A from tensor memory, B from shared
//                memory) and commits their completion to mbarriers.
//   warp 9       lane 0 bulk-copies each quad's prepared B-operand stage.
//   warps 10..13 epilogue, one per tensor-memory lane quarter (one thread per
//                row): sum the row's residual entries (bf16 value x x^T
//                column, fp32, entry order) while the mmas of the item run,
//                then read the item's sums (tcgen05.ld), add the residual sum
//                and the bias, round once and store y.
// A and B share a ring of stages (one quad = 256 columns of K); the
// accumulator is double-buffered so the epilogue of item i overlaps the mmas
// of item i + 1.
//
// Every wait is bounded (kSpinLimit polls); a wait that gives up raises a
// shared abort flag and the kernel error code 3, every warp then drains what
// it has in flight and leaves, and tensor memory is always released.

namespace tile {

constexpr int kDecodeWarps = 8;
constexpr int kMmaWarp = 8;
constexpr int kXWarp = 9;
constexpr int kEpiWarp0 = 10;  // warps 10..13: lane quarters 2, 3, 0, 1
constexpr int kEpiWarps = 4;
constexpr int kThreads = 32 * (kDecodeWarps + 2 + kEpiWarps);
constexpr uint32_t kStageCols = 128;  // tensor-memory columns of one A stage (4 units x 32)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kXRowBytes = 512;    // one batch row of one stage (256 bf16)
constexpr uint32_t kXGroupBytes = 4096; // 8 batch rows: the stride between core-matrix groups
// shared-memory map (absolute shared-window addresses): activation stages from
// 128K, then as many rings as fit below the window's end; the other rings
// from 1K (below the pair table)
constexpr uint32_t kXBase = 128u << 10;
constexpr uint32_t kRingLow = 1024;
constexpr uint32_t kWindowEnd = 232448;
constexpr uint32_t kSlotBars = kBarAddr;  // one per ring slot: 8 warps x up to 3 slots
constexpr uint32_t kPipeBars = kBarAddr + kDecodeWarps * 3 * 8;
constexpr uint32_t kTmemHolder = kBarAddr + 320;
constexpr uint32_t kAbortFlag = kBarAddr + 328;

template <int NB>
struct Cfg {
    static constexpr int kStages = NB == 64 ? 2 : 3;        // A / activation stages
    static constexpr int kRingSlots = NB == 64 ? 2 : 3;     // quads in flight per decode warp
    static constexpr uint32_t kXStage = NB * kXRowBytes;
    static constexpr uint32_t kRingBytes = kRingSlots * 4 * 672;  // sized for the 26-state quad
    static constexpr uint32_t kRingHigh = kXBase + kStages * kXStage;
    static constexpr int kHighRings0 = (int)((kWindowEnd - kRingHigh) / kRingBytes);
    static constexpr int kHighRings = kHighRings0 < kDecodeWarps ? kHighRings0 : kDecodeWarps;
    static constexpr uint32_t kDCol = kStages * kStageCols;  // first accumulator column
    // instruction descriptor: f32 accumulators, bf16 A and B, both K-major, N, M = 128
    static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NB >> 3) << 17) |
                                       ((128u >> 4) << 24);
    // mbarriers after the slot barriers: a_full[S], a_empty[S], d_full[2], d_empty[2], fin
    static constexpr uint32_t kAFull = kPipeBars;
    static constexpr uint32_t kAEmpty = kPipeBars + 8 * kStages;
    static constexpr uint32_t kDFull = kPipeBars + 16 * kStages;
    static constexpr uint32_t kDEmpty = kDFull + 16;
    static constexpr uint32_t kFin = kDEmpty + 16;
    static_assert(kRingLow + (kDecodeWarps - kHighRings) * kRingBytes <= (32u << 10), "low rings overlap the table");
    static_assert(kFin + 8 <= kTmemHolder, "barrier block overflow");
    static_assert(kDCol + 2 * NB <= kTmemCols, "tensor-memory budget");
};
static_assert(kAbortFlag + 4 <= (512u << 7) && kBarAddr + 24 * 8 <= kPipeBars, "barrier block overflow");

template <int NB>
__device__ __forceinline__ uint32_t ring_base(int warp) {
    using C = Cfg<NB>;
    return warp < C::kHighRings ? C::kRingHigh + warp * C::kRingBytes
                                : kRingLow + (warp - C::kHighRings) * C::kRingBytes;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mbar_init_n(uint32_t bar, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ bool aborted() {
    uint32_t v;
    asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(kAbortFlag) : "memory");
    return v != 0;
}
__device__ __forceinline__ void raise_abort() {
    asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(kAbortFlag), "r"(1u) : "memory");
    atomicExch(&g_gemv_error, 3);
}
// A bounded wait that also gives up once another warp has aborted.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity) {
    if (mbar_wait(bar, parity)) return true;
    raise_abort();
    return false;
}

// D[128 x NB] (+)= A[128 x 16] (tensor memory) * B[16 x NB] (shared memory)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// K-major, no swizzle: 8-row x 16-byte core matrices, LBO = 128 B between the
// two core matrices of a k16 step, SBO = 4096 B between 8-row groups.
__device__ __forceinline__ uint64_t b_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 16) |
           ((uint64_t)(kXGroupBytes >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

// One unit's w_hat pairs into the A operand: rows g, g + 8 of the warp's row
// block; store register 4r + {0, 1, 2, 3} = (row g, column 8r + 2c),
// (row g, 8r + 2c + 1), (row g + 8, 8r + 2c), (row g + 8, 8r + 2c + 1).
template <int NS, int SH>
__device__ __forceinline__ void unit_to_tmem(const uint4& a, uint32_t w4, uint32_t sw, uint32_t lane_base,
                                             uint32_t sig_base, uint32_t taddr) {
    const uint32_t w[5] = {a.x, a.y, a.z, a.w, w4};
    const uint32_t lo = SH <= 2 ? (sw << (2 - SH)) : (sw >> (SH - 2));
    const uint32_t hi = sw >> (SH + 6);
    const uint32_t ss0 = lds((lo & 0x3FCu) | sig_base);  // (sigma, sigma) of row g
    const uint32_t ss1 = lds((hi & 0x3FCu) | sig_base);  // row g + 8
    const uint32_t v[16] = {
        what_pair<NS, 0>(w, lane_base, ss0),  what_pair<NS, 2>(w, lane_base, ss0),
        what_pair<NS, 1>(w, lane_base, ss1),  what_pair<NS, 3>(w, lane_base, ss1),
        what_pair<NS, 4>(w, lane_base, ss0),  what_pair<NS, 6>(w, lane_base, ss0),
        what_pair<NS, 5>(w, lane_base, ss1),  what_pair<NS, 7>(w, lane_base, ss1),
        what_pair<NS, 8>(w, lane_base, ss0),  what_pair<NS, 10>(w, lane_base, ss0),
        what_pair<NS, 9>(w, lane_base, ss1),  what_pair<NS, 11>(w, lane_base, ss1),
        what_pair<NS, 12>(w, lane_base, ss0), what_pair<NS, 14>(w, lane_base, ss0),
        what_pair<NS, 13>(w, lane_base, ss1), what_pair<NS, 15>(w, lane_base, ss1)};
    tmem_st_16x256b_x4(taddr, v);
}


struct Item {
    int job, rb, grp, cp0, n_units;
};

// The items of a job are its ceil(r16 / 8) tiles; keys (first item of every
// job) in shared memory.
template <int MAXJ>
__device__ __forceinline__ Item item_at(const GemvBatch<MAXJ>& batch, int64_t item) {
    Item I;
    int j = 0;
    if constexpr (MAXJ > 1) {
        int lo = 0, hi = batch.n - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if ((int64_t)(int32_t)lds(kBeginAddr + 4 * mid) <= item) lo = mid; else hi = mid - 1;
        }
        j = lo;
    }
    const GemvJob& J = batch.jobs[j];
    I.job = j;
    I.rb = (int)(item - J.item_begin);
    I.grp = 0;
    I.cp0 = 0;
    I.n_units = J.kp;
    return I;
}

// Residual sum of one output row: sum over the row's residual entries (one
// consecutive range of the row-major CSR, columns ascending) of bf16 value x
// activation, fp32, for each batch row n < m. xt: x^T, mp8 bf16 per column
// (the batch padded to 8). Eight entries and their activation vectors are in
// flight at once.
template <int NB>
__device__ __forceinline__ void row_residuals(const GemvJob& J, const uint16_t* xt, int mp8, int row, int m,
                                              float (&acc)[NB]) {
#pragma unroll
    for (int n = 0; n < NB; ++n) acc[n] = 0.f;
    const uint32_t cols = (uint32_t)J.cols;
    const uint32_t eb = __ldg(J.res_ptr + (int64_t)row * J.kg);
    const uint32_t ee = min(__ldg(J.res_ptr + (int64_t)(row + 1) * J.kg), J.n_res);
    constexpr int kB = NB <= 16 ? 8 : 4;
    for (uint32_t e0 = eb; e0 < ee; e0 += kB) {
        uint32_t en[kB];
#pragma unroll
        for (int t = 0; t < kB; ++t) en[t] = e0 + t < ee ? __ldg(J.res_ent + e0 + t) : 0u;
#pragma unroll
        for (int n8 = 0; n8 < NB / 8; ++n8) {
            if (8 * n8 < m) {
                uint4 q[kB];
#pragma unroll
                for (int t = 0; t < kB; ++t) {
                    const uint32_t col = en[t] >> 16;
                    q[t] = e0 + t < ee && col < cols
                               ? __ldg(reinterpret_cast<const uint4*>(xt + (int64_t)col * mp8) + n8)
                               : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
                for (int t = 0; t < kB; ++t) {
                    const float v = __uint_as_float(en[t] << 16);  // zero for absent entries
                    const uint32_t w[4] = {q[t].x, q[t].y, q[t].z, q[t].w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc[8 * n8 + 2 * k] = fmaf(v, __uint_as_float(w[k] << 16), acc[8 * n8 + 2 * k]);
                        acc[8 * n8 + 2 * k + 1] =
                            fmaf(v, __uint_as_float(w[k] & 0xFFFF0000u), acc[8 * n8 + 2 * k + 1]);
                    }
                }
            }
        }
    }
}

// The prepared activations of a job: x_perm (the B-operand stage of quad q at
// q * NB * 512 bytes) then x^T.
template <int NB>
__device__ __forceinline__ const uint16_t* prep_xt(const GemvJob& J) {
    const int64_t xperm = ((int64_t)(J.kp + 3) / 4 * NB * 512 + 255) / 256 * 256;
    return reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(J.reserved_ptr) + xperm);
}

// Lays out the activations of every job whose rb_begin-th block range covers
// blockIdx.x (jobs with the same x share one preparation): block = (job, quad).
// x_perm row n of quad q, permuted column k' = 64u + 2t + e with
// t = 8r + 2c + j holds x[n, 256q + 64u + 16c + 4r + 2j + e]; batch rows past
// m and the phantom tile's columns are zero. x^T[col][n] for n < mp8.
template <int NB, int MAXJ>
__global__ void __launch_bounds__(256) x_prep_kernel(const __grid_constant__ GemvBatch<MAXJ> batch) {
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
    if (!J.reserved0) return;  // prepared by another job with the same activations
    const int q = (int)blockIdx.x - J.rb_begin;
    if (q >= (J.kp + 3) / 4) return;
    const int m = batch.m, mp8 = (m + 7) / 8 * 8, ng = (m + 7) / 8;
    const int t = threadIdx.x;           // column within the quad
    const int col = 256 * q + t;
    const bool live = col < J.cols;
    uint16_t* xperm = static_cast<uint16_t*>(J.reserved_ptr) + (int64_t)q * NB * 256;
    uint16_t* xt = const_cast<uint16_t*>(prep_xt<NB>(J));
    // permuted position of column t: unit u, c = bits 4..5, r = bits 2..3, j = bit 1, e = bit 0
    const int u = t >> 6, c64 = t & 63;
    const int c = c64 >> 4, r = (c64 >> 2) & 3, jj = (c64 >> 1) & 1, e = c64 & 1;
    const int kperm = 64 * u + 2 * (8 * r + 2 * c + jj) + e;  // permuted column within the quad
    const int kb = kperm >> 3, pos = kperm & 7;
    if (col < 64 * J.kp) {
        for (int n = 0; n < 8 * ng; ++n) {
            const uint16_t v = live && n < m ? J.x[(int64_t)n * J.cols + col] : (uint16_t)0;
            xperm[(n >> 3) * 2048 + kb * 64 + (n & 7) * 8 + pos] = v;
        }
        for (int n = 0; n < mp8; ++n)
            xt[(int64_t)col * mp8 + n] = live && n < m ? J.x[(int64_t)n * J.cols + col] : (uint16_t)0;
    }
}

template <int NS, int NB, int MAXJ>
__global__ void __launch_bounds__(kThreads, 1) tile_kernel(const __grid_constant__ GemvBatch<MAXJ> batch) {
    using Tr = PackTraits<NS>;
    using C = Cfg<NB>;
    constexpr uint32_t kU = Tr::kUnit;
    constexpr uint32_t kQuad = 4 * kU;
    constexpr int S = C::kStages;
    constexpr int R = C::kRingSlots;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
    if (s0 > kRingLow || s0 + kSmemBytes < kWindowEnd) {
        if (threadIdx.x == 0) atomicExch(&g_gemv_error, 1);
        return;
    }
    uint8_t* const base = smem - s0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- tables, keys, barriers, zeroed activation stages, tensor memory ----
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
    for (uint32_t i = threadIdx.x; i < S * C::kXStage / 16; i += blockDim.x)
        *reinterpret_cast<uint4*>(base + kXBase + 16 * i) = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (MAXJ > 1) {
        for (int i = warp; i < batch.n; i += kThreads / 32)
            if (lane == 0) *reinterpret_cast<int32_t*>(base + kBeginAddr + 4 * i) = (int32_t)batch.jobs[i].item_begin;
    }
    if (threadIdx.x == 0) {
        for (int k = 0; k < kDecodeWarps * R; ++k) mbar_init(kSlotBars + 8 * k);
        for (int k = 0; k < S; ++k) {
            mbar_init_n(C::kAFull + 8 * k, kDecodeWarps + 1);
            mbar_init_n(C::kAEmpty + 8 * k, 1);
        }
        for (int k = 0; k < 2; ++k) {
            mbar_init_n(C::kDFull + 8 * k, 1);
            mbar_init_n(C::kDEmpty + 8 * k, kEpiWarps);
        }
        mbar_init_n(C::kFin, 1);
        *reinterpret_cast<uint32_t*>(base + kAbortFlag) = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(kTmemHolder),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the activation stages were zeroed through the generic proxy; the mmas read them through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(base + kTmemHolder);

    const int64_t total = batch.total_items;
    const int64_t stride = gridDim.x;

    if (warp < kDecodeWarps) {
        // ------------------------------ decode warps ------------------------------
        const int bb = 2 * (warp & 3) + (warp >> 2);  // row block within the tile
        const uint32_t t_lane = (uint32_t)(16 * bb) << 16;
        const uint32_t ring = ring_base<NB>(warp);
        const uint32_t bars = kSlotBars + warp * R * 8;
        const uint32_t lane_base = NS == 26 ? (kLat26Xor | (4u * lane)) : (kLat16Base + 4u * lane);
        const uint32_t sig_base = kSigAddr;

        // producer cursor over this CTA's items in which this warp has a row block
        int64_t p_item = blockIdx.x;
        int p_q = 0, p_nq = 0, p_units = 0;
        const uint8_t* p_src = nullptr;
        uint32_t p_slot = 0;
        auto p_load = [&]() {
            for (; p_item < total; p_item += stride) {
                const Item I = item_at(batch, p_item);
                const GemvJob& J = batch.jobs[I.job];
                const int b16 = 8 * I.rb + bb;
                if (b16 < J.r16) {
                    p_src = J.units + ((int64_t)b16 * J.kp + I.cp0) * kU;
                    p_units = I.n_units;
                    p_nq = (I.n_units + 3) >> 2;
                    p_q = 0;
                    return;
                }
            }
        };
        auto produce = [&]() {
            if (p_item >= total) return;
            const int left = p_units - 4 * p_q;
            const uint32_t bytes = (uint32_t)(left < 4 ? left : 4) * kU;
            if (lane == 0) {
                const uint32_t bar = bars + 8 * p_slot;
                slot_arm(bar, bytes);
                bulk_copy(ring + p_slot * kQuad, p_src + (int64_t)p_q * kQuad, bytes, bar);
            }
            p_slot = p_slot + 1 == (uint32_t)R ? 0u : p_slot + 1;
            if (++p_q == p_nq) {
                p_item += stride;
                p_load();
            }
        };
        p_load();
#pragma unroll
        for (int k = 0; k < R; ++k) produce();

        uint32_t c_slot = 0, c_phase = 0;
        uint32_t cc = 0;  // chunks (stages) consumed
        bool ok = true;
        for (int64_t item = blockIdx.x; item < total && ok; item += stride) {
            const Item I = item_at(batch, item);
            const GemvJob& J = batch.jobs[I.job];
            const bool valid = 8 * I.rb + bb < J.r16;
            const int nq = (I.n_units + 3) >> 2;
            for (int q = 0; q < nq; ++q, ++cc) {
                if (aborted()) {
                    ok = false;
                    break;
                }
                const uint32_t s = cc % S;
                uint4 A[4] = {};
                uint4 W = make_uint4(0u, 0u, 0u, 0u);
                uint2 Sg = make_uint2(0u, 0u);
                const int uq = min(4, I.n_units - 4 * q);
                if (valid) {
                    if (!wait_or_abort(bars + 8 * c_slot, c_phase)) {
                        ok = false;
                        break;
                    }
                    const uint32_t slot = ring + c_slot * kQuad;
                    if (uq == 4) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) A[i] = lds_slot4(slot + 512 * i + 16 * lane);
                        if constexpr (NS == 26) W = lds_slot4(slot + 2048 + 16 * lane);
                        Sg = lds_slot2(slot + 4 * Tr::kSigOff + 8 * (lane >> 1));
                    } else {
                        uint32_t w4[3] = {0u, 0u, 0u}, h[3] = {0u, 0u, 0u};
#pragma unroll
                        for (int i = 0; i < 3; ++i) {
                            if (i < uq) {
                                A[i] = lds_slot4(slot + 512 * i + 16 * lane);
                                if constexpr (NS == 26) w4[i] = lds_slot(slot + 512 * uq + 4 * (uq * lane + i));
                                h[i] = lds_slot_u16(slot + Tr::kSigOff * uq + 2 * (uq * (lane >> 1) + i));
                            }
                        }
                        W = make_uint4(w4[0], w4[1], w4[2], 0u);
                        Sg = make_uint2(h[0] | (h[1] << 16), h[2]);
                    }
                    // one register of every slot read: each read has landed before the slot is reused
                    uint32_t dep = A[0].x ^ A[1].x ^ A[2].x ^ A[3].x ^ W.x ^ W.y ^ W.z ^ Sg.x ^ Sg.y;
                    asm volatile("" ::"r"(dep));
                    __syncwarp();
                    produce();
                    c_slot = c_slot + 1 == (uint32_t)R ? 0u : c_slot + 1;
                    c_phase ^= c_slot == 0 ? 1u : 0u;
                }
                // the mmas that last read stage s are done
                if (!wait_or_abort(C::kAEmpty + 8 * s, ((cc / S) & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (valid) {
                    const uint32_t ta = tmem + t_lane + s * kStageCols;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (i < uq) {
                            const uint32_t w4 = i == 0 ? W.x : i == 1 ? W.y : i == 2 ? W.z : W.w;
                            const uint32_t sw = i < 2 ? Sg.x : Sg.y;
                            if (i & 1) unit_to_tmem<NS, 16>(A[i], w4, sw, lane_base, sig_base, ta + 32 * i);
                            else unit_to_tmem<NS, 0>(A[i], w4, sw, lane_base, sig_base, ta + 32 * i);
                        }
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(C::kAFull + 8 * s);
            }
        }
        if (!ok) {
            // copies still in flight into this warp's ring get a bounded chance to land
            for (int k = 0; k < R; ++k) {
                (void)mbar_wait(bars + 8 * c_slot, c_phase);
                c_slot = c_slot + 1 == (uint32_t)R ? 0u : c_slot + 1;
                c_phase ^= c_slot == 0 ? 1u : 0u;
            }
        }
    } else if (warp == kXWarp) {
        // --------------------------- activation staging ---------------------------
        // one bulk copy per quad of the prepared stage (the batch rows' 8-row
        // groups that hold data; the other rows stay zero from the set-up)
        if (lane == 0) {
            const uint32_t xbytes = (uint32_t)((batch.m + 7) / 8) * kXGroupBytes;
            uint32_t cc = 0;
            bool ok = true;
            for (int64_t item = blockIdx.x; item < total && ok; item += stride) {
                const Item I = item_at(batch, item);
                const GemvJob& J = batch.jobs[I.job];
                const int nq = (I.n_units + 3) >> 2;
                const uint8_t* xp = static_cast<const uint8_t*>(J.reserved_ptr);
                for (int q = 0; q < nq; ++q, ++cc) {
                    const uint32_t s = cc % S;
                    if (aborted() || !wait_or_abort(C::kAEmpty + 8 * s, ((cc / S) & 1u) ^ 1u)) {
                        ok = false;
                        break;
                    }
                    slot_arm(C::kAFull + 8 * s, xbytes);
                    bulk_copy(kXBase + s * C::kXStage, xp + (int64_t)q * C::kXStage, xbytes, C::kAFull + 8 * s);
                }
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ------------------------------ mma issuer ------------------------------
        if (lane == 0) {
            uint32_t cc = 0, it = 0;
            bool ok = true;
            for (int64_t item = blockIdx.x; item < total && ok; item += stride, ++it) {
                const Item I = item_at(batch, item);
                const int nq = (I.n_units + 3) >> 2;
                const uint32_t b = it & 1u;
                if (!wait_or_abort(C::kDEmpty + 8 * b, ((it >> 1) & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + C::kDCol + NB * b;
                for (int q = 0; q < nq; ++q, ++cc) {
                    const uint32_t s = cc % S;
                    if (aborted() || !wait_or_abort(C::kAFull + 8 * s, (cc / S) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int ksteps = 4 * min(4, I.n_units - 4 * q);
                    const uint32_t a = tmem + s * kStageCols;
                    const uint64_t bd = b_desc(kXBase + s * C::kXStage);
                    for (int k = 0; k < ksteps; ++k)
                        mma_ts(d, a + 8 * k, bd + (uint64_t)(16 * k), C::kIdesc, (q | k) != 0 ? 1u : 0u);
                    tc_commit(C::kAEmpty + 8 * s);
                }
                if (!ok) break;
                tc_commit(C::kDFull + 8 * b);
            }
            // every mma issued by this thread has completed before tensor memory is released
            tc_commit(C::kFin);
            (void)mbar_wait(C::kFin, 0);
        }
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------------
        const int qw = warp & 3;  // tensor-memory lane quarter of this warp
        const int m = batch.m, mp8 = (m + 7) / 8 * 8;
        uint32_t it = 0;
        for (int64_t item = blockIdx.x; item < total; item += stride, ++it) {
            const Item I = item_at(batch, item);
            const GemvJob& J = batch.jobs[I.job];
            const uint32_t b = it & 1u;
            const int row = I.rb * 128 + 32 * qw + lane;
            const bool live = row < J.rows;
            // the residual sum does not depend on the mmas: it runs while they do
            float acc[NB];
            if (live) row_residuals<NB>(J, prep_xt<NB>(J), mp8, row, m, acc);
            if (aborted() || !wait_or_abort(C::kDFull + 8 * b, (it >> 1) & 1u)) break;
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(32 * qw) << 16) + C::kDCol + NB * b;
#pragma unroll
            for (int cb = 0; cb < NB / 8; ++cb) {
                if (8 * cb < m) {
                    uint32_t v[8];
                    tmem_ld_32x32b_x8(taddr + 8 * cb, v);
                    // the destination registers are defined only after the wait
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int k = 0; k < 8; ++k) acc[8 * cb + k] += __uint_as_float(v[k]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(C::kDEmpty + 8 * b);  // the accumulator may be reused
            if (live) {
                const float bv = J.bias ? bf16_to_f32(J.bias[row]) : 0.f;
#pragma unroll
                for (int n = 0; n < NB; ++n) {
                    if (n < m) {
                        const float v = acc[n] + bv;
                        if (J.out_f32) reinterpret_cast<float*>(J.y)[(int64_t)n * J.rows + row] = v;
                        else reinterpret_cast<uint16_t*>(J.y)[(int64_t)n * J.rows + row] =
                                __bfloat16_as_ushort(__float2bfloat16_rn(v));
                    }
                }
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace tile
