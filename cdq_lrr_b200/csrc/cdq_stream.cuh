// The streaming fused linear for batches of 1 to 8 rows, and the residual
// pre-pass shared by both streaming paths. Included by cdq_gemv.cu (it shares
// that file's bulk-copy ring, pair tables and unit decode).
//
// Residual pre-pass (res_sum_kernel). One thread per CSR bucket (row, group
// of 32 tile columns) of every job of the launch:
//     R[n][group][row] = sum over the bucket's entries, in order, starting
//                        from zero, of bf16 value x activation (fp32 fma),
// written to the job's per-group sums in the workspace. The buckets of a row
// are consecutive, so a warp reads one stretch of the entry array; a thread's
// loads are issued in batches so that several are in flight.
//
// Streaming kernel (stream_kernel). The units of every job of a launch form
// one sequence: job by job, row block by row block, which is also the order
// of the units buffers in memory. A work item is (job, 16-row block, residual
// group of up to 16 units, i.e. 32 tile columns). Warp w of the W warps of
// the grid owns the items whose first unit lies in [U*w/W, U*(w+1)/W) (U =
// units of the launch), so each warp walks one contiguous stretch of the
// units buffers: its producer lane copies quad after quad into the warp's
// two-slot ring, and the cursor moves from item to item without a search.
// Per item the quads are decoded into exact w_hat pairs and fed to mma.sync
// (as in the wide kernel), and the group's value is the mma sum plus the
// group's residual sum from the pre-pass (read at the item's start, used at
// its end). An output is
//     y = sum over the row's groups, in group order and starting from zero,
//         of (mma sum of the group + residual sum of the group), + bias,
// rounded once. A row block whose groups all lie in one warp's stretch is
// summed in registers. A row block cut by a stretch boundary writes each
// group's value to the workspace (over the group's residual sum, which its
// own lane has read); the warp that brings the row block's arrival counter to
// its group count adds the values in group order, stores y and resets the
// counter to zero. Either way the arithmetic is the same, so y does not
// depend on how a launch is cut into stretches (or grouped with other jobs),
// and the output is deterministic. The wide kernel (batches above 8) and its
// fix-up pass use the same per-group values.
namespace stream {

#ifndef CDQ_STREAM_WARPS
#define CDQ_STREAM_WARPS 16
#endif
constexpr int kSWarps = CDQ_STREAM_WARPS;
constexpr int kSThreads = 32 * kSWarps;
constexpr int kSLowWarps = 5;  // rings below the pair table, in [1K, 32K)

// A slot holds one quad (the activations come through the L1 cache).
template <int NS>
struct Ring {
    static constexpr uint32_t kQuad = 4 * PackTraits<NS>::kUnit;
    static constexpr uint32_t kBytes = kSlots * kQuad;
    static constexpr uint32_t kTop = kHighStage + (kSWarps - kSLowWarps) * kBytes;
};
static_assert(kLowStage + kSLowWarps * Ring<26>::kBytes <= (32u << 10), "low rings overlap the table");
static_assert(Ring<26>::kTop <= kSmemBytes && Ring<16>::kTop <= kSmemBytes, "rings exceed the window");
static_assert(kBarAddr + kSWarps * kSlots * 8 <= (512u << 7), "barriers overlap the table");

template <int NS>
__device__ __forceinline__ uint32_t ring_of(int warp) {
    return warp < kSLowWarps ? kLowStage + warp * Ring<NS>::kBytes
                             : kHighStage + (warp - kSLowWarps) * Ring<NS>::kBytes;
}

// A work item: job, 16-row block, residual group.
struct Cursor {
    int j, b16, grp;
};

// First unit of the item (the launch's unit count once past the last job).
// B: a batch view with n, total_units and jobs[] (GemvBatch, or the
// persistent decode kernel's per-projection-group view).
template <class B>
__device__ __forceinline__ int item_start(const B& b, const Cursor& c) {
    if (c.j >= b.n) return (int)b.total_units;
    const GemvJob& J = b.jobs[c.j];
    return (int)J.unit_begin + c.b16 * J.kp + 16 * c.grp;
}

// The first item whose first unit is >= u (u in [0, total_units]).
template <class B>
__device__ __forceinline__ Cursor first_at(const B& b, int u) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {  // last job with unit_begin <= u (uniform reads of the launch record)
        const int mid = (lo + hi + 1) >> 1;
        if (b.jobs[mid].unit_begin <= u) lo = mid; else hi = mid - 1;
    }
    const GemvJob& J = b.jobs[lo];
    const uint32_t rel = (uint32_t)(u - J.unit_begin);  // launches hold fewer than 2^31 units
    Cursor c;
    c.j = lo;
    c.b16 = (int)(rel / (uint32_t)J.kp);
    c.grp = ((int)(rel - (uint32_t)c.b16 * (uint32_t)J.kp) + 15) >> 4;
    if (c.grp >= J.kg) {
        c.grp = 0;
        ++c.b16;
    }
    if (c.b16 >= J.r16) {
        c.b16 = 0;
        ++c.j;
    }
    return c;
}

// Residual pre-pass: a block takes 256 consecutive buckets of one job (one
// thread per bucket). Their entries are one contiguous stretch of the entry
// array: thread 0 bulk-copies it into shared memory (the 16-byte-aligned
// part; a ragged edge of up to three entries at either end is read with
// plain loads) together with the activation row, then each thread adds its
// bucket's entries in order, activations read from shared memory. A stretch
// longer than the entry buffer goes in chunks (the thread's sum carries
// over); batches of several rows repeat the pass per row. The one wait on the
// copies is bounded (error code 4 of the fused linear on timeout). Block ->
// job through rb_begin (set by the launcher).
constexpr int kResThreads = 256;
constexpr int kResCap = 4096;  // entries staged per chunk (16 KB)

__host__ __device__ constexpr int res_smem_bytes(int cols) { return 16 + (kResCap + 4) * 4 + cols * 2; }

template <int MAXJ>
__global__ void __launch_bounds__(kResThreads) res_sum_kernel(const __grid_constant__ GemvBatch<MAXJ> batch) {
    // the streaming kernel may be scheduled now (it waits for this grid's
    // completion before it reads any residual sum); this grid itself waits
    // for the kernel that wrote the activations
    pdl_release();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t rsm[];
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(rsm);
    uint32_t* const ent = reinterpret_cast<uint32_t*>(rsm + 16);  // entry e of a chunk at e - (c0 & ~3)
    uint16_t* const xs = reinterpret_cast<uint16_t*>(rsm + 16 + (kResCap + 4) * 4);
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
    const int kg = J.kg, cols = J.cols, tid = threadIdx.x;
    const uint32_t buckets = (uint32_t)J.r16 * 16u * (uint32_t)kg;
    const uint32_t bb = ((uint32_t)blockIdx.x - (uint32_t)J.rb_begin) * kResThreads;
    const uint32_t b = bb + tid;
    const bool live = b < buckets;
    const uint32_t n_res = J.n_res;
    const uint32_t last = min(bb + kResThreads, buckets);  // one past the block's last bucket
    const bool bulk = ((uintptr_t)J.res_ent & 15u) == 0;   // entries 16-byte aligned: copy in bulk
    if (tid == 0) {
        mbar_init(bar);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the block's stretch [E0, E1) and this thread's bucket [s, t) (the CSR is ascending)
    const uint32_t E0 = min(__ldg(J.res_ptr + bb), n_res);
    const uint32_t E1 = max(min(__ldg(J.res_ptr + last), n_res), E0);
    const uint32_t s = live ? min(max(__ldg(J.res_ptr + b), E0), E1) : E1;
    const uint32_t t = live ? min(max(__ldg(J.res_ptr + b + 1), s), E1) : E1;
    const uint32_t row = b / (uint32_t)kg, grp = b - row * (uint32_t)kg;
    const int64_t rpad = (int64_t)J.r16 * 16;
    const int m = batch.m;
    __syncthreads();
    uint32_t phase = 0;
    for (int n = 0; n < m; ++n) {
        float acc = 0.f;
        for (uint32_t c0 = E0; c0 < E1; c0 += kResCap) {
            const uint32_t c1 = min(c0 + (uint32_t)kResCap, E1), base = c0 & ~3u;
            // [a0, a1): the chunk's 16-byte-aligned entries (bulk-copied); [c0, a0)
            // and [a1, c1) hold at most three entries each (plain loads)
            const uint32_t a0 = bulk ? min((c0 + 3u) & ~3u, c1) : c1, a1 = bulk ? max(c1 & ~3u, a0) : c1;
            __syncthreads();  // the previous chunk's (or row's) readers are done
            if (tid == 0) {
                const uint32_t xbytes = c0 == E0 ? (uint32_t)cols * 2 : 0u;
                slot_arm(bar, xbytes + (a1 - a0) * 4);
                if (xbytes) bulk_copy(bar + 16 + (kResCap + 4) * 4, J.x + (int64_t)n * cols, xbytes, bar);
                if (a1 > a0) bulk_copy(bar + 16 + (a0 - base) * 4, J.res_ent + a0, (a1 - a0) * 4, bar);
            }
            for (uint32_t e = c0 + tid; e < a0; e += kResThreads) ent[e - base] = __ldg(J.res_ent + e);
            for (uint32_t e = a1 + tid; e < c1; e += kResThreads) ent[e - base] = __ldg(J.res_ent + e);
            const bool landed = mbar_wait(bar, phase);
            phase ^= 1u;
            if (!__syncthreads_and(landed)) {
                if (tid == 0) atomicExch(&g_gemv_error, 4);
                return;
            }
            const uint32_t lo = max(s, c0), hi = min(t, c1);
            for (uint32_t e = lo; e < hi; ++e) {
                const uint32_t en = ent[e - base];
                const uint32_t col = en >> 16;
                if (col < (uint32_t)cols)
                    acc = fmaf(__uint_as_float(en << 16), __uint_as_float((uint32_t)xs[col] << 16), acc);
            }
        }
        if (live) J.partial[((int64_t)n * kg + grp) * rpad + row] = acc;
    }
}

// The pre-pass over every job of the launch (a batch of m rows).
template <int MAXJ>
cudaError_t launch_res(const GemvBatch<MAXJ>& b, int m, cudaStream_t stream) {
    GemvBatch<MAXJ> rb = b;
    int64_t blocks = 0;
    int max_cols = 32;
    for (int j = 0; j < b.n; ++j) {
        rb.jobs[j].rb_begin = (int32_t)blocks;
        blocks += ((int64_t)b.jobs[j].r16 * 16 * b.jobs[j].kg + kResThreads - 1) / kResThreads;
        max_cols = std::max(max_cols, (int)b.jobs[j].cols);
    }
    if (blocks >= INT32_MAX) return cudaErrorInvalidValue;
    rb.m = m;
    const int smem = res_smem_bytes(max_cols);  // at most 160 KB
    auto kern = res_sum_kernel<MAXJ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, res_smem_bytes(CDQ_MAX_COLS));
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3((unsigned)std::max<int64_t>(blocks, 1)), dim3(kResThreads), (size_t)smem, stream, rb);
}

// floor(U * k / n) for U < 2^31 and k <= n < 2^16, without a 64-bit division:
// the double quotient is within one of the answer, then fixed exactly.
__device__ __forceinline__ int64_t stretch_bound(int64_t U, int64_t k, int64_t n) {
    const int64_t num = U * k;
    int64_t q = (int64_t)((double)num / (double)n);
    if (q * n > num) --q;
    if ((q + 1) * n <= num) ++q;
    return q;
}

// A group of a row block cut by a stretch boundary: store the group's value;
// the warp's last group of the row block reports its `done` groups on the
// row block's counter, and the warp that completes the count adds the groups
// in order, stores y and resets the counter. Kept out of line: it runs for at
// most two row blocks per warp.
template <int M>
__device__ __noinline__ void cut_group(const GemvJob& J, int b16, int grp, const float (&v)[4], bool report,
                                       int done, int g, int c, int lane) {
    const int kg = J.kg;
    const int64_t rpad = (int64_t)J.r16 * 16;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int64_t row = b16 * 16 + g + 8 * h;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int n = 2 * c + jj;
            if (n < M) J.partial[((int64_t)n * kg + grp) * rpad + row] = v[2 * h + jj];
        }
    }
    if (!report) return;
    fence_acq_rel_gpu();  // release: the group values before the count
    __syncwarp();
    uint32_t before = 0;
    if (lane == 0) before = atomicAdd(J.counters + b16, (uint32_t)done);
    before = __shfl_sync(0xFFFFFFFFu, before, 0);
    if (before + (uint32_t)done != (uint32_t)kg) return;
    // every group has arrived: add them in group order
    fence_acq_rel_gpu();  // acquire: the other groups' values after the count
    __syncwarp();         // ... for every lane, through lane 0's acquire
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int row = b16 * 16 + g + 8 * h;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int n = 2 * c + jj;
            if (n < M) {
                const float* sp = J.partial + (int64_t)n * kg * rpad + row;
                float s = 0.f;
                for (int k = 0; k < kg; ++k) s += __ldcg(sp + (int64_t)k * rpad);
                if (row < J.rows) store_out(J, n, row, s);
            }
        }
    }
    if (lane == 0) J.counters[b16] = 0u;
}

// Activations of a unit: 16 bf16 per lane as two 16-byte loads, from global
// memory through the L1 cache (XGlobal) or from shared memory (XShared: the
// persistent decode kernel keeps each projection group's input there).
struct XGlobal {
    const uint16_t* p;
    __device__ __forceinline__ XGlobal at(int64_t off) const { return XGlobal{p + off}; }
    __device__ __forceinline__ void load(int off, uint4& a, uint4& b) const {
        a = ldg_x4(p + off);
        b = ldg_x4(p + off + 8);
    }
};
struct XShared {
    uint32_t addr;
    __device__ __forceinline__ XShared at(int64_t off) const { return XShared{addr + 2u * (uint32_t)off}; }
    __device__ __forceinline__ void load(int off, uint4& a, uint4& b) const {
        const uint32_t q = addr + 2u * (uint32_t)off;
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w) : "r"(q));
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
                     : "r"(q + 16));
    }
};

// One quad of UQ units (4: a full quad; 1..3: the compact last quad of a row
// block) read from its ring slot: the lane's code words and scale half-words
// into registers, then the slot goes back to the producer (`refill`, after
// one register of every read has arrived, so the next copy cannot overwrite
// bytes still being read), then the units' mmas. PH: the item holds the
// phantom second tile of an odd tile count (unit `phantom` of this quad, -1
// if none here), whose lanes c >= 2 take zero activations.
template <int NS, int UQ, bool PH, class X, typename Refill>
__device__ __forceinline__ void quad_step(uint32_t slot, int lane, int c, const X& xq, int phantom,
                                          uint32_t lane_base, uint32_t sig_base, float (&d)[4], Refill&& refill) {
    using Tr = PackTraits<NS>;
    uint4 A[4];
    uint32_t w4[4] = {0u, 0u, 0u, 0u};
    uint32_t s01, s23, dep;
    if constexpr (UQ == 4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) A[i] = lds_slot4(slot + 512 * i + 16 * lane);
        const uint4 W = NS == 26 ? lds_slot4(slot + 2048 + 16 * lane) : make_uint4(0u, 0u, 0u, 0u);
        const uint2 S = lds_slot2(slot + 4 * Tr::kSigOff + 8 * (lane >> 1));
        w4[0] = W.x;
        w4[1] = W.y;
        w4[2] = W.z;
        w4[3] = W.w;
        s01 = S.x;
        s23 = S.y;
        dep = W.x ^ S.x ^ A[0].x ^ A[1].x ^ A[2].x ^ A[3].x;
    } else {
        uint32_t h[3] = {0u, 0u, 0u};
        dep = 0u;
#pragma unroll
        for (int i = 0; i < UQ; ++i) {
            A[i] = lds_slot4(slot + 512 * i + 16 * lane);
            if constexpr (NS == 26) w4[i] = lds_slot(slot + 512 * UQ + 4 * (UQ * lane + i));
            h[i] = lds_slot_u16(slot + Tr::kSigOff * UQ + 2 * (UQ * (lane >> 1) + i));
            dep ^= A[i].x ^ w4[i] ^ h[i];
        }
        s01 = h[0] | (h[1] << 16);
        s23 = h[2];
    }
    asm volatile("" ::"r"(dep));
    __syncwarp();
    refill();
#pragma unroll
    for (int i = 0; i < UQ; ++i) {
        uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
        // the phantom tile's lanes c >= 2 take zero activations
        if (!PH || i != phantom || c < 2) xq.load(64 * i, xa, xb);
        if (i & 1) unit_mma<NS, 16>(A[i], w4[i], i < 2 ? s01 : s23, xa, xb, lane_base, sig_base, d);
        else unit_mma<NS, 0>(A[i], w4[i], i < 2 ? s01 : s23, xa, xb, lane_base, sig_base, d);
    }
}

// The pair table (lane-private copies) and the fp8 scale table of a
// streaming kernel's shared window; every thread of the block takes part (no
// barrier inside).
template <int NS>
__device__ __forceinline__ void build_tables(uint8_t* base) {
    using Tr = PackTraits<NS>;
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
}

// Where a warp's two-slot ring stands between calls of stream_warp: the slot
// the next quad lands in and that slot's mbarrier phase. Every call consumes
// every copy it issues, so the next call starts with an empty ring.
struct RingState {
    uint32_t slot, phase;
};

// A warp's place in one stretch [u_lo, u_hi) of a batch's unit sequence: the
// consumer's first item and the producer's position. The producer (lane 0
// issues; every lane keeps the same cursor) walks the quads of
// [u_first, u_end), which are consecutive in each job's units buffer.
struct Stretch {
    Cursor cur;
    int u_lo, u_hi, u_first, grp_first;
    int pj, p_left, p_kp, p_r, p_rb;
    const uint8_t* p_ptr;
    int opened;  // copies stretch_open issued (0 .. 2)
};

// Issues the next quad's copy into `slot` (the slot the consumer has just
// read, or one of the first two).
template <int NS, class B>
__device__ __forceinline__ void stretch_produce(Stretch& st, const B& batch, uint32_t slot, uint32_t ring,
                                                uint32_t bars) {
    constexpr uint32_t kU = PackTraits<NS>::kUnit;
    if (st.p_left <= 0) return;
    const int u = min(4, st.p_kp - st.p_r);
    const uint32_t bytes = (uint32_t)u * kU;
    if ((threadIdx.x & 31) == 0) {
        const uint32_t bar = bars + 8 * slot;
        slot_arm(bar, bytes);
        bulk_copy(ring + slot * Ring<NS>::kQuad, st.p_ptr, bytes, bar);
    }
    st.p_ptr += bytes;
    st.p_left -= u;
    st.p_r += u;
    if (st.p_r == st.p_kp) {
        st.p_r = 0;
        if (--st.p_rb == 0 && st.p_left > 0) {
            const GemvJob& J = batch.jobs[++st.pj];
            st.p_kp = J.kp;
            st.p_rb = J.r16;
            st.p_ptr = J.units;
        }
    }
}

// Opens a warp's stretch: finds its first item, issues the first two copies
// into the ring (rs: where the ring stands) and, with prefetch_l2, asks L2 for
// every other byte of the stretch's weights (small stretches, so the later
// copies come from L2).
template <int NS, class B>
__device__ __forceinline__ Stretch stretch_open(const B& batch, int u_lo, int u_hi, uint32_t ring, uint32_t bars,
                                                const RingState& rs, bool prefetch_l2) {
    constexpr uint32_t kU = PackTraits<NS>::kUnit;
    Stretch st;
    st.opened = 0;
    st.cur = first_at(batch, u_lo);
    st.u_lo = u_lo;
    st.u_hi = u_hi;
    st.u_first = item_start(batch, st.cur);
    st.grp_first = st.cur.grp;  // first group of a row block cut at the stretch's start
    st.p_left = 0;
    if (st.u_first >= u_hi) return st;  // no item starts in this stretch
    const int u_end = item_start(batch, first_at(batch, u_hi));
    st.pj = st.cur.j;
    st.p_left = u_end - st.u_first;
    const GemvJob& J = batch.jobs[st.pj];
    st.p_kp = J.kp;
    st.p_r = 16 * st.cur.grp;
    st.p_rb = J.r16 - st.cur.b16;
    st.p_ptr = J.units + ((int64_t)st.cur.b16 * J.kp + st.p_r) * kU;
    if (prefetch_l2 && (threadIdx.x & 31) == 0) {
        int left = st.p_left, pj = st.pj;
        const uint8_t* ptr = st.p_ptr;
        int in_job = st.p_rb * st.p_kp - st.p_r;  // units from p_ptr to the job's end
        while (left > 0) {
            const int u = min(left, in_job);
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"((uint32_t)u * kU) : "memory");
            left -= u;
            if (left > 0) {
                const GemvJob& Jn = batch.jobs[++pj];
                ptr = Jn.units;
                in_job = Jn.r16 * Jn.kp;
            }
        }
    }
    const int before = st.p_left;
    stretch_produce<NS>(st, batch, rs.slot, ring, bars);
    const int after1 = st.p_left;
    stretch_produce<NS>(st, batch, rs.slot ^ 1u, ring, bars);
    st.opened = (before > 0) + (after1 > 0);
    return st;
}

// Lets the copies an opened stretch issued land before the warp leaves
// without running it (an error path): bounded waits, ring state unchanged.
template <int NS>
__device__ __forceinline__ void stretch_drain(const Stretch& st, uint32_t bars, const RingState& rs) {
    uint32_t slot = rs.slot, phase = rs.phase;
    for (int k = 0; k < st.opened; ++k) {
        (void)mbar_wait(bars + 8 * slot, phase);
        slot ^= 1u;
        phase ^= slot == 0 ? 1u : 0u;
    }
}

// Runs an opened stretch: its items decoded, multiplied, finished with the
// residual sums from the workspace, and the outputs written (cut row blocks
// through the arrival counters). xsrc(J.x) gives a job's activation source
// (XGlobal or XShared). Returns false if a copy never landed (error code 2
// recorded, in-flight copies drained).
// The residual-sum wait of stretch_run: poll() says without waiting whether
// the sums are published, operator() waits for them (bounded; false: gave
// up). RReady: no wait, the sums are complete before the stretch runs.
struct RReady {
    __device__ __forceinline__ bool poll() const { return true; }
    __device__ __forceinline__ bool operator()() const { return true; }
};

template <int NS, int M, class X, class B, class XSrc, class RWait = RReady>
__device__ __forceinline__ bool stretch_run(Stretch& st, const B& batch, uint32_t ring, uint32_t bars,
                                            RingState& rs, XSrc&& xsrc, RWait&& r_ready = RWait{}) {
    // LATE: the residual sums may still be in the making while the stretch
    // runs: an item reads them as soon as a poll between its quads finds them
    // published, else at its end after r_ready() has waited for them
    constexpr bool LATE = !std::is_same<std::decay_t<RWait>, RReady>::value;
    constexpr uint32_t kQuad = Ring<NS>::kQuad;
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    if (st.u_first >= st.u_hi) return true;
    const uint32_t lane_base = NS == 26 ? (kLat26Xor | (4u * lane)) : (kLat16Base + 4u * lane);
    const uint32_t sig_base = kSigAddr;
    const int xrow = g < M ? g : 0;  // batch rows >= M: their mma columns are never stored

    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t c_slot = rs.slot, c_phase = rs.phase;
    bool failed = false;
    // the current job's fields, held in registers (reloaded when the cursor
    // enters the next job), and the current item's first unit (items are
    // consecutive in the unit sequence, so it advances by the item's units)
    int jk = -1, kg = 1, kp = 1, r16 = 1, cols = 0;
    bool odd_kt = false;
    const uint16_t* jx = nullptr;
    float* jpart = nullptr;
    int ustart = st.u_first;
    Cursor cur = st.cur;
    const int u_lo = st.u_lo, u_hi = st.u_hi, grp_first = st.grp_first;
    auto refill = [&]() { stretch_produce<NS>(st, batch, c_slot, ring, bars); };
    while (ustart < u_hi) {
        if (cur.j != jk) {
            const GemvJob& J = batch.jobs[cur.j];
            jk = cur.j;
            kg = J.kg;
            kp = J.kp;
            r16 = J.r16;
            cols = J.cols;
            odd_kt = (J.kt & 1) != 0;
            jx = J.x;
            jpart = J.partial;
        }
        const int cp0 = 16 * cur.grp;
        const int n_units = min(16, kp - cp0);
        // a phantom second tile (odd tile count) sits in the row block's last unit
        const bool phantom_item = odd_kt && cp0 + n_units == kp;
        const X xp = xsrc(jx).at((int64_t)xrow * cols + 64 * cp0 + 16 * c);

        // the group's residual sums of rows g and g + 8 (batch columns 2c, 2c + 1),
        // from the pre-pass: in flight while the quads stream
        const int64_t rpad = (int64_t)r16 * 16;
        float R[4] = {0.f, 0.f, 0.f, 0.f};
        auto load_r = [&]() {
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int jj = 0; jj < 2; ++jj)
                    if (2 * c + jj < M)
                        R[2 * h + jj] = __ldcg(jpart + ((int64_t)(2 * c + jj) * kg + cur.grp) * rpad +
                                               cur.b16 * 16 + g + 8 * h);
        };
        bool r_have = !LATE;
        if (!LATE) load_r();
        auto poll_r = [&]() {
            if constexpr (LATE) {
                if (!r_have && r_ready.poll()) {
                    r_have = true;
                    load_r();
                }
            }
        };

        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const int nq = (n_units + 3) >> 2;
        const int nfull = phantom_item ? 0 : (n_units >> 2);
        int q0 = 0;
        for (; q0 < nfull; ++q0) {  // full quads: no per-quad dispatch
            if (!mbar_wait(bars + 8 * c_slot, c_phase)) {
                failed = true;
                break;
            }
            quad_step<NS, 4, false>(ring + c_slot * kQuad, lane, c, xp.at(256 * q0), -1, lane_base, sig_base, d,
                                    refill);
            c_slot ^= 1u;
            c_phase ^= c_slot == 0 ? 1u : 0u;
            poll_r();
        }
        if (failed) break;
        for (int q = q0; q < nq; ++q) {  // the short last quad, or every quad of a phantom item
            if (!mbar_wait(bars + 8 * c_slot, c_phase)) {
                failed = true;
                break;
            }
            const uint32_t slot = ring + c_slot * kQuad;
            const int uq = min(4, n_units - 4 * q);
            const X xq = xp.at(256 * q);
            if (!phantom_item) {
                if (uq == 4) quad_step<NS, 4, false>(slot, lane, c, xq, -1, lane_base, sig_base, d, refill);
                else if (uq == 2) quad_step<NS, 2, false>(slot, lane, c, xq, -1, lane_base, sig_base, d, refill);
                else if (uq == 3) quad_step<NS, 3, false>(slot, lane, c, xq, -1, lane_base, sig_base, d, refill);
                else quad_step<NS, 1, false>(slot, lane, c, xq, -1, lane_base, sig_base, d, refill);
            } else {
                // the phantom tile is in the item's last unit, so in its last quad
                const int ph = q == nq - 1 ? uq - 1 : -1;
                if (uq == 4) quad_step<NS, 4, true>(slot, lane, c, xq, ph, lane_base, sig_base, d, refill);
                else if (uq == 2) quad_step<NS, 2, true>(slot, lane, c, xq, ph, lane_base, sig_base, d, refill);
                else if (uq == 3) quad_step<NS, 3, true>(slot, lane, c, xq, ph, lane_base, sig_base, d, refill);
                else quad_step<NS, 1, true>(slot, lane, c, xq, ph, lane_base, sig_base, d, refill);
            }
            c_slot ^= 1u;
            c_phase ^= c_slot == 0 ? 1u : 0u;
        }
        if (failed) break;

        if (LATE && !r_have) {
            if (!r_ready()) {
                failed = true;
                break;
            }
            load_r();
        }
        // (row g + 8h, batch column 2c + j) of this lane's mma fragment: e = 2h + j
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = d[e] + R[e];

        const int rb0 = ustart - cp0;  // first unit of the row block
        const int grp = cur.grp, b16 = cur.b16;
        const bool last_grp = grp == kg - 1;
        ustart += n_units;
        const bool has_next = ustart < u_hi;
        const bool cut = kg > 1 && (rb0 < u_lo || rb0 + 16 * (kg - 1) >= u_hi);
        const GemvJob& J = batch.jobs[jk];
        if (!cut) {
#pragma unroll
            for (int e = 0; e < 4; ++e) tot[e] += v[e];
            if (last_grp) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = b16 * 16 + g + 8 * h;
#pragma unroll
                    for (int jj = 0; jj < 2; ++jj)
                        if (row < J.rows && 2 * c + jj < M) store_out(J, 2 * c + jj, row, tot[2 * h + jj]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) tot[e] = 0.f;
            }
        } else {
            cut_group<M>(J, b16, grp, v, last_grp || !has_next, grp - (rb0 < u_lo ? grp_first : 0) + 1, g, c,
                         lane);
        }
        if (++cur.grp == kg) {
            cur.grp = 0;
            if (++cur.b16 == r16) {
                cur.b16 = 0;
                ++cur.j;
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
    rs.slot = c_slot;
    rs.phase = c_phase;
    return !failed;
}

// One warp's stretch [u_lo, u_hi) of `batch` in one go: open it, run
// `after_issue` once the first two copies are in flight (before any
// activation or workspace read: the standalone kernel's programmatic-
// dependency wait), then run it.
template <int NS, int M, class X, class B, class XSrc, class AfterIssue>
__device__ __forceinline__ bool stream_warp(const B& batch, int u_lo, int u_hi, uint32_t ring, uint32_t bars,
                                            RingState& rs, XSrc&& xsrc, AfterIssue&& after_issue) {
    Stretch st = stretch_open<NS>(batch, u_lo, u_hi, ring, bars, rs, false);
    after_issue();
    return stretch_run<NS, M, X>(st, batch, ring, bars, rs, xsrc);
}

template <int NS, int M, int MAXJ>
__global__ void __launch_bounds__(kSThreads, 1)
stream_kernel(const __grid_constant__ GemvBatch<MAXJ> batch) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
    if (s0 > kLowStage || s0 + kSmemBytes < Ring<NS>::kTop) {
        if (threadIdx.x == 0) atomicExch(&g_gemv_error, 1);
        return;
    }
    build_tables<NS>(smem - s0);  // smem - s0: generic pointer of shared address 0
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ring = ring_of<NS>(warp);
    const uint32_t bars = kBarAddr + warp * kSlots * 8;
    if (lane == 0) {
        for (int k = 0; k < kSlots; ++k) mbar_init(bars + 8 * k);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // this warp's stretch of the unit sequence
    const int64_t U = batch.total_units;
    const int64_t nw = (int64_t)gridDim.x * kSWarps;
    const int64_t gw = (int64_t)blockIdx.x * kSWarps + warp;
    RingState rs{0u, 0u};
    // The residual pre-pass is this launch's programmatic predecessor: the
    // table set-up and the first copies overlap it; its sums (and the
    // workspace it shares with the cut row blocks) are read only after it has
    // completed (a no-op when the launch has no such predecessor).
    (void)stream_warp<NS, M, XGlobal>(
        batch, (int)stretch_bound(U, gw, nw), (int)stretch_bound(U, gw + 1, nw), ring, bars, rs,
        [](const uint16_t* x) { return XGlobal{x}; }, []() { pdl_wait(); });
}

// Two launches: the residual pre-pass, then the streaming kernel (the jobs'
// unit offsets laid out on the host; one CTA per SM at most, none beyond the
// number of work items).
template <int NS, int M, int MAXJ>
cudaError_t launch(const GemvBatch<MAXJ>& b, cudaStream_t stream, int num_sms) {
    auto kern = stream_kernel<NS, M, MAXJ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    GemvBatch<MAXJ> sb = b;
    int64_t units = 0, items = 0;
    for (int j = 0; j < b.n; ++j) {
        sb.jobs[j].unit_begin = units;
        units += (int64_t)b.jobs[j].r16 * b.jobs[j].kp;
        items += (int64_t)b.jobs[j].r16 * b.jobs[j].kg;
    }
    if (units >= INT32_MAX) return cudaErrorInvalidValue;
    sb.total_units = units;
    e = launch_res(b, M, stream);
    if (e != cudaSuccess) return e;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, num_sms));
    // programmatic dependent launch: the kernel starts while the pre-pass runs
    return launch_pdl(kern, dim3(grid), dim3(kSThreads), kSmemBytes, stream, sb);
}

}  // namespace stream
