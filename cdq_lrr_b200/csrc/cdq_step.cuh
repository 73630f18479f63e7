// The persistent decode step: one cooperative launch runs a whole batch-1
// token of a Qwen2-style decoder (every layer's norms, CDQ projections,
// attention and MLP, then the lm_head with its argmax and the token advance),
// with grid-wide barriers between the steps that depend on one another, so
// no launch latency, no prologue and no pair-table build is paid per
// operation. Included by cdq_gemv.cu (it runs the streaming kernel's per-warp
// stretch code, stretch_open and stretch_run, on every projection group).
//
// Per layer, every CTA:
//   A  h' = h + down (layer 0: the embedding row), x = RMSNorm(h') into its own
//      shared memory (CTA 0 also writes h' to the other hidden buffer), the
//      residual sums of its q/k/v items from that x, then its q/k/v stretches
//      (activations from shared memory)                         -> barrier
//   B  CTAs 0 .. heads-1: rotary embedding, cache append and attention of
//      one query head                                           -> barrier
//   C  x = the attention output, residual sums and o_proj       -> barrier
//   D  h'' = h' + o, x = RMSNorm(h''), gate/up                  -> barrier
//   E  x = SiLU(gate) * up, down_proj                           -> barrier
// then RMSNorm of h'' + down, the lm_head rows of every warp with their argmax
// keys (atomicMax), a barrier, and CTA 0 turns the key into the next token.
// Every operation uses the same device functions and arithmetic as the
// one-kernel-per-operation step (cdq_decode_math.cuh, the stretch code, the
// residual pre-pass's per-bucket sums), so the two steps give the same bits.
//
// The barrier: thread 0 of each CTA adds an arrival to a monotonic counter
// and polls it until every CTA has arrived (bounded; on timeout the error word
// is set and every CTA leaves at its next barrier). After a projection step a
// CTA arrives first, then opens the next projection group (descriptors,
// residual stage, first weight copies), then waits: the opening overlaps the
// wait for the slowest CTA instead of delaying this CTA's arrival.
// The cooperative launch guarantees that all CTAs are resident, one per SM.

namespace step {

using namespace stream;

constexpr uint32_t kBarrierPolls = 1u << 22;

// The scratch region of the shared window (offsets from its start): the
// attention scratch, the norm's warp partials, the barrier flag, then copies
// of the step's parameters and two buffers of a projection group's
// descriptor with this CTA's stage descriptor: the group being run and the
// next one, fetched while this one runs (read many times per group: shared
// memory instead of L2 round trips).
constexpr uint32_t al16(uint32_t b) { return (b + 15u) / 16u * 16u; }
constexpr uint32_t kScrRed = al16(sizeof(dm::AttnScratch));
constexpr uint32_t kScrFlag = kScrRed + 16 * 4;
constexpr uint32_t kScrParams = al16(kScrFlag + 16);
constexpr uint32_t kScrGroupBuf = al16(sizeof(StepGroup) + sizeof(StepStage));  // a group and its stage
constexpr uint32_t kScrGroup = al16(kScrParams + sizeof(StepParams));            // two such buffers
constexpr uint32_t kScrSync = kScrGroup + 2 * kScrGroupBuf;
constexpr uint32_t kScrBytes = al16(kScrSync + 32);
static_assert(sizeof(StepParams) % 16 == 0 && sizeof(StepGroup) % 16 == 0 && sizeof(StepStage) % 16 == 0,
              "shared copies go in 16-byte words");

// Copies n bytes (a multiple of 16, both 16-byte aligned) from global to
// shared memory with the CTA's threads; the caller synchronises.
__device__ __forceinline__ void copy_to_shared(void* dst, const void* src, uint32_t n) {
    for (uint32_t i = threadIdx.x; i < n / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Sync words of the step's table (32-bit word offsets).
constexpr int kSyncArrivals = 0;  // u64: barrier arrivals, monotonic over launches
constexpr int kSyncLaunches = 2;  // u64: completed launches
constexpr int kSyncError = 4;     // u32: the sticky error code

// The grid barrier: thread 0 of every CTA adds one arrival to a monotonic
// counter and waits until it reaches `target` (this barrier's count: every
// CTA of every earlier barrier of every earlier launch), so no reset and no
// second word are needed. false: the barrier gave up (or found the error word
// set by a CTA that failed while it waited):
// the caller leaves. ok_s: a word of the CTA's shared window (no static
// shared memory: the streaming layout needs the dynamic window at the start
// of the CTA's).
// It comes in two halves: grid_arrive (the CTA's writes are done and its
// arrival counted) and grid_wait; work between them must not read anything
// another CTA wrote before the barrier (the step opens its next projection
// group there, which reads only weights and descriptors).
__device__ __forceinline__ void grid_arrive(uint32_t* sync) {
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_acq_rel_gpu();  // release: the CTA's writes before its arrival
        atomicAdd(reinterpret_cast<unsigned long long*>(sync + kSyncArrivals), 1ull);
    }
}

__device__ __forceinline__ bool grid_wait(uint32_t* sync, unsigned long long target, volatile uint32_t& ok_s) {
    if (threadIdx.x == 0) {
        uint32_t ok = 1u;
        auto* arrivals = reinterpret_cast<unsigned long long*>(sync + kSyncArrivals);
        uint32_t polls = 0;
        while (ld_acquire64(arrivals) < target) {
            if (++polls >= kBarrierPolls) {
                atomicExch(sync + kSyncError, 1u);
                ok = 0u;
                break;
            }
            if ((polls & 255u) == 0u) {
                if (ld_acquire(sync + kSyncError) != 0u) {  // another CTA gave up
                    ok = 0u;
                    break;
                }
                __nanosleep(64);
            }
        }
        // Reaching the target needs no second look at the error word: a CTA
        // that fails leaves without arriving, so the barrier after its
        // failure never completes and the others find the error in their
        // polls. The acquire load that saw the target orders this CTA's later
        // reads (through the CTA barrier below) after every arrival's writes.
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0u;
}

__device__ __forceinline__ bool grid_barrier(uint32_t* sync, unsigned long long target, volatile uint32_t& ok_s) {
    grid_arrive(sync);
    return grid_wait(sync, target, ok_s);
}

// Residual sums of the items of `batch` whose first unit lies in
// [u_lo, u_hi) (this CTA's stretches), with the activation row x in shared
// memory: one thread per (item, row) bucket, each bucket's entries added in
// order (the residual pre-pass's arithmetic), into the workspace slots the
// items' warps read.
__device__ __forceinline__ void cta_residual_sums(const StepGroup& batch, int u_lo, int u_hi, const uint16_t* xs,
                                                  int tid, int nthreads) {
    const Cursor c0 = first_at(batch, u_lo), c1 = first_at(batch, u_hi);
    for (int j = c0.j; j <= c1.j && j < batch.n; ++j) {
        const GemvJob& J = batch.jobs[j];
        const int kg = J.kg, cols = J.cols;
        const int i_lo = j == c0.j ? c0.b16 * kg + c0.grp : 0;
        const int i_hi = j == c1.j ? c1.b16 * kg + c1.grp : J.r16 * kg;
        const uint32_t n_res = J.n_res;
        const int64_t rpad = (int64_t)J.r16 * 16;
        const uint32_t* __restrict__ rp = J.res_ptr;
        const uint32_t* __restrict__ re = J.res_ent;
        for (int e = tid; e < (i_hi - i_lo) * 16; e += nthreads) {
            const int it = i_lo + (e >> 4), ri = e & 15;
            const int b16 = it / kg, grp = it - b16 * kg;
            const int row = b16 * 16 + ri;
            const int64_t bucket = (int64_t)row * kg + grp;
            const uint32_t s = min(__ldg(rp + bucket), n_res);
            const uint32_t t = min(max(__ldg(rp + bucket + 1), s), n_res);
            float acc = 0.f;
            for (uint32_t k0 = s; k0 < t; k0 += 8) {  // eight loads in flight, then the fmas in order
                uint32_t en[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) en[i] = k0 + i < t ? __ldg(re + k0 + i) : 0xFFFF0000u;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t col = en[i] >> 16;
                    if (k0 + i < t && col < (uint32_t)cols)
                        acc = fmaf(__uint_as_float(en[i] << 16), __uint_as_float((uint32_t)xs[col] << 16), acc);
                }
            }
            J.partial[(int64_t)grp * rpad + row] = acc;
        }
    }
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Issues this CTA's residual stage copies for a group (every thread; one
// cp.async group per thread, waited for in run_group).
__device__ __forceinline__ void stage_issue(const StepStage& d, const StepGroup& G, const StepParams& P) {
    if (d.ok) {
        uint32_t bo = P.rst_addr, eo = P.rst_addr + 4u * (uint32_t)P.rst_bnd_cap;
        for (int k = 0; k < d.n; ++k) {
            const GemvJob& J = G.jobs[k];
            for (int i = threadIdx.x; i < d.nb[k]; i += kSThreads) cp_async4(bo + 4u * i, J.res_ptr + d.b0[k] + i);
            for (int i = threadIdx.x; i < d.ne[k]; i += kSThreads) cp_async4(eo + 4u * i, J.res_ent + d.e0[k] + i);
            bo += 4u * (uint32_t)d.nb[k];
            eo += 4u * (uint32_t)d.ne[k];
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// cta_residual_sums from the staged bounds and entries (the same buckets, the
// same order of fmas).
__device__ __forceinline__ void cta_residual_sums_staged(const StepGroup& batch, const StepStage& d, int u_lo,
                                                         int u_hi, const uint16_t* xs, const uint32_t* bnd,
                                                         const uint32_t* ent, int tid, int nthreads) {
    const Cursor c0 = first_at(batch, u_lo), c1 = first_at(batch, u_hi);
    int bo = 0, eo = 0;
    for (int j = 0; j < batch.n; ++j) {
        const GemvJob& J = batch.jobs[j];
        if (j >= c0.j && j <= c1.j) {
            const int kg = J.kg, cols = J.cols;
            const int i_lo = j == c0.j ? c0.b16 * kg + c0.grp : 0;
            const int i_hi = j == c1.j ? c1.b16 * kg + c1.grp : J.r16 * kg;
            const int64_t rpad = (int64_t)J.r16 * 16;
            const uint32_t e0 = (uint32_t)d.e0[j], e1 = e0 + (uint32_t)d.ne[j];
            for (int e = tid; e < (i_hi - i_lo) * 16; e += nthreads) {
                const int it = i_lo + (e >> 4), ri = e & 15;
                const int b16 = it / kg, grp = it - b16 * kg;
                const int row = b16 * 16 + ri;
                const int bl = row * kg + grp - d.b0[j];  // the bucket in the stage
                const uint32_t s = min(max(bnd[bo + bl], e0), e1);
                const uint32_t t = min(max(bnd[bo + bl + 1], s), e1);
                float acc = 0.f;
                for (uint32_t k = s; k < t; ++k) {
                    const uint32_t en = ent[eo + (k - e0)], col = en >> 16;
                    if (col < (uint32_t)cols)
                        acc = fmaf(__uint_as_float(en << 16), __uint_as_float((uint32_t)xs[col] << 16), acc);
                }
                J.partial[(int64_t)grp * rpad + row] = acc;
            }
        }
        bo += d.nb[j];
        eo += d.ne[j];
    }
}

// Projection group (l, gi) of the table and this CTA's stage descriptor for it.
__device__ __forceinline__ const StepGroup* group_of(const StepParams& P, int l, int gi) {
    return &P.layer[l].qkv + gi;  // qkv, o, gu, down are consecutive
}
__device__ __forceinline__ const StepStage* stage_of(const StepParams& P, int l, int gi) {
    return &P.stage[((int64_t)l * 4 + gi) * P.n_ctas + blockIdx.x];
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// Issues the copies of group (l, gi)'s descriptors into the shared buffer at
// `dst` (every thread; one cp.async group per thread, waited for with the
// stage copies in run_group).
__device__ __forceinline__ void fetch_group(const StepParams& P, int l, int gi, uint32_t dst) {
    const uint4* g = reinterpret_cast<const uint4*>(group_of(P, l, gi));
    const uint4* d = reinterpret_cast<const uint4*>(stage_of(P, l, gi));
    for (uint32_t i = threadIdx.x; i < sizeof(StepGroup) / 16; i += blockDim.x) cp_async16(dst + 16 * i, g + i);
    for (uint32_t i = threadIdx.x; i < sizeof(StepStage) / 16; i += blockDim.x)
        cp_async16(dst + sizeof(StepGroup) + 16 * i, d + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// A warp's stretch of a projection group: opened (first two weight copies
// issued, the rest of its weights prefetched into L2) before the barrier that
// precedes the group, so those copies fly during the barrier and the steps
// before the group. G, D: the group's descriptors, already in shared memory
// (fetched while the previous group ran); the next group's are fetched into
// the other buffer (next_buf) now.
template <int NS>
__device__ __forceinline__ Stretch open_group(const StepParams& P, int l, int gi, uint32_t ring, uint32_t bars,
                                              const RingState& rs, const StepGroup& G, const StepStage& D,
                                              uint32_t next_buf) {
    const int nl = gi == 3 ? l + 1 : l, ngi = gi == 3 ? 0 : gi + 1;
    if (nl < P.layers) fetch_group(P, nl, ngi, next_buf);
    stage_issue(D, G, P);
    const int64_t U = G.total_units;
    const int64_t nw = (int64_t)gridDim.x * kSWarps;
    const int64_t gw = (int64_t)blockIdx.x * kSWarps + (threadIdx.x >> 5);
    return stretch_open<NS>(G, (int)stretch_bound(U, gw, nw), (int)stretch_bound(U, gw + 1, nw), ring, bars, rs,
                            true);
}

// Shared words of run_group: a byte per warp (it has items) and the flag that
// publishes the group's residual sums.
struct GroupSync {
    uint8_t busy[kSWarps];
    uint32_t r_flag;
};

// stretch_run's residual-sum wait in run_group: the group's sums are
// published all at once, by the flag taking the group's token. The writers
// are warps of this CTA that fence at GPU scope before the flag is set, so a
// reader that has seen the flag needs only CTA-scope ordering before its
// loads of the sums (a GPU-scope fence here cost about a microsecond).
struct RToken {
    const uint32_t* flag;
    uint32_t token;
    __device__ __forceinline__ bool poll() const {
        if (*reinterpret_cast<const volatile uint32_t*>(flag) != token) return false;
        __threadfence_block();
        return true;
    }
    __device__ __forceinline__ bool operator()() const {
        const volatile uint32_t* f = flag;
        for (uint32_t polls = 0; *f != token; ++polls) {
            if (polls >= kBarrierPolls) return false;
            if (polls > 64) __nanosleep(32);
        }
        __threadfence_block();
        return true;
    }
};

// Runs an opened projection group: the CTA builds the group's input in shared
// memory (`prep`, every thread, CTA barriers allowed), then the warps that
// have items start streaming while the others compute this CTA's residual
// sums; an item's warp reads them once a poll between its quads finds the
// flag `token` set (a bounded wait at the item's end at the latest). Without
// idle warps everyone sums first. CTA-uniform result.
template <int NS, class Prep>
__device__ __forceinline__ bool run_group(Stretch& st, const StepGroup& G, const StepStage& d, const uint16_t* xs,
                                          uint32_t xs_addr, const uint32_t* bnd, const uint32_t* ent, uint32_t ring,
                                          uint32_t bars, RingState& rs, GroupSync& gs, uint32_t token,
                                          Prep&& prep) {
    const int64_t U = G.total_units;
    const int64_t nw = (int64_t)gridDim.x * kSWarps;
    const int64_t cta0 = (int64_t)blockIdx.x * kSWarps;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool has = st.u_first < st.u_hi;
    prep();
    asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's stage copies
    if (lane == 0) gs.busy[warp] = has ? 1 : 0;
    __syncthreads();  // everyone's stage copies and busy bytes
    uint32_t mask = 0;
#pragma unroll
    for (int w = 0; w < kSWarps; ++w) mask |= (uint32_t)gs.busy[w] << w;
    const int n_busy = __popc(mask);
    const int lo = (int)stretch_bound(U, cta0, nw), hi = (int)stretch_bound(U, cta0 + kSWarps, nw);
    auto sums = [&](int tid, int nthreads) {
        if (d.ok) cta_residual_sums_staged(G, d, lo, hi, xs, bnd, ent, tid, nthreads);
        else cta_residual_sums(G, lo, hi, xs, tid, nthreads);
    };
    if (n_busy == kSWarps) {  // no idle warp: sum first
        sums(threadIdx.x, kSThreads);
        fence_acq_rel_gpu();  // release: the sums before the flag
        __syncthreads();
        if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(&gs.r_flag) = token;
        __syncthreads();
    } else if (!has) {  // an idle warp: its share of the sums, then the flag
        const int rank = __popc(~mask & ((1u << warp) - 1u)), n_idle = kSWarps - n_busy;
        sums(rank * 32 + lane, n_idle * 32);
        fence_acq_rel_gpu();  // release: the sums before the flag
        asm volatile("bar.sync 1, %0;" ::"r"(n_idle * 32) : "memory");
        if (rank == 0 && lane == 0) *reinterpret_cast<volatile uint32_t*>(&gs.r_flag) = token;
    }
    bool ok = true;
    if (has) {
        ok = stretch_run<NS, 1, XShared>(st, G, ring, bars, rs,
                                         [xs_addr](const uint16_t*) { return XShared{xs_addr}; },
                                         RToken{&gs.r_flag, token});
    }
    return __syncthreads_and(ok) != 0;
}

// x = RMSNorm(h_in (+ delta)) with weight w into xs (shared, bf16), threads
// 0 .. 255 in the one-kernel step's order; h_out (CTA 0 only) receives the
// residual sum. emb: the embedding row instead of h_in + delta (layer 0).
__device__ __forceinline__ void norm_into(const uint16_t* h_in, const uint16_t* delta, const uint16_t* emb,
                                          bool emb_ok, const uint16_t* w, float eps, int n, uint16_t* h_out,
                                          uint16_t* xs, float* red) {
    using namespace dm;
    constexpr int kKeep = 4;  // weights of the first kKeep strides held from the first pass
    const int tid = threadIdx.x;
    float ss = 0.f;
    uint16_t wk[kKeep];
    if (tid < kNormThreads) {
        // kKeep strides at a time: every load of a batch issued before its stores
        for (int i0 = tid; i0 < n; i0 += kKeep * kNormThreads) {
            uint16_t a[kKeep], b[kKeep];
#pragma unroll
            for (int k = 0; k < kKeep; ++k) {
                const int i = i0 + k * kNormThreads;
                a[k] = i < n ? (emb ? (emb_ok ? emb[i] : (uint16_t)0) : h_in[i]) : (uint16_t)0;
                b[k] = i < n && !emb ? delta[i] : (uint16_t)0;
                if (i0 == tid) wk[k] = i < n ? w[i] : (uint16_t)0;
            }
#pragma unroll
            for (int k = 0; k < kKeep; ++k) {
                const int i = i0 + k * kNormThreads;
                if (i < n) {
                    const uint16_t hv = emb ? a[k] : add_bf(a[k], b[k]);
                    xs[i] = hv;
                    if (h_out) h_out[i] = hv;
                    ss = fmaf(bf(hv), bf(hv), ss);
                }
            }
        }
    }
    const float r = norm_scale(norm_total(ss, red), n, eps);
    if (tid < kNormThreads) {
#pragma unroll
        for (int k = 0; k < kKeep; ++k)
            if (tid + k * kNormThreads < n) xs[tid + k * kNormThreads] = norm_out(wk[k], xs[tid + k * kNormThreads], r);
        for (int i = tid + kKeep * kNormThreads; i < n; i += kNormThreads) xs[i] = norm_out(w[i], xs[i], r);
    }
    __syncthreads();
}

// A projection group succeeded in every warp of the CTA (CTA-uniform, so the
// CTA leaves the layer loop as a whole).
__device__ __forceinline__ bool group_ok(bool warp_ok) { return __syncthreads_and(warp_ok) != 0; }

template <int NS>
__global__ void __launch_bounds__(kSThreads, 1) decode_step_kernel(const StepParams* __restrict__ params) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const StepParams& Pg = *params;
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
    if (s0 > kLowStage || s0 + kSmemBytes < Ring<NS>::kTop) {
        if (threadIdx.x == 0) atomicExch(&g_gemv_error, 1);
        return;
    }
    if (Pg.n_states != NS) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(Pg.sync + kSyncError, 3u);
        return;
    }
    if (ld_acquire(Pg.sync + kSyncError) != 0u) return;  // an earlier step failed: reset first
    if ((int)gridDim.x != Pg.n_ctas) {           // the stage descriptors are per CTA
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(Pg.sync + kSyncError, 4u);
        return;
    }
    uint8_t* const base = smem - s0;  // generic pointer of shared address 0
    StepParams& P = *reinterpret_cast<StepParams*>(base + Pg.scr_addr + kScrParams);
    copy_to_shared(&P, &Pg, sizeof(StepParams));
    build_tables<NS>(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ring = ring_of<NS>(warp);
    const uint32_t bars = kBarAddr + warp * kSlots * 8;
    if (lane == 0) {
        for (int k = 0; k < kSlots; ++k) mbar_init(bars + 8 * k);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    uint16_t* const xs = reinterpret_cast<uint16_t*>(base + Pg.xs_addr);
    float* const xf = reinterpret_cast<float*>(base + Pg.xf_addr);
    float* const scores = reinterpret_cast<float*>(base + Pg.sc_addr);
    dm::AttnScratch& S = *reinterpret_cast<dm::AttnScratch*>(base + Pg.scr_addr);
    float* const red = reinterpret_cast<float*>(base + Pg.scr_addr + kScrRed);
    volatile uint32_t& bar_ok = *reinterpret_cast<volatile uint32_t*>(base + Pg.scr_addr + kScrFlag);
    const uint32_t gbuf0 = Pg.scr_addr + kScrGroup;  // shared addresses of the two group buffers
    GroupSync& gsync = *reinterpret_cast<GroupSync*>(base + Pg.scr_addr + kScrSync);
    if (threadIdx.x == 0) gsync.r_flag = 0u;  // tokens of this launch start at 1
    copy_to_shared(base + gbuf0, group_of(Pg, 0, 0), sizeof(StepGroup));  // the first group's descriptors
    copy_to_shared(base + gbuf0 + sizeof(StepGroup), stage_of(Pg, 0, 0), sizeof(StepStage));
    const uint32_t* const bnd = reinterpret_cast<const uint32_t*>(base + Pg.rst_addr);
    const uint32_t* const ent = reinterpret_cast<const uint32_t*>(base + Pg.rst_addr + 4u * (uint32_t)Pg.rst_bnd_cap);
    __syncthreads();

    const uint32_t n_ctas = gridDim.x;
    const int H = P.hidden, I = P.inter;
    const int pos = *P.pos;
    const bool pos_ok = pos >= 0 && pos < P.max_len;
    const int64_t id = *P.ids;
    RingState rs{0u, 0u};
    bool ok = true;
    // this launch's barriers: 5 per layer and the final one, n_ctas arrivals each
    unsigned long long target = 0ull;
    if (threadIdx.x == 0) {
        const unsigned long long launches =
            ld_acquire64(reinterpret_cast<const unsigned long long*>(P.sync + kSyncLaunches));
        target = (launches * (unsigned long long)(5 * P.layers + 1) + 1ull) * n_ctas;
    }
    auto arrive = [&]() { grid_arrive(P.sync); };
    auto wait = [&]() {
        const bool b = grid_wait(P.sync, target, bar_ok);
        target += n_ctas;
        return b;
    };
    auto barrier = [&]() {
        arrive();
        return wait();
    };
    // the group descriptors in use alternate between the two shared buffers:
    // a group's are fetched while the group before it runs
    int cur = 1;
    auto Gs = [&]() -> const StepGroup& { return *reinterpret_cast<const StepGroup*>(base + gbuf0 + cur * kScrGroupBuf); };
    auto Ds = [&]() -> const StepStage& {
        return *reinterpret_cast<const StepStage*>(base + gbuf0 + cur * kScrGroupBuf + sizeof(StepGroup));
    };
    auto open = [&](int l, int gi) {
        cur ^= 1;
        return open_group<NS>(P, l, gi, ring, bars, rs, Gs(), Ds(), gbuf0 + (cur ^ 1) * kScrGroupBuf);
    };
    Stretch st = open(0, 0);
    bool live = true;  // st holds copies in flight
    for (int l = 0; l < P.layers; ++l) {
        const StepLayer& L = P.layer[l];
        // the cache rows 0 .. pos-1 that step B reads, asked of L2 now (the
        // first block of each kv head's query group), so that the attention's
        // key and value loads do not wait on HBM
        if (pos_ok && pos > 0 && threadIdx.x == 0 && (int)blockIdx.x < P.heads &&
            (int)blockIdx.x % (P.heads / P.kv_heads) == 0) {
            const int64_t off = (int64_t)((int)blockIdx.x / (P.heads / P.kv_heads)) * P.max_len * dm::kHd;
            const uint32_t bytes = (uint32_t)pos * dm::kHd * 2u;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(L.kc + off), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(L.vc + off), "r"(bytes) : "memory");
        }
        // A: x = RMSNorm(h + down) (layer 0: the embedding row); q, k, v
        ok = run_group<NS>(st, Gs(), Ds(), xs, P.xs_addr, bnd, ent, ring,
                           bars, rs, gsync, 4u * l + 1u, [&]() {
            if (l == 0)
                norm_into(nullptr, nullptr, P.embed + (id >= 0 && id < P.vocab ? id : 0) * (int64_t)H,
                          id >= 0 && id < P.vocab, L.ln1, P.eps, H, blockIdx.x == 0 ? P.h[1] : nullptr, xs, red);
            else
                norm_into(P.h[0], P.dn, nullptr, false, L.ln1, P.eps, H, blockIdx.x == 0 ? P.h[1] : nullptr, xs,
                          red);
        });
        live = false;
        if (!ok) break;
        arrive();  // this group's outputs are written: the next group opens while the others finish
        st = open(l, 1);
        live = true;
        if (!wait()) break;
        // B: attention, one CTA per query head
        if ((int)blockIdx.x < P.heads && pos_ok)
            dm::attn_head(blockIdx.x, threadIdx.x, P.q, P.k, P.v, P.cos_t + (int64_t)pos * dm::kHd,
                          P.sin_t + (int64_t)pos * dm::kHd, pos, L.kc, L.vc, P.max_len, P.heads, P.kv_heads,
                          P.scale, P.att, scores, S);
        if (!barrier()) break;
        // C: o_proj of the attention output
        ok = run_group<NS>(st, Gs(), Ds(), xs, P.xs_addr, bnd, ent, ring,
                           bars, rs, gsync, 4u * l + 2u, [&]() {
            const uint16_t* ap = P.att;
            const int na = P.heads * dm::kHd;
            for (int i0 = threadIdx.x; i0 < na; i0 += 4 * kSThreads) {
                uint16_t a[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) a[k] = i0 + k * kSThreads < na ? ap[i0 + k * kSThreads] : (uint16_t)0;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (i0 + k * kSThreads < na) xs[i0 + k * kSThreads] = a[k];
            }
            __syncthreads();
        });
        live = false;
        if (!ok) break;
        arrive();  // this group's outputs are written: the next group opens while the others finish
        st = open(l, 2);
        live = true;
        if (!wait()) break;
        // D: x = RMSNorm(h' + o); gate, up
        ok = run_group<NS>(st, Gs(), Ds(), xs, P.xs_addr, bnd, ent, ring,
                           bars, rs, gsync, 4u * l + 3u, [&]() {
            norm_into(P.h[1], P.o, nullptr, false, L.ln2, P.eps, H, blockIdx.x == 0 ? P.h[0] : nullptr, xs, red);
        });
        live = false;
        if (!ok) break;
        arrive();  // this group's outputs are written: the next group opens while the others finish
        st = open(l, 3);
        live = true;
        if (!wait()) break;
        // E: x = SiLU(gate) * up; down
        ok = run_group<NS>(st, Gs(), Ds(), xs, P.xs_addr, bnd, ent, ring,
                           bars, rs, gsync, 4u * l + 4u, [&]() {
            const uint16_t* gp = P.g;
            const uint16_t* up = P.u;
            for (int i0 = threadIdx.x; i0 < I; i0 += 8 * kSThreads) {  // eight loads in flight per thread
                uint16_t a[8], b[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int i = i0 + k * kSThreads;
                    a[k] = i < I ? gp[i] : (uint16_t)0;
                    b[k] = i < I ? up[i] : (uint16_t)0;
                }
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (i0 + k * kSThreads < I) xs[i0 + k * kSThreads] = dm::silu_mul(a[k], b[k]);
            }
            __syncthreads();
        });
        live = false;
        if (!ok) break;
        arrive();
        if (l + 1 < P.layers) {
            st = open(l + 1, 0);
            live = true;
        }
        if (!wait()) break;
    }
    if (live) stretch_drain<NS>(st, bars, rs);  // left early with copies in flight
    asm volatile("cp.async.wait_all;" ::: "memory");  // a descriptor fetch still in flight (error paths)
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(P.sync + kSyncError, 2u);
        return;
    }
    if (ld_acquire(P.sync + kSyncError) != 0u) return;
    // the final norm of h'' + down, then this CTA's lm_head rows
    norm_into(P.h[0], P.dn, nullptr, false, P.norm_w, P.eps, H, nullptr, xs, red);
    for (int i = threadIdx.x; i < H; i += kSThreads) xf[i] = dm::bf(xs[i]);
    __syncthreads();
    unsigned long long key[1] = {0ull};
    const int64_t nwarps = (int64_t)n_ctas * kSWarps;
    for (int64_t r0 = ((int64_t)blockIdx.x * kSWarps + warp) * dm::kLmRows; r0 < P.vocab;
         r0 += nwarps * dm::kLmRows)
        dm::lm_rows<1, dm::kLmRows>(P.lm_w, xf, H, P.vocab, r0, lane, P.logits, key);
    if (lane == 0 && key[0]) atomicMax(P.best, key[0]);
    if (!barrier()) return;
    // the greedy token, recorded; the next step's input and position
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(reinterpret_cast<unsigned long long*>(P.sync + kSyncLaunches), 1ull);  // every CTA has passed
        const int64_t tok = dm::key_token(*P.best);
        *P.best = 0ull;
        *P.next = tok;
        const int c = *P.count;
        if (c < P.token_cap) P.tokens[c] = tok;
        *P.ids = tok;
        *P.pos = pos + 1;
        *P.count = c + 1;
    }
}

}  // namespace step
