// Batch-1 decode-step kernels around the fused CDQ linear, for a Qwen2-style
// decoder (the reference runs HF's Qwen2 layers around its CDQLinear:
// code/cdq_lrr_qwen05.py:300-330). Each kernel reproduces the rounding steps
// of the HF bf16 module it replaces:
//   add_rmsnorm  h = bf16(h + delta) (the residual add), then
//                out = bf16(w * bf16(h_f32 * rsqrt(mean(h_f32^2) + eps)))
//                (Qwen2RMSNorm);
//   attn_decode  rotary embedding of q and k at the step's position
//                (bf16(bf16(x * cos) + bf16(rotate_half(x) * sin))), append of
//                k and v to the static cache, and grouped-query attention over
//                positions 0..pos (fp32 scores, softmax and weighted sum, one
//                bf16 rounding of the output);
//   silu_mul     out = bf16(bf16(silu(g)) * u) (Qwen2MLP's act_fn(gate) * up);
//   embed_rmsnorm  h = embedding row of the step's token, then add_rmsnorm's
//                norm (the first layer's input norm);
//   lm_head_argmax  logits = bf16(x . w_row) for every vocabulary row (the tied
//                bf16 lm_head GEMV, fp32 accumulation) and their argmax (first
//                index among equal values, NaN above everything, torch.argmax's
//                rule) folded into one 64-bit key per step;
//   advance      the step's greedy token becomes the next step's input, is
//                recorded, and the position moves on, all on the device, so a
//                CUDA graph of the whole step replays without the host.
// Every kernel is launched programmatically dependent on its predecessor: it
// waits for the predecessor's completion before touching data, then lets its
// own successor be scheduled, so launch latencies overlap execution.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "cdq.h"
#include "cdq_decode_math.cuh"
#include "cdq_internal.cuh"

using cdq::launch_pdl;
using cdq::pdl_release;
using cdq::pdl_wait;
using namespace cdq::dm;

namespace {

// One block per row: row r of h / delta / out is the r-th vector of n values.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(uint16_t* __restrict__ h,
                                                                   const uint16_t* __restrict__ delta,
                                                                   const uint16_t* __restrict__ w, float eps,
                                                                   uint16_t* __restrict__ out, int n) {
    __shared__ float red[kNormThreads / 32];
    pdl_wait();
    pdl_release();
    const int64_t ro = (int64_t)blockIdx.x * n;
    h += ro;
    out += ro;
    if (delta) delta += ro;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += kNormThreads) {
        uint16_t hv = h[i];
        if (delta) {
            hv = add_bf(hv, delta[i]);
            h[i] = hv;
        }
        ss = fmaf(bf(hv), bf(hv), ss);
    }
    const float r = norm_scale(norm_total(ss, red), n, eps);
    for (int i = threadIdx.x; i < n; i += kNormThreads) out[i] = norm_out(w[i], h[i], r);
}

// One block per query head.
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
    const uint16_t* __restrict__ cos_t, const uint16_t* __restrict__ sin_t, const int32_t* __restrict__ pos_p,
    uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int max_len, int n_heads, int n_kv, float scale,
    uint16_t* __restrict__ out, int cap) {
    extern __shared__ float scores[];
    __shared__ AttnScratch S;
    pdl_wait();
    pdl_release();
    const int P = *pos_p;
    if (P < 0 || P >= max_len || P >= cap) return;  // the host sizes the cache; nothing to attend otherwise
    attn_head(blockIdx.x, threadIdx.x, q, k, v, cos_t + (int64_t)P * kHd, sin_t + (int64_t)P * kHd, P, kc, vc,
              max_len, n_heads, n_kv, scale, out, scores, S);
}

__global__ void silu_mul_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u,
                                uint16_t* __restrict__ out, int n) {
    pdl_wait();
    pdl_release();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = silu_mul(g[i], u[i]);
}

__global__ void advance_kernel(const int64_t* __restrict__ next, int64_t* __restrict__ ids,
                               int64_t* __restrict__ tokens, int32_t* __restrict__ pos, int32_t* __restrict__ count,
                               int cap) {
    pdl_wait();
    pdl_release();
    const int c = *count;
    if (c < cap) tokens[c] = *next;
    *ids = *next;
    *pos += 1;
    *count = c + 1;
}

__global__ void __launch_bounds__(kNormThreads) embed_rmsnorm_kernel(const int64_t* __restrict__ ids,
                                                                     const uint16_t* __restrict__ table,
                                                                     int64_t vocab, uint16_t* __restrict__ h,
                                                                     const uint16_t* __restrict__ w, float eps,
                                                                     uint16_t* __restrict__ out, int n) {
    __shared__ float red[kNormThreads / 32];
    pdl_wait();
    pdl_release();
    const int64_t ro = (int64_t)blockIdx.x * n;
    h += ro;
    out += ro;
    const int64_t id = ids[blockIdx.x];
    const bool ok = id >= 0 && id < vocab;  // an out-of-range id gives a zero row
    const uint16_t* row = table + (ok ? id : 0) * (int64_t)n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += kNormThreads) {
        const uint16_t v = ok ? row[i] : (uint16_t)0;
        h[i] = v;
        ss = fmaf(bf(v), bf(v), ss);
    }
    const float r = norm_scale(norm_total(ss, red), n, eps);
    for (int i = threadIdx.x; i < n; i += kNormThreads) out[i] = norm_out(w[i], h[i], r);
}

constexpr int kLmThreads = 256;

// For each of the M activation rows m: logits[m][r] = bf16(sum_k x[m][k] *
// w[r][k]) (fp32, lane-chunk order then a warp reduction: the same
// arithmetic for every M) and the row's argmax key (atomicMax into best[m],
// which the token kernel reads and clears). x is staged in shared memory as
// fp32.
template <int M>
__global__ void __launch_bounds__(kLmThreads) lm_head_argmax_kernel(const uint16_t* __restrict__ w,
                                                                    const uint16_t* __restrict__ x, int vocab,
                                                                    int n, uint16_t* __restrict__ logits,
                                                                    unsigned long long* __restrict__ best) {
    extern __shared__ float xs[];  // [M][n]
    pdl_wait();
    pdl_release();
    for (int i = threadIdx.x; i < M * n; i += kLmThreads) xs[i] = bf(x[i]);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t nw = (int64_t)gridDim.x * (kLmThreads / 32);
    unsigned long long key[M];
#pragma unroll
    for (int m = 0; m < M; ++m) key[m] = 0ull;
    constexpr int kRows = M == 1 ? kLmRows : 1;  // vocabulary rows per warp step
    for (int64_t r0 = ((int64_t)blockIdx.x * (kLmThreads / 32) + warp) * kRows; r0 < vocab; r0 += nw * kRows)
        lm_rows<M, kRows>(w, xs, n, vocab, r0, lane, logits, key);
#pragma unroll
    for (int m = 0; m < M; ++m)
        if (lane == 0 && key[m]) atomicMax(best + m, key[m]);
}

// The argmax keys -> the rows' tokens, then the keys are cleared for the next call.
__global__ void argmax_token_kernel(unsigned long long* __restrict__ best, int64_t* __restrict__ next, int m) {
    pdl_wait();
    pdl_release();
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
        next[i] = key_token(best[i]);
        best[i] = 0ull;
    }
}

// Speculative verification: the rotary embedding of the keys of n_q
// consecutive positions base..base+n_q-1 and their append (with the values)
// to the cache, one block per (kv head, position); the same arithmetic as the
// single-token kernel's append.
__global__ void __launch_bounds__(kHd) rope_append_kernel(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                                                          const uint16_t* __restrict__ cos_t,
                                                          const uint16_t* __restrict__ sin_t,
                                                          const int32_t* __restrict__ pos_p, uint16_t* __restrict__ kc,
                                                          uint16_t* __restrict__ vc, int max_len, int n_kv) {
    pdl_wait();
    pdl_release();
    const int kvh = blockIdx.x, qi = blockIdx.y, d = threadIdx.x;
    const int P = *pos_p + qi;
    if (P < 0 || P >= max_len) return;
    const uint16_t* kq = k + (int64_t)qi * n_kv * kHd;
    const uint16_t* vq = v + (int64_t)qi * n_kv * kHd;
    const uint16_t* cs = cos_t + (int64_t)P * kHd;
    const uint16_t* sn = sin_t + (int64_t)P * kHd;
    const int o = d < kHd / 2 ? d + kHd / 2 : d - kHd / 2;
    const float sgn = d < kHd / 2 ? -1.f : 1.f;
    const float kd = bf(kq[kvh * kHd + d]), ko = bf(kq[kvh * kHd + o]);
    kc[((int64_t)kvh * max_len + P) * kHd + d] = tobf(rbf(rbf(kd * bf(cs[d])) + rbf(sgn * ko * bf(sn[d]))));
    vc[((int64_t)kvh * max_len + P) * kHd + d] = vq[kvh * kHd + d];
}

// Speculative verification: attention of n_q consecutive query positions, one
// block per (head, position), each exactly the single-token kernel's
// attention at that position (its own key and value read back from the
// cache, where rope_append_kernel put the same bits the single-token kernel
// keeps in registers).
__global__ void __launch_bounds__(kAttnThreads) attn_multi_kernel(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ cos_t, const uint16_t* __restrict__ sin_t,
    const int32_t* __restrict__ pos_p, const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc, int max_len,
    int n_heads, int n_kv, float scale, uint16_t* __restrict__ out, int cap) {
    extern __shared__ float scores[];
    __shared__ AttnScratch S;
    const int h = blockIdx.x, qi = blockIdx.y, tid = threadIdx.x;
    pdl_wait();
    pdl_release();
    const int group = n_heads / n_kv, kvh = h / group;
    const int P = *pos_p + qi;
    if (P < 0 || P >= max_len || P >= cap) return;
    const uint16_t* kb = kc + (int64_t)kvh * max_len * kHd;
    const uint16_t* vb = vc + (int64_t)kvh * max_len * kHd;
    if (tid < kHd) {
        const int d = tid;
        S.qe[d] = rope(q + (int64_t)qi * n_heads * kHd + h * kHd, d, cos_t + (int64_t)P * kHd,
                       sin_t + (int64_t)P * kHd);
        // the position's own key and value, as rope_append_kernel stored them
        // (the same bits the single-token kernel keeps in registers)
        S.ke[d] = bf(kb[(int64_t)P * kHd + d]);
        S.ve[d] = bf(vb[(int64_t)P * kHd + d]);
    }
    __syncthreads();
    attn_core(tid, kb, vb, P, scale, out + (int64_t)qi * n_heads * kHd + h * kHd, scores, S);
}

}  // namespace

extern "C" {

cdq_status cdq_add_rmsnorm_rows(uint16_t* h, const uint16_t* delta, const uint16_t* w, float eps, uint16_t* out,
                                int32_t n, int32_t rows, void* stream) {
    if (!h || !w || !out || n < 1 || rows < 1 || rows > 65535) return CDQ_ERR_ARG;
    return launch_pdl(add_rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, (cudaStream_t)stream, h, delta, w, eps,
                      out, n) == cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

cdq_status cdq_add_rmsnorm(uint16_t* h, const uint16_t* delta, const uint16_t* w, float eps, uint16_t* out,
                           int32_t n, void* stream) {
    return cdq_add_rmsnorm_rows(h, delta, w, eps, out, n, 1, stream);
}

cdq_status cdq_attn_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* cos_t,
                           const uint16_t* sin_t, const int32_t* pos, uint16_t* k_cache, uint16_t* v_cache,
                           int32_t max_len, int32_t n_heads, int32_t n_kv, int32_t head_dim, float scale,
                           uint16_t* out, void* stream) {
    if (!q || !k || !v || !cos_t || !sin_t || !pos || !k_cache || !v_cache || !out) return CDQ_ERR_ARG;
    if (head_dim != kHd || n_kv < 1 || n_heads < n_kv || n_heads % n_kv || max_len < 1 || max_len > 16384)
        return CDQ_ERR_UNSUPPORTED;
    if ((uintptr_t)k_cache % 16 || (uintptr_t)v_cache % 16) return CDQ_ERR_ARG;
    const int smem = max_len * 4;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return CDQ_ERR_CUDA;
    return launch_pdl(attn_decode_kernel, dim3(n_heads), dim3(kAttnThreads), (size_t)smem, (cudaStream_t)stream, q,
                      k, v, cos_t, sin_t, pos, k_cache, v_cache, (int)max_len, (int)n_heads, (int)n_kv, scale, out,
                      (int)max_len) == cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

cdq_status cdq_silu_mul(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n, void* stream) {
    if (!g || !u || !out || n < 1 || n > ((int64_t)1 << 30)) return CDQ_ERR_ARG;
    const int blocks = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
    return launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), 0, (cudaStream_t)stream, g, u, out, (int)n) ==
                   cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

cdq_status cdq_decode_advance(const int64_t* next, int64_t* ids, int64_t* tokens, int32_t* pos, int32_t* count,
                              int32_t cap, void* stream) {
    if (!next || !ids || !tokens || !pos || !count || cap < 1) return CDQ_ERR_ARG;
    return launch_pdl(advance_kernel, dim3(1), dim3(1), 0, (cudaStream_t)stream, next, ids, tokens, pos, count,
                      (int)cap) == cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

cdq_status cdq_embed_rmsnorm_rows(const int64_t* ids, const uint16_t* table, int64_t vocab, uint16_t* h,
                                  const uint16_t* w, float eps, uint16_t* out, int32_t n, int32_t rows, void* stream) {
    if (!ids || !table || vocab < 1 || !h || !w || !out || n < 1 || rows < 1 || rows > 65535) return CDQ_ERR_ARG;
    return launch_pdl(embed_rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, (cudaStream_t)stream, ids, table, vocab,
                      h, w, eps, out, (int)n) == cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

cdq_status cdq_embed_rmsnorm(const int64_t* ids, const uint16_t* table, int64_t vocab, uint16_t* h,
                             const uint16_t* w, float eps, uint16_t* out, int32_t n, void* stream) {
    return cdq_embed_rmsnorm_rows(ids, table, vocab, h, w, eps, out, n, 1, stream);
}

cdq_status cdq_lm_head_argmax_rows(const uint16_t* w, const uint16_t* x, int32_t vocab, int32_t n, int32_t m,
                                   uint16_t* logits, uint64_t* best, int64_t* next, void* stream) {
    if (!w || !x || !best || !next || vocab < 1 || n < 8 || n % 8 || n > 16384 || m < 1 || m > 8)
        return CDQ_ERR_ARG;
    if ((uintptr_t)w % 16 || (uintptr_t)best % 8) return CDQ_ERR_ARG;
    int sms = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return CDQ_ERR_CUDA;
    const int64_t rows_per_block = (kLmThreads / 32) * (m == 1 ? kLmRows : 1);
    const int blocks = (int)std::min<int64_t>((vocab + rows_per_block - 1) / rows_per_block, (int64_t)sms * 8);
    const size_t smem = (size_t)m * n * 4;
    auto* best64 = reinterpret_cast<unsigned long long*>(best);
    cudaError_t e = cudaSuccess;
    switch (m) {
#define CDQ_LM_CASE(MM)                                                                                           \
    case MM:                                                                                                      \
        if (smem > 48 * 1024 && cudaFuncSetAttribute(lm_head_argmax_kernel<MM>,                                   \
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=   \
                                    cudaSuccess)                                                                  \
            return CDQ_ERR_CUDA;                                                                                  \
        e = launch_pdl(lm_head_argmax_kernel<MM>, dim3(blocks), dim3(kLmThreads), smem, (cudaStream_t)stream, w, x, \
                       (int)vocab, (int)n, logits, best64);                                                       \
        break;
        CDQ_LM_CASE(1)
        CDQ_LM_CASE(2)
        CDQ_LM_CASE(3)
        CDQ_LM_CASE(4)
        CDQ_LM_CASE(5)
        CDQ_LM_CASE(6)
        CDQ_LM_CASE(7)
        CDQ_LM_CASE(8)
#undef CDQ_LM_CASE
    }
    if (e != cudaSuccess) return CDQ_ERR_CUDA;
    return launch_pdl(argmax_token_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, best64, next, (int)m) ==
                   cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

cdq_status cdq_lm_head_argmax(const uint16_t* w, const uint16_t* x, int32_t vocab, int32_t n, uint16_t* logits,
                              uint64_t* best, int64_t* next, void* stream) {
    return cdq_lm_head_argmax_rows(w, x, vocab, n, 1, logits, best, next, stream);
}

cdq_status cdq_attn_decode_multi(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* cos_t,
                                 const uint16_t* sin_t, const int32_t* pos, uint16_t* k_cache, uint16_t* v_cache,
                                 int32_t max_len, int32_t n_heads, int32_t n_kv, int32_t head_dim, float scale,
                                 uint16_t* out, int32_t n_q, void* stream) {
    if (!q || !k || !v || !cos_t || !sin_t || !pos || !k_cache || !v_cache || !out || n_q < 1 || n_q > 64)
        return CDQ_ERR_ARG;
    if (head_dim != kHd || n_kv < 1 || n_heads < n_kv || n_heads % n_kv || max_len < 1 || max_len > 16384)
        return CDQ_ERR_UNSUPPORTED;
    if ((uintptr_t)k_cache % 16 || (uintptr_t)v_cache % 16) return CDQ_ERR_ARG;
    if (launch_pdl(rope_append_kernel, dim3(n_kv, n_q), dim3(kHd), 0, (cudaStream_t)stream, k, v, cos_t, sin_t, pos,
                   k_cache, v_cache, (int)max_len, (int)n_kv) != cudaSuccess)
        return CDQ_ERR_CUDA;
    const int smem = max_len * 4;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(attn_multi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return CDQ_ERR_CUDA;
    return launch_pdl(attn_multi_kernel, dim3(n_heads, n_q), dim3(kAttnThreads), (size_t)smem, (cudaStream_t)stream,
                      q, cos_t, sin_t, pos, k_cache, v_cache, (int)max_len, (int)n_heads, (int)n_kv, scale, out,
                      (int)max_len) == cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

}  // extern "C"
