// Decode-step arithmetic shared by the one-kernel-per-operation decode step
// (cdq_decode.cu) and the persistent decode-step kernel (cdq_step.cuh): the
// same device functions, so both produce the same bits. Each reproduces the
// rounding steps of the HF bf16 module it replaces (Qwen2RMSNorm, rotary
// embedding + grouped-query attention, Qwen2MLP's act_fn(gate) * up, the tied
// lm_head GEMV and torch.argmax).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace cdq {
namespace dm {

__device__ __forceinline__ float bf(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
__device__ __forceinline__ uint16_t tobf(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float rbf(float v) { return bf(tobf(v)); }

// ---- RMSNorm: the sum of squares of threads 0 .. kNormThreads-1 ----
constexpr int kNormThreads = 256;

// Every thread of the block calls this with its own partial (threads at or
// beyond kNormThreads pass 0 and are ignored); the warp partials of the first
// kNormThreads / 32 warps are added in warp order. red: kNormThreads / 32
// floats of shared memory. Returns the total in every thread.
__device__ __forceinline__ float norm_total(float ss, float* red) {
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0 && threadIdx.x < kNormThreads) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < kNormThreads / 32; ++k) tot += red[k];
    __syncthreads();  // red may be reused after the call
    return tot;
}

__device__ __forceinline__ float norm_scale(float tot, int n, float eps) { return rsqrtf(tot / (float)n + eps); }

// out = bf16(w * bf16(h * r)) for one element (h already the bf16 residual sum)
__device__ __forceinline__ uint16_t norm_out(uint16_t w, uint16_t h, float r) { return tobf(bf(w) * rbf(bf(h) * r)); }

// the residual add h + delta in bf16
__device__ __forceinline__ uint16_t add_bf(uint16_t h, uint16_t delta) { return tobf(bf(h) + bf(delta)); }

// SiLU(g) * u in Qwen2MLP's rounding steps
__device__ __forceinline__ uint16_t silu_mul(uint16_t g, uint16_t u) {
    const float x = bf(g);
    return tobf(rbf(x / (1.f + expf(-x))) * bf(u));
}

// ---- attention of one query head at position P ----
constexpr int kHd = 64;             // head dimension
constexpr int kAttnThreads = 512;   // threads working on one head
constexpr int kVSlices = kAttnThreads / kHd;  // position slices of the weighted value sum

// Shared scratch of one head's attention.
struct AttnScratch {
    float qe[kHd], ke[kHd], ve[kHd], red[kAttnThreads / 32], part[kVSlices][kHd];
};

// Rotary embedding of element d of a head vector at the position of (cs, sn).
__device__ __forceinline__ float rope(const uint16_t* x, int d, const uint16_t* cs, const uint16_t* sn) {
    const int o = d < kHd / 2 ? d + kHd / 2 : d - kHd / 2;
    const float sgn = d < kHd / 2 ? -1.f : 1.f;
    return rbf(rbf(bf(x[d]) * bf(cs[d])) + rbf(sgn * bf(x[o]) * bf(sn[d])));
}

// Attention of one query head at position P (S.qe: the rotary-embedded query;
// S.ke, S.ve: the position's own key and value, which the cache may not hold
// yet) over the kv head's cache rows kb / vb (rows 0 .. P-1), threads
// 0 .. kAttnThreads-1 of the block:
//   scores s_j = scale * (q . k_j) (fp32 fmas in element order), j = 0 .. P;
//   m = max s_j; e_j = exp(s_j - m); sum = the threads' partial sums (each over
//   its positions j = tid, tid + kAttnThreads, ...) added in thread order
//   through a warp reduction and the warps' partials in warp order;
//   out_d = bf16((sum over slices t = 0 .. kVSlices-1, in order, of
//           sum over j = t, t + kVSlices, ... of e_j v_jd) / sum).
// Called by every thread of the block (block barriers inside); threads at or
// beyond kAttnThreads only take part in the barriers. scores: P + 1 floats of
// shared memory.
__device__ __forceinline__ void attn_core(int tid, const uint16_t* kb, const uint16_t* vb, int P, float scale,
                                          uint16_t* out, float* scores, AttnScratch& S) {
    const bool act = tid < kAttnThreads;
    float mx = -INFINITY;
    if (act) {
        for (int j = tid; j <= P; j += kAttnThreads) {
            float s = 0.f;
            if (j < P) {
                const uint4* kr = reinterpret_cast<const uint4*>(kb + (int64_t)j * kHd);
#pragma unroll
                for (int c = 0; c < kHd / 8; ++c) {
                    const uint4 u = kr[c];
                    const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        s = fmaf(S.qe[8 * c + 2 * t], __uint_as_float(wv[t] << 16), s);
                        s = fmaf(S.qe[8 * c + 2 * t + 1], __uint_as_float(wv[t] & 0xFFFF0000u), s);
                    }
                }
            } else {
#pragma unroll 8
                for (int d = 0; d < kHd; ++d) s = fmaf(S.qe[d], S.ke[d], s);
            }
            s *= scale;
            scores[j] = s;
            mx = fmaxf(mx, s);
        }
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        if ((tid & 31) == 0) S.red[tid >> 5] = mx;
    }
    // the weighted values: thread (slice t, element d) takes positions j = t mod
    // kVSlices; the value loads of its first 16 positions are issued here, in
    // flight during the two reductions
    const int d = tid & (kHd - 1), t = (tid / kHd) % kVSlices;
    constexpr int kBatch = 16;
    uint16_t vv0[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
        const int j = t + k * kVSlices;
        vv0[k] = act && j < P ? vb[(int64_t)j * kHd + d] : (uint16_t)0;
    }
    __syncthreads();
    mx = S.red[0];
    for (int k2 = 1; k2 < kAttnThreads / 32; ++k2) mx = fmaxf(mx, S.red[k2]);
    __syncthreads();
    float sum = 0.f;
    if (act) {
        for (int j = tid; j <= P; j += kAttnThreads) {
            const float e = expf(scores[j] - mx);
            scores[j] = e;
            sum += e;
        }
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
        if ((tid & 31) == 0) S.red[tid >> 5] = sum;
    }
    __syncthreads();
    sum = 0.f;
    for (int k2 = 0; k2 < kAttnThreads / 32; ++k2) sum += S.red[k2];
    if (act) {
        // positions j = t, t + kVSlices, ... below P in order; the value loads of
        // 16 positions are issued before their fmas
        float acc = 0.f;
        for (int j0 = t; j0 < P; j0 += kBatch * kVSlices) {
            uint16_t vv[kBatch];
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const int j = j0 + k * kVSlices;
                vv[k] = j0 == t ? vv0[k] : j < P ? vb[(int64_t)j * kHd + d] : (uint16_t)0;
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k)
                if (j0 + k * kVSlices < P) acc = fmaf(scores[j0 + k * kVSlices], bf(vv[k]), acc);
        }
        if (P % kVSlices == t) acc = fmaf(scores[P], S.ve[d], acc);  // the position's own value
        S.part[t][d] = acc;
    }
    __syncthreads();
    if (act && t == 0) {
        float v = S.part[0][d];
        for (int k2 = 1; k2 < kVSlices; ++k2) v += S.part[k2][d];
        out[d] = tobf(v / sum);
    }
    __syncthreads();  // the scratch may be reused after the call
}

// Head h's attention at position P for the single-token step: the query, the
// step's key (rotary-embedded here) and value; the block of the kv head's
// first query head appends that key and value to the cache at P. (q, k, v
// may be rewritten by the caller between calls in one kernel: no
// read-only-cache loads.)
__device__ __forceinline__ void attn_head(int h, int tid, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                          const uint16_t* cs, const uint16_t* sn, int P, uint16_t* kc,
                                          uint16_t* vc, int max_len, int n_heads, int n_kv, float scale,
                                          uint16_t* out, float* scores, AttnScratch& S) {
    const int group = n_heads / n_kv, kvh = h / group;
    if (tid < kHd) {
        const int d = tid;
        S.qe[d] = rope(q + h * kHd, d, cs, sn);
        S.ke[d] = rope(k + kvh * kHd, d, cs, sn);
        S.ve[d] = bf(v[kvh * kHd + d]);
        if (h % group == 0) {  // one block per kv head appends the step's k and v
            kc[((int64_t)kvh * max_len + P) * kHd + d] = tobf(S.ke[d]);
            vc[((int64_t)kvh * max_len + P) * kHd + d] = v[kvh * kHd + d];
        }
    }
    __syncthreads();
    attn_core(tid, kc + (int64_t)kvh * max_len * kHd, vc + (int64_t)kvh * max_len * kHd, P, scale, out + h * kHd,
              scores, S);
}

// ---- lm_head GEMV and argmax ----
// The argmax key of a bf16 logit: orderable bits of the value (NaN above
// every number) above the complemented index (the first index wins ties).
__device__ __forceinline__ unsigned long long argmax_key(uint16_t v, uint32_t idx) {
    uint32_t b = v == 0x8000u ? 0u : v;        // -0 equals +0
    if ((b & 0x7FFFu) > 0x7F80u) b = 0xFFFFu;  // every NaN: the largest key
    else b = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - idx);
}

constexpr int kLmRows = 4;  // vocabulary rows per warp step at batch 1 (loads in flight)

// Vocabulary rows r0 .. r0 + R - 1 for M activation rows, one warp: lane-chunk
// order (16-byte chunks ch = lane, lane + 32, ...) then a warp reduction, the
// same arithmetic for every M and every caller. xs: [M][n] fp32 in shared
// memory. Writes the logits (if given) and folds the rows into key[m].
template <int M, int R>
__device__ __forceinline__ void lm_rows(const uint16_t* __restrict__ w, const float* xs, int n, int64_t vocab,
                                        int64_t r0, int lane, uint16_t* logits, unsigned long long (&key)[M]) {
    const int nch = n / 8;
    float acc[R][M];
#pragma unroll
    for (int t = 0; t < R; ++t)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[t][m] = 0.f;
    for (int ch = lane; ch < nch; ch += 32) {
        uint4 u[R];
#pragma unroll
        for (int t = 0; t < R; ++t)
            u[t] = r0 + t < vocab ? __ldcs(reinterpret_cast<const uint4*>(w + (r0 + t) * (int64_t)n) + ch)
                                  : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float4 xa = *reinterpret_cast<const float4*>(xs + m * n + 8 * ch);
            const float4 xb = *reinterpret_cast<const float4*>(xs + m * n + 8 * ch + 4);
#pragma unroll
            for (int t = 0; t < R; ++t) {
                float a = acc[t][m];
                a = fmaf(__uint_as_float(u[t].x << 16), xa.x, a);
                a = fmaf(__uint_as_float(u[t].x & 0xFFFF0000u), xa.y, a);
                a = fmaf(__uint_as_float(u[t].y << 16), xa.z, a);
                a = fmaf(__uint_as_float(u[t].y & 0xFFFF0000u), xa.w, a);
                a = fmaf(__uint_as_float(u[t].z << 16), xb.x, a);
                a = fmaf(__uint_as_float(u[t].z & 0xFFFF0000u), xb.y, a);
                a = fmaf(__uint_as_float(u[t].w << 16), xb.z, a);
                a = fmaf(__uint_as_float(u[t].w & 0xFFFF0000u), xb.w, a);
                acc[t][m] = a;
            }
        }
    }
#pragma unroll
    for (int t = 0; t < R; ++t) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float a = acc[t][m];
            for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
            if (r0 + t < vocab) {
                const uint16_t v = tobf(a);
                if (lane == 0 && logits) logits[(int64_t)m * vocab + r0 + t] = v;
                const unsigned long long k = argmax_key(v, (uint32_t)(r0 + t));
                key[m] = k > key[m] ? k : key[m];
            }
        }
    }
}

// The token of an argmax key.
__device__ __forceinline__ int64_t key_token(unsigned long long k) {
    return (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}

}  // namespace dm
}  // namespace cdq
