// C-ABI entry points that launch device work: argument checks, per-device
// set-up and the mapping of device packs onto kernel launches.
#include <cuda_runtime.h>

#include <algorithm>
#include <memory>
#include <mutex>
#include <vector>

#include "cdq.h"
#include "cdq_common.cuh"
#include "cdq_internal.cuh"

using namespace cdq;

namespace {

std::mutex g_mu;
bool g_ready[128] = {};
int g_sms[128] = {};

// Once per device: constant lattice tables and the SM count.
cdq_status device_setup(int* sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return CDQ_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ready[dev]) {
        if (upload_lattices() != cudaSuccess || dequant_setup() != cudaSuccess ||
            quantize_setup() != cudaSuccess)
            return CDQ_ERR_CUDA;
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return CDQ_ERR_CUDA;
        g_sms[dev] = n;
        g_ready[dev] = true;
    }
    *sms = g_sms[dev];
    return CDQ_OK;
}

inline bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }
inline int64_t al256(int64_t b) { return (b + 255) / 256 * 256; }

cdq_status check_pack(const cdq_packed* w) {
    if (!w) return CDQ_ERR_ARG;
    if (w->n_states != 26 && w->n_states != 16) return CDQ_ERR_STATES;
    if (w->rows <= 0 || w->cols <= 0 || w->cols % 32 || w->cols > CDQ_MAX_COLS) return CDQ_ERR_SHAPE;
    if (!w->units || !w->res_ptr || (w->n_res > 0 && !w->res_ent)) return CDQ_ERR_ARG;
    if (!aligned(w->units, 16) || !aligned(w->res_ptr, 4)) return CDQ_ERR_ARG;
    return CDQ_OK;
}

cdq_status fill_job(const cdq_packed* w, const uint16_t* x, int64_t m, void* y, int out_f32,
                    const uint16_t* bias, void* ws, size_t ws_bytes, GemvJob* J) {
    cdq_status st = check_pack(w);
    if (st) return st;
    if (m < 1 || m > CDQ_MAX_BATCH) return CDQ_ERR_ARG;
    if (!x || !y || !aligned(x, 16) || !aligned(y, out_f32 ? 4 : 2) || (bias && !aligned(bias, 2)))
        return CDQ_ERR_ARG;
    const Geometry g = geometry(w->rows, w->cols, w->n_states);
    J->units = w->units;
    J->res_ptr = w->res_ptr;
    J->res_ent = w->res_ent;
    J->x = x;
    J->y = y;
    J->bias = bias;
    J->rows = w->rows;
    J->cols = w->cols;
    J->r16 = (int32_t)g.r16;
    J->kt = (int32_t)g.kt;
    J->kp = (int32_t)g.kp;
    J->kg = (int32_t)g.kg;
    J->out_f32 = out_f32;
    J->n_res = (uint32_t)w->n_res;
    J->reserved_ptr = nullptr;
    J->rb_begin = 0;
    J->reserved0 = 0;
    // the caller's workspace: the row-block arrival counters, then the
    // streaming path's per-group sums or the tile path's prepared activations
    const int64_t need = linear_workspace_need(g, m);
    if (!ws || (int64_t)ws_bytes < need || !aligned(ws, 256)) return CDQ_ERR_WORKSPACE;
    J->counters = reinterpret_cast<uint32_t*>(ws);
    J->partial = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + gemv_counter_bytes(g));
    J->unit_begin = 0;
    return CDQ_OK;
}

cdq_status linear_common(const cdq_packed* w, const uint16_t* x, int64_t m, void* y, int out_f32,
                         const uint16_t* bias, void* ws, size_t ws_bytes, void* stream) {
    int sms = 0;
    cdq_status st = device_setup(&sms);
    if (st) return st;
    GemvBatch<1> b;
    b.n = 1;
    st = fill_job(w, x, m, y, out_f32, bias, ws, ws_bytes, &b.jobs[0]);
    if (st) return st;
    b.jobs[0].item_begin = 0;
    b.total_items = (int64_t)b.jobs[0].r16 * b.jobs[0].kg;
    b.total_row_blocks = b.jobs[0].r16;
    b.m = (int32_t)m;
    b.finish_single = 0;
    cudaError_t e = gemv_launch_single(b, w->n_states, (int)m, (cudaStream_t)stream, sms);
    return e == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

cdq_status quantize_common(const uint16_t* w, int32_t rows, int32_t cols, int32_t n_states, double stc_frac,
                           int32_t flags, int64_t res_capacity, cdq_packed* out, cdq_quant_info* info,
                           void* workspace, size_t workspace_bytes, void* stream) {
    int sms = 0;
    cdq_status st = device_setup(&sms);
    if (st) return st;
    cdq_sizes sz;
    st = cdq_get_sizes(rows, cols, n_states, stc_frac, 1, &sz);
    if (st) return st;
    if (flags & ~CDQ_QUANT_NO_TOPK_GUARD) return CDQ_ERR_ARG;
    if (!w || !aligned(w, 16) || !out || !info || !out->units || !out->res_ptr || !out->res_ent ||
        !out->res_q || !aligned(out->units, 16) || !aligned(out->res_ptr, 4) ||
        !aligned(out->res_ent, 4) || !aligned(info, 8) || res_capacity < 0)
        return CDQ_ERR_ARG;
    if (!workspace || (int64_t)workspace_bytes < sz.quantize_workspace_bytes ||
        !aligned(workspace, 256))
        return CDQ_ERR_WORKSPACE;
    QuantArgs a;
    a.w = w;
    a.rows = rows;
    a.cols = cols;
    a.n_states = n_states;
    a.stc_frac = stc_frac;
    a.no_guard = (flags & CDQ_QUANT_NO_TOPK_GUARD) ? 1 : 0;
    a.res_cap = res_capacity;
    a.out = *out;
    a.out.rows = rows;
    a.out.cols = cols;
    a.out.n_states = n_states;
    a.info = info;
    a.ws = reinterpret_cast<uint8_t*>(workspace);
    a.ws_bytes = workspace_bytes;
    cudaError_t e = quantize_launch(a, (cudaStream_t)stream, sms);
    return e == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

}  // namespace

extern "C" {

cdq_status cdq_linear(const cdq_packed* w, const uint16_t* x, int64_t m, uint16_t* y,
                      const uint16_t* bias, void* workspace, size_t workspace_bytes, void* stream) {
    return linear_common(w, x, m, y, 0, bias, workspace, workspace_bytes, stream);
}

cdq_status cdq_linear_f32(const cdq_packed* w, const uint16_t* x, int64_t m, float* y,
                          const uint16_t* bias, void* workspace, size_t workspace_bytes,
                          void* stream) {
    return linear_common(w, x, m, y, 1, bias, workspace, workspace_bytes, stream);
}

cdq_status cdq_linear_grouped(const cdq_gemv_job* jobs, int32_t n, int64_t m, void* stream) {
    if (!jobs || n < 0) return CDQ_ERR_ARG;
    if (n == 0) return CDQ_OK;
    int sms = 0;
    cdq_status st = device_setup(&sms);
    if (st) return st;
    for (int i = 0; i < n; ++i)
        if (jobs[i].w.n_states != 26 && jobs[i].w.n_states != 16) return CDQ_ERR_STATES;
    // one launch per lattice size, at most kMaxJobs jobs each
    for (int ns : {26, 16}) {
        std::vector<int> idx;
        for (int i = 0; i < n; ++i)
            if (jobs[i].w.n_states == ns) idx.push_back(i);
        for (size_t s0 = 0; s0 < idx.size(); s0 += kMaxJobs) {
            std::unique_ptr<GemvBatch<kMaxJobs>> b(new GemvBatch<kMaxJobs>);
            b->n = 0;
            b->m = (int32_t)m;
            b->finish_single = 0;
            int64_t items = 0, blocks = 0;
            for (size_t s1 = s0; s1 < std::min(idx.size(), s0 + (size_t)kMaxJobs); ++s1) {
                const cdq_gemv_job& jb = jobs[idx[s1]];
                GemvJob& J = b->jobs[b->n];
                st = fill_job(&jb.w, jb.x, m, jb.y, jb.out_f32 ? 1 : 0, jb.bias, jb.workspace,
                              (size_t)std::max<int64_t>(0, jb.workspace_bytes), &J);
                if (st) return st;
                J.item_begin = items;
                J.rb_begin = (int32_t)blocks;
                items += (int64_t)J.r16 * J.kg;
                blocks += J.r16;
                b->n++;
                if (items >= INT32_MAX || blocks >= INT32_MAX) return CDQ_ERR_SHAPE;
            }
            b->total_items = items;
            b->total_row_blocks = (int32_t)blocks;
            cudaError_t e = gemv_launch_grouped(*b, ns, (int)m, (cudaStream_t)stream, sms);
            if (e != cudaSuccess) return CDQ_ERR_CUDA;
        }
    }
    return CDQ_OK;
}

cdq_status cdq_dequant(const cdq_packed* w, uint16_t* w_hat, void* stream) {
    int sms = 0;
    cdq_status st = device_setup(&sms);
    if (st) return st;
    st = check_pack(w);
    if (st) return st;
    if (!w_hat || !aligned(w_hat, 16)) return CDQ_ERR_ARG;
    cudaError_t e = dequant_launch(*w, w_hat, (cudaStream_t)stream);
    return e == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

cdq_status cdq_quantize(const uint16_t* w, int32_t rows, int32_t cols, int32_t n_states,
                        double stc_frac, cdq_packed* out, cdq_quant_info* info, void* workspace,
                        size_t workspace_bytes, void* stream) {
    cdq_sizes sz;
    cdq_status st = cdq_get_sizes(rows, cols, n_states, stc_frac, 1, &sz);
    if (st) return st;
    return quantize_common(w, rows, cols, n_states, stc_frac, 0, sz.max_res, out, info, workspace,
                           workspace_bytes, stream);
}

cdq_status cdq_quantize_ex(const uint16_t* w, int32_t rows, int32_t cols, int32_t n_states,
                           double stc_frac, int32_t flags, int64_t res_capacity, cdq_packed* out,
                           cdq_quant_info* info, void* workspace, size_t workspace_bytes, void* stream) {
    return quantize_common(w, rows, cols, n_states, stc_frac, flags, res_capacity, out, info, workspace,
                           workspace_bytes, stream);
}

cdq_status cdq_set_tile_min_batch(int32_t m) {
    if (m < 1) return CDQ_ERR_ARG;
    gemv_set_tile_min_batch(m);
    return CDQ_OK;
}

cdq_status cdq_kernel_error(int32_t* code) {
    if (!code) return CDQ_ERR_ARG;
    int v = 0;
    if (gemv_read_error(&v) != cudaSuccess) return CDQ_ERR_CUDA;
    *code = v;
    return CDQ_OK;
}

}  // extern "C"
