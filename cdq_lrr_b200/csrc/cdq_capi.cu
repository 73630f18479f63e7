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
    b.m = (int32_t)m;
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
            cudaError_t e = gemv_launch_grouped(*b, ns, (int)m, (cudaStream_t)stream, sms);
            if (e != cudaSuccess) return CDQ_ERR_CUDA;
        }
    }
    return CDQ_OK;
}

// Table layout: the parameters, the layers, the stage descriptors
// [layer][group][CTA] (one CTA per SM of the current device), the sync words.
struct StepTableLayout {
    int64_t layers_off, stage_off, sync_off, bytes;
};
StepTableLayout step_table_layout(int32_t layers, int sms) {
    StepTableLayout t;
    t.layers_off = al256((int64_t)sizeof(StepParams));
    t.stage_off = al256(t.layers_off + (int64_t)layers * (int64_t)sizeof(StepLayer));
    t.sync_off = al256(t.stage_off + (int64_t)layers * 4 * sms * (int64_t)sizeof(StepStage));
    t.bytes = t.sync_off + 256;
    return t;
}

// floor(u * k / n), the kernel's stretch_bound
int64_t host_stretch_bound(int64_t U, int64_t k, int64_t n) { return U * k / n; }

// The kernel's first_at over a group (first item whose first unit is >= u).
void host_first_at(const StepGroup& G, int64_t u, int* j, int* b16, int* grp) {
    int lo = 0, hi = G.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (G.jobs[mid].unit_begin <= u) lo = mid; else hi = mid - 1;
    }
    const GemvJob& J = G.jobs[lo];
    const int64_t rel = u - J.unit_begin;
    int b = (int)(rel / J.kp), g = (int)((rel - (int64_t)b * J.kp + 15) >> 4), jj = lo;
    if (g >= J.kg) {
        g = 0;
        ++b;
    }
    if (b >= J.r16) {
        b = 0;
        ++jj;
    }
    *j = jj;
    *b16 = b;
    *grp = g;
}

// The residual data CTA c of `sms` needs for group G: per job, the buckets of
// the row blocks its items touch (with the closing bound) and their entries.
StepStage host_stage(const StepGroup& G, const std::vector<const std::vector<uint32_t>*>& ptrs, int c, int sms,
                     int bnd_cap, int ent_cap) {
    StepStage d = {};
    d.n = G.n;
    const int64_t U = G.total_units, nw = (int64_t)sms * 16;
    int j0, b0, g0, j1, b1, g1;
    host_first_at(G, host_stretch_bound(U, (int64_t)c * 16, nw), &j0, &b0, &g0);
    host_first_at(G, host_stretch_bound(U, (int64_t)(c + 1) * 16, nw), &j1, &b1, &g1);
    for (int j = 0; j < G.n; ++j) {
        const GemvJob& J = G.jobs[j];
        if (j < j0 || j > j1) continue;
        const int64_t i_lo = j == j0 ? (int64_t)b0 * J.kg + g0 : 0;
        const int64_t i_hi = j == j1 ? (int64_t)b1 * J.kg + g1 : (int64_t)J.r16 * J.kg;
        if (i_lo >= i_hi) continue;
        const int64_t rb_lo = i_lo / J.kg, rb_hi = (i_hi + J.kg - 1) / J.kg;
        const int64_t B0 = rb_lo * 16 * J.kg, B1 = rb_hi * 16 * J.kg;
        const std::vector<uint32_t>& rp = *ptrs[j];
        const uint32_t e0 = std::min<uint32_t>(rp[B0], J.n_res);
        const uint32_t e1 = std::min<uint32_t>(std::max(rp[B1], e0), J.n_res);
        d.b0[j] = (int32_t)B0;
        d.nb[j] = (int32_t)(B1 - B0 + 1);
        d.e0[j] = (int32_t)e0;
        d.ne[j] = (int32_t)(e1 - e0);
        d.nb_total += d.nb[j];
        d.ne_total += d.ne[j];
    }
    d.ok = d.nb_total <= bnd_cap && d.ne_total <= ent_cap;
    return d;
}

cdq_status cdq_step_table_bytes(int32_t layers, int64_t* bytes) {
    if (layers < 1 || layers > 4096 || !bytes) return CDQ_ERR_ARG;
    int sms = 0;
    cdq_status st = device_setup(&sms);
    if (st) return st;
    *bytes = step_table_layout(layers, sms).bytes;
    return CDQ_OK;
}

cdq_status cdq_step_prepare(const cdq_step_model* md, const cdq_step_layer* layers, void* table) {
    if (!md || !layers || !table || !aligned(table, 256)) return CDQ_ERR_ARG;
    int sms = 0;
    cdq_status st = device_setup(&sms);
    if (st) return st;
    const cdq_step_model& M = *md;
    if (M.layers < 1 || M.hidden < 8 || M.hidden % 8 || M.heads < 1 || M.kv_heads < 1 || M.inter < 1 ||
        M.max_len < 1 || M.token_cap < 1 || M.vocab < 1 || M.vocab >= INT32_MAX)
        return CDQ_ERR_ARG;
    if (M.head_dim != 64 || M.heads % M.kv_heads || M.heads > sms) return CDQ_ERR_UNSUPPORTED;
    const void* need[] = {M.embed, M.norm_w, M.lm_w, M.cos_t, M.sin_t, M.pos,  M.ids, M.tokens, M.count,
                          M.best,  M.next,   M.h0,   M.h1,    M.q,     M.k,    M.v,   M.att,    M.o,
                          M.g,     M.u,      M.dn};
    for (const void* p : need)
        if (!p) return CDQ_ERR_ARG;
    if (!aligned(M.lm_w, 16) || !aligned(M.best, 8)) return CDQ_ERR_ARG;
    const StepTableLayout lay = step_table_layout(M.layers, sms);
    const int64_t bytes = lay.bytes;
    std::vector<uint8_t> img((size_t)bytes, 0);
    auto* P = reinterpret_cast<StepParams*>(img.data());
    auto* L = reinterpret_cast<StepLayer*>(img.data() + lay.layers_off);
    auto* STG = reinterpret_cast<StepStage*>(img.data() + lay.stage_off);
    uint8_t* dev = static_cast<uint8_t*>(table);
    P->layers = M.layers;
    P->hidden = M.hidden;
    P->heads = M.heads;
    P->kv_heads = M.kv_heads;
    P->inter = M.inter;
    P->max_len = M.max_len;
    P->token_cap = M.token_cap;
    P->vocab = M.vocab;
    P->eps = M.eps;
    P->scale = M.scale;
    P->embed = M.embed;
    P->norm_w = M.norm_w;
    P->lm_w = M.lm_w;
    P->cos_t = M.cos_t;
    P->sin_t = M.sin_t;
    P->pos = M.pos;
    P->ids = M.ids;
    P->tokens = M.tokens;
    P->count = M.count;
    P->best = reinterpret_cast<unsigned long long*>(M.best);
    P->next = M.next;
    P->logits = M.logits;
    P->h[0] = M.h0;
    P->h[1] = M.h1;
    P->q = M.q;
    P->k = M.k;
    P->v = M.v;
    P->att = M.att;
    P->o = M.o;
    P->g = M.g;
    P->u = M.u;
    P->dn = M.dn;
    if (!step_smem_layout(*P)) return CDQ_ERR_UNSUPPORTED;
    P->layer = reinterpret_cast<const StepLayer*>(dev + lay.layers_off);
    P->stage = reinterpret_cast<const StepStage*>(dev + lay.stage_off);
    P->sync = reinterpret_cast<uint32_t*>(dev + lay.sync_off);
    P->n_ctas = sms;
    const int qd = M.heads * 64, kvd = M.kv_heads * 64;
    int ns = 0;
    for (int l = 0; l < M.layers; ++l) {
        const cdq_step_layer& S = layers[l];
        if (!S.ln1 || !S.ln2 || !S.k_cache || !S.v_cache || !aligned(S.k_cache, 16) || !aligned(S.v_cache, 16))
            return CDQ_ERR_ARG;
        struct Want {
            const cdq_gemv_job* j;
            int rows, cols;
            const void* y;
        } want[7] = {{&S.q, qd, M.hidden, M.q},         {&S.k, kvd, M.hidden, M.k},
                     {&S.v, kvd, M.hidden, M.v},        {&S.o, M.hidden, qd, M.o},
                     {&S.gate, M.inter, M.hidden, M.g}, {&S.up, M.inter, M.hidden, M.u},
                     {&S.down, M.hidden, M.inter, M.dn}};
        GemvJob J[7];
        for (int i = 0; i < 7; ++i) {
            const cdq_gemv_job& jb = *want[i].j;
            if (jb.w.rows != want[i].rows || jb.w.cols != want[i].cols) return CDQ_ERR_SHAPE;
            if (jb.y != want[i].y || jb.out_f32) return CDQ_ERR_ARG;
            if (ns == 0) ns = jb.w.n_states;
            if (jb.w.n_states != ns) return CDQ_ERR_STATES;
            st = fill_job(&jb.w, jb.x, 1, jb.y, 0, jb.bias, jb.workspace,
                          (size_t)std::max<int64_t>(0, jb.workspace_bytes), &J[i]);
            if (st) return st;
        }
        StepLayer& D = L[l];
        auto group = [&](StepGroup& G, std::initializer_list<int> idx) {
            G.n = 0;
            G.total_units = 0;
            for (int i : idx) {
                GemvJob& g = G.jobs[G.n++];
                g = J[i];
                g.unit_begin = G.total_units;
                G.total_units += (int64_t)g.r16 * g.kp;
            }
        };
        group(D.qkv, {0, 1, 2});
        group(D.o, {3});
        group(D.gu, {4, 5});
        group(D.down, {6});
        // the CSR bounds of the seven projections, for the stage descriptors
        std::vector<uint32_t> rp[7];
        for (int i = 0; i < 7; ++i) {
            rp[i].resize((size_t)J[i].r16 * 16 * J[i].kg + 1);
            if (cudaMemcpy(rp[i].data(), J[i].res_ptr, rp[i].size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
                return CDQ_ERR_CUDA;
        }
        const StepGroup* groups[4] = {&D.qkv, &D.o, &D.gu, &D.down};
        const std::vector<std::vector<int>> members = {{0, 1, 2}, {3}, {4, 5}, {6}};
        for (int gi = 0; gi < 4; ++gi) {
            std::vector<const std::vector<uint32_t>*> ptrs;
            for (int i : members[gi]) ptrs.push_back(&rp[i]);
            for (int c = 0; c < sms; ++c)
                STG[((int64_t)l * 4 + gi) * sms + c] =
                    host_stage(*groups[gi], ptrs, c, sms, P->rst_bnd_cap, P->rst_ent_cap);
        }
        D.ln1 = S.ln1;
        D.ln2 = S.ln2;
        D.kc = S.k_cache;
        D.vc = S.v_cache;
    }
    P->n_states = ns;
    return cudaMemcpy(table, img.data(), (size_t)bytes, cudaMemcpyHostToDevice) == cudaSuccess ? CDQ_OK
                                                                                               : CDQ_ERR_CUDA;
}

cdq_status cdq_decode_step(const void* table, int32_t n_states, void* stream) {
    if (!table || !aligned(table, 256)) return CDQ_ERR_ARG;
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    int sms = 0;
    cdq_status st = device_setup(&sms);
    if (st) return st;
    return step_launch(static_cast<const StepParams*>(table), n_states, sms, (cudaStream_t)stream) == cudaSuccess
               ? CDQ_OK
               : CDQ_ERR_CUDA;
}

cdq_status cdq_step_error(const void* table, int32_t* code) {
    if (!table || !code) return CDQ_ERR_ARG;
    StepParams p;
    if (cudaMemcpy(&p, table, sizeof p, cudaMemcpyDeviceToHost) != cudaSuccess) return CDQ_ERR_CUDA;
    uint32_t w = 0;
    if (cudaMemcpy(&w, p.sync + 4, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return CDQ_ERR_CUDA;
    *code = (int32_t)w;
    return CDQ_OK;
}

cdq_status cdq_step_reset(void* table, void* stream) {
    if (!table) return CDQ_ERR_ARG;
    StepParams p;
    if (cudaMemcpy(&p, table, sizeof p, cudaMemcpyDeviceToHost) != cudaSuccess) return CDQ_ERR_CUDA;
    return cudaMemsetAsync(p.sync, 0, 32, (cudaStream_t)stream) == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
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
