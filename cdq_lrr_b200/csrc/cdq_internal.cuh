// Internal launch interfaces shared by the C-ABI layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "cdq.h"
#include "cdq_common.cuh"

namespace cdq {

// One GEMV of a launch, with geometry precomputed on the host.
struct GemvJob {
    const uint8_t* units;
    const uint32_t* res_ptr;
    const uint32_t* res_ent;
    const uint16_t* x;
    void* y;
    const uint16_t* bias;
    float* partial;       // per-group partial sums [m][kg][r16*16] (workspace)
    void* reserved_ptr;
    int64_t item_begin;   // first work item (row block x residual group) of this job
    int64_t unit_begin;   // first unit of this job in the launch's unit sequence (streaming kernel)
    uint32_t* counters;   // per-row-block arrival counters after the partial sums (streaming kernel)
    int32_t rows, cols, r16, kt, kp, kg;
    int32_t out_f32;
    uint32_t n_res;       // residual entries; bucket pointers are clamped to it
    int32_t rb_begin;     // first fix-up block of this job (set by the launcher)
    int32_t reserved0;
};
static_assert(sizeof(GemvJob) == 128, "GemvJob layout");

constexpr int kMaxJobs = 192;  // 192 x 128-byte jobs fit the 32 KB kernel-parameter space

template <int MAXJ>
struct GemvBatch {
    int64_t total_items;
    int32_t n;
    int32_t m;                 // batch rows of every job of the launch
    int64_t total_units;       // units of every job of the launch (streaming kernel)
    GemvJob jobs[MAXJ];
};

// Launch with programmatic stream serialization: the kernel may start while
// its predecessor on the stream is still running; it must execute
// griddepcontrol.wait before it reads anything that predecessor writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Device side of a programmatic launch: wait for the predecessor's completion
// (and its memory), then let the successor be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;"); }
// Release/acquire fence at GPU scope: with a relaxed atomic or flag after it
// (release) or before it (acquire), the ordering that a GPU-wide hand-off of
// data needs, without the total order of a sequentially consistent fence.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

cudaError_t upload_lattices();
// allow_tile: the launch may take the tcgen05 tile path (the jobs' workspaces
// hold linear_workspace_need bytes); false keeps the streaming path.
cudaError_t gemv_launch_single(const GemvBatch<1>& b, int ns, int m, cudaStream_t s, int sms,
                               bool allow_tile = true);
cudaError_t gemv_launch_grouped(const GemvBatch<kMaxJobs>& b, int ns, int m, cudaStream_t s,
                                int sms);
cudaError_t gemv_read_error(int* out);
void gemv_set_tile_min_batch(int m);

// ---- persistent decode step (one cooperative launch per token) ----
constexpr int kStepPhaseJobs = 3;
// One projection group of a decoder layer (the jobs that share an input: q/k/v,
// o, gate/up, down), laid out as the streaming kernel's batch view: units of
// the jobs in job order (unit_begin set), x unused (the input is in shared
// memory), m = 1.
struct StepGroup {
    int32_t n;
    int32_t reserved0;
    int64_t total_units;
    GemvJob jobs[kStepPhaseJobs];
};
struct StepLayer {
    StepGroup qkv, o, gu, down;
    const uint16_t* ln1;
    const uint16_t* ln2;
    uint16_t* kc;
    uint16_t* vc;
};
// The residual data one CTA needs for one projection group (the CSR bounds
// and entries of the buckets of its items, per job), staged into its shared
// memory by asynchronous copies issued before the barrier that precedes the
// group: per job k, bounds [b0, b0 + nb) and entries [e0, e0 + ne). ok = 0:
// too large for the stage buffers (the CTA reads them from global memory).
struct StepStage {
    int32_t n, ok, nb_total, ne_total;
    int32_t b0[kStepPhaseJobs], nb[kStepPhaseJobs], e0[kStepPhaseJobs], ne[kStepPhaseJobs];
};
static_assert(sizeof(StepStage) == 64, "StepStage layout");

// Everything the persistent kernel reads, in device memory: this record, then
// the layers, then the stage descriptors [layer][group][CTA], then the sync
// words (64-bit barrier arrivals, 64-bit completed launches, 32-bit error).
struct StepParams {
    int32_t layers, hidden, heads, kv_heads, inter, max_len, token_cap, n_states;
    int64_t vocab;
    float eps, scale;
    const uint16_t* embed;
    const uint16_t* norm_w;
    const uint16_t* lm_w;
    const uint16_t* cos_t;
    const uint16_t* sin_t;
    int32_t* pos;
    int64_t* ids;
    int64_t* tokens;
    int32_t* count;
    unsigned long long* best;
    int64_t* next;
    uint16_t* logits;
    uint16_t* h[2];
    uint16_t *q, *k, *v, *att, *o, *g, *u, *dn;
    uint32_t xs_addr, xf_addr, sc_addr, scr_addr;  // shared-window addresses of the kernel's buffers
    uint32_t rst_addr;                             // residual stage: bounds, then entries
    int32_t rst_bnd_cap, rst_ent_cap;              // stage capacities (uint32 words)
    int32_t n_ctas;                                // the grid the stage descriptors were made for
    const StepLayer* layer;
    const StepStage* stage;
    uint32_t* sync;
    int64_t reserved_tail;  // 16-byte multiple (the kernel copies this record into shared memory)
};
// Shared-window layout of the persistent kernel above the streaming rings:
// returns false if the model's buffers do not fit.
bool step_smem_layout(StepParams& p);
cudaError_t step_launch(const StepParams* dev_params, int ns, int sms, cudaStream_t s);

cudaError_t dequant_setup();
cudaError_t quantize_setup();
cudaError_t dequant_launch(const cdq_packed& w, uint16_t* out, cudaStream_t s);

struct QuantArgs {
    const uint16_t* w;
    int32_t rows, cols, n_states;
    double stc_frac;
    int32_t no_guard;  // 1: no top-k tie guard (the packer CLI's quantizer)
    int64_t res_cap;   // residual entries the output buffers hold
    cdq_packed out;
    cdq_quant_info* info;
    uint8_t* ws;
    size_t ws_bytes;
};
cudaError_t quantize_launch(const QuantArgs& a, cudaStream_t s, int sms);

}  // namespace cdq
