// Internal launch interfaces shared by the C-ABI layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cdq.h"

namespace cdq {

// One GEMV of a launch, with geometry precomputed on the host.
struct GemvJob {
    const uint32_t* codes;
    const uint8_t* scales;
    const uint32_t* res_ptr;
    const uint32_t* res_ent;
    const uint16_t* x;
    void* y;
    const uint16_t* bias;
    float* partial;       // split-K slots [m][kg][rb*32]
    uint32_t* counters;   // [rb], zero between calls
    int64_t item_begin;   // first work item of this job in the launch
    int32_t rows, cols, rb, kt, kt4, kg;
    int32_t out_f32;
    int32_t pad_;
};

constexpr int kMaxJobs = 192;  // 192 x 104-byte jobs fit the 32 KB kernel-parameter space

template <int MAXJ>
struct GemvBatch {
    int64_t total_items;
    int32_t n;
    int32_t pad_;
    GemvJob jobs[MAXJ];
};

cudaError_t upload_lattices();
cudaError_t gemv_launch_single(const GemvBatch<1>& b, int ns, int m, cudaStream_t s, int sms);
cudaError_t gemv_launch_grouped(const GemvBatch<kMaxJobs>& b, int ns, int m, cudaStream_t s,
                                int sms);

cudaError_t dequant_setup();
cudaError_t quantize_setup();
cudaError_t dequant_launch(const cdq_packed& w, uint16_t* out, cudaStream_t s);

struct QuantArgs {
    const uint16_t* w;
    int32_t rows, cols, n_states;
    double stc_frac;
    cdq_packed out;
    cdq_quant_info* info;
    uint8_t* ws;
    size_t ws_bytes;
};
cudaError_t quantize_launch(const QuantArgs& a, cudaStream_t s, int sms);

}  // namespace cdq
