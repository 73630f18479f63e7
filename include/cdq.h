/*
 * cdq.h - C ABI of the B200 (sm_100a) CDQ-LRR decode path.
 *
 * CDQ-LRR stores a projection weight [rows, cols] (cols % 32 == 0) as tiles of
 * 32 consecutive weights of one row. Each tile keeps one float8 e4m3fn scale
 * sigma = max|w|, one lattice index per weight (26-state lattice, 5 bits, or
 * 16-state lattice, 4 bits) and, for the top fraction of weights by saliency,
 * the original bf16 value (a "residual"). Decoding is
 *     w_hat = bf16(LATTICE[q] * bf16(sigma)), residual positions take their value.
 *
 * Every function borrows raw pointers and never frees them. Device pointers
 * are CUDA global memory of the current device; stream arguments are
 * cudaStream_t passed as void*. All functions return a cdq_status (0 = OK).
 * Kernels are enqueued asynchronously on the given stream unless the
 * comment says otherwise. bf16 values travel as uint16_t bit patterns.
 *
 * Citations name the reference interface each entry point replaces
 * (file:line within the CDQ-LRR project).
 */
#ifndef CDQ_B200_H
#define CDQ_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CDQ_API __attribute__((visibility("default")))
#else
#define CDQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum cdq_status {
    CDQ_OK = 0,
    CDQ_ERR_SHAPE = 1,       /* cols % 32 != 0, a zero or oversized dimension   */
    CDQ_ERR_STATES = 2,      /* lattice size other than 26 or 16               */
    CDQ_ERR_ARG = 3,         /* null pointer or out-of-range argument          */
    CDQ_ERR_CUDA = 4,        /* a CUDA runtime call or kernel launch failed     */
    CDQ_ERR_FORMAT = 5,      /* malformed or truncated .cdq bytes              */
    CDQ_ERR_CAPACITY = 6,    /* a caller buffer is too small                    */
    CDQ_ERR_WORKSPACE = 7,   /* workspace missing or smaller than required     */
    CDQ_ERR_UNSUPPORTED = 8  /* valid request this build cannot serve          */
} cdq_status;

/* Largest supported cols: residual entries store the column in 16 bits. */
#define CDQ_MAX_COLS 65536
#define CDQ_TILE 32
#define CDQ_MAX_BATCH 64        /* cdq_linear serves M <= CDQ_MAX_BATCH      */

/*
 * Device layout of one packed weight ("device pack"), built so that one
 * 128-bit (+32-bit) load per lane gives each lane of a warp exactly the pair
 * codes of its m16n8k16 tensor-core A fragment.
 *
 * Rows form blocks of 16 (R16 = ceil(rows/16)), tile columns (32 weights of
 * a row) form pairs (KP = ceil(KT/2), KT = cols/32). A unit = one 16-row block
 * x one tile-column pair = 32 tiles, stored as 672 bytes (26 states) or 544
 * bytes (16 states), units ordered [R16][KP]:
 *   bytes [0, 512)   lane l's code words 0..3 (16 bytes at 16*l);
 *   bytes [512, 640) lane l's code word 4 (26 states only);
 *   then 32 bytes of fp8 e4m3fn scales: word g holds the scales of
 *   (row g, tile 0), (row g, tile 1), (row g+8, tile 0), (row g+8, tile 1).
 * Lane l = 4g + c carries 16 slots q = 8t + 4s + i (t: tile of the pair, s:
 * 16-element half of the tile, i = h + 2j): slot q is the element pair
 * p = 8s + c + 4j (weights 2p, 2p+1) of row g + 8h of tile t.
 *   26 states: slot q is the 10-bit code s[2p]*27 + s[2p+1] at bits
 *   [10q, 10q+10) of the lane's 160-bit word stream, s = lattice index 0..25,
 *   or 26 at a residual position (contributes zero);
 *   16 states: byte q = s[2p] | s[2p+1] << 4, residual positions hold index 7
 *   (the lattice's exact zero).
 * Rows beyond `rows` and the missing tile of an odd KT hold zero codes and
 * scale 0.
 *   res_ptr : residual CSR offsets, R16*16*KG + 1 entries (KG = ceil(KT/32));
 *             bucket row * KG + g lists row `row` (0 <= row < R16*16), tile
 *             columns [32g, 32g + 32), so one row's entries are the range
 *             [res_ptr[row*KG], res_ptr[(row+1)*KG]).
 *   res_ent : n_res words (col << 16) | bf16 bits, sorted by bucket then col
 *             (by row, then column).
 *   res_q   : n_res lattice indices the quantizer chose at the residual
 *             positions (read only by format conversion, never by cdq_linear).
 */
typedef struct cdq_packed {
    int32_t rows;
    int32_t cols;
    int32_t n_states;      /* 26 or 16 */
    int32_t reserved0;
    int64_t n_res;         /* residual entries in res_ent / res_q */
    uint8_t* units;        /* R16 * KP units of 672 or 544 bytes */
    uint32_t* res_ptr;
    uint32_t* res_ent;
    uint8_t* res_q;
} cdq_packed;

/* Byte and element counts of a device pack and of the workspaces. */
typedef struct cdq_sizes {
    int64_t row_blocks;        /* R16 */
    int64_t tile_pairs;        /* KP */
    int64_t res_groups;        /* KG */
    int64_t units_bytes;
    int64_t res_ptr_count;     /* uint32 entries */
    int64_t max_res;           /* upper bound on n_res from cdq_quantize: 2k */
    int64_t linear_workspace_bytes;    /* per call of cdq_linear (group sums or prepared x) */
    int64_t quantize_workspace_bytes;
} cdq_sizes;

/* Sizes for a [rows, cols] weight, the given lattice and residual fraction
 * (stc_frac only affects max_res) and largest batch. No CUDA calls. */
CDQ_API cdq_status cdq_get_sizes(int32_t rows, int32_t cols, int32_t n_states, double stc_frac,
                                 int32_t max_batch, cdq_sizes* out);

/* Library version string and the compiled device architecture. */
CDQ_API const char* cdq_version(void);

/*
 * y[M, rows] = x[M, cols] * w_hat^T (+ bias), fused: the packed weight is
 * streamed from HBM and dequantized in registers (bit-exact w_hat pairs fed
 * to the tensor cores), FP32 accumulation, result rounded once to bf16.
 * M <= CDQ_MAX_BATCH. bias may be NULL. x, y, bias: bf16 bit patterns,
 * row-major.
 * workspace: linear_workspace_bytes of device memory. Its first
 * ceil(R16 * 4 / 256) * 256 bytes hold one arrival counter per 16-row block:
 * they must be zero before the first call (zero-fill a new workspace once),
 * and every completed call leaves them zero again; the rest needs no
 * initialisation. After a call that recorded a kernel error
 * (cdq_kernel_error), zero the workspace again. Calls that share one
 * workspace must not overlap on the GPU.
 * Paths: M <= 8, two launches: a residual pre-pass (the sum of every
 * (row, residual group) bucket, bf16 value x activation in fp32, entries in
 * order) and the streaming kernel, which adds each group's mma sum to its
 * residual sum, sums the groups of a row in order (in registers, or through
 * the workspace and the counters where a warp's work boundary cuts a row
 * block) and adds the bias. M = 9..64 on the streaming path: the pre-pass,
 * the wide streaming kernel and a fix-up launch that adds the groups; same
 * arithmetic per output, so a row's result does not depend on the batch it
 * is computed in. M >= the tile threshold with enough 128-row tiles: the
 * tcgen05 tile path, two launches (activation layout, tile kernel whose
 * epilogue adds the residual entries and the bias).
 * Replaces CDQLinear.forward, code/cdq_lrr_qwen05.py:196-198, and the
 * loader's CDQLinear.forward, code/cdq_loader.py:53-58.
 */
CDQ_API cdq_status cdq_linear(const cdq_packed* w, const uint16_t* x, int64_t m, uint16_t* y,
                              const uint16_t* bias, void* workspace, size_t workspace_bytes,
                              void* stream);

/* As cdq_linear, output in float32 (no final bf16 rounding). */
CDQ_API cdq_status cdq_linear_f32(const cdq_packed* w, const uint16_t* x, int64_t m, float* y,
                                  const uint16_t* bias, void* workspace, size_t workspace_bytes,
                                  void* stream);

/*
 * As cdq_linear (bf16 output), for callers that cannot allocate device
 * memory: a plugin whose host process owns all device memory through its own
 * pool, or a path where a cudaMalloc, which may synchronise the device, is
 * not allowed. It allocates nothing and takes no workspace: its scratch (the
 * row-block counters and per-group sums of the streaming paths) is a 4 MiB
 * array that the library holds on every GPU that loads it, until the process
 * exits. Weights whose scratch would exceed 4 MiB (ceil(rows/16) * 4 bytes
 * rounded up to 256, plus m * ceil(cols/1024) * ceil(rows/16) * 64 bytes
 * rounded up to 256) are rejected with CDQ_ERR_WORKSPACE. Always the
 * streaming paths (no tcgen05 tile path), any m <= CDQ_MAX_BATCH. All calls
 * share the one array: calls that overlap on the GPU race, so issue them on
 * one stream. The first call on a device sets up the scratch address and
 * lattice tables (host-side runtime calls); make it before any stream
 * capture. The address is remembered per device ordinal, so it does not
 * survive a cudaDeviceReset of that device within the process.
 * No counterpart in the reference.
 */
CDQ_API cdq_status cdq_linear_noalloc(const cdq_packed* w, const uint16_t* x, int64_t m,
                                      uint16_t* y, const uint16_t* bias, void* stream);

/* One GEMV of a grouped launch. */
typedef struct cdq_gemv_job {
    cdq_packed w;          /* by value */
    const uint16_t* x;     /* [m, cols] bf16 */
    void* y;               /* [m, rows] bf16 or float32 */
    const uint16_t* bias;  /* NULL or [rows] */
    void* workspace;       /* this job's linear workspace (distinct per job) */
    int64_t workspace_bytes;
    int32_t out_f32;       /* 0: bf16 y, 1: float32 y */
    int32_t reserved0;
} cdq_gemv_job;

/*
 * Runs n independent jobs (same batch m) in one launch: the work of all jobs
 * is spread over every SM, which a decode step uses for the projections that
 * share an input (q/k/v, gate/up) or that are otherwise independent.
 * jobs: host array, copied by the call. No counterpart in the reference (it
 * runs one projection per F.linear call, code/cdq_lrr_qwen05.py:198).
 */
CDQ_API cdq_status cdq_linear_grouped(const cdq_gemv_job* jobs, int32_t n, int64_t m, void* stream);

/*
 * Kernel selection for the fused linear (process-wide, all devices): batches
 * of at least m rows take the tcgen05 tile path (the weight rows are the
 * M = 128 side of a tensor-core mma with tensor-memory accumulators, the
 * batch its N side, padded to 16, 32 or 64); smaller batches take the
 * streaming mma.sync path. Default 16; a value above CDQ_MAX_BATCH turns the
 * tile path off. The tile path adds a row's products in its own order (one
 * tensor-memory accumulator over the whole row, then the row's residual
 * entries), so its outputs differ from the streaming path's in the last
 * bits. Not thread-safe against concurrent calls of the linear entry points.
 * No counterpart in the reference.
 */
CDQ_API cdq_status cdq_set_tile_min_batch(int32_t m);

/*
 * The sticky in-kernel error code of the fused linear on the current device
 * (0: none; 1: shared-memory window misplaced; 2: a weight copy never landed
 * within the wait limit; 3: a tile-path pipeline wait gave up; 4: a residual
 * pre-pass copy never landed within the wait limit). A kernel that
 * records an error leaves its outputs incomplete but returns normally, so the
 * context stays usable. Reads after a device synchronisation; does not reset.
 */
CDQ_API cdq_status cdq_kernel_error(int32_t* code);

/*
 * One-shot all-reduce of float32 vectors over NVLink peer memory (the
 * row-parallel partial outputs of tensor parallelism). Each rank creates a
 * region on its device (staging buffers of 2 x cap floats, a signal pad and
 * epoch counters; allocated and zeroed by the library), exports its CUDA IPC
 * handle, and maps every peer's region with cdq_ar_open. cdq_allreduce_f32
 * then sums data[0, n) across the ranks in place: each rank publishes its
 * vector in its own region, flags every peer (system-scope release), waits for
 * every peer's flag (acquire; a bounded wait that records error code 1 of
 * cdq_ar_error and leaves data unreduced), and adds the ranks' vectors in rank
 * order, so every rank holds bit-identical sums. regions[q] is rank q's region
 * as mapped on this rank (regions[rank] = own region). Every rank must make
 * the same sequence of calls with the same n; calls on one rank must be
 * stream-ordered. No multicast objects, no collective library.
 * The reference has no multi-GPU path.
 */
#define CDQ_AR_MAX_RANKS 8
#define CDQ_AR_BLOCKS 16
typedef struct cdq_ipc_handle {
    uint8_t bytes[64];
} cdq_ipc_handle;
CDQ_API cdq_status cdq_ar_create(int64_t cap, void** region, cdq_ipc_handle* handle);
CDQ_API cdq_status cdq_ar_open(const cdq_ipc_handle* handle, void** peer_region);
CDQ_API cdq_status cdq_ar_close(void* peer_region);
CDQ_API cdq_status cdq_ar_destroy(void* region);
CDQ_API cdq_status cdq_allreduce_f32(void* const* regions, int32_t world, int32_t rank, int64_t cap,
                                     float* data, int64_t n, void* stream);
/* Sticky error code of the all-reduce on the current device (0: none; 1: a
 * peer's flag did not arrive within the wait limit). Reading does not reset
 * it; cdq_ar_clear_error does. After error 1 the ranks' epochs and staging
 * parities are out of step: every rank must destroy its region and create a
 * new one (zeroed pads and epochs) and exchange handles again before the
 * next cdq_allreduce_f32. */
CDQ_API cdq_status cdq_ar_error(int32_t* code);
CDQ_API cdq_status cdq_ar_clear_error(void);
/* Polls of a peer's flag before a wait gives up (process-wide, read at each
 * cdq_allreduce_f32 call; default 2^24, 1 <= polls < 2^32). A short limit
 * lets a test see the give-up path without a peer. */
CDQ_API cdq_status cdq_ar_set_spin_limit(int64_t polls);

/*
 * Device-side ingest of a reference-format pack: q [rows*cols/32][32] lattice
 * indices, scales_f8 [rows*cols/32] e4m3fn bytes, ridx [n_res] strictly
 * ascending flat indices (int64) and rval [n_res] bf16 bits, all in device
 * memory (for example the arrays of a .cdq file copied to the GPU), into the
 * device buffers of `out` (sized by cdq_get_sizes with n_res <= max_res).
 * Byte-identical to cdq_host_from_reference; three launches on `stream`, no
 * temporary memory. *error (device int32, zeroed by the caller) becomes 1 on
 * malformed input (an index >= n_states, residual positions out of range or
 * not ascending), in which case the pack is incomplete.
 * Replaces the per-tile Python parse of the loader (code/cdq_loader.py:79-87)
 * and CDQLinear's buffer set-up (code/cdq_lrr_qwen05.py:155-166).
 */
CDQ_API cdq_status cdq_pack_from_reference_device(int32_t rows, int32_t cols, int32_t n_states,
                                                  const uint8_t* q, const uint8_t* scales_f8,
                                                  const int64_t* ridx, const uint16_t* rval, int64_t n_res,
                                                  cdq_packed* out, int32_t* error, void* stream);

/*
 * Persistent decode step: one cooperative launch (one CTA per SM, all
 * resident) runs a whole batch-1 greedy token of a Qwen2-style decoder with
 * CDQ projections: per layer the residual add + RMSNorm, q/k/v (with biases),
 * rotary embedding + cache append + grouped-query attention, o_proj, the
 * second add + RMSNorm, gate/up, SiLU(gate) * up, down_proj; then the final
 * norm, the tied bf16 lm_head with its argmax, and the token advance
 * (tokens[count] = token, ids = token, pos + 1, count + 1), with grid-wide
 * barriers between dependent steps. Every operation computes exactly what the
 * one-kernel-per-operation step computes (cdq_embed_rmsnorm, cdq_add_rmsnorm,
 * cdq_linear_grouped, cdq_attn_decode, cdq_silu_mul, cdq_lm_head_argmax,
 * cdq_decode_advance), bit for bit. Replaces the reference's generate loop
 * step (code/cdq_lrr_qwen05.py:335-340: one HF forward of the patched model).
 */
typedef struct cdq_step_layer {
    /* m = 1 jobs: w, bias, workspace as for cdq_linear; y must be the model's
     * buffer of that projection (q, k, v, o, g, u, dn below); x a valid
     * activation buffer as for cdq_linear (not read: the persistent kernel
     * keeps each projection group's input in shared memory); out_f32 = 0.
     * All seven of one lattice size. */
    cdq_gemv_job q, k, v, o, gate, up, down;
    const uint16_t* ln1;  /* input_layernorm weight [hidden] */
    const uint16_t* ln2;  /* post_attention_layernorm weight [hidden] */
    uint16_t* k_cache;    /* [kv_heads, max_len, 64] bf16, 16-byte aligned */
    uint16_t* v_cache;
} cdq_step_layer;

typedef struct cdq_step_model {
    int32_t layers, hidden, heads, kv_heads, head_dim, inter, max_len, token_cap;
    int64_t vocab;
    float eps, scale;                  /* RMSNorm epsilon, attention scale */
    const uint16_t* embed;             /* [vocab, hidden] */
    const uint16_t* norm_w;            /* final norm weight [hidden] */
    const uint16_t* lm_w;              /* [vocab, hidden], 16-byte aligned */
    const uint16_t* cos_t;             /* [max_len, 64] rotary tables */
    const uint16_t* sin_t;
    int32_t* pos;                      /* the step's position (device) */
    int64_t* ids;                      /* the step's input token */
    int64_t* tokens;                   /* [token_cap] generated tokens */
    int32_t* count;                    /* tokens generated so far */
    uint64_t* best;                    /* argmax key, zero between steps */
    int64_t* next;                     /* the step's greedy token */
    uint16_t* logits;                  /* NULL or [vocab] bf16 */
    uint16_t* h0;                      /* two hidden-state buffers [hidden] */
    uint16_t* h1;
    uint16_t *q, *k, *v, *att, *o, *g, *u, *dn; /* projection inputs and outputs */
} cdq_step_model;

/* Bytes of device memory the step's table takes for `layers` layers on the
 * current device (it holds per-SM residual stage descriptors). */
CDQ_API cdq_status cdq_step_table_bytes(int32_t layers, int64_t* bytes);
/* Checks the model and writes its table to `table` (device memory of
 * cdq_step_table_bytes, 256-byte aligned; synchronous copy). The table holds
 * pointers: every buffer must outlive it. CDQ_ERR_UNSUPPORTED when the shapes
 * do not fit the kernel (head_dim != 64, more heads than SMs, buffers beyond
 * the shared window), CDQ_ERR_SHAPE on projection shapes that do not match the
 * model. */
CDQ_API cdq_status cdq_step_prepare(const cdq_step_model* model, const cdq_step_layer* layers, void* table);
/* One token on `stream` (capturable in a CUDA graph). n_states: the lattice
 * size the table was prepared with. */
CDQ_API cdq_status cdq_decode_step(const void* table, int32_t n_states, void* stream);
/* The step's sticky error word (0: none; 1: a grid barrier gave up; 2: a
 * weight copy never landed; 3: the table was prepared for another lattice
 * size); synchronous read. cdq_step_reset clears it and the barrier state. */
CDQ_API cdq_status cdq_step_error(const void* table, int32_t* code);
CDQ_API cdq_status cdq_step_reset(void* table, void* stream);

/*
 * Validation of a device pack that did not come from this library's
 * converters or quantizer (a saved state dict, a pack built elsewhere):
 * adds to *bad (device int32, zeroed by the caller) one per lane whose 26-state
 * pair codes exceed 728, one per CSR bound out of order (bounds must start at
 * 0, never decrease and end at n_res) and one per residual entry whose column
 * is >= cols. The linear kernels trust the pack they are given; a pack with
 * *bad != 0 must not be used. Up to two launches on `stream`.
 * Guards the reference's CDQLinear buffer load (code/cdq_lrr_qwen05.py:155-166,
 * via load_state_dict) when the buffers are in this library's own layout.
 */
CDQ_API cdq_status cdq_check_device_pack(const cdq_packed* pack, int32_t* bad, void* stream);

/*
 * Quality statistics on the device (the reference's report after quantizing,
 * code/run_any_model.py:89-110): out[0..3] (device float64) = sum (a-b)^2,
 * sum a*b, sum a^2, sum b^2 over n values of a and b (dtype 0: bf16 bits,
 * 1: float32), from which the caller forms MSE and cosine (weights vs w_hat,
 * or baseline vs quantized logits). workspace: >= 32 KiB of device memory for
 * the block partial sums, added in block order (deterministic).
 */
CDQ_API cdq_status cdq_compare_stats(const void* a, const void* b, int64_t n, int32_t dtype, double* out,
                                     double* workspace, int64_t workspace_bytes, void* stream);

/*
 * Batch-1 decode-step kernels around the fused linear, for a Qwen2-style
 * decoder layer (the reference runs HF's Qwen2 modules around CDQLinear,
 * code/cdq_lrr_qwen05.py:300-330; these replace Qwen2RMSNorm, the rotary
 * embedding, the static-cache update, attention and Qwen2MLP's act_fn(gate)*up
 * with the same bf16 rounding steps). All tensors bf16 bit patterns on the
 * device, enqueued on `stream`.
 *   cdq_add_rmsnorm: h = h + delta (if delta), out = w * norm(h); n <= 1 block.
 *   cdq_attn_decode: q [n_heads*64], k, v [n_kv*64]; cos_t/sin_t [max_len][64];
 *     *pos (device int32) the step's position; k_cache/v_cache [n_kv][max_len][64]
 *     (HF StaticCache layout, batch 1), the step's k and v written at *pos;
 *     out [n_heads*64]. head_dim must be 64.
 *   cdq_silu_mul: out = silu(g) * u.
 *   cdq_decode_advance: tokens[*count] = *next (if *count < cap), *ids = *next,
 *     ++*pos, ++*count: the step's greedy token feeds the next step on the device.
 */
CDQ_API cdq_status cdq_add_rmsnorm(uint16_t* h, const uint16_t* delta, const uint16_t* w, float eps,
                                   uint16_t* out, int32_t n, void* stream);
CDQ_API cdq_status cdq_attn_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                   const uint16_t* cos_t, const uint16_t* sin_t, const int32_t* pos,
                                   uint16_t* k_cache, uint16_t* v_cache, int32_t max_len, int32_t n_heads,
                                   int32_t n_kv, int32_t head_dim, float scale, uint16_t* out, void* stream);
CDQ_API cdq_status cdq_silu_mul(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n, void* stream);
CDQ_API cdq_status cdq_decode_advance(const int64_t* next, int64_t* ids, int64_t* tokens, int32_t* pos,
                                      int32_t* count, int32_t cap, void* stream);
/*
 *   cdq_embed_rmsnorm: h = table[*ids] (embedding row, a zero row for an id
 *     outside [0, vocab)), out = w * norm(h): the embedding lookup and the
 *     first layer's input norm in one launch.
 *   cdq_lm_head_argmax: logits[r] = bf16(x . w[r]) for the vocab rows of the
 *     bf16 lm_head w [vocab][n] (fp32 accumulation; logits may be NULL), and
 *     *next = their argmax (first index among equal values, NaN above every
 *     number: torch.argmax on the bf16 logits). best: device uint64, zero
 *     before the first call; the call leaves it zero. n % 8 == 0, n <= 16384.
 *     Replaces the tied lm_head F.linear and argmax of the reference's greedy
 *     generate (code/cdq_lrr_qwen05.py:335-340).
 * All of these kernels, and the fused linear's, are launched programmatically
 * dependent on their predecessor on the stream (each waits for it before
 * touching data), so consecutive launches overlap their launch latency.
 */
CDQ_API cdq_status cdq_embed_rmsnorm(const int64_t* ids, const uint16_t* table, int64_t vocab, uint16_t* h,
                                     const uint16_t* w, float eps, uint16_t* out, int32_t n, void* stream);
CDQ_API cdq_status cdq_lm_head_argmax(const uint16_t* w, const uint16_t* x, int32_t vocab, int32_t n,
                                      uint16_t* logits, uint64_t* best, int64_t* next, void* stream);

/*
 * Several rows or positions at once, for the speculative verify pass (k + 1
 * consecutive positions of one sequence); every row gets exactly the
 * arithmetic of the single-row call, so a verify pass reproduces sequential
 * decode steps bit for bit.
 *   cdq_add_rmsnorm_rows / cdq_embed_rmsnorm_rows: rows vectors of n (ids:
 *     rows tokens).
 *   cdq_lm_head_argmax_rows: m <= 8 activation rows x [m][n] -> logits
 *     [m][vocab] (or NULL), next[m]; best: m device uint64 keys, zero before
 *     the first call and left zero.
 *   cdq_attn_decode_multi: n_q <= 64 queries at positions *pos .. *pos+n_q-1
 *     (q [n_q][n_heads*64], k, v [n_q][n_kv*64], out [n_q][n_heads*64]): the
 *     keys and values of all n_q positions are appended to the cache first,
 *     then each query attends over positions 0..its own, as cdq_attn_decode
 *     does for one.
 * The reference decodes one token per step (code/cdq_lrr_qwen05.py:335-340);
 * the draft/verify use of its two lattices follows its README's description
 * of the 16-state tier.
 */
CDQ_API cdq_status cdq_add_rmsnorm_rows(uint16_t* h, const uint16_t* delta, const uint16_t* w, float eps,
                                        uint16_t* out, int32_t n, int32_t rows, void* stream);
CDQ_API cdq_status cdq_embed_rmsnorm_rows(const int64_t* ids, const uint16_t* table, int64_t vocab, uint16_t* h,
                                          const uint16_t* w, float eps, uint16_t* out, int32_t n, int32_t rows,
                                          void* stream);
CDQ_API cdq_status cdq_lm_head_argmax_rows(const uint16_t* w, const uint16_t* x, int32_t vocab, int32_t n,
                                           int32_t m, uint16_t* logits, uint64_t* best, int64_t* next,
                                           void* stream);
CDQ_API cdq_status cdq_attn_decode_multi(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                         const uint16_t* cos_t, const uint16_t* sin_t, const int32_t* pos,
                                         uint16_t* k_cache, uint16_t* v_cache, int32_t max_len, int32_t n_heads,
                                         int32_t n_kv, int32_t head_dim, float scale, uint16_t* out, int32_t n_q,
                                         void* stream);

/*
 * Bit-exact w_hat [rows, cols] bf16 from a device pack.
 * Replaces dequantize, code/cdq_lrr_qwen05.py:141-152, and
 * CDQLinear.dequant_weight, code/cdq_lrr_qwen05.py:188-194.
 */
CDQ_API cdq_status cdq_dequant(const cdq_packed* w, uint16_t* w_hat, void* stream);

/* Diagnostics of one cdq_quantize call, written to device memory. */
typedef struct cdq_quant_info {
    int64_t n_res;          /* residual count (<= max_res) */
    int64_t k;              /* max(1, round(numel * stc_frac)) */
    float threshold;        /* saliency quantile */
    int32_t topk_fallback;  /* 1 if more than 2k weights reached the threshold */
    int64_t mask_count;     /* weights with saliency >= threshold */
} cdq_quant_info;

/*
 * GPU tile quantizer: bf16 weight [rows, cols] (device) -> device pack.
 * Bit-exact with quantize_cdq_lrr, code/cdq_lrr_qwen05.py:63-133 (and its
 * packer twin code/cdq_pack.py:283-305, which lacks the top-k tie guard):
 * sigma = max|w| as float8 e4m3fn, unbiased float64-Welford tile variance,
 * saliency |w|*(var+1e-6), linear quantile threshold at 1 - stc_frac,
 * top-k fallback on severe ties (lowest flat indices win ties), nearest
 * lattice centroid of w / sigma_q (first index on ties).
 * out: buffers sized by cdq_get_sizes (res_ent / res_q hold max_res entries);
 * out->n_res is not touched (read info->n_res). info: device memory.
 * workspace: quantize_workspace_bytes of device memory (no zeroing needed).
 */
CDQ_API cdq_status cdq_quantize(const uint16_t* w, int32_t rows, int32_t cols, int32_t n_states,
                                double stc_frac, cdq_packed* out, cdq_quant_info* info,
                                void* workspace, size_t workspace_bytes, void* stream);

/*
 * cdq_quantize with options. flags: 0, or CDQ_QUANT_NO_TOPK_GUARD to quantize
 * as the reference packer CLI does (code/cdq_pack.py:279-291: the same steps
 * without the top-k tie guard of code/cdq_lrr_qwen05.py:93-96, so every weight
 * whose saliency reaches the threshold becomes a residual; that can be every
 * weight, e.g. an all-zero tensor). res_capacity: the residual entries
 * out->res_ent / out->res_q hold (cdq_get_sizes' max_res suffices with the
 * guard; rows * cols always suffices). Entries beyond the capacity are not
 * written; info->n_res always reports the full count, so n_res > res_capacity
 * means the pack is incomplete and the call must be repeated with larger
 * buffers.
 */
#define CDQ_QUANT_NO_TOPK_GUARD 1
CDQ_API cdq_status cdq_quantize_ex(const uint16_t* w, int32_t rows, int32_t cols, int32_t n_states,
                                   double stc_frac, int32_t flags, int64_t res_capacity, cdq_packed* out,
                                   cdq_quant_info* info, void* workspace, size_t workspace_bytes,
                                   void* stream);

/*
 * Bit packers of the .cdq tile records (host memory, n_tiles tiles or count
 * residuals per call), byte-exact with the reference's:
 *   cdq_pack_tile_indices / cdq_unpack_tile_indices: q [n_tiles][32] <-> 20
 *     bytes per tile (26 states: 5 bits per index, LSB first; pack_5bit_row /
 *     unpack_5bit_row, code/cdq_pack.py:50-64) or 16 (16 states: two indices
 *     per byte, the even one in the low nibble; pack_indices_nibble /
 *     unpack_nibble_row, code/cdq_pack.py:67-81). Indices are masked to 5 or
 *     4 bits.
 *   cdq_pack_residual_stream / cdq_unpack_residual_stream: count residuals of
 *     one tile <-> ceil(21 * count / 8) bytes, each a 5-bit offset then the
 *     16 bf16 bits, LSB first (pack_residuals / unpack_residuals,
 *     code/cdq_pack.py:84-119).
 */
CDQ_API cdq_status cdq_pack_tile_indices(const uint8_t* q, int64_t n_tiles, int32_t n_states, uint8_t* out);
CDQ_API cdq_status cdq_unpack_tile_indices(const uint8_t* packed, int64_t n_tiles, int32_t n_states, uint8_t* q);
CDQ_API cdq_status cdq_pack_residual_stream(const uint8_t* offsets, const uint16_t* values, int64_t count,
                                            uint8_t* out);
CDQ_API cdq_status cdq_unpack_residual_stream(const uint8_t* packed, int64_t count, uint8_t* offsets,
                                              uint16_t* values);

/*
 * Host-side conversions between the reference's pack tensors and the device
 * layout. All pointers are HOST memory; synchronous.
 * Reference pack tensors (code/cdq_lrr_qwen05.py:121-133):
 *   quant_indices uint8 [n_tiles, 32] (row-major tile order),
 *   scales_f8 uint8 [n_tiles] (e4m3fn codes), residual_indices int64 [n_res]
 *   (flat, ascending), residual_values uint16 [n_res] (bf16 bits).
 * The loader (code/cdq_loader.py:94-105) holds the same data as q, the
 * decoded scales, offs (= residual_indices) and vals.
 */
CDQ_API cdq_status cdq_host_from_reference(int32_t rows, int32_t cols, int32_t n_states,
                                           const uint8_t* quant_indices, const uint8_t* scales_f8,
                                           const int64_t* residual_indices,
                                           const uint16_t* residual_values, int64_t n_res,
                                           cdq_packed* out_host);

CDQ_API cdq_status cdq_host_to_reference(const cdq_packed* in_host, uint8_t* quant_indices,
                                         uint8_t* scales_f8, int64_t* residual_indices,
                                         uint16_t* residual_values);

/*
 * .cdq file codec (host memory, synchronous), byte-exact with write_cdq /
 * read_cdq, code/cdq_pack.py:162-234, and the loader's parser,
 * code/cdq_loader.py:61-100. Layout: "CDQ1", u16 version (1: 26-state, 2:
 * 16-state), u16 tensor count, bf16 lattice; per tensor u16 name length,
 * name, u32 rows, u32 cols, u32 n_tiles; per tile u8 scale, u8 residual
 * count, 20 or 16 index bytes, residual stream of ceil(21*count/8) bytes.
 */
typedef struct cdq_file_tensor {
    char name[256];
    int32_t rows;
    int32_t cols;
    int64_t n_tiles;
    int64_t n_res;
    int64_t record_offset;   /* byte offset of the first tile record */
    int64_t record_bytes;    /* bytes of all tile records */
} cdq_file_tensor;

/* Parses the header and tensor table. *n_states gets 26 or 16. At most
 * max_tensors entries are written; *n_tensors gets the file's count. */
CDQ_API cdq_status cdq_file_scan(const uint8_t* data, int64_t len, int32_t* n_states,
                                 cdq_file_tensor* tensors, int32_t max_tensors, int32_t* n_tensors);

/* Decodes one scanned tensor into reference pack tensors (sizes from t). */
CDQ_API cdq_status cdq_file_decode(const uint8_t* data, int64_t len, int32_t n_states,
                                   const cdq_file_tensor* t, uint8_t* quant_indices,
                                   uint8_t* scales_f8, int64_t* residual_indices,
                                   uint16_t* residual_values);

/*
 * .cdq tile records decoded on the device. cdq_file_checkpoints (host) walks
 * one tensor's records (a tensor of cdq_file_scan) and writes, for every span
 * of `every` tiles, the span's byte offset from record_offset and its first
 * residual index (ceil(n_tiles / every) entries each). cdq_file_decode_device
 * then unpacks every span in parallel from the records copied to the device
 * (the record_bytes bytes from record_offset) into the reference arrays
 * (q [n_tiles][32], scales_f8 [n_tiles], ridx / rval [n_res], as
 * cdq_file_decode writes them); *error (device int32, zeroed by the caller)
 * becomes 1 on malformed records. Replaces the per-tile Python loop of the
 * loader (code/cdq_loader.py:79-87) and read_cdq (code/cdq_pack.py:218-229).
 */
CDQ_API cdq_status cdq_file_checkpoints(const uint8_t* data, int64_t len, int32_t n_states,
                                        const cdq_file_tensor* t, int32_t every, int64_t* byte_off,
                                        int64_t* res_off);
CDQ_API cdq_status cdq_file_decode_device(const uint8_t* records, int64_t record_bytes, int32_t n_states,
                                          int64_t n_tiles, int64_t n_res, int32_t every,
                                          const int64_t* byte_off, const int64_t* res_off, uint8_t* q,
                                          uint8_t* scales_f8, int64_t* ridx, uint16_t* rval, int32_t* error,
                                          void* stream);


/* Encodes the header (magic, version, count, lattice) into out (capacity
 * cap); *written gets the byte count (8 + 52 or 8 + 32). */
CDQ_API cdq_status cdq_file_encode_header(int32_t n_states, int32_t n_tensors, uint8_t* out,
                                          int64_t cap, int64_t* written);

/* Encodes one tensor (name, dims, tile records) from reference pack tensors.
 * With out == NULL only *written (the required bytes) is computed. */
CDQ_API cdq_status cdq_file_encode_tensor(const char* name, int32_t rows, int32_t cols,
                                          int32_t n_states, const uint8_t* quant_indices,
                                          const uint8_t* scales_f8,
                                          const int64_t* residual_indices,
                                          const uint16_t* residual_values, int64_t n_res,
                                          uint8_t* out, int64_t cap, int64_t* written);

#ifdef __cplusplus
}
#endif

#endif /* CDQ_B200_H */
