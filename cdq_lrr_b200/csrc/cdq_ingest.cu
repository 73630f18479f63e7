// Device-side conversion of a reference-format pack (the dict of
// code/cdq_lrr_qwen05.py:121-133, as read from a .cdq file by
// code/cdq_loader.py:61-100) into the device layout, byte-identical to the
// host converter cdq_host_from_reference. Three launches, no host work on the
// data, no temporary memory:
//   1. units: one thread per (row block, tile-column pair, lane) builds the
//      lane's code words from the indices (every position with its lattice
//      index) and writes the lane's one scale byte of the unit; every byte of
//      the units buffer is written (zero codes and scale 0 outside the weight);
//   2. residuals: one thread per residual (flat indices strictly ascending, so
//      entry i of the row-major CSR is residual i): writes res_ent / res_q and
//      turns its element of the pair code into the residual symbol with one
//      XOR per touched word (pairs whose two elements are both residuals are
//      rewritten once, by the even element's thread; XORs on disjoint bit
//      fields of a word commute);
//   3. bucket bounds: one thread per (row, residual group) bucket finds its
//      first entry by binary search over the sorted residuals.
// Malformed input (an index >= n_states, residual positions out of range or
// not ascending) sets *error to 1; the pack is then incomplete.
//
// The reference arrays themselves can come from the .cdq bytes on the device
// too (cdq_file_decode_device): the file's tile records are variable-length,
// so a host pass over their count bytes (cdq_file_checkpoints) records where
// every span of tiles starts, and one thread per span unpacks it.
#include <cuda_runtime.h>

#include "cdq.h"
#include "cdq_common.cuh"

namespace {

using namespace cdq;

__device__ __forceinline__ uint32_t pair_code_d(int ns, uint32_t a, uint32_t b) {
    return ns == 26 ? a * 27u + b : (a & 0xFu) | ((b & 0xFu) << 4);
}

__global__ void ingest_units(Geometry g, int ns, const uint8_t* __restrict__ q, const uint8_t* __restrict__ sc,
                             uint8_t* __restrict__ units, int* __restrict__ error) {
    const int64_t n = g.r16 * g.kp * 32;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < n; id += (int64_t)gridDim.x * blockDim.x) {
        const int lane = (int)(id & 31);
        const int64_t unit = id >> 5, b16 = unit / g.kp, cp = unit - b16 * g.kp;
        uint32_t w[5] = {0u, 0u, 0u, 0u, 0u};
        bool bad = false;
        for (int s = 0; s < 16; ++s) {
            int ri, t, p;
            slot_pos(lane, s, &ri, &t, &p);
            const int64_t row = b16 * 16 + ri, c = cp * 2 + t;
            if (row >= g.rows || c >= g.kt) continue;
            const uint8_t* e = q + (row * g.kt + c) * 32 + 2 * p;
            const uint32_t a = e[0], b = e[1];
            bad |= a >= (uint32_t)ns || b >= (uint32_t)ns;
            const uint32_t code = pair_code_d(ns, a, b);
            if (ns == 26) {
                const int bit = 10 * s, wd = bit >> 5, off = bit & 31;
                w[wd] |= code << off;
                if (off > 22) w[wd + 1] |= code >> (32 - off);
            } else {
                w[s >> 2] |= (code & 0xFFu) << (8 * (s & 3));
            }
        }
        if (bad) atomicExch(error, 1);
        for (int wd = 0; wd < g.words; ++wd)
            *reinterpret_cast<uint32_t*>(units + word_offset(g, b16, cp, lane, wd)) = w[wd];
        const int ri = lane >> 1, t = lane & 1;
        const int64_t row = b16 * 16 + ri, c = cp * 2 + t;
        units[scale_offset(g, b16, cp, ri, t)] = row < g.rows && c < g.kt ? sc[row * g.kt + c] : (uint8_t)0;
    }
}

__global__ void ingest_residuals(Geometry g, int ns, const uint8_t* __restrict__ q, const int64_t* __restrict__ ridx,
                                 const uint16_t* __restrict__ rval, int64_t n_res, uint8_t* __restrict__ units,
                                 uint32_t* __restrict__ res_ent, uint8_t* __restrict__ res_q, int* __restrict__ error) {
    const int64_t numel = g.rows * g.cols;
    const uint32_t rs = ns == 26 ? (uint32_t)kResidualSym26 : (uint32_t)kResidualSym16;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_res; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t f = ridx[i];
        if (f < 0 || f >= numel || (i > 0 && ridx[i - 1] >= f)) {
            atomicExch(error, 1);
            continue;
        }
        const int64_t row = f / g.cols, col = f - row * g.cols;
        res_ent[i] = ((uint32_t)col << 16) | rval[i];
        res_q[i] = q[f];
        const int e = (int)(col & 31), half = e & 1;
        const bool nb = half ? (i > 0 && ridx[i - 1] == f - 1) : (i + 1 < n_res && ridx[i + 1] == f + 1);
        if (half && nb) continue;  // the even element's thread rewrites the pair
        const int64_t f0 = f - half;
        const uint32_t a = q[f0], b = q[f0 + 1];
        const uint32_t na = (!half || nb) ? rs : a, nbv = (half || nb) ? rs : b;
        const uint32_t delta = pair_code_d(ns, a, b) ^ pair_code_d(ns, na, nbv);
        int lane, slot;
        slot_of((int)(row & 15), (int)((col >> 5) & 1), e >> 1, &lane, &slot);
        const int64_t b16 = row >> 4, cp = col >> 6;
        if (ns == 26) {
            const int bit = 10 * slot, wd = bit >> 5, off = bit & 31;
            atomicXor(reinterpret_cast<unsigned int*>(units + word_offset(g, b16, cp, lane, wd)), delta << off);
            if (off > 22)
                atomicXor(reinterpret_cast<unsigned int*>(units + word_offset(g, b16, cp, lane, wd + 1)),
                          delta >> (32 - off));
        } else {
            atomicXor(reinterpret_cast<unsigned int*>(units + word_offset(g, b16, cp, lane, slot >> 2)),
                      (delta & 0xFFu) << (8 * (slot & 3)));
        }
    }
}

// bucket of residual i: (row, group of 32 tiles), row major
__device__ __forceinline__ int64_t bucket_of(const Geometry& g, int64_t f) {
    const int64_t row = f / g.cols, col = f - row * g.cols;
    return row * g.kg + (col >> 5) / kGroupTiles;
}

__global__ void ingest_bounds(Geometry g, const int64_t* __restrict__ ridx, int64_t n_res,
                              uint32_t* __restrict__ res_ptr) {
    const int64_t nb = g.r16 * 16 * g.kg;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b <= nb; b += (int64_t)gridDim.x * blockDim.x) {
        int64_t lo = 0, hi = n_res;  // first entry whose bucket >= b
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (bucket_of(g, ridx[mid]) < b) lo = mid + 1; else hi = mid;
        }
        res_ptr[b] = (uint32_t)lo;
    }
}

// Tile records of a .cdq tensor (code/cdq_pack.py:183-190): scale byte,
// residual count tc, 20 (5-bit LSB-first) or 16 (nibble) index bytes, then
// tc residuals of 21 bits (5-bit offset, 16-bit bf16) LSB-first. One thread per
// span of `every` tiles, from the span's checkpoint (byte offset within the
// records, first residual index); residuals of a tile sorted by offset.
__global__ void file_decode_spans(const uint8_t* __restrict__ rec, int64_t rec_bytes, int ns, int64_t n_tiles,
                                  int64_t n_res, int every, const int64_t* __restrict__ byte_off,
                                  const int64_t* __restrict__ res_off, uint8_t* __restrict__ q,
                                  uint8_t* __restrict__ sc, int64_t* __restrict__ ridx, uint16_t* __restrict__ rval,
                                  int* __restrict__ error) {
    const int64_t spans = (n_tiles + every - 1) / every;
    const int ib = ns == 26 ? 20 : 16;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < spans; c += (int64_t)gridDim.x * blockDim.x) {
        int64_t pos = byte_off[c], n = res_off[c];
        const int64_t k1 = (c + 1) * every < n_tiles ? (c + 1) * every : n_tiles;
        bool bad = false;
        for (int64_t k = c * every; k < k1 && !bad; ++k) {
            if (pos + 2 + ib > rec_bytes) {
                bad = true;
                break;
            }
            sc[k] = rec[pos];
            const int tc = rec[pos + 1];
            const uint8_t* in = rec + pos + 2;
            uint8_t* qk = q + k * 32;
            if (ns == 26) {
                for (int i = 0; i < 32; ++i) {
                    const int bit = 5 * i, by = bit >> 3, sh = bit & 7;
                    const uint32_t v = in[by] | (by + 1 < 20 ? (uint32_t)in[by + 1] << 8 : 0u);
                    const uint8_t s = (uint8_t)((v >> sh) & 0x1Fu);
                    bad |= s >= 26;
                    qk[i] = s;
                }
            } else {
                for (int i = 0; i < 16; ++i) {
                    qk[2 * i] = in[i] & 0xF;
                    qk[2 * i + 1] = in[i] >> 4;
                }
            }
            pos += 2 + ib;
            const int64_t bb = ((int64_t)tc * 21 + 7) / 8;
            if (tc > 32 || pos + bb > rec_bytes || n + tc > n_res) {
                bad = true;
                break;
            }
            int offs[32];
            uint16_t vals[32];
            for (int j = 0; j < tc; ++j) {
                uint32_t w[2] = {0u, 0u};
                for (int f = 0; f < 2; ++f) {
                    const int64_t p0 = 21LL * j + (f ? 5 : 0);
                    uint32_t v = 0;
                    for (int i = 0; i < 3; ++i) {
                        const int64_t by = (p0 >> 3) + i;
                        if (by < bb) v |= (uint32_t)rec[pos + by] << (8 * i);
                    }
                    w[f] = (v >> (p0 & 7)) & (f ? 0xFFFFu : 0x1Fu);
                }
                // insertion by offset (the packer writes them ascending)
                int at = j;
                while (at > 0 && offs[at - 1] > (int)w[0]) {
                    offs[at] = offs[at - 1];
                    vals[at] = vals[at - 1];
                    --at;
                }
                offs[at] = (int)w[0];
                vals[at] = (uint16_t)w[1];
            }
            for (int j = 0; j < tc; ++j) {
                bad |= j > 0 && offs[j] == offs[j - 1];
                ridx[n + j] = k * 32 + offs[j];
                rval[n + j] = vals[j];
            }
            n += tc;
            pos += bb;
        }
        const int64_t end_pos = c + 1 < spans ? byte_off[c + 1] : rec_bytes;
        const int64_t end_n = c + 1 < spans ? res_off[c + 1] : n_res;
        if (bad || pos != end_pos || n != end_n) atomicExch(error, 1);
    }
}

// Validation of a device pack from an untrusted source (a state dict, a file
// written by another build): one thread per (unit, lane) checks the lane's 16
// pair codes (26 states: at most 26 * 27 + 26 = 728, the last entry of the
// pair table the linear kernels index with the code); one thread per CSR
// bucket checks that the bounds start at 0, never decrease and end at n_res;
// one thread per entry checks its column against cols. Every malformed part
// adds one to *bad.
__global__ void check_units(Geometry g, const uint8_t* __restrict__ units, int* __restrict__ bad) {
    const int64_t n = g.r16 * g.kp * 32;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < n; id += (int64_t)gridDim.x * blockDim.x) {
        const int lane = (int)(id & 31);
        const int64_t unit = id >> 5, b16 = unit / g.kp, cp = unit - b16 * g.kp;
        uint32_t w[5];
        for (int wd = 0; wd < 5; ++wd)
            w[wd] = *reinterpret_cast<const uint32_t*>(units + word_offset(g, b16, cp, lane, wd));
        int n_bad = 0;
        for (int s = 0; s < 16; ++s) {
            const int bit = 10 * s, wd = bit >> 5, off = bit & 31;
            const uint64_t win = w[wd] | (wd + 1 < 5 ? (uint64_t)w[wd + 1] << 32 : 0ull);
            n_bad += ((uint32_t)(win >> off) & 0x3FFu) > 728u;
        }
        if (n_bad) atomicAdd(bad, 1);
    }
}

__global__ void check_csr(const uint32_t* __restrict__ res_ptr, int64_t buckets, const uint32_t* __restrict__ res_ent,
                          int64_t n_res, int32_t cols, int* __restrict__ bad) {
    const int64_t n = buckets > n_res ? buckets : n_res;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (i < buckets) {
            const uint32_t a = res_ptr[i], b = res_ptr[i + 1];
            if (b < a || (i == 0 && a != 0u) || (i == buckets - 1 && (int64_t)b != n_res)) atomicAdd(bad, 1);
        }
        if (i < n_res && (int32_t)(res_ent[i] >> 16) >= cols) atomicAdd(bad, 1);
    }
}

int grid_for(int64_t n, int threads) {
    const int64_t b = (n + threads - 1) / threads;
    return (int)(b < 1 ? 1 : (b > 65535 ? 65535 : b));
}

}  // namespace

extern "C" cdq_status cdq_pack_from_reference_device(int32_t rows, int32_t cols, int32_t n_states, const uint8_t* q,
                                                     const uint8_t* scales_f8, const int64_t* ridx,
                                                     const uint16_t* rval, int64_t n_res, cdq_packed* out,
                                                     int32_t* error, void* stream) {
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    if (rows <= 0 || cols <= 0 || cols % 32 || cols > CDQ_MAX_COLS) return CDQ_ERR_SHAPE;
    if (!q || !scales_f8 || !out || !out->units || !out->res_ptr || !error || n_res < 0 ||
        (n_res > 0 && (!ridx || !rval || !out->res_ent || !out->res_q)) || n_res >= (int64_t)UINT32_MAX)
        return CDQ_ERR_ARG;
    if ((uintptr_t)out->units % 16 || (uintptr_t)out->res_ptr % 4 || (n_res > 0 && (uintptr_t)ridx % 8))
        return CDQ_ERR_ARG;
    const Geometry g = geometry(rows, cols, n_states);
    cudaStream_t s = (cudaStream_t)stream;
    constexpr int kT = 256;
    ingest_units<<<grid_for(g.r16 * g.kp * 32, kT), kT, 0, s>>>(g, n_states, q, scales_f8, out->units, error);
    if (n_res > 0)
        ingest_residuals<<<grid_for(n_res, kT), kT, 0, s>>>(g, n_states, q, ridx, rval, n_res, out->units,
                                                             out->res_ent, out->res_q, error);
    ingest_bounds<<<grid_for(g.r16 * 16 * g.kg + 1, kT), kT, 0, s>>>(g, ridx, n_res, out->res_ptr);
    if (cudaGetLastError() != cudaSuccess) return CDQ_ERR_CUDA;
    out->rows = rows;
    out->cols = cols;
    out->n_states = n_states;
    out->n_res = n_res;
    return CDQ_OK;
}

extern "C" cdq_status cdq_file_decode_device(const uint8_t* records, int64_t record_bytes, int32_t n_states,
                                            int64_t n_tiles, int64_t n_res, int32_t every,
                                            const int64_t* byte_off, const int64_t* res_off, uint8_t* q,
                                            uint8_t* scales_f8, int64_t* ridx, uint16_t* rval, int32_t* error,
                                            void* stream) {
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    if (!records || record_bytes < 0 || n_tiles < 1 || n_res < 0 || every < 1 || !byte_off || !res_off || !q ||
        !scales_f8 || !error || (n_res > 0 && (!ridx || !rval)))
        return CDQ_ERR_ARG;
    const int64_t spans = (n_tiles + every - 1) / every;
    file_decode_spans<<<grid_for(spans, 128), 128, 0, (cudaStream_t)stream>>>(
        records, record_bytes, n_states, n_tiles, n_res, every, byte_off, res_off, q, scales_f8, ridx, rval, error);
    return cudaGetLastError() == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}

extern "C" cdq_status cdq_check_device_pack(const cdq_packed* pack, int32_t* bad, void* stream) {
    if (!pack || !bad || !pack->units || !pack->res_ptr || pack->n_res < 0 || (pack->n_res > 0 && !pack->res_ent))
        return CDQ_ERR_ARG;
    if (pack->n_states != 26 && pack->n_states != 16) return CDQ_ERR_STATES;
    if (pack->rows <= 0 || pack->cols <= 0 || pack->cols % 32 || pack->cols > CDQ_MAX_COLS) return CDQ_ERR_SHAPE;
    if ((uintptr_t)pack->units % 4 || (uintptr_t)pack->res_ptr % 4 || (uintptr_t)pack->res_ent % 4)
        return CDQ_ERR_ARG;
    const Geometry g = geometry(pack->rows, pack->cols, pack->n_states);
    cudaStream_t s = (cudaStream_t)stream;
    constexpr int kT = 256;
    if (pack->n_states == 26)
        check_units<<<grid_for(g.r16 * g.kp * 32, kT), kT, 0, s>>>(g, pack->units, bad);
    const int64_t buckets = g.r16 * 16 * g.kg;
    check_csr<<<grid_for(buckets > pack->n_res ? buckets : pack->n_res, kT), kT, 0, s>>>(
        pack->res_ptr, buckets, pack->res_ent, pack->n_res, pack->cols, bad);
    return cudaGetLastError() == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}
