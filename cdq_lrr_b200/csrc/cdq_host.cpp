// Host-side part of the C ABI: sizes, conversion between the reference's
// pack tensors and the device layout, and the .cdq file codec.
//
// Reference interfaces restated here (CDQ-LRR project paths):
//   pack tensors      code/cdq_lrr_qwen05.py:121-133 (quantize_cdq_lrr's dict)
//   5-bit / nibble    code/cdq_pack.py:50-88 (LSB-first; even lane = low nibble)
//   residual stream   code/cdq_pack.py:91-119 (5-bit offset + 16-bit value,
//                     LSB-first, ceil(21*count/8) bytes per tile)
//   file layout       code/cdq_pack.py:12-18, writer :162-190, reader :193-234,
//                     loader parser code/cdq_loader.py:61-100
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "cdq.h"
#include "cdq_common.cuh"

using namespace cdq;

namespace {

int64_t residual_budget(int64_t numel, double stc_frac) {
    // k = max(1, round(numel * stc_frac)) with Python's round-half-even.
    double k = std::nearbyint((double)numel * stc_frac);
    int64_t ki = std::max<int64_t>(1, (int64_t)k);
    return std::min<int64_t>(2 * ki, numel);
}

inline int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

cdq_status check_shape(int32_t rows, int32_t cols, int32_t n_states) {
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    if (rows <= 0 || cols <= 0 || cols % 32 != 0 || cols > CDQ_MAX_COLS) return CDQ_ERR_SHAPE;
    return CDQ_OK;
}

// Slot code of two symbols, and its inverse.
inline uint32_t pair_code(int n_states, uint32_t a, uint32_t b) {
    return n_states == 26 ? a * 27u + b : (a & 0xFu) | ((b & 0xFu) << 4);
}
inline void pair_syms(int n_states, uint32_t code, uint8_t* a, uint8_t* b) {
    if (n_states == 26) {
        *a = (uint8_t)(code / 27u);
        *b = (uint8_t)(code % 27u);
    } else {
        *a = (uint8_t)(code & 0xFu);
        *b = (uint8_t)(code >> 4);
    }
}
// Place / read slot q of a lane's word stream.
inline void put_slot(int n_states, uint32_t* w, int q, uint32_t code) {
    if (n_states == 26) {
        const int bit = 10 * q, wd = bit >> 5, off = bit & 31;
        w[wd] |= code << off;
        if (off > 22) w[wd + 1] |= code >> (32 - off);
    } else {
        w[q >> 2] |= (code & 0xFFu) << (8 * (q & 3));
    }
}
inline uint32_t get_slot(int n_states, const uint32_t* w, int q) {
    if (n_states == 26) {
        const int bit = 10 * q, wd = bit >> 5, off = bit & 31;
        uint64_t win = w[wd] | (wd + 1 < 5 ? (uint64_t)w[wd + 1] << 32 : 0);
        return (uint32_t)(win >> off) & 0x3FFu;
    }
    return (w[q >> 2] >> (8 * (q & 3))) & 0xFFu;
}

// ---- little-endian byte stream helpers for the .cdq codec ----
struct Reader {
    const uint8_t* p;
    int64_t len, pos;
    bool need(int64_t n) const { return n >= 0 && pos + n <= len; }
    uint16_t u16() { uint16_t v = (uint16_t)(p[pos] | (p[pos + 1] << 8)); pos += 2; return v; }
    uint32_t u32() {
        uint32_t v = (uint32_t)p[pos] | ((uint32_t)p[pos + 1] << 8) | ((uint32_t)p[pos + 2] << 16) |
                     ((uint32_t)p[pos + 3] << 24);
        pos += 4;
        return v;
    }
};

inline int64_t blob_bytes(int64_t tc) { return (tc * 21 + 7) / 8; }
inline int idx_bytes(int n_states) { return n_states == 26 ? 20 : 16; }

void unpack_indices(const uint8_t* in, int n_states, uint8_t* q) {
    if (n_states == 26) {
        // 32 x 5 bits LSB-first over 20 bytes
        for (int i = 0; i < 32; ++i) {
            int bit = 5 * i, by = bit >> 3, sh = bit & 7;
            uint32_t v = in[by] | (by + 1 < 20 ? (uint32_t)in[by + 1] << 8 : 0u);
            q[i] = (uint8_t)((v >> sh) & 0x1Fu);
        }
    } else {
        for (int i = 0; i < 16; ++i) {
            q[2 * i] = in[i] & 0xF;
            q[2 * i + 1] = in[i] >> 4;
        }
    }
}

void pack_indices(const uint8_t* q, int n_states, uint8_t* out) {
    if (n_states == 26) {
        memset(out, 0, 20);
        for (int i = 0; i < 32; ++i) {
            int bit = 5 * i, by = bit >> 3, sh = bit & 7;
            uint32_t v = (uint32_t)(q[i] & 0x1F) << sh;
            out[by] |= (uint8_t)v;
            if (sh > 3) out[by + 1] |= (uint8_t)(v >> 8);
        }
    } else {
        for (int i = 0; i < 16; ++i) out[i] = (uint8_t)((q[2 * i] & 0xF) | ((q[2 * i + 1] & 0xF) << 4));
    }
}

// Reads `nbits` (<= 16) bits at bit position `pos` of a little-endian stream.
inline uint32_t get_bits(const uint8_t* b, int64_t nbytes, int64_t pos, int nbits) {
    uint32_t v = 0;
    for (int i = 0; i < 3; ++i) {
        int64_t by = (pos >> 3) + i;
        if (by < nbytes) v |= (uint32_t)b[by] << (8 * i);
    }
    return (v >> (pos & 7)) & ((1u << nbits) - 1u);
}

inline void put_bits(uint8_t* b, int64_t pos, uint32_t val, int nbits) {
    for (int i = 0; i < nbits; ++i, ++pos)
        if ((val >> i) & 1u) b[pos >> 3] |= (uint8_t)(1u << (pos & 7));
}

}  // namespace

extern "C" {

cdq_status cdq_get_sizes(int32_t rows, int32_t cols, int32_t n_states, double stc_frac,
                         int32_t max_batch, cdq_sizes* out) {
    if (!out) return CDQ_ERR_ARG;
    cdq_status st = check_shape(rows, cols, n_states);
    if (st) return st;
    if (max_batch < 1 || max_batch > CDQ_MAX_BATCH) return CDQ_ERR_ARG;
    if (!(stc_frac >= 0.0 && stc_frac <= 1.0)) return CDQ_ERR_ARG;
    Geometry g = geometry(rows, cols, n_states);
    int64_t numel = (int64_t)rows * cols;
    int64_t n_tiles = numel / 32;
    out->row_blocks = g.r16;
    out->tile_pairs = g.kp;
    out->res_groups = g.kg;
    out->units_bytes = g.r16 * g.kp * g.unit;
    out->res_ptr_count = g.r16 * g.kg * 16 + 1;
    out->max_res = residual_budget(numel, stc_frac);
    // streaming-path group sums or tile-path prepared activations, whichever is larger
    out->linear_workspace_bytes = linear_workspace_need(g, max_batch);
    // tile variance f32, tie counts u32 (n_tiles + 1), histograms, scalars
    out->quantize_workspace_bytes = align256(n_tiles * 4) + align256((n_tiles + 1) * 4) +
                                    align256(4 * 2048 * 4) + align256(1024);
    return CDQ_OK;
}

const char* cdq_version(void) { return "cdq-b200 1.1 (sm_100a)"; }

cdq_status cdq_host_from_reference(int32_t rows, int32_t cols, int32_t n_states,
                                   const uint8_t* q, const uint8_t* scales_f8,
                                   const int64_t* ridx, const uint16_t* rval, int64_t n_res,
                                   cdq_packed* out) {
    cdq_status st = check_shape(rows, cols, n_states);
    if (st) return st;
    if (!q || !scales_f8 || !out || !out->units || !out->res_ptr ||
        (n_res > 0 && (!ridx || !rval || !out->res_ent || !out->res_q)) || n_res < 0)
        return CDQ_ERR_ARG;
    Geometry g = geometry(rows, cols, n_states);
    const int64_t numel = (int64_t)rows * cols, n_tiles = numel / 32;
    const uint8_t res_sym = n_states == 26 ? kResidualSym26 : kResidualSym16;

    // residual positions: strictly ascending flat indices
    std::vector<uint32_t> mask(n_tiles, 0u);
    for (int64_t i = 0; i < n_res; ++i) {
        int64_t f = ridx[i];
        if (f < 0 || f >= numel || (i && f <= ridx[i - 1])) return CDQ_ERR_ARG;
        mask[f / 32] |= 1u << (f % 32);
    }
    for (int64_t t = 0; t < n_tiles; ++t)
        for (int e = 0; e < 32; ++e)
            if (q[t * 32 + e] >= n_states) return CDQ_ERR_ARG;
    auto sym = [&](int64_t t, int e) -> uint32_t {
        return ((mask[t] >> e) & 1u) ? res_sym : q[t * 32 + e];
    };
    memset(out->units, 0, (size_t)(g.r16 * g.kp * g.unit));
    for (int64_t b16 = 0; b16 < g.r16; ++b16) {
        for (int64_t cp = 0; cp < g.kp; ++cp) {
            for (int lane = 0; lane < 32; ++lane) {
                uint32_t w[5] = {0, 0, 0, 0, 0};
                for (int s = 0; s < 16; ++s) {
                    int ri, t, p;
                    slot_pos(lane, s, &ri, &t, &p);
                    const int64_t row = b16 * 16 + ri, c = cp * 2 + t;
                    if (row >= rows || c >= g.kt) continue;
                    const int64_t tile = row * g.kt + c;
                    put_slot(n_states, w, s, pair_code(n_states, sym(tile, 2 * p), sym(tile, 2 * p + 1)));
                }
                for (int wd = 0; wd < g.words; ++wd) memcpy(out->units + word_offset(g, b16, cp, lane, wd), &w[wd], 4);
            }
            for (int ri = 0; ri < 16; ++ri)
                for (int t = 0; t < 2; ++t) {
                    const int64_t row = b16 * 16 + ri, c = cp * 2 + t;
                    if (row < rows && c < g.kt) out->units[scale_offset(g, b16, cp, ri, t)] = scales_f8[row * g.kt + c];
                }
        }
    }
    // residual CSR: bucket (row, group), row major
    const int64_t nb = g.r16 * g.kg * 16;
    std::vector<int64_t> cnt(nb + 1, 0);
    auto bucket_of = [&](int64_t f) {
        const int64_t row = f / cols, col = f % cols;
        return bucket_index(g, row / 16, (col / 32) / kGroupTiles, (int)(row % 16));
    };
    for (int64_t i = 0; i < n_res; ++i) cnt[bucket_of(ridx[i])]++;
    int64_t run = 0;
    for (int64_t b = 0; b < nb; ++b) {
        out->res_ptr[b] = (uint32_t)run;
        int64_t c = cnt[b];
        cnt[b] = run;
        run += c;
    }
    out->res_ptr[nb] = (uint32_t)run;
    for (int64_t i = 0; i < n_res; ++i) {
        const int64_t pos = cnt[bucket_of(ridx[i])]++;
        out->res_ent[pos] = ((uint32_t)(ridx[i] % cols) << 16) | rval[i];
        out->res_q[pos] = q[ridx[i]];
    }
    out->rows = rows;
    out->cols = cols;
    out->n_states = n_states;
    out->n_res = n_res;
    return CDQ_OK;
}

cdq_status cdq_host_to_reference(const cdq_packed* in, uint8_t* q, uint8_t* scales_f8,
                                 int64_t* ridx, uint16_t* rval) {
    if (!in || !q || !scales_f8 || !in->units || !in->res_ptr) return CDQ_ERR_ARG;
    cdq_status st = check_shape(in->rows, in->cols, in->n_states);
    if (st) return st;
    if (in->n_res > 0 && (!ridx || !rval || !in->res_ent || !in->res_q)) return CDQ_ERR_ARG;
    const int ns = in->n_states;
    Geometry g = geometry(in->rows, in->cols, ns);
    for (int64_t b16 = 0; b16 < g.r16; ++b16) {
        for (int64_t cp = 0; cp < g.kp; ++cp) {
            for (int lane = 0; lane < 32; ++lane) {
                uint32_t w[5] = {0, 0, 0, 0, 0};
                for (int wd = 0; wd < g.words; ++wd) memcpy(&w[wd], in->units + word_offset(g, b16, cp, lane, wd), 4);
                for (int s = 0; s < 16; ++s) {
                    int ri, t, p;
                    slot_pos(lane, s, &ri, &t, &p);
                    const int64_t row = b16 * 16 + ri, c = cp * 2 + t;
                    if (row >= in->rows || c >= g.kt) continue;
                    const int64_t tile = row * g.kt + c;
                    pair_syms(ns, get_slot(ns, w, s), &q[tile * 32 + 2 * p], &q[tile * 32 + 2 * p + 1]);
                }
            }
            for (int ri = 0; ri < 16; ++ri)
                for (int t = 0; t < 2; ++t) {
                    const int64_t row = b16 * 16 + ri, c = cp * 2 + t;
                    if (row < in->rows && c < g.kt) scales_f8[row * g.kt + c] = in->units[scale_offset(g, b16, cp, ri, t)];
                }
        }
    }
    // residual positions: the quantizer's index, and the flat residual list in
    // row-major order (rows ascending, then groups, then columns)
    int64_t n = 0;
    for (int64_t row = 0; row < in->rows; ++row) {
        for (int64_t gr = 0; gr < g.kg; ++gr) {
            const int64_t b = bucket_index(g, row / 16, gr, (int)(row % 16));
            for (uint32_t e = in->res_ptr[b]; e < in->res_ptr[b + 1]; ++e) {
                if (n >= in->n_res) return CDQ_ERR_FORMAT;
                const int64_t f = row * in->cols + (in->res_ent[e] >> 16);
                q[f] = in->res_q[e];
                ridx[n] = f;
                rval[n] = (uint16_t)(in->res_ent[e] & 0xFFFFu);
                ++n;
            }
        }
    }
    return n == in->n_res ? CDQ_OK : CDQ_ERR_FORMAT;
}

cdq_status cdq_file_scan(const uint8_t* data, int64_t len, int32_t* n_states,
                         cdq_file_tensor* tensors, int32_t max_tensors, int32_t* n_tensors) {
    if (!data || !n_states || !n_tensors || len < 0 || max_tensors < 0 ||
        (max_tensors > 0 && !tensors))
        return CDQ_ERR_ARG;
    Reader r{data, len, 0};
    if (!r.need(8) || memcmp(data, "CDQ1", 4) != 0) return CDQ_ERR_FORMAT;
    r.pos = 4;
    uint16_t ver = r.u16(), n = r.u16();
    if (ver != 1 && ver != 2) return CDQ_ERR_FORMAT;
    const int ns = ver == 1 ? 26 : 16;
    const int ib = idx_bytes(ns);
    if (!r.need(ver == 1 ? 52 : 32)) return CDQ_ERR_FORMAT;
    r.pos += ver == 1 ? 52 : 32;
    for (int i = 0; i < n; ++i) {
        if (!r.need(2)) return CDQ_ERR_FORMAT;
        uint16_t nl = r.u16();
        if (!r.need(nl + 12)) return CDQ_ERR_FORMAT;
        cdq_file_tensor t;
        memset(&t, 0, sizeof t);
        memcpy(t.name, data + r.pos, std::min<int>(nl, 255));
        r.pos += nl;
        uint32_t rows = r.u32(), cols = r.u32(), nt = r.u32();
        if (rows == 0 || cols == 0 || cols % 32 || (int64_t)rows * cols != (int64_t)nt * 32 ||
            rows > 0x7FFFFFFFu || cols > CDQ_MAX_COLS || nl > 255)
            return CDQ_ERR_FORMAT;
        t.rows = (int32_t)rows;
        t.cols = (int32_t)cols;
        t.n_tiles = nt;
        t.record_offset = r.pos;
        int64_t nres = 0;
        for (uint32_t k = 0; k < nt; ++k) {
            if (!r.need(2 + ib)) return CDQ_ERR_FORMAT;
            int64_t tc = data[r.pos + 1];
            if (tc > 32) return CDQ_ERR_FORMAT;
            r.pos += 2 + ib;
            int64_t bb = blob_bytes(tc);
            if (!r.need(bb)) return CDQ_ERR_FORMAT;
            r.pos += bb;
            nres += tc;
        }
        t.record_bytes = r.pos - t.record_offset;
        t.n_res = nres;
        if (i < max_tensors) tensors[i] = t;
    }
    *n_states = ns;
    *n_tensors = n;
    return CDQ_OK;
}

cdq_status cdq_file_checkpoints(const uint8_t* data, int64_t len, int32_t n_states, const cdq_file_tensor* t,
                                int32_t every, int64_t* byte_off, int64_t* res_off) {
    if (!data || !t || !byte_off || !res_off || every < 1) return CDQ_ERR_ARG;
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    if (t->record_offset < 0 || t->record_offset + t->record_bytes > len) return CDQ_ERR_FORMAT;
    const int ib = idx_bytes(n_states);
    int64_t pos = t->record_offset, n = 0;
    for (int64_t k = 0; k < t->n_tiles; ++k) {
        if (k % every == 0) {
            byte_off[k / every] = pos - t->record_offset;
            res_off[k / every] = n;
        }
        if (pos + 2 + ib > len) return CDQ_ERR_FORMAT;
        const int tc = data[pos + 1];
        if (tc > 32) return CDQ_ERR_FORMAT;
        pos += 2 + ib + blob_bytes(tc);
        if (pos > len) return CDQ_ERR_FORMAT;
        n += tc;
    }
    return n == t->n_res && pos - t->record_offset == t->record_bytes ? CDQ_OK : CDQ_ERR_FORMAT;
}

cdq_status cdq_file_decode(const uint8_t* data, int64_t len, int32_t n_states,
                           const cdq_file_tensor* t, uint8_t* q, uint8_t* scales_f8,
                           int64_t* ridx, uint16_t* rval) {
    if (!data || !t || !q || !scales_f8 || (t->n_res > 0 && (!ridx || !rval))) return CDQ_ERR_ARG;
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    if (t->record_offset < 0 || t->record_offset + t->record_bytes > len) return CDQ_ERR_FORMAT;
    const int ib = idx_bytes(n_states);
    int64_t pos = t->record_offset, n = 0;
    for (int64_t k = 0; k < t->n_tiles; ++k) {
        if (pos + 2 + ib > len) return CDQ_ERR_FORMAT;
        scales_f8[k] = data[pos];
        int tc = data[pos + 1];
        unpack_indices(data + pos + 2, n_states, q + k * 32);
        if (n_states == 26)
            for (int e = 0; e < 32; ++e)
                if (q[k * 32 + e] >= 26) return CDQ_ERR_FORMAT;
        pos += 2 + ib;
        int64_t bb = blob_bytes(tc);
        if (pos + bb > len || n + tc > t->n_res) return CDQ_ERR_FORMAT;
        int64_t first = n;
        for (int j = 0; j < tc; ++j) {
            int off = (int)get_bits(data + pos, bb, 21LL * j, 5);
            uint16_t v = (uint16_t)get_bits(data + pos, bb, 21LL * j + 5, 16);
            ridx[n] = k * 32 + off;
            rval[n] = v;
            ++n;
        }
        // offsets inside a tile are written in ascending order by the packer;
        // accept any order of distinct offsets, reject duplicates
        if (tc > 1) {
            std::vector<std::pair<int64_t, uint16_t>> e(tc);
            for (int j = 0; j < tc; ++j) e[j] = {ridx[first + j], rval[first + j]};
            std::sort(e.begin(), e.end(),
                      [](const std::pair<int64_t, uint16_t>& a, const std::pair<int64_t, uint16_t>& b) {
                          return a.first < b.first;
                      });
            for (int j = 0; j < tc; ++j) {
                if (j && e[j].first == e[j - 1].first) return CDQ_ERR_FORMAT;
                ridx[first + j] = e[j].first;
                rval[first + j] = e[j].second;
            }
        }
        pos += bb;
    }
    return n == t->n_res ? CDQ_OK : CDQ_ERR_FORMAT;
}

cdq_status cdq_pack_tile_indices(const uint8_t* q, int64_t n_tiles, int32_t n_states, uint8_t* out) {
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    if (n_tiles < 0 || (n_tiles && (!q || !out))) return CDQ_ERR_ARG;
    const int ib = idx_bytes(n_states);
    for (int64_t t = 0; t < n_tiles; ++t) pack_indices(q + t * 32, n_states, out + t * ib);
    return CDQ_OK;
}

cdq_status cdq_unpack_tile_indices(const uint8_t* packed, int64_t n_tiles, int32_t n_states, uint8_t* q) {
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    if (n_tiles < 0 || (n_tiles && (!q || !packed))) return CDQ_ERR_ARG;
    const int ib = idx_bytes(n_states);
    for (int64_t t = 0; t < n_tiles; ++t) unpack_indices(packed + t * ib, n_states, q + t * 32);
    return CDQ_OK;
}

cdq_status cdq_pack_residual_stream(const uint8_t* offsets, const uint16_t* values, int64_t count, uint8_t* out) {
    if (count < 0 || (count && (!offsets || !values || !out))) return CDQ_ERR_ARG;
    memset(out, 0, (size_t)blob_bytes(count));
    for (int64_t i = 0; i < count; ++i) {
        put_bits(out, 21 * i, offsets[i] & 0x1Fu, 5);
        put_bits(out, 21 * i + 5, values[i], 16);
    }
    return CDQ_OK;
}

cdq_status cdq_unpack_residual_stream(const uint8_t* packed, int64_t count, uint8_t* offsets, uint16_t* values) {
    if (count < 0 || (count && (!offsets || !values || !packed))) return CDQ_ERR_ARG;
    const int64_t nb = blob_bytes(count);
    for (int64_t i = 0; i < count; ++i) {
        offsets[i] = (uint8_t)get_bits(packed, nb, 21 * i, 5);
        values[i] = (uint16_t)get_bits(packed, nb, 21 * i + 5, 16);
    }
    return CDQ_OK;
}

cdq_status cdq_file_encode_header(int32_t n_states, int32_t n_tensors, uint8_t* out, int64_t cap,
                                  int64_t* written) {
    if (!written || n_tensors < 0 || n_tensors > 0xFFFF) return CDQ_ERR_ARG;
    if (n_states != 26 && n_states != 16) return CDQ_ERR_STATES;
    const int ns = n_states;
    const int64_t need = 8 + 2 * ns;
    *written = need;
    if (!out) return CDQ_OK;
    if (cap < need) return CDQ_ERR_CAPACITY;
    memcpy(out, "CDQ1", 4);
    uint16_t ver = ns == 26 ? 1 : 2;
    out[4] = (uint8_t)ver;
    out[5] = (uint8_t)(ver >> 8);
    out[6] = (uint8_t)n_tensors;
    out[7] = (uint8_t)(n_tensors >> 8);
    const uint16_t* lat = ns == 26 ? kLattice26 : kLattice16;
    for (int i = 0; i < ns; ++i) {
        out[8 + 2 * i] = (uint8_t)lat[i];
        out[9 + 2 * i] = (uint8_t)(lat[i] >> 8);
    }
    return CDQ_OK;
}

cdq_status cdq_file_encode_tensor(const char* name, int32_t rows, int32_t cols, int32_t n_states,
                                  const uint8_t* q, const uint8_t* scales_f8,
                                  const int64_t* ridx, const uint16_t* rval, int64_t n_res,
                                  uint8_t* out, int64_t cap, int64_t* written) {
    if (!name || !written || !q || !scales_f8 || n_res < 0 || (n_res > 0 && (!ridx || !rval)))
        return CDQ_ERR_ARG;
    cdq_status st = check_shape(rows, cols, n_states);
    if (st) return st;
    const int64_t nl = (int64_t)strlen(name);
    if (nl > 0xFFFF) return CDQ_ERR_ARG;
    const int64_t numel = (int64_t)rows * cols, nt = numel / 32;
    if (nt > 0xFFFFFFFFLL) return CDQ_ERR_SHAPE;
    const int ib = idx_bytes(n_states);
    // per-tile residual counts
    std::vector<int> tc(nt, 0);
    for (int64_t i = 0; i < n_res; ++i) {
        if (ridx[i] < 0 || ridx[i] >= numel || (i && ridx[i] <= ridx[i - 1])) return CDQ_ERR_ARG;
        tc[ridx[i] / 32]++;
    }
    int64_t need = 2 + nl + 12;
    for (int64_t k = 0; k < nt; ++k) need += 2 + ib + blob_bytes(tc[k]);
    *written = need;
    if (!out) return CDQ_OK;
    if (cap < need) return CDQ_ERR_CAPACITY;
    memset(out, 0, need);
    int64_t p = 0;
    out[p++] = (uint8_t)nl;
    out[p++] = (uint8_t)(nl >> 8);
    memcpy(out + p, name, nl);
    p += nl;
    uint32_t hdr[3] = {(uint32_t)rows, (uint32_t)cols, (uint32_t)nt};
    for (int i = 0; i < 3; ++i)
        for (int b = 0; b < 4; ++b) out[p++] = (uint8_t)(hdr[i] >> (8 * b));
    int64_t r = 0;
    for (int64_t k = 0; k < nt; ++k) {
        out[p] = scales_f8[k];
        out[p + 1] = (uint8_t)tc[k];
        for (int e = 0; e < 32; ++e)
            if (q[k * 32 + e] >= n_states) return CDQ_ERR_ARG;
        pack_indices(q + k * 32, n_states, out + p + 2);
        p += 2 + ib;
        for (int j = 0; j < tc[k]; ++j, ++r) {
            put_bits(out + p, 21LL * j, (uint32_t)(ridx[r] % 32), 5);
            put_bits(out + p, 21LL * j + 5, rval[r], 16);
        }
        p += blob_bytes(tc[k]);
    }
    return CDQ_OK;
}

}  // extern "C"
