// Shared constants, number-format helpers and the device-pack geometry of the
// CDQ-LRR B200 library.
//
// Lattices: the bf16 bit patterns of CAMKII_LATTICE (26 states,
// code/cdq_lrr_qwen05.py:27-32) and CAMKII_LATTICE_16 (16 states, zero at
// index 7, index 15 duplicating 14, code/cdq_lrr_qwen05.py:39-44).
// Float8 e4m3fn: round to nearest even, NaN at 0x7F/0xFF, no infinities;
// magnitudes that round to 480 or beyond become NaN (torch's conversion used
// at code/cdq_lrr_qwen05.py:52 and :117).
//
// Device pack geometry ("fragment units" in "quads"). Rows are grouped in
// blocks of 16 (R16 = ceil(rows/16)), tile columns (32 weights of a row) in
// pairs (KP = ceil(KT/2), KT = cols/32). One unit = (16-row block, tile-column
// pair) = 32 tiles = 640 code bytes + 32 scale bytes (26 states) or 512 + 32
// (16 states). Units of a row block are stored in quads of four consecutive
// units (the last quad of a row block holds KP mod 4 units when that is not
// zero); a quad of u units, starting at byte (b16 * KP + 4 * quad) * unit, is
//   [0, 512u)           unit i, lane l: code words 0..3 (uint4 at 512i + 16l)
//   [512u, 640u)        26 states: code word 4 of unit i, lane l at 4(u*l + i)
//                       from the start of this part (lane-major)
//   next 32u bytes      scale half-words: lane pair k = l >> 1, unit i at
//                       2(u*k + i): fp8 codes (row g, tile t), (row g+8, tile t)
// so a full quad is read with four 16-byte loads per lane for the code words,
// one 16-byte load for the four fifth words and one 8-byte load for the four
// scale half-words.
// Lane l = 4g + c holds the 16 pair codes of the m16n8k16 A fragments of rows
// g and g+8 of the block over the unit's columns 16c .. 16c+15 (all in tile
// t = c>>1): slot q = 4s + i (s = k16 slice, i = h + 2j) is row g + 8h,
// unit columns 16c + 4s + 2j and +1, i.e. element pair p = 8(c&1) + 2s + j
// of tile t. The k order inside a slice is permuted so that a lane's
// activation operands are 16 contiguous columns (two 16-byte loads).
// A pair code covers weights 2p, 2p+1 of the tile:
// 26 states -> s[2p]*27 + s[2p+1] (10 bits, symbol 26 = residual slot, value
// zero) at bits [10q, 10q+10) of the lane's 160-bit word stream; 16 states ->
// byte q = s[2p] | s[2p+1] << 4 (residual slots use index 7, the exact zero).
// A phantom tile (odd KT) and rows beyond `rows` hold residual slots, scale 0.
// Residual CSR buckets: (16-row block, group of 32 tile columns, row 0..15).
#pragma once

#include <stdint.h>
#include <string.h>
#include <math.h>

#ifdef __CUDACC__
#define CDQ_HD __host__ __device__ __forceinline__
#else
#define CDQ_HD inline
#endif

namespace cdq {

constexpr int kTile = 32;
constexpr int kGroupTiles = 32;      // residual CSR group: 32 tile columns (16 pairs)
constexpr int kGroupPairs = 16;
constexpr int kResidualSym26 = 26;   // 26-state pair-code symbol of a residual slot
constexpr int kResidualSym16 = 7;    // 16-state: the lattice's exact zero
constexpr int kPairs26 = 27 * 27;    // 729 pair codes (26 states + residual slot)
constexpr int kPairs16 = 256;

static const uint16_t kLattice26[26] = {
    0xBF80, 0xBF3B, 0xBF07, 0xBEC0, 0xBE86, 0xBE36, 0xBDEF, 0xBD96, 0xBD31,
    0xBCBC, 0xBC25, 0xBB4B, 0xBA03, 0x3A03, 0x3B4B, 0x3C25, 0x3CBC, 0x3D31,
    0x3D96, 0x3DEF, 0x3E36, 0x3E86, 0x3EC0, 0x3F07, 0x3F3B, 0x3F80};
static const uint16_t kLattice16[16] = {
    0xBF78, 0xBF41, 0xBF15, 0xBEE2, 0xBEA3, 0xBE52, 0xBDCC, 0x0000,
    0x3DCC, 0x3E52, 0x3EA3, 0x3EE2, 0x3F15, 0x3F41, 0x3F78, 0x3F78};

CDQ_HD uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
CDQ_HD float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
CDQ_HD float bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

// float32 -> bf16 bits, round to nearest even, every NaN -> 0x7FC0.
CDQ_HD uint16_t f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// float32 -> float8 e4m3fn code.
CDQ_HD uint8_t fp8_encode(float f) {
    uint32_t u = f32_bits(f);
    uint32_t sign = (u >> 24) & 0x80u;
    u &= 0x7FFFFFFFu;
    if (u >= 0x7F800000u) return (uint8_t)(sign | 0x7Fu);  // inf, NaN
    if (u < (121u << 23)) {                                // below 2^-6
        // quantum 2^-9: scaling by 512 is exact, rintf rounds half to even
        float s = bits_f32(u) * 512.0f;
        return (uint8_t)(sign | (uint32_t)rintf(s));        // 8 lands on 2^-6
    }
    uint32_t e = (u >> 23) - 120u;  // (E - 127) + 7
    uint32_t m = u & 0x7FFFFFu;
    uint32_t keep = m >> 20, rest = m & 0xFFFFFu;
    if (rest > 0x80000u || (rest == 0x80000u && (keep & 1u))) ++keep;
    if (keep == 8u) {
        keep = 0;
        ++e;
    }
    if (e > 15u || (e == 15u && keep == 7u)) return (uint8_t)(sign | 0x7Fu);
    return (uint8_t)(sign | (e << 3) | keep);
}

// float8 e4m3fn code -> bf16 bits (exact; NaN -> 0x7FC0).
CDQ_HD uint16_t fp8_to_bf16(uint8_t c) {
    uint32_t s = (uint32_t)(c & 0x80u) << 8;
    uint32_t e = (c >> 3) & 0xFu, m = c & 7u;
    if ((c & 0x7Fu) == 0x7Fu) return 0x7FC0;
    if (e) return (uint16_t)(s | ((e + 120u) << 7) | (m << 4));
    if (!m) return (uint16_t)s;
    // subnormal m * 2^-9: normalise the 3-bit mantissa
    uint32_t sh = (m >= 4) ? 2 : (m >= 2 ? 1 : 0);     // floor(log2 m)
    uint32_t exp = 118u + sh;                         // 2^-9 * 2^sh
    uint32_t mant = (m << (7 - sh)) & 0x7Fu;
    return (uint16_t)(s | (exp << 7) | mant);
}

// ---- device pack geometry ----
struct Geometry {
    int64_t rows, cols, kt, r16, kp, kg;
    int words;        // code words per lane: 5 (26 states) or 4 (16 states)
    int64_t unit;     // bytes per unit: 672 or 544
    int64_t sig_off;  // code bytes per unit: 640 or 512
};

CDQ_HD Geometry geometry(int64_t rows, int64_t cols, int n_states) {
    Geometry g;
    g.rows = rows;
    g.cols = cols;
    g.kt = cols / 32;
    g.r16 = (rows + 15) / 16;
    g.kp = (g.kt + 1) / 2;
    g.kg = (g.kt + kGroupTiles - 1) / kGroupTiles;
    g.words = n_states == 26 ? 5 : 4;
    g.sig_off = n_states == 26 ? 640 : 512;
    g.unit = g.sig_off + 32;
    return g;
}

// Workspace of one fused-linear call with batch m (bytes). It starts with one
// uint32 arrival counter per row block (the streaming kernel's split-K
// hand-off; zero before the first call, every call leaves them zero), then
// the path's own data: the streaming path's float32 sums per (batch row,
// residual group, padded row), or the tcgen05 tile path's prepared
// activations: the B-operand stages of every quad (batch padded to N = 16, 32
// or 64, 512 bytes per batch row per quad) and x^T (64 * kp columns x the
// batch padded to 8, bf16).
CDQ_HD int64_t ws_align256(int64_t b) { return (b + 255) / 256 * 256; }
CDQ_HD int tile_nb(int64_t m) { return m <= 16 ? 16 : m <= 32 ? 32 : 64; }
CDQ_HD int64_t tile_xperm_bytes(const Geometry& g, int64_t m) { return (g.kp + 3) / 4 * tile_nb(m) * 512; }
CDQ_HD int64_t tile_prep_bytes(const Geometry& g, int64_t m) {
    return ws_align256(tile_xperm_bytes(g, m)) + ws_align256(g.kp * 64 * ((m + 7) / 8 * 8) * 2);
}
CDQ_HD int64_t gemv_counter_bytes(const Geometry& g) { return ws_align256(g.r16 * 4); }
CDQ_HD int64_t gemv_sums_bytes(const Geometry& g, int64_t m) {
    return ws_align256(m * g.kg * g.r16 * 16 * 4);
}
// the streaming path alone (counters + sums)
CDQ_HD int64_t gemv_partial_bytes(const Geometry& g, int64_t m) {
    return gemv_counter_bytes(g) + gemv_sums_bytes(g, m);
}
CDQ_HD int64_t linear_workspace_need(const Geometry& g, int64_t m) {
    const int64_t a = gemv_sums_bytes(g, m), b = tile_prep_bytes(g, m);
    return gemv_counter_bytes(g) + (a > b ? a : b);
}

// Quad holding unit (b16, cp): byte offset of the quad, its unit count u and
// the unit's index i inside it.
CDQ_HD int64_t quad_base(const Geometry& g, int64_t b16, int64_t cp, int* u, int* i) {
    const int64_t q = cp >> 2;
    const int64_t left = g.kp - 4 * q;
    *u = (int)(left < 4 ? left : 4);
    *i = (int)(cp & 3);
    return (b16 * g.kp + 4 * q) * g.unit;
}

// Byte offset (in the units buffer) of code word wd of lane l of unit (b16, cp).
CDQ_HD int64_t word_offset(const Geometry& g, int64_t b16, int64_t cp, int lane, int wd) {
    int u, i;
    const int64_t base = quad_base(g, b16, cp, &u, &i);
    return wd < 4 ? base + 512 * i + 16 * lane + 4 * wd : base + 512 * u + 4 * (u * lane + i);
}

// (row within block ri, tile of the pair t, element pair p of the tile)
// -> (lane, slot)
CDQ_HD void slot_of(int ri, int t, int p, int* lane, int* slot) {
    const int g = ri & 7, h = ri >> 3, c = 2 * t + (p >> 3), s = (p >> 1) & 3, j = p & 1;
    *lane = 4 * g + c;
    *slot = 4 * s + (h | (j << 1));
}

// (lane, slot) -> (row within block, tile of the pair, element pair)
CDQ_HD void slot_pos(int lane, int slot, int* ri, int* t, int* p) {
    const int g = lane >> 2, c = lane & 3, s = slot >> 2, i = slot & 3;
    *t = c >> 1;
    *ri = g + 8 * (i & 1);
    *p = 8 * (c & 1) + 2 * s + (i >> 1);
}

// Byte offset (in the units buffer) of the scale of (row within block ri,
// tile t) of unit (b16, cp).
CDQ_HD int64_t scale_offset(const Geometry& g, int64_t b16, int64_t cp, int ri, int t) {
    int u, i;
    const int64_t base = quad_base(g, b16, cp, &u, &i);
    const int k = 2 * (ri & 7) + t;
    return base + g.sig_off * u + 2 * (u * k + i) + (ri >> 3);
}

// Residual CSR bucket of (16-row block, residual group, row in block): row
// major, so the buckets of one row (all its groups, columns ascending) are
// consecutive and [res_ptr[row * kg], res_ptr[(row + 1) * kg]) is the row.
CDQ_HD int64_t bucket_index(const Geometry& g, int64_t r16, int64_t grp, int ri) {
    return (r16 * 16 + ri) * g.kg + grp;
}

}  // namespace cdq
