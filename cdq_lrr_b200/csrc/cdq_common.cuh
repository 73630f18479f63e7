// Shared constants and number-format helpers of the CDQ-LRR B200 library.
//
// Lattices: the bf16 bit patterns of CAMKII_LATTICE (26 states,
// code/cdq_lrr_qwen05.py:27-32) and CAMKII_LATTICE_16 (16 states, zero at
// index 7, index 15 duplicating 14, code/cdq_lrr_qwen05.py:39-44).
// Float8 e4m3fn: round to nearest even, NaN at 0x7F/0xFF, no infinities;
// magnitudes that round to 480 or beyond become NaN (torch's conversion used
// at code/cdq_lrr_qwen05.py:52 and :117).
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
constexpr int kGroupTiles = 32;      // residual CSR group: 32 tile columns
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

// ---- device pack geometry (see include/cdq.h) ----
struct Geometry {
    int64_t rows, cols, rb, kt, kt4, kg;
    int words;  // code words per tile: 5 (26-state) or 4 (16-state)
};

CDQ_HD Geometry geometry(int64_t rows, int64_t cols, int n_states) {
    Geometry g;
    g.rows = rows;
    g.cols = cols;
    g.rb = (rows + 31) / 32;
    g.kt = cols / 32;
    g.kt4 = (g.kt + 3) / 4;
    g.kg = (g.kt + kGroupTiles - 1) / kGroupTiles;
    g.words = n_states == 26 ? 5 : 4;
    return g;
}

// Word index (uint32 units) of word wd of lane l in tile column (rb, c).
CDQ_HD int64_t code_word_index(const Geometry& g, int64_t rb, int64_t c, int lane, int wd) {
    int64_t base = (rb * g.kt + c) * (int64_t)(g.words * 32);
    return wd < 4 ? base + lane * 4 + wd : base + 128 + lane;
}

CDQ_HD int64_t scale_index(const Geometry& g, int64_t rb, int64_t c, int lane) {
    return ((rb * g.kt4 + c / 4) * 32 + lane) * 4 + (c & 3);
}

CDQ_HD int64_t bucket_index(const Geometry& g, int64_t rb, int64_t grp, int lane) {
    return (rb * g.kg + grp) * 32 + lane;
}

}  // namespace cdq
