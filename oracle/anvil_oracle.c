/*
 * anvil_oracle.c -- CPU restatement of the MMVQ hot path, used ONLY as test
 * infrastructure: the parity checker for tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py.  Nothing in the product links or calls it.
 *
 * What it restates, and from where:
 *   - GGUF block layouts and per-weight dequantisation of Q4_0, Q4_1, Q5_0, Q5_1, Q2_K,
 *     Q3_K, Q4_K, Q5_K, Q6_K, Q8_0, IQ4_NL and IQ4_XS: gguf-py (the reference's declared
 *     dependency, kernel-anvil pyproject.toml:19, gguf 0.19.0) gguf/quants.py Q4_0..Q5_1,
 *     Q2_K, Q3_K, IQ4_NL and IQ4_XS dequantize_blocks, 378-401 (Q8_0), 474-523 (Q4_K incl. get_scale_min), 525-549
 *     (Q5_K), 552-572 (Q6_K).
 *     The seven lattice I-quants IQ2_XXS, IQ2_XS, IQ2_S, IQ3_XXS, IQ3_S, IQ1_S and IQ1_M
 *     (the reference's QUANT_TYPES, kernel_anvil/hip_codegen.py:89-96): gguf-py
 *     gguf/quants.py <type>.dequantize_blocks with the grids of <type>.grid_hex /
 *     grid_map and IQ2_XXS.ksigns, here as the generated table header
 *     kernel-anvil_b200/csrc/iq_grids.h.
 *     Pinned in tests against gguf.quants.dequantize (fixtures and live).
 *   - Q8_1 activation quantisation: llama.cpp's CUDA quantize_q8_1 semantics (the
 *     reference's runtime path: kernel_anvil/hip_codegen.py:392-396 layout, 101-102 size;
 *     docs/decode-pipeline-breakdown.md:21): per 32 values d = max|x|/127,
 *     q = roundf(x/d), stored {half(d), half(sum x)}; the sum is taken in the
 *     xor-butterfly order of a 32-lane warp reduction.  gguf-py has no Q8_1; its Q8_0
 *     quantiser (gguf/quants.py:381-392) is the closest pinned relative and tests
 *     compare against it.
 *   - Chained-input Q8_1 (the persistent chain's group input computed from an earlier
 *     GEMV's output; no counterpart in the reference, whose decode quantises every input
 *     with quantize_q8_1 after ops outside this path): the quants of quantize_q8_1 with d kept
 *     in fp32, and a per-column power of two 2^-e (e the exponent of the column's largest
 *     magnitude) applied to the GEMV's result.
 *   - Block dots: the MMVQ arithmetic of vec_dot_{q4_K,q5_K,q6_K,q8_0}_q8_1 as restated
 *     in kernel_anvil/hip_codegen.py:430-491 (with qi = 32, the correct QI4_K of
 *     kernel_anvil/hip_codegen.py:86) and docs/llama-cpp-kernel-analysis.md:200-224:
 *     exact int32 sums per sub-block, then
 *     y = sum_b d_b * sum_j d8_j * sc_j * sumi_j - dmin_b * sum_j d8_j * m_j * sumq_j,
 *     evaluated here in double.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off, no fast-math: IEEE
 * division and rounding must match the GPU bit for bit).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11,
       T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18,
       T_IQ1_S = 19, T_IQ4_NL = 20, T_IQ3_S = 21, T_IQ2_S = 22, T_IQ4_XS = 23, T_IQ1_M = 29 };

#define ANVIL_IQ_TABLE static const
#include "iq_grids.h"

/* The 16 levels of IQ4_NL / IQ4_XS (gguf-py quants.py IQ4_NL.kvalues). */
static const int iq4_levels[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                   1,    13,   25,  38,  53,  69,  89,  113};

/* IQ4_NL (18 B: d @0, qs[16] @2): weight e is level qs[e] & 15 (e < 16) or qs[e - 16] >> 4.
 * IQ4_XS (136 B: d @0, scales_h u16 @2, scales_l[4] @4, qs[128] @8): group j (32 weights)
 * reads qs[16j + e] low nibble for e < 16 and qs[16j + e - 16] high nibble above; its scale
 * is (scales_l[j / 2] nibble j % 2 | bits 2j..2j+1 of scales_h << 4) - 32. */
static inline int iq4nl_level(const uint8_t *qs, int e) {
    return iq4_levels[e < 16 ? (qs[e] & 15) : (qs[e - 16] >> 4)];
}
static inline int iq4xs_scale(const uint8_t *blk, int j) {
    const int sh = blk[2] | (blk[3] << 8);
    const int lo = (blk[4 + j / 2] >> (4 * (j & 1))) & 15;
    return (lo | (((sh >> (2 * j)) & 3) << 4)) - 32;
}

/* ---- IEEE binary16 conversions (written from the format definition) ---------- */

float oracle_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1F;
    const uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: value = man * 2^-24 */
            float v = (float)man * 5.9604644775390625e-8f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> binary16, round to nearest, ties to even. */
uint16_t oracle_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) { /* inf or nan */
        return sign | 0x7C00 | (ax > 0x7F800000u ? 0x200 : 0);
    }
    const int e = (int)(ax >> 23) - 127; /* unbiased exponent */
    if (e > 15) return sign | 0x7C00;    /* overflow to inf (>= 65536 before rounding) */
    uint32_t mant = (ax & 0x7FFFFF) | 0x800000; /* 24-bit significand with hidden bit */
    int shift;                                  /* right shift to the half ulp grid */
    uint32_t hexp;
    if (e >= -14) {
        shift = 13;
        hexp = (uint32_t)(e + 15);
    } else {
        if (ax == 0) return sign;
        shift = 13 + (-14 - e); /* subnormal half */
        hexp = 0;
        if (shift > 24) return sign; /* below half the smallest subnormal */
    }
    const uint32_t q = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1);
    const uint32_t halfway = 1u << (shift - 1);
    uint32_t r = q;
    if (rem > halfway || (rem == halfway && (q & 1))) r += 1;
    uint32_t out;
    if (hexp == 0) {
        out = r; /* may carry into the smallest normal: still the right encoding */
    } else {
        /* r has 11 bits (hidden bit at 10); a carry to bit 11 bumps the exponent */
        if (r & 0x800) {
            r >>= 1;
            hexp += 1;
        }
        if (hexp >= 31) return sign | 0x7C00;
        out = (hexp << 10) | (r & 0x3FF);
    }
    return sign | (uint16_t)out;
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ---- Q8_1 quantiser ---------------------------------------------------------- */

void oracle_quantize_q8_1(const float *x, uint8_t *xq, int64_t K, int64_t ncols) {
    const int64_t nb = K / 32 * ncols;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; ++b) {
        const float *v = x + b * 32;
        float amax = 0.0f;
        float s[32];
        for (int l = 0; l < 32; ++l) {
            const float a = fabsf(v[l]);
            amax = a > amax ? a : amax;
            s[l] = v[l];
        }
        for (int o = 16; o > 0; o >>= 1) { /* xor-butterfly: lane l adds lane l^o */
            float t[32];
            for (int l = 0; l < 32; ++l) t[l] = s[l] + s[l ^ o];
            memcpy(s, t, sizeof(s));
        }
        const float d = amax / 127.0f;
        uint8_t *blk = xq + b * 36;
        for (int l = 0; l < 32; ++l) {
            const int q = amax == 0.0f ? 0 : (int)roundf(v[l] / d);
            blk[4 + l] = (uint8_t)(int8_t)q;
        }
        const uint16_t hd = oracle_float_to_half(d), hs = oracle_float_to_half(s[0]);
        blk[0] = (uint8_t)hd;
        blk[1] = (uint8_t)(hd >> 8);
        blk[2] = (uint8_t)hs;
        blk[3] = (uint8_t)(hs >> 8);
    }
}

/* Chained-input quantisation (the persistent chain's group input computed from an earlier
 * GEMV's output): per 32-value block the quants of quantize_q8_1 (q = roundf(x / d),
 * d = amax / 127) with d kept in fp32 at bytes 0-3 of the block; per column the scale
 * 2^(E - 127), E = clamp(254 - biased exponent of max|x|, 1, 254), which the GEMV applies to
 * its result (y = scale * sum over blocks). */
void oracle_quantize_q8_1_chained(const float *x, uint8_t *xq, float *scale, int64_t K,
                                  int64_t ncols) {
    for (int64_t c = 0; c < ncols; ++c) {
        const float *col = x + c * K;
        float m = 0.0f;
        for (int64_t i = 0; i < K; ++i) {
            const float a = fabsf(col[i]);
            m = a > m ? a : m;
        }
        uint32_t mb;
        memcpy(&mb, &m, 4);
        int E = 254 - (int)((mb >> 23) & 0xFF);
        E = E < 1 ? 1 : E > 254 ? 254 : E;
        const uint32_t sb = (uint32_t)E << 23;
        memcpy(&scale[c], &sb, 4);
        for (int64_t b = 0; b < K / 32; ++b) {
            const float *v = col + b * 32;
            float amax = 0.0f;
            for (int l = 0; l < 32; ++l) {
                const float a = fabsf(v[l]);
                amax = a > amax ? a : amax;
            }
            const float d = amax / 127.0f;
            uint8_t *blk = xq + (c * (K / 32) + b) * 36;
            for (int l = 0; l < 32; ++l) {
                const int q = amax == 0.0f ? 0 : (int)roundf(v[l] / d);
                blk[4 + l] = (uint8_t)(int8_t)q;
            }
            memcpy(blk, &d, 4);
        }
    }
}

/* ---- K-quant scale unpacking (gguf/quants.py:478-501) ------------------------- */

static void q4k_scale_min(const uint8_t *s, int j, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Unsigned quant of weight e (0..31) of sub-block j (0..7). */
static inline int q4k_quant(const uint8_t *blk, int j, int e) {
    const uint8_t b = blk[16 + 32 * (j >> 1) + e];
    return (j & 1) ? (b >> 4) : (b & 0xF);
}
static inline int q5k_quant(const uint8_t *blk, int j, int e) {
    const uint8_t b = blk[48 + 32 * (j >> 1) + e];
    const int lo = (j & 1) ? (b >> 4) : (b & 0xF);
    const int hi = (blk[16 + e] >> j) & 1;
    return lo | (hi << 4);
}
/* Signed quant (q - 32) of weight e (0..31) of 32-weight sub-block j (0..7) of a Q6_K
 * block: j = 4h + 2s + t uses ql[64h + 32t + e] nibble s and qh[32h + e] bits 2(2s+t). */
static inline int q6k_quant(const uint8_t *blk, int j, int e) {
    const int h = j >> 2, s = (j >> 1) & 1, t = j & 1;
    const uint8_t l = blk[64 * h + 32 * t + e];
    const int lo = s ? (l >> 4) : (l & 0xF);
    const int hi = (blk[128 + 32 * h + e] >> (2 * (j & 3))) & 3;
    return (lo | (hi << 4)) - 32;
}

/* Q2_K (84 B: scales[16] @0, qs[64] @16, d @80, dmin @82) and Q3_K (110 B: hmask[32] @0,
 * qs[64] @32, scales[12] @96, d @108), gguf-py Q2_K / Q3_K dequantize_blocks.  Weight w of
 * the 256: its 2-bit quant is bits 2s of qs byte 32h + l with h = w / 128, s = (w % 128) / 32,
 * l = w % 32; Q3_K subtracts 4 unless bit w / 32 of hmask[l] is set.  Sub-block j = w / 16
 * has Q2_K scale scales[j] & 15 and min scales[j] >> 4, and Q3_K 6-bit scale (low nibble of
 * scales[j] for j < 8, high nibble of scales[j - 8] above; bits 4-5 from bits 2(j / 4) of
 * scales[8 + j % 4]) minus 32. */
static inline int q23_low(const uint8_t *qs, int w) {
    return (qs[32 * (w >> 7) + (w & 31)] >> (2 * ((w >> 5) & 3))) & 3;
}
static inline int q2k_quant(const uint8_t *blk, int w) { return q23_low(blk + 16, w); }
static inline int q3k_quant(const uint8_t *blk, int w) {
    const int hbit = (blk[w & 31] >> (w >> 5)) & 1;
    return q23_low(blk + 32, w) - (hbit ? 0 : 4);
}
static inline int q3k_scale(const uint8_t *blk, int j) {
    const uint8_t *s = blk + 96;
    const int lo = j < 8 ? (s[j] & 15) : (s[j - 8] >> 4);
    const int hi = (s[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

static int type_bytes(int t) {
    switch (t) {
    case T_IQ2_XXS: return 66;
    case T_IQ2_XS: return 74;
    case T_IQ2_S: return 82;
    case T_IQ3_XXS: return 98;
    case T_IQ3_S: return 110;
    case T_IQ1_S: return 50;
    case T_IQ1_M: return 56;
    case T_IQ4_NL: return 18;
    case T_IQ4_XS: return 136;
    case T_Q2_K: return 84;
    case T_Q3_K: return 110;
    case T_Q4_0: return 18;
    case T_Q4_1: return 20;
    case T_Q5_0: return 22;
    case T_Q5_1: return 24;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    default: return 0;
    }
}
static int is_basic(int t) { return t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_1; }
static int type_qk(int t) { return (t == T_Q8_0 || t == T_IQ4_NL || is_basic(t)) ? 32 : 256; }

/* Q4_0 / Q4_1 / Q5_0 / Q5_1 (gguf-py quants.py Q4_0..Q5_1 dequantize_blocks): 32 weights;
 * element e < 16 is the low nibble of qs[e], element e >= 16 the high nibble of qs[e - 16];
 * the _5 types add bit e of the little-endian uint32 qh as bit 4.  Q4_0 subtracts 8, Q5_0
 * subtracts 16; the _1 types keep the unsigned value and add m. */
static int basic_qs_off(int t) { return t == T_Q4_0 ? 2 : t == T_Q4_1 ? 4 : t == T_Q5_0 ? 6 : 8; }
static inline int basic_quant(int t, const uint8_t *blk, int e) {
    const uint8_t *qs = blk + basic_qs_off(t);
    int q = e < 16 ? (qs[e] & 15) : (qs[e - 16] >> 4);
    if (t == T_Q5_0 || t == T_Q5_1) {
        const uint8_t *h = blk + (t == T_Q5_0 ? 2 : 4);
        const uint32_t qh = (uint32_t)h[0] | ((uint32_t)h[1] << 8) | ((uint32_t)h[2] << 16) |
                            ((uint32_t)h[3] << 24);
        q |= (int)((qh >> e) & 1u) << 4;
    }
    if (t == T_Q4_0) q -= 8;
    if (t == T_Q5_0) q -= 16;
    return q;
}

/* ---- lattice I-quants ---------------------------------------------------------------
 * Block layouts (256 weights; sub-block j = weights 32j..32j+31, group k = weights 8k..8k+7):
 *   IQ2_XXS  66 B: d @0; per j at 2+8j: 4 grid bytes (one 8-value row of the 256-row grid per
 *            group), then a u32 whose bits 7l..7l+6 index the sign byte of group 4j+l and
 *            whose bits 28-31 are the scale ls.              w = d (0.5 + ls) / 4 * grid * sign
 *   IQ2_XS   74 B: d @0; u16 qs[32] @2 (bits 0-8 a row of the 512-row grid, 9-15 a sign
 *            index, one per group); scales[8] @66, a nibble per 16 weights (low first).
 *   IQ2_S    82 B: d @0; qs[32] @2 (row index bits 0-7), signs[32] @34 (one byte per group),
 *            qh[8] @66 (2 bits per group: index bits 8-9 of group 4j+l at bit 2l of qh[j]),
 *            scales[8] @74 as IQ2_XS; grid of 1024 rows.
 *   IQ3_XXS  98 B: d @0; qs[64] @2 (one 4-value row of the 256-row grid per 4 weights);
 *            u32 @66+4j: sign indices and scale as IQ2_XXS.  w = d (0.5 + ls) / 2 * grid * sign
 *   IQ3_S   110 B: d @0; qs[64] @2 (row index bits 0-7), qh[8] @66 (bit 8 of row 8j+b at bit
 *            b of qh[j]), signs[32] @74, scales[4] @106 (a nibble per sub-block).
 *                                                            w = d (1 + 2 ls) * grid * sign
 *   IQ1_S    50 B: d @0; qs[32] @2 (row index bits 0-7 per group); u16 qh[8] @34: bits
 *            3l..3l+2 index bits 8-10 of group 4j+l, bits 12-14 the scale s, bit 15 the sign
 *            of the delta.                   w = d (2 s + 1) * (grid + (bit 15 ? -1 : 1) / 8)
 *   IQ1_M    56 B: qs[32] @0; qh[16] @32 (a nibble per group, low first: bits 0-2 index bits
 *            8-10, bit 3 the delta sign); u16 scales[4] @48: 3-bit scales at bits 3t of word
 *            i for the 16 weights 16(4i + t).., and bits 12-15 of word i are bits 4i..4i+3
 *            of the fp16 d.                                   w = d (2 s + 1) * (grid + delta)
 * The IQ1 grid holds -1, 0, 1.  For the integer arithmetic every weight is
 * d * F * M_g * L_w: the level L_w (the signed grid value, or 8 * grid +- 1 for IQ1), the
 * scale multiplier M_g of its 16- or 32-weight group and the type's factor F (1/8 for IQ2
 * and IQ1, 1/4 for IQ3_XXS, 1 for IQ3_S). */
static int is_iq(int t) {
    return t == T_IQ2_XXS || t == T_IQ2_XS || t == T_IQ2_S || t == T_IQ3_XXS || t == T_IQ3_S ||
           t == T_IQ1_S || t == T_IQ1_M;
}
static int iq_group16(int t) { return t == T_IQ2_XS || t == T_IQ2_S || t == T_IQ1_M; }
static double iq_factor(int t) { return t == T_IQ3_XXS ? 0.25 : t == T_IQ3_S ? 1.0 : 0.125; }
static inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline int row8(uint64_t row, int i) { return (int)(int8_t)(uint8_t)(row >> (8 * i)); }
static inline int row4(uint32_t row, int i) { return (int)(int8_t)(uint8_t)(row >> (8 * i)); }
static inline uint16_t iq1m_d_bits(const uint8_t *blk) {
    uint16_t d = 0;
    for (int i = 0; i < 4; ++i) d |= (uint16_t)((rd16(blk + 48 + 2 * i) >> 12) << (4 * i));
    return d;
}
static float iq_d(int t, const uint8_t *blk) {
    return oracle_half_to_float(t == T_IQ1_M ? iq1m_d_bits(blk) : rd16(blk));
}
/* Grid value of weight w (before its sign; IQ1: -1, 0 or 1). */
static int iq_grid(int t, const uint8_t *blk, int w) {
    const int j = w >> 5, l = (w >> 3) & 3, k = w >> 3, i = w & 7;
    switch (t) {
    case T_IQ2_XXS: return row8(kIq2xxsGrid[blk[2 + 8 * j + l]], i);
    case T_IQ2_XS: return row8(kIq2xsGrid[rd16(blk + 2 + 2 * k) & 511], i);
    case T_IQ2_S: return row8(kIq2sGrid[blk[2 + k] | (((blk[66 + j] >> (2 * l)) & 3) << 8)], i);
    case T_IQ3_XXS: return row4(kIq3xxsGrid[blk[2 + (w >> 2)]], w & 3);
    case T_IQ3_S: {
        const int r = w >> 2;
        return row4(kIq3sGrid[blk[2 + r] | (((blk[66 + j] >> (r & 7)) & 1) << 8)], w & 3);
    }
    case T_IQ1_S: return row8(kIq1sGrid[blk[2 + k] | (((rd16(blk + 34 + 2 * j) >> (3 * l)) & 7) << 8)], i);
    case T_IQ1_M: {
        const int nib = (blk[32 + (k >> 1)] >> (4 * (k & 1))) & 15;
        return row8(kIq1sGrid[blk[k] | ((nib & 7) << 8)], i);
    }
    default: return 0;
    }
}
/* 1 when weight w is negated (IQ2 / IQ3 sign bits); for IQ1 when its delta is -1/8. */
static int iq_neg(int t, const uint8_t *blk, int w) {
    const int j = w >> 5, l = (w >> 3) & 3, k = w >> 3, i = w & 7;
    switch (t) {
    case T_IQ2_XXS: return (kIqSigns[(rd32(blk + 2 + 8 * j + 4) >> (7 * l)) & 127] >> i) & 1;
    case T_IQ2_XS: return (kIqSigns[rd16(blk + 2 + 2 * k) >> 9] >> i) & 1;
    case T_IQ2_S: return (blk[34 + k] >> i) & 1;
    case T_IQ3_XXS: return (kIqSigns[(rd32(blk + 66 + 4 * j) >> (7 * l)) & 127] >> i) & 1;
    case T_IQ3_S: return (blk[74 + k] >> i) & 1;
    case T_IQ1_S: return rd16(blk + 34 + 2 * j) >> 15;
    case T_IQ1_M: return (blk[32 + (k >> 1)] >> (4 * (k & 1) + 3)) & 1;
    default: return 0;
    }
}
/* The integer level L_w. */
static int iq_level(int t, const uint8_t *blk, int w) {
    const int g = iq_grid(t, blk, w), neg = iq_neg(t, blk, w);
    if (t == T_IQ1_S || t == T_IQ1_M) return 8 * g + (neg ? -1 : 1);
    return neg ? -g : g;
}
/* The raw scale field of scale group sg (a 32-weight sub-block, or 16 weights for the
 * iq_group16 types) and its integer multiplier M. */
static int iq_scale(int t, const uint8_t *blk, int sg) {
    switch (t) {
    case T_IQ2_XXS: return blk[2 + 8 * sg + 7] >> 4;
    case T_IQ2_XS: return (blk[66 + (sg >> 1)] >> (4 * (sg & 1))) & 15;
    case T_IQ2_S: return (blk[74 + (sg >> 1)] >> (4 * (sg & 1))) & 15;
    case T_IQ3_XXS: return blk[66 + 4 * sg + 3] >> 4;
    case T_IQ3_S: return (blk[106 + (sg >> 1)] >> (4 * (sg & 1))) & 15;
    case T_IQ1_S: return (rd16(blk + 34 + 2 * sg) >> 12) & 7;
    case T_IQ1_M: return (rd16(blk + 48 + 2 * (sg >> 2)) >> (3 * (sg & 3))) & 7;
    default: return 0;
    }
}
static int iq_mult(int t, const uint8_t *blk, int sg) { return 2 * iq_scale(t, blk, sg) + 1; }

/* gguf-py's float32 order per type: IQ2 db = d * (0.5 + ls) * 0.25, IQ3_XXS d * (0.5 + ls)
 * * 0.5, then db * grid * sign; IQ3_S d * (1 + 2 ls) * grid * sign; IQ1 d * (2 s + 1) *
 * (grid + delta). */
static void iq_dequant_block(int t, const uint8_t *blk, float *o) {
    const float d = iq_d(t, blk);
    for (int w = 0; w < 256; ++w) {
        const int sg = iq_group16(t) ? w >> 4 : w >> 5;
        const int g = iq_grid(t, blk, w), neg = iq_neg(t, blk, w);
        const int ls = iq_scale(t, blk, sg);
        if (t == T_IQ1_S || t == T_IQ1_M) {
            const float dl = d * (float)(2 * ls + 1);
            o[w] = dl * ((float)g + (neg ? -0.125f : 0.125f));
        } else if (t == T_IQ3_S) {
            const float db = d * (float)(1 + 2 * ls);
            o[w] = neg ? -(db * (float)g) : db * (float)g;
        } else {
            const float db = d * (0.5f + (float)ls) * (t == T_IQ3_XXS ? 0.5f : 0.25f);
            o[w] = neg ? -(db * (float)g) : db * (float)g;
        }
    }
}

/* ---- dequantisation (gguf-py float32 operation order) -------------------------- */

int oracle_dequant(int type, const uint8_t *W, float *out, int64_t nrows, int64_t K) {
    const int bytes = type_bytes(type), qk = type_qk(type);
    if (!bytes || K % qk) return -1;
    const int64_t nblk = nrows * (K / qk);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) {
        const uint8_t *blk = W + b * bytes;
        float *o = out + b * qk;
        if (type == T_Q8_0) {
            const float d = oracle_half_to_float(rd16(blk));
            for (int e = 0; e < 32; ++e) o[e] = (float)(int8_t)blk[2 + e] * d;
        } else if (is_basic(type)) {
            const float d = oracle_half_to_float(rd16(blk));
            if (type == T_Q4_1 || type == T_Q5_1) {
                const float m = oracle_half_to_float(rd16(blk + 2));
                for (int e = 0; e < 32; ++e) o[e] = d * (float)basic_quant(type, blk, e) + m;
            } else {
                for (int e = 0; e < 32; ++e) o[e] = d * (float)basic_quant(type, blk, e);
            }
        } else if (is_iq(type)) {
            iq_dequant_block(type, blk, o);
        } else if (type == T_IQ4_NL) {
            const float d = oracle_half_to_float(rd16(blk));
            for (int e = 0; e < 32; ++e) o[e] = d * (float)iq4nl_level(blk + 2, e);
        } else if (type == T_IQ4_XS) {
            const float d = oracle_half_to_float(rd16(blk));
            for (int j = 0; j < 8; ++j) {
                const float dl = d * (float)iq4xs_scale(blk, j);
                for (int e = 0; e < 32; ++e) o[32 * j + e] = dl * (float)iq4nl_level(blk + 8 + 16 * j, e);
            }
        } else if (type == T_Q2_K) {
            const float d = oracle_half_to_float(rd16(blk + 80));
            const float dmin = oracle_half_to_float(rd16(blk + 82));
            for (int w = 0; w < 256; ++w) {
                const uint8_t sc = blk[w >> 4];
                const float dl = d * (float)(sc & 15), ml = dmin * (float)(sc >> 4);
                o[w] = dl * (float)q2k_quant(blk, w) - ml;
            }
        } else if (type == T_Q3_K) {
            const float d = oracle_half_to_float(rd16(blk + 108));
            for (int w = 0; w < 256; ++w) {
                const float dl = d * (float)q3k_scale(blk, w >> 4);
                o[w] = dl * (float)q3k_quant(blk, w);
            }
        } else if (type == T_Q6_K) {
            const float d = oracle_half_to_float(rd16(blk + 208));
            for (int j = 0; j < 8; ++j)
                for (int e = 0; e < 32; ++e) {
                    const float dl = d * (float)(int8_t)blk[192 + 2 * j + (e >> 4)];
                    o[32 * j + e] = dl * (float)q6k_quant(blk, j, e);
                }
        } else {
            const float d = oracle_half_to_float(rd16(blk));
            const float dmin = oracle_half_to_float(rd16(blk + 2));
            for (int j = 0; j < 8; ++j) {
                int sc, m;
                q4k_scale_min(blk + 4, j, &sc, &m);
                const float dl = d * (float)sc, ml = dmin * (float)m;
                for (int e = 0; e < 32; ++e) {
                    const int q = type == T_Q4_K ? q4k_quant(blk, j, e) : q5k_quant(blk, j, e);
                    o[32 * j + e] = dl * (float)q - ml;
                }
            }
        }
    }
    return 0;
}

/* ---- integer block sums and y -------------------------------------------------- */

/* Exact integer dots.  sums[(c*nrows + r)*nsub + s] with nsub = K/16 for Q2_K, Q3_K and
 * Q6_K (one per 16-weight scale group) and K/32 otherwise (one per Q8_1 block).  Q2_K, Q4_K
 * and Q5_K use the unsigned quant (the min term is separate), Q3_K q with its offset, Q6_K
 * q - 32, Q8_0 the int8 quant. */
int oracle_block_sums(int type, const uint8_t *W, const uint8_t *xq, int32_t *sums,
                      int64_t nrows, int64_t K, int64_t ncols) {
    const int bytes = type_bytes(type), qk = type_qk(type);
    if (!bytes || K % qk) return -1;
    const int64_t nblk = K / qk, nkb = K / 32;
    const int64_t nsub = (type == T_Q6_K || type == T_Q2_K || type == T_Q3_K || iq_group16(type))
                             ? K / 16 : K / 32;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t c = 0; c < ncols; ++c)
        for (int64_t r = 0; r < nrows; ++r) {
            const uint8_t *row = W + r * nblk * bytes;
            const uint8_t *xc = xq + c * nkb * 36;
            int32_t *out = sums + (c * nrows + r) * nsub;
            for (int64_t b = 0; b < nblk; ++b) {
                const uint8_t *blk = row + b * bytes;
                if (type == T_Q8_0) {
                    const int8_t *a = (const int8_t *)(xc + b * 36 + 4);
                    int32_t s = 0;
                    for (int e = 0; e < 32; ++e) s += (int32_t)(int8_t)blk[2 + e] * a[e];
                    out[b] = s;
                    continue;
                }
                if (is_basic(type)) {
                    const int8_t *a = (const int8_t *)(xc + b * 36 + 4);
                    int32_t s = 0;
                    for (int e = 0; e < 32; ++e) s += basic_quant(type, blk, e) * a[e];
                    out[b] = s;
                    continue;
                }
                if (is_iq(type)) {
                    /* sum of L_w * q8 per scale group */
                    const int gs = iq_group16(type) ? 16 : 32, ng = 256 / gs;
                    for (int g = 0; g < ng; ++g) {
                        int32_t s = 0;
                        for (int e = 0; e < gs; ++e) {
                            const int w = gs * g + e;
                            s += iq_level(type, blk, w) * (int8_t)xc[(8 * b + (w >> 5)) * 36 + 4 + (w & 31)];
                        }
                        out[ng * b + g] = s;
                    }
                    continue;
                }
                if (type == T_IQ4_NL) {
                    const int8_t *a = (const int8_t *)(xc + b * 36 + 4);
                    int32_t s = 0;
                    for (int e = 0; e < 32; ++e) s += iq4nl_level(blk + 2, e) * a[e];
                    out[b] = s;
                    continue;
                }
                if (type == T_IQ4_XS) {
                    for (int j = 0; j < 8; ++j) {
                        const int8_t *a = (const int8_t *)(xc + (8 * b + j) * 36 + 4);
                        int32_t s = 0;
                        for (int e = 0; e < 32; ++e) s += iq4nl_level(blk + 8 + 16 * j, e) * a[e];
                        out[8 * b + j] = s;
                    }
                    continue;
                }
                if (type == T_Q2_K || type == T_Q3_K) {
                    for (int j = 0; j < 16; ++j) {
                        const int8_t *a = (const int8_t *)(xc + (8 * b + (j >> 1)) * 36 + 4) + 16 * (j & 1);
                        int32_t s = 0;
                        for (int e = 0; e < 16; ++e) {
                            const int w = 16 * j + e;
                            s += (type == T_Q2_K ? q2k_quant(blk, w) : q3k_quant(blk, w)) * a[e];
                        }
                        out[16 * b + j] = s;
                    }
                    continue;
                }
                for (int j = 0; j < 8; ++j) {
                    const int8_t *a = (const int8_t *)(xc + (8 * b + j) * 36 + 4);
                    if (type == T_Q6_K) {
                        int32_t s0 = 0, s1 = 0;
                        for (int e = 0; e < 16; ++e) s0 += q6k_quant(blk, j, e) * a[e];
                        for (int e = 16; e < 32; ++e) s1 += q6k_quant(blk, j, e) * a[e];
                        out[16 * b + 2 * j] = s0;
                        out[16 * b + 2 * j + 1] = s1;
                    } else {
                        int32_t s = 0;
                        for (int e = 0; e < 32; ++e)
                            s += (type == T_Q4_K ? q4k_quant(blk, j, e) : q5k_quant(blk, j, e)) * a[e];
                        out[8 * b + j] = s;
                    }
                }
            }
        }
    return 0;
}

/* The activation block's d8: fp16 at byte 0 (Q8_1), or fp32 at bytes 0-3 (the chained-input
 * blocks of the persistent chain). */
static inline double act_d8(const uint8_t *ab, int d32) {
    if (!d32) return (double)oracle_half_to_float(rd16(ab));
    float f;
    memcpy(&f, ab, 4);
    return (double)f;
}

/* y[c*nrows + r] in double from the exact block sums (same formula as the kernels). */
static int mmvq_impl(int type, const uint8_t *W, const uint8_t *xq, double *y, int64_t nrows,
                     int64_t K, int64_t ncols, int d32) {
    const int bytes = type_bytes(type), qk = type_qk(type);
    if (!bytes || K % qk) return -1;
    const int64_t nblk = K / qk, nkb = K / 32;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t c = 0; c < ncols; ++c)
        for (int64_t r = 0; r < nrows; ++r) {
            const uint8_t *row = W + r * nblk * bytes;
            const uint8_t *xc = xq + c * nkb * 36;
            double acc = 0.0;
            for (int64_t b = 0; b < nblk; ++b) {
                const uint8_t *blk = row + b * bytes;
                if (type == T_Q8_0) {
                    const uint8_t *ab = xc + b * 36;
                    const int8_t *a = (const int8_t *)(ab + 4);
                    int32_t s = 0;
                    for (int e = 0; e < 32; ++e) s += (int32_t)(int8_t)blk[2 + e] * a[e];
                    acc += (double)oracle_half_to_float(rd16(blk)) *
                           (double)act_d8(ab, d32) * (double)s;
                    continue;
                }
                if (is_basic(type)) {
                    /* d * d8 * sum(q * q8), plus m * d8 * sum(q8) for the _1 types */
                    const uint8_t *ab = xc + b * 36;
                    const int8_t *a = (const int8_t *)(ab + 4);
                    int32_t s = 0, sq = 0;
                    for (int e = 0; e < 32; ++e) {
                        s += basic_quant(type, blk, e) * a[e];
                        sq += a[e];
                    }
                    const double d8 = act_d8(ab, d32);
                    acc += (double)oracle_half_to_float(rd16(blk)) * d8 * (double)s;
                    if (type == T_Q4_1 || type == T_Q5_1)
                        acc += (double)oracle_half_to_float(rd16(blk + 2)) * d8 * (double)sq;
                    continue;
                }
                if (is_iq(type)) {
                    /* d * F * sum_g d8 * M_g * sum(L_w q8) */
                    const int gs = iq_group16(type) ? 16 : 32, ng = 256 / gs;
                    double sb = 0.0;
                    for (int g = 0; g < ng; ++g) {
                        const uint8_t *ab = xc + (8 * b + (gs * g >> 5)) * 36;
                        int32_t s = 0;
                        for (int e = 0; e < gs; ++e) {
                            const int w = gs * g + e;
                            s += iq_level(type, blk, w) * (int8_t)ab[4 + (w & 31)];
                        }
                        sb += act_d8(ab, d32) * (double)iq_mult(type, blk, g) * (double)s;
                    }
                    acc += (double)iq_d(type, blk) * iq_factor(type) * sb;
                    continue;
                }
                if (type == T_IQ4_NL) {
                    const uint8_t *ab = xc + b * 36;
                    const int8_t *a = (const int8_t *)(ab + 4);
                    int32_t s = 0;
                    for (int e = 0; e < 32; ++e) s += iq4nl_level(blk + 2, e) * a[e];
                    acc += (double)oracle_half_to_float(rd16(blk)) *
                           (double)act_d8(ab, d32) * (double)s;
                    continue;
                }
                if (type == T_IQ4_XS) {
                    /* d * sum_j d8_j * scale_j * sum(level * q8) */
                    double sb = 0.0;
                    for (int j = 0; j < 8; ++j) {
                        const uint8_t *ab = xc + (8 * b + j) * 36;
                        const int8_t *a = (const int8_t *)(ab + 4);
                        int32_t s = 0;
                        for (int e = 0; e < 32; ++e) s += iq4nl_level(blk + 8 + 16 * j, e) * a[e];
                        sb += (double)act_d8(ab, d32) * (double)iq4xs_scale(blk, j) * (double)s;
                    }
                    acc += (double)oracle_half_to_float(rd16(blk)) * sb;
                    continue;
                }
                if (type == T_Q2_K || type == T_Q3_K) {
                    /* per 16-weight group j: d * sc_j * d8 * sum(q q8), and for Q2_K
                     * - dmin * m_j * d8 * sum(q8) */
                    const double d = oracle_half_to_float(rd16(blk + (type == T_Q2_K ? 80 : 108)));
                    const double dmin = type == T_Q2_K ? oracle_half_to_float(rd16(blk + 82)) : 0.0;
                    double sd = 0.0, sm = 0.0;
                    for (int j = 0; j < 16; ++j) {
                        const uint8_t *ab = xc + (8 * b + (j >> 1)) * 36;
                        const int8_t *a = (const int8_t *)(ab + 4) + 16 * (j & 1);
                        int32_t si = 0, sq = 0;
                        for (int e = 0; e < 16; ++e) {
                            const int w = 16 * j + e;
                            si += (type == T_Q2_K ? q2k_quant(blk, w) : q3k_quant(blk, w)) * a[e];
                            sq += a[e];
                        }
                        const double d8 = act_d8(ab, d32);
                        const int sc = type == T_Q2_K ? (blk[j] & 15) : q3k_scale(blk, j);
                        sd += d8 * (double)sc * (double)si;
                        if (type == T_Q2_K) sm += d8 * (double)(blk[j] >> 4) * (double)sq;
                    }
                    acc += d * sd - dmin * sm;
                    continue;
                }
                if (type == T_Q6_K) {
                    const double d = oracle_half_to_float(rd16(blk + 208));
                    double sb = 0.0;
                    for (int j = 0; j < 8; ++j) {
                        const uint8_t *ab = xc + (8 * b + j) * 36;
                        const int8_t *a = (const int8_t *)(ab + 4);
                        int32_t s0 = 0, s1 = 0;
                        for (int e = 0; e < 16; ++e) s0 += q6k_quant(blk, j, e) * a[e];
                        for (int e = 16; e < 32; ++e) s1 += q6k_quant(blk, j, e) * a[e];
                        const int32_t sc0 = (int8_t)blk[192 + 2 * j], sc1 = (int8_t)blk[193 + 2 * j];
                        sb += (double)act_d8(ab, d32) *
                              ((double)sc0 * (double)s0 + (double)sc1 * (double)s1);
                    }
                    acc += d * sb;
                    continue;
                }
                const double d = oracle_half_to_float(rd16(blk));
                const double dmin = oracle_half_to_float(rd16(blk + 2));
                double sd = 0.0, sm = 0.0;
                for (int j = 0; j < 8; ++j) {
                    const uint8_t *ab = xc + (8 * b + j) * 36;
                    const int8_t *a = (const int8_t *)(ab + 4);
                    int32_t si = 0, sq = 0;
                    for (int e = 0; e < 32; ++e) {
                        si += (type == T_Q4_K ? q4k_quant(blk, j, e) : q5k_quant(blk, j, e)) * a[e];
                        sq += a[e];
                    }
                    int sc, m;
                    q4k_scale_min(blk + 4, j, &sc, &m);
                    const double d8 = act_d8(ab, d32);
                    sd += d8 * (double)sc * (double)si;
                    sm += d8 * (double)m * (double)sq;
                }
                acc += d * sd - dmin * sm;
            }
            y[c * nrows + r] = acc;
        }
    return 0;
}

int oracle_mmvq(int type, const uint8_t *W, const uint8_t *xq, double *y, int64_t nrows,
                int64_t K, int64_t ncols) {
    return mmvq_impl(type, W, xq, y, nrows, K, ncols, 0);
}

/* oracle_mmvq on blocks whose d8 is fp32 (bytes 0-3), unscaled. */
int oracle_mmvq_d32(int type, const uint8_t *W, const uint8_t *xq, double *y, int64_t nrows,
                    int64_t K, int64_t ncols) {
    return mmvq_impl(type, W, xq, y, nrows, K, ncols, 1);
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
