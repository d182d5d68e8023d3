// mmvq.cuh -- sm_100a MMVQ (quantized GEMV) kernel template.
//
// The reference's kernel is a CTA of (32, nwarps) threads computing rows_per_block rows,
// with the warps splitting K and a shared-memory cross-warp reduction (grid ceil(N/rpb);
// kernel_anvil/hip_codegen.py:228-333; docs/llama-cpp-kernel-analysis.md:107-148).  Here the
// same two knobs keep their roles -- nwarps = warps per CTA, rows_per_block = rows per tile
// -- but the bytes move the B200 way:
//
//   1. Persistent CTAs (the host sizes the grid to what is resident).  Each warp is an
//      autonomous consumer owning a ring of `nstages` tiles of RPB rows; tiles are dealt
//      round-robin over all warps of the grid.  A tile is one contiguous byte range of W,
//      streamed into shared memory by one bulk async copy (cp.async.bulk, the TMA
//      engine's untiled form) issued by lane 0 and completing on the stage's mbarrier.
//      The first copies go out BEFORE the programmatic-dependent-launch wait, so inside a
//      chain the weight stream of GEMV i+1 starts while GEMV i drains.  No register is
//      tied up by bytes in flight and no CTA-wide barrier sits in the tile loop.
//   2. After the wait the activation is staged once per CTA: either Q8_1 blocks from
//      global memory, or fp32 values brought in by one bulk copy and quantised to Q8_1 in
//      shared memory with the quantiser's exact arithmetic (the fused prologue that
//      removes the separate quantize_q8_1 launch).  Quants are stored in 16-byte chunks
//      with an XOR swizzle matched to the read pattern, plus fp32 scales d8, d8 * sum(q)
//      and int half-block sums of q.
//   3. Each lane owns whole weight blocks of its rows (lanes split a row's blocks the way
//      the reference loop splits kbx, kernel_anvil/hip_codegen.py:266-285).  Per block the
//      header is read once and the units (64-weight pairs of sub-blocks, or the single
//      Q8_0 block) are walked in a compile-time sequence, so the 6-bit scale unpacking is
//      a fixed bit extraction.  Dots are __dp4a; Q4_K high nibbles go through the
//      unsigned x signed form on the unshifted byte (x16, removed exactly by a shift).
//   4. Row sums are reduced with warp shuffles across the lanes sharing the row.
//
// Modes: kModeQ81 (Q8_1 input), kModeF32 (fp32 input, fused quantisation), kModeSums
// (Q8_1 input; the exact int32 block dots are written instead of y: the parity probe
// behind anvil_mmvq_block_sums).
#pragma once

#include "anvil_common.cuh"

namespace anvil {

constexpr int kMaxWarps = 8;       // 256 threads: llama.cpp's MMVQ upper bound
constexpr int kMaxCols = 8;        // MMVQ_MAX_BATCH_SIZE
constexpr int kMaxSmem = 227 * 1024;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // default bound on any device wait (2 s)

constexpr int kModeQ81 = 0;
constexpr int kModeF32 = 1;
constexpr int kModeSums = 2;
// kModeGLU: y = silu(W_gate x) * (W_up x) for one column.  Weights segW[0] (gate) and
// segW[1] (up); a tile stages RPB/2 rows of each, gate rows first, and the lane that owns
// gate row i owns up row i, so the epilogue combines them without leaving registers.
constexpr int kModeGLU = 3;

constexpr int kMaxSeg = 4;  // matrices of one launch (GEMVs sharing the activation)

struct MmvqArgs {
    const void *x;      // Q8_1 blocks (kModeQ81 / kModeSums) or fp32 values (kModeF32)
    int32_t *sums;      // kModeSums output (one segment)
    uint64_t wait_ns;   // bound on every mbarrier wait
    int K, nstages;
    // Segments: GEMVs of one weight type reading x, dealt as one tile sequence.
    // Segment s: weights segW[s] (raw GGUF blocks, row-major), segRows[s] rows, outputs
    // segY[s] (ncols x segRows[s]); its tiles are [segTile[s], segTile[s + 1]).
    int nseg;
    const uint8_t *segW[kMaxSeg];
    float *segY[kMaxSeg];
    int segRows[kMaxSeg];
    int segTile[kMaxSeg + 1];
};

// Segment holding tile `tile` (segments are few: a linear scan).
__device__ __forceinline__ int mmvq_segment(const MmvqArgs &a, int tile) {
    int s = 0;
    while (s + 1 < a.nseg && tile >= a.segTile[s + 1]) ++s;
    return s;
}

// The Q8_1 block scale d = RN32(amax / 127), the correctly rounded IEEE quotient, without a
// division (the IEEE division and reciprocal intrinsics cost on the order of a thousand
// cycles here): the fp64 product amax * RN64(1/127), rounded to fp32.  That is exact for every
// float amax: amax / 127 = m 2^e / 127 with m < 2^24 is never a float32 rounding midpoint (a
// midpoint has an even numerator over an odd 127) and lies at least 2^-32 (relative) away
// from one, while the fp64 product is within 2^-52 of amax / 127 (also checked on the host
// for every float32 mantissa, every subnormal and the top binade).
__device__ __forceinline__ float q8_scale(float amax) { return float(double(amax) * (1.0 / 127.0)); }

// roundf(RN32(x / d)), the quantiser's q, for d > 0 and |x| <= 127 d, given rd64 = RN64(1/d)
// and rd = RN32(rd64) = RN32(1/d) (fp64 then fp32 rounding equals direct fp32 rounding, since
// 53 >= 2 * 24 + 2).  Fast path: t = x * rd differs from x / d by at most |x/d| (2^-24 +
// 2^-24 + 2^-48) < 127.5 * 2^-23 ~ 1.6e-5, and RN32(x / d) differs from x / d by at most
// 0.5 ulp < 7.6e-6, so both round to the same integer unless t lies within 2.4e-5 of a
// half-integer (1e-4 is the margin used).  There the quotient is RN32(double(x) * rd64): its
// error is below 2^-51.9 (relative), and x / d = X 2^a / (D 2^b) (X, D < 2^24) is never a
// float32 midpoint and lies at least 2^-49 (relative) away from one, so rounding to fp32 gives
// RN32(x / d) exactly.
__device__ __forceinline__ int quant_q8(float x, float rd, double rd64) {
    const float t = x * rd;
    const float f = fabsf(t) - floorf(fabsf(t));  // fractional part of |t|
    if (fabsf(f - 0.5f) > 1e-4f) return int(roundf(t));
    return int(roundf(float(double(x) * rd64)));
}

// True where t = x * rd needs the exact quotient: within 1e-4 of a half-integer, or not a
// finite number (rd = inf for a subnormal d).
__device__ __forceinline__ bool near_half(float t) {
    const float a = fabsf(t);
    return !(fabsf(a - floorf(a) - 0.5f) > 1e-4f);
}

// The quants of 16 values of one Q8_1 block half (quant_q8 for each), packed four to a word
// (value 4k + i in byte i of word k), and their sum.  The fast path runs for all 16 values
// without a branch, so their instruction chains overlap; the exact quotient is taken in a
// second pass only when some value needs it.  amax == 0 gives all zeros.
__device__ __forceinline__ void quant16(const float (&v)[16], float amax, float rd, double rd64,
                                        uint32_t (&w)[4], int &sum) {
    int q[16];
    bool near = false;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float t = v[i] * rd;
        near |= near_half(t);
        q[i] = int(roundf(t));
    }
    if (near && amax != 0.0f) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (near_half(v[i] * rd)) q[i] = int(roundf(float(double(v[i]) * rd64)));
    }
    sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) word |= (amax == 0.0f ? 0u : uint32_t(q[4 * k + i]) & 0xFFu) << (8 * i);
        w[k] = word;
        sum = __dp4a(int(word), 0x01010101, sum);
    }
}

struct MmvqSmem {
    int bar, w, stage, xbuf, aq, ad, ads, as, total;
};

__host__ __device__ inline int mmvq_type_bytes(int qt) {
    switch (qt) {
    case kTypeQ4_0: return 18;
    case kTypeQ4_1: return 20;
    case kTypeQ5_0: return 22;
    case kTypeQ5_1: return 24;
    case kTypeIQ4_NL: return 18;
    case kTypeIQ4_XS: return 136;
    case kTypeIQ2_XXS: return 66;
    case kTypeIQ2_XS: return 74;
    case kTypeIQ2_S: return 82;
    case kTypeIQ3_XXS: return 98;
    case kTypeIQ3_S: return 110;
    case kTypeIQ1_S: return 50;
    case kTypeIQ1_M: return 56;
    case kTypeQ2_K: return 84;
    case kTypeQ3_K: return 110;
    case kTypeQ4_K: return 144;
    case kTypeQ5_K: return 176;
    case kTypeQ6_K: return 210;
    default: return 34;
    }
}
__host__ __device__ inline int mmvq_type_qk(int qt) {
    return qt == kTypeQ8_0 || qt == kTypeQ4_0 || qt == kTypeQ4_1 || qt == kTypeQ5_0 ||
                   qt == kTypeQ5_1 || qt == kTypeIQ4_NL
               ? 32
               : 256;
}

// The 32-weight "basic" types (one Q8_1 block per weight block, one unit per block).
template <int QT>
constexpr bool kBasic = QT == kTypeQ4_0 || QT == kTypeQ4_1 || QT == kTypeQ5_0 || QT == kTypeQ5_1;
template <int QT>
constexpr bool kBlock32 = QT == kTypeQ8_0 || kBasic<QT> || QT == kTypeIQ4_NL;
// The lattice I-quants (256-weight super-blocks of signed grid rows).
template <int QT>
constexpr bool kIQLattice = QT == kTypeIQ2_XXS || QT == kTypeIQ2_XS || QT == kTypeIQ2_S ||
                            QT == kTypeIQ3_XXS || QT == kTypeIQ3_S || QT == kTypeIQ1_S ||
                            QT == kTypeIQ1_M;
// The types with 16-weight scale groups (two per Q8_1 block): one block sum per group.
template <int QT>
constexpr bool kSub16 = QT == kTypeQ6_K || QT == kTypeQ2_K || QT == kTypeQ3_K ||
                        QT == kTypeIQ2_XS || QT == kTypeIQ2_S || QT == kTypeIQ1_M;

// Bytes of one column's swizzled activation quants: 2 chunks of 16 B per Q8_1 block,
// padded to whole 16-chunk groups so the XOR swizzle never leaves the column.
__host__ __device__ inline int act_col_bytes(int nkb) { return ((2 * nkb + 15) & ~15) * 16; }

// Dynamic shared memory layout; identical on host (launch size) and device.
// [mbarriers][nwarps x nstages weight stages][fp32 x (fused mode)][act quants][d8][d8*sum q][sums]
__host__ __device__ inline MmvqSmem mmvq_smem_layout(int qt, int K, int ncols, int rpb,
                                                     int nwarps, int nstages, int mode) {
    const int row_bytes = (K / mmvq_type_qk(qt)) * mmvq_type_bytes(qt);
    const int nkb = K / 32;
    MmvqSmem L;
    L.bar = 0;
    L.w = (8 * (nwarps * nstages + 1) + 15) & ~15;
    // +32 per stage: up to 15 bytes of head misalignment plus one word of funnel over-read.
    L.stage = ((rpb * row_bytes + 32) + 15) & ~15;
    L.xbuf = L.w + nwarps * nstages * L.stage;
    L.aq = L.xbuf;  // the fused mode quantises straight from registers (no fp32 copy)
    L.ad = L.aq + ncols * act_col_bytes(nkb);
    L.ads = L.ad + ncols * nkb * 4;
    L.as = (L.ads + ncols * nkb * 4 + 15) & ~15;
    L.total = L.as + ncols * nkb * 8;
    return L;
}

// Swizzled position of 16-byte activation chunk `ci` (chunks 2kb, 2kb+1 hold Q8_1 block kb).
// K-quants: a quarter warp reads the same chunk of 8 consecutive super-blocks (chunk
// stride 16), so the chunk's slot in its 128-byte line is XORed with bits 4-6 of ci.
// Q8_0: a quarter warp reads chunk 2b+h of 8 consecutive blocks (stride 2), so the odd
// line of each pair of lines is shifted by one slot.
template <int QT>
__device__ __forceinline__ int act_chunk(int ci) {
    if constexpr (kBlock32<QT>) {
        return ci ^ ((ci >> 3) & 1);
    } else {
        return ci ^ ((ci >> 4) & 7);
    }
}

// ---- small device helpers ------------------------------------------------------------

// 32 bytes starting at a 2-byte aligned shared-memory address, as 8 little-endian words:
// nine aligned word loads and a funnel shift by the address's byte offset.
__device__ __forceinline__ void lds32_a2(const uint8_t *p, uint32_t (&w)[8]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = uint32_t(a & 3) * 8;
    uint32_t prev = q[0];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t nx = q[k + 1];
        w[k] = __funnelshift_r(prev, nx, sh);
        prev = nx;
    }
}

// 16 bytes starting at a 2-byte aligned shared-memory address, as 4 little-endian words:
// five aligned word loads (at most 3 bytes read past the 16) and a funnel shift.
__device__ __forceinline__ void lds16B_a2(const uint8_t *p, uint32_t (&w)[4]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = uint32_t(a & 3) * 8;
    uint32_t prev = q[0];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t nx = q[k + 1];
        w[k] = __funnelshift_r(prev, nx, sh);
        prev = nx;
    }
}

// 32 / 16 bytes at a 4-byte aligned shared-memory address as little-endian words.  Used
// where the block size keeps the quants word aligned: weights start 16-byte aligned (checked
// on the host) and every row is a whole number of 84-, 20-, 24- or 136-byte blocks (Q2_K,
// Q4_1, Q5_1, IQ4_XS), so row, block and quant offsets are multiples of 4.
__device__ __forceinline__ void lds32_a4(const uint8_t *p, uint32_t (&w)[8]) {
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p);
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = q[k];
}
__device__ __forceinline__ void lds16B_a4(const uint8_t *p, uint32_t (&w)[4]) {
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p);
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = q[k];
}

// Bits 0..3 of h moved to bit 4 of bytes 0..3 (the fifth bit of four 5-bit quants): one
// multiply places copies of h at bits 4, 11, 18 and 25 (they do not overlap, so nothing
// carries) and the mask keeps bit i of copy i.
__device__ __forceinline__ uint32_t spread_bit4(uint32_t h) {
    return ((h & 0xFu) * 0x02040810u) & 0x10101010u;
}

__device__ __forceinline__ uint32_t lds16(const uint8_t *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}

__device__ __forceinline__ void lds32_a16(const uint8_t *p, uint32_t (&w)[8]) {
    const uint4 a = *reinterpret_cast<const uint4 *>(p);
    const uint4 b = *reinterpret_cast<const uint4 *>(p + 16);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}

// Unsigned bytes of `a` dotted with signed bytes of `b`, plus c (PTX dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One Q8_1 activation block as seen by a dot: 32 quants, d8, d8 * sum(q), half sums.
struct ActBlk {
    uint32_t q[8];
    float d, ds;
    int slo, shi;
};

struct ActView {  // one column's staged activation
    const uint8_t *aq;
    const float *ad, *ads;
    const int2 *as;
};

template <int QT>
__device__ __forceinline__ void load_act(const ActView &v, int kb, ActBlk &a) {
    const uint4 c0 = *reinterpret_cast<const uint4 *>(v.aq + act_chunk<QT>(2 * kb) * 16);
    const uint4 c1 = *reinterpret_cast<const uint4 *>(v.aq + act_chunk<QT>(2 * kb + 1) * 16);
    a.q[0] = c0.x; a.q[1] = c0.y; a.q[2] = c0.z; a.q[3] = c0.w;
    a.q[4] = c1.x; a.q[5] = c1.y; a.q[6] = c1.z; a.q[7] = c1.w;
    a.d = v.ad[kb];
    a.ds = 0.f;
    a.slo = a.shi = 0;
    if constexpr (QT == kTypeQ4_K || QT == kTypeQ5_K || QT == kTypeQ4_1 || QT == kTypeQ5_1)
        a.ds = v.ads[kb];
    if constexpr (kSub16<QT> || QT == kTypeQ4_0 || QT == kTypeQ5_0 || QT == kTypeIQ1_S) {
        const int2 s = v.as[kb];
        a.slo = s.x;
        a.shi = s.y;
    }
}

// ---- per-type block decode and dot ------------------------------------------------------
//
// A lane handling (row, block) first reads the block header (BlkHdr), then for each unit U
// (compile time) decodes the unit's weight bytes and dots them with the unit's activation
// blocks.  Units: Q4_K/Q5_K U = sub-block pair (2U, 2U+1); Q6_K U = (h, t) = (U>>1, U&1),
// sub-blocks 4h+t and 4h+2+t; Q2_K/Q3_K U = weights [64U, 64U+64) (Q8_1 blocks 2U, 2U+1 of
// the super-block, scale groups 4U..4U+3); Q8_0 one unit, the block itself.

struct BlkHdr {
    float d, dmin;
    uint32_t s0, s1, s2;  // K4/K5 packed scales[12]
};

template <int QT> struct Units { static constexpr int n = 4; };
template <> struct Units<kTypeQ8_0> { static constexpr int n = 1; };
template <> struct Units<kTypeQ4_0> { static constexpr int n = 1; };
template <> struct Units<kTypeQ4_1> { static constexpr int n = 1; };
template <> struct Units<kTypeQ5_0> { static constexpr int n = 1; };
template <> struct Units<kTypeQ5_1> { static constexpr int n = 1; };
template <> struct Units<kTypeIQ4_NL> { static constexpr int n = 1; };

// The 16 non-linear int8 levels of IQ4_NL / IQ4_XS (ggml's kvalues_iq4nl, as listed by
// gguf-py quants.py IQ4_NL.kvalues), four per little-endian word.
constexpr uint32_t iq4_word(int a, int b, int c, int d) {
    return uint32_t(uint8_t(a)) | uint32_t(uint8_t(b)) << 8 | uint32_t(uint8_t(c)) << 16 |
           uint32_t(uint8_t(d)) << 24;
}
constexpr uint32_t kIQ4Levels0 = iq4_word(-127, -104, -83, -65);
constexpr uint32_t kIQ4Levels1 = iq4_word(-49, -35, -22, -10);
constexpr uint32_t kIQ4Levels2 = iq4_word(1, 13, 25, 38);
constexpr uint32_t kIQ4Levels3 = iq4_word(53, 69, 89, 113);

// Levels of four 4-bit indices held as the four nibbles of s (bits 0..15): two byte permutes
// look each index up in the low and high halves of the table (selector bits 0-2), a third
// takes byte n from the high-half result where bit 3 of nibble n is set.
__device__ __forceinline__ uint32_t iq4_levels4(uint32_t s) {
    const uint32_t lo = __byte_perm(kIQ4Levels0, kIQ4Levels1, s & 0x7777u);
    const uint32_t hi = __byte_perm(kIQ4Levels2, kIQ4Levels3, s & 0x7777u);
    return __byte_perm(lo, hi, 0x3210u | ((s & 0x8888u) >> 1));
}

// The eight level indices packed in one word of quants (byte i: low nibble and high nibble)
// -> lo: the levels of the four low nibbles, hi: those of the four high nibbles, byte i each.
__device__ __forceinline__ void iq4_levels8(uint32_t v, uint32_t &lo, uint32_t &hi) {
    const uint32_t a = iq4_levels4(v & 0xFFFFu);  // bytes 0, 1: (lo, hi, lo, hi)
    const uint32_t b = iq4_levels4(v >> 16);      // bytes 2, 3
    lo = __byte_perm(a, b, 0x6420u);
    hi = __byte_perm(a, b, 0x7531u);
}

// Q8_1 blocks consumed by unit U of super-block b.
template <int QT, int U>
__device__ __forceinline__ void unit_kb(int b, int &kb0, int &kb1) {
    if constexpr (kBlock32<QT>) {
        kb0 = b;
        kb1 = b;
    } else if constexpr (QT == kTypeQ6_K) {
        kb0 = 8 * b + 4 * (U >> 1) + (U & 1);
        kb1 = kb0 + 2;
    } else {
        kb0 = 8 * b + 2 * U;
        kb1 = kb0 + 1;
    }
}

template <int QT>
__device__ __forceinline__ BlkHdr load_hdr(const uint8_t *blk) {
    BlkHdr h;
    h.dmin = 0.f;
    h.s0 = h.s1 = h.s2 = 0;
    if constexpr (QT == kTypeQ4_K || QT == kTypeQ5_K) {
        const uint4 v = *reinterpret_cast<const uint4 *>(blk);
        h.d = h2f(v.x);
        h.dmin = h2f(v.x >> 16);
        h.s0 = v.y;
        h.s1 = v.z;
        h.s2 = v.w;
    } else if constexpr (QT == kTypeQ6_K) {
        h.d = h2f(lds16(blk + 208));
    } else if constexpr (QT == kTypeIQ4_XS) {
        h.d = h2f(lds16(blk));
        h.s0 = lds16(blk + 2);                                 // scales_h
        h.s1 = lds16(blk + 4) | (lds16(blk + 6) << 16);        // scales_l[4]
    } else if constexpr (QT == kTypeQ2_K) {
        h.d = h2f(lds16(blk + 80));
        h.dmin = h2f(lds16(blk + 82));
    } else if constexpr (QT == kTypeQ3_K) {
        // the 12 scale bytes as three words (2-byte aligned block)
        h.d = h2f(lds16(blk + 108));
        h.s0 = lds16(blk + 96) | (lds16(blk + 98) << 16);
        h.s1 = lds16(blk + 100) | (lds16(blk + 102) << 16);
        h.s2 = lds16(blk + 104) | (lds16(blk + 106) << 16);
    } else if constexpr (QT == kTypeQ4_1 || QT == kTypeQ5_1) {
        h.d = h2f(lds16(blk));
        h.dmin = h2f(lds16(blk + 2));  // m, the block's added minimum
    } else if constexpr (QT == kTypeIQ1_M) {
        // bits 12-15 of scale word i (bytes 48 + 2i) are bits 4i..4i+3 of the fp16 d
        h.d = h2f((lds16(blk + 48) >> 12) | ((lds16(blk + 50) >> 12) << 4) |
                  ((lds16(blk + 52) >> 12) << 8) | ((lds16(blk + 54) >> 12) << 12));
    } else {
        h.d = h2f(lds16(blk));
    }
    return h;
}

// Six-bit scale and min of sub-blocks 2U and 2U+1 (gguf-py quants.py:478-501,
// Q4_K.get_scale_min): for j < 4 sc = s[j] & 63, m = s[j+4] & 63; for j >= 4
// sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4, m = (s[j+4] >> 4) | (s[j] >> 6) << 4.
template <int U>
__device__ __forceinline__ void scale_min_pair(const BlkHdr &h, int &sc0, int &sc1, int &m0,
                                               int &m1) {
    constexpr int sh = (U & 1) * 16;  // bytes 2U%4 and 2U%4+1 of each word
    if constexpr (U < 2) {
        const uint32_t scp = (h.s0 >> sh) & 0x3F3Fu, mp = (h.s1 >> sh) & 0x3F3Fu;
        sc0 = scp & 0xFF;
        sc1 = scp >> 8;
        m0 = mp & 0xFF;
        m1 = mp >> 8;
    } else {
        const uint32_t b0 = h.s0 >> sh, b1 = h.s1 >> sh, b2 = h.s2 >> sh;
        const uint32_t scp = (b2 & 0x0F0Fu) | ((b0 >> 2) & 0x3030u);
        const uint32_t mp = ((b2 >> 4) & 0x0F0Fu) | ((b1 >> 2) & 0x3030u);
        sc0 = scp & 0xFF;
        sc1 = (scp >> 8) & 0xFF;
        m0 = mp & 0xFF;
        m1 = (mp >> 8) & 0xFF;
    }
}

// ---- lattice I-quants ----------------------------------------------------------------
// Grid rows are read through L1 from the generated tables (one word of 8 or 4 int8 values
// per row, value 0 in the lowest byte).  Layouts, with sub-block j = weights 32j..32j+31
// and group k = weights 8k..8k+7 (gguf-py gguf/quants.py IQ*.dequantize_blocks):
//   IQ2_XXS  66 B: d @0; at 2+8j: 4 row bytes (256-row grid), then a u32 of four 7-bit sign
//            indices (bits 7l) and the scale (bits 28-31)
//   IQ2_XS   74 B: d @0; u16 per group @2+2k: row (bits 0-8, 512 rows), sign index (9-15);
//            scale nibbles @66, one per 16 weights
//   IQ2_S    82 B: d @0; row bits 0-7 @2+k, sign byte @34+k, row bits 8-9 at bit 2l of
//            byte 66+j (1024 rows), scale nibbles @74
//   IQ3_XXS  98 B: d @0; a row byte per 4 weights @2 (256 rows of 4); u32 @66+4j: sign
//            indices and scale as IQ2_XXS
//   IQ3_S   110 B: d @0; row bits 0-7 per 4 weights @2, bit 8 at bit r of byte 66+j (512
//            rows of 4), sign byte @74+k, scale nibble j @106
//   IQ1_S    50 B: d @0; row bits 0-7 @2+k; u16 @34+2j: row bits 8-10 of group 4j+l at
//            bits 3l, scale bits 12-14, delta sign bit 15 (2048 rows of -1/0/1)
//   IQ1_M    56 B: row bits 0-7 @k; nibble k @32 (low first): row bits 8-10, delta sign
//            bit 3; u16 scale words @48: 3-bit scale of 16 weights 16(4i+t) at bits 3t of
//            word i, d in the top nibbles (load_hdr)
// A weight is d * F * M * L: L the signed grid value (IQ1: 8 grid +- 1 with the delta),
// M = 2 scale + 1 (IQ3_S: 1 + 2 scale) for its 16- or 32-weight group, F = 1/8 (IQ2, IQ1),
// 1/4 (IQ3_XXS) or 1 (IQ3_S).
#define ANVIL_IQ_TABLE static __device__ const
#include "iq_grids.h"
#undef ANVIL_IQ_TABLE

// The sign byte of 7-bit index i: bit 7 completes an even count of set bits (the rule of
// the kIqSigns table, computed instead of loaded).
__device__ __forceinline__ uint32_t iq_sign_byte(uint32_t i) {
    return i | ((__popc(i) & 1u) << 7);
}

// Four positive int8 values with bits 0..3 of b negating values 0..3: b's bits spread to
// 0x00 / 0xFF byte masks, then -v = (v ^ 0xFF) + 1 per byte (grid values are >= 1, so no
// byte carries into the next).
__device__ __forceinline__ uint32_t iq_signed4(uint32_t v, uint32_t b) {
    const uint32_t m = (((b & 15u) * 0x00204081u) & 0x01010101u) * 0xFFu;
    return (v ^ m) + (m & 0x01010101u);
}

// One 8-value grid row with its sign byte, as two words.
__device__ __forceinline__ void iq_row8(uint64_t row, uint32_t sgn, uint32_t &lo, uint32_t &hi) {
    lo = iq_signed4(uint32_t(row), sgn);
    hi = iq_signed4(uint32_t(row >> 32), sgn >> 4);
}

__device__ __forceinline__ uint32_t lds32_2(const uint8_t *p) { return lds16(p) | (lds16(p + 2) << 16); }

// The 32 signed levels of sub-block j as 8 words (word w = values 4w..4w+3).
template <int QT>
__device__ __forceinline__ void iq_sub(const uint8_t *blk, int j, uint32_t (&q)[8]) {
    if constexpr (QT == kTypeIQ2_XXS) {
        const uint32_t rows = lds32_2(blk + 2 + 8 * j), aux = lds32_2(blk + 6 + 8 * j);
#pragma unroll
        for (int l = 0; l < 4; ++l)
            iq_row8(__ldg(&kIq2xxsGrid[(rows >> (8 * l)) & 0xFFu]),
                    iq_sign_byte((aux >> (7 * l)) & 127u), q[2 * l], q[2 * l + 1]);
    } else if constexpr (QT == kTypeIQ2_XS) {
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t e = lds16(blk + 2 + 8 * j + 2 * l);
            iq_row8(__ldg(&kIq2xsGrid[e & 511u]), iq_sign_byte(e >> 9), q[2 * l], q[2 * l + 1]);
        }
    } else if constexpr (QT == kTypeIQ2_S) {
        const uint32_t lo = lds32_2(blk + 2 + 4 * j), sg = lds32_2(blk + 34 + 4 * j);
        const uint32_t hb = blk[66 + j];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t r = ((lo >> (8 * l)) & 0xFFu) | (((hb >> (2 * l)) & 3u) << 8);
            iq_row8(__ldg(&kIq2sGrid[r]), sg >> (8 * l), q[2 * l], q[2 * l + 1]);
        }
    } else if constexpr (QT == kTypeIQ3_XXS) {
        const uint32_t r0 = lds32_2(blk + 2 + 8 * j), r1 = lds32_2(blk + 6 + 8 * j);
        const uint32_t aux = lds32_2(blk + 66 + 4 * j);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t rr = l < 2 ? r0 : r1;
            const uint32_t sgn = iq_sign_byte((aux >> (7 * l)) & 127u);
            q[2 * l] = iq_signed4(__ldg(&kIq3xxsGrid[(rr >> (16 * (l & 1))) & 0xFFu]), sgn);
            q[2 * l + 1] = iq_signed4(__ldg(&kIq3xxsGrid[(rr >> (16 * (l & 1) + 8)) & 0xFFu]), sgn >> 4);
        }
    } else if constexpr (QT == kTypeIQ3_S) {
        const uint32_t r0 = lds32_2(blk + 2 + 8 * j), r1 = lds32_2(blk + 6 + 8 * j);
        const uint32_t hb = blk[66 + j], sg = lds32_2(blk + 74 + 4 * j);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const uint32_t idx = (((r < 4 ? r0 : r1) >> (8 * (r & 3))) & 0xFFu) | (((hb >> r) & 1u) << 8);
            q[r] = iq_signed4(__ldg(&kIq3sGrid[idx]), sg >> (4 * r));
        }
    } else if constexpr (QT == kTypeIQ1_S) {
        const uint32_t lo = lds32_2(blk + 2 + 4 * j), qh = lds16(blk + 34 + 2 * j);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint64_t row = __ldg(&kIq1sGrid[((lo >> (8 * l)) & 0xFFu) | (((qh >> (3 * l)) & 7u) << 8)]);
            q[2 * l] = uint32_t(row);
            q[2 * l + 1] = uint32_t(row >> 32);
        }
    } else if constexpr (QT == kTypeIQ1_M) {
        const uint32_t lo = lds32_2(blk + 4 * j), nb = lds16(blk + 32 + 2 * j);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint64_t row = __ldg(&kIq1sGrid[((lo >> (8 * l)) & 0xFFu) | (((nb >> (4 * l)) & 7u) << 8)]);
            q[2 * l] = uint32_t(row);
            q[2 * l + 1] = uint32_t(row >> 32);
        }
    }
}

// Scale multiplier M of scale group sg (a sub-block, or 16 weights for the kSub16 types).
template <int QT>
__device__ __forceinline__ int iq_mult(const uint8_t *blk, int sg) {
    if constexpr (QT == kTypeIQ2_XXS) return 2 * int(blk[2 + 8 * sg + 7] >> 4) + 1;
    if constexpr (QT == kTypeIQ2_XS) return 2 * int((blk[66 + (sg >> 1)] >> (4 * (sg & 1))) & 15) + 1;
    if constexpr (QT == kTypeIQ2_S) return 2 * int((blk[74 + (sg >> 1)] >> (4 * (sg & 1))) & 15) + 1;
    if constexpr (QT == kTypeIQ3_XXS) return 2 * int(blk[66 + 4 * sg + 3] >> 4) + 1;
    if constexpr (QT == kTypeIQ3_S) return 1 + 2 * int((blk[106 + (sg >> 1)] >> (4 * (sg & 1))) & 15);
    if constexpr (QT == kTypeIQ1_S) return 2 * int((lds16(blk + 34 + 2 * sg) >> 12) & 7) + 1;
    if constexpr (QT == kTypeIQ1_M) return 2 * int((lds16(blk + 48 + 2 * (sg >> 2)) >> (3 * (sg & 3))) & 7) + 1;
    return 0;
}

template <int QT>
constexpr float kIQFactor = QT == kTypeIQ3_XXS ? 0.25f : QT == kTypeIQ3_S ? 1.0f : 0.125f;

// Decoded weight bytes of one unit of one row (q0 pairs with Q8_1 block kb0, q1 with kb1).
struct WBytes {
    uint32_t q0[8], q1[8];
};

template <int QT, int U>
__device__ __forceinline__ void load_unit(const uint8_t *blk, WBytes &w) {
    if constexpr (QT == kTypeQ4_K) {
        uint32_t v[8];
        lds32_a16(blk + 16 + 32 * U, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            w.q0[k] = v[k] & 0x0F0F0F0Fu;
            w.q1[k] = v[k] & 0xF0F0F0F0u;  // high nibbles in place (x16)
        }
    } else if constexpr (QT == kTypeQ5_K) {
        uint32_t v[8], qh[8];
        lds32_a16(blk + 48 + 32 * U, v);
        lds32_a16(blk + 16, qh);  // fifth bit of weight e of sub-block j = bit j of qh[e]
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            w.q0[k] = (v[k] & 0x0F0F0F0Fu) | (((qh[k] >> (2 * U)) & 0x01010101u) << 4);
            w.q1[k] = ((v[k] >> 4) & 0x0F0F0F0Fu) | (((qh[k] >> (2 * U + 1)) & 0x01010101u) << 4);
        }
    } else if constexpr (QT == kTypeQ6_K) {
        // unit (h, t): ql bytes [64h+32t, +32) hold sub-block 4h+t (low nibbles) and
        // 4h+2+t (high nibbles); qh bytes [32h, +32) hold their top two bits at shifts
        // 2t and 4+2t (gguf-py quants.py:563-569).
        constexpr int h = U >> 1, t = U & 1;
        uint32_t ql[8], qh[8];
        lds32_a2(blk + 64 * h + 32 * t, ql);
        lds32_a2(blk + 128 + 32 * h, qh);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            w.q0[k] = (ql[k] & 0x0F0F0F0Fu) | (((qh[k] >> (2 * t)) & 0x03030303u) << 4);
            w.q1[k] = ((ql[k] >> 4) & 0x0F0F0F0Fu) | ((qh[k] >> (2 * t)) & 0x30303030u);
        }
    } else if constexpr (QT == kTypeIQ4_XS) {
        // groups 2U and 2U+1: qs bytes [32U, 32U + 32); within a group byte e holds weight e
        // (low nibble) and weight 16 + e (high nibble)
        uint32_t v[8];
        lds32_a4(blk + 8 + 32 * U, v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            iq4_levels8(v[k], w.q0[k], w.q0[4 + k]);
            iq4_levels8(v[4 + k], w.q1[k], w.q1[4 + k]);
        }
    } else if constexpr (kIQLattice<QT>) {
        iq_sub<QT>(blk, 2 * U, w.q0);
        iq_sub<QT>(blk, 2 * U + 1, w.q1);
    } else if constexpr (QT == kTypeIQ4_NL) {
        uint32_t v[4];
        lds16B_a2(blk + 2, v);
#pragma unroll
        for (int k = 0; k < 4; ++k) iq4_levels8(v[k], w.q0[k], w.q0[4 + k]);
    } else if constexpr (QT == kTypeQ2_K || QT == kTypeQ3_K) {
        // weight 64U + 32i + l (i = 0, 1: Q8_1 block kb0, kb1) is bits 2(2(U&1) + i) of qs
        // byte 32(U>>1) + l; Q3_K adds bit 2U + i of hmask[l] as bit 2 (q + 4 when set)
        constexpr int qs_off = QT == kTypeQ2_K ? 16 : 32;
        constexpr int s0 = 4 * (U & 1);
        uint32_t v[8];
        if constexpr (QT == kTypeQ2_K) {
            lds32_a4(blk + qs_off + 32 * (U >> 1), v);
        } else {
            lds32_a2(blk + qs_off + 32 * (U >> 1), v);  // 110-byte blocks: 2-byte aligned
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            w.q0[k] = (v[k] >> s0) & 0x03030303u;
            w.q1[k] = (v[k] >> (s0 + 2)) & 0x03030303u;
        }
        if constexpr (QT == kTypeQ3_K) {
            uint32_t hm[8];
            lds32_a2(blk, hm);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                w.q0[k] |= ((hm[k] >> (2 * U)) & 0x01010101u) << 2;
                w.q1[k] |= ((hm[k] >> (2 * U + 1)) & 0x01010101u) << 2;
            }
        }
    } else if constexpr (kBasic<QT>) {
        // quants in Q8_1 element order: words 0..3 the low nibbles of qs[0..15] (weights
        // 0..15), words 4..7 the high nibbles (weights 16..31); the 5-bit types add bit e of
        // qh as bit 4 of weight e (gguf-py quants.py Q4_0..Q5_1 dequantize_blocks)
        constexpr int qs_off = QT == kTypeQ4_0 ? 2 : QT == kTypeQ4_1 ? 4 : QT == kTypeQ5_0 ? 6 : 8;
        uint32_t v[4];
        if constexpr (QT == kTypeQ4_1 || QT == kTypeQ5_1) {
            lds16B_a4(blk + qs_off, v);
        } else {
            lds16B_a2(blk + qs_off, v);  // 18- and 22-byte blocks: 2-byte aligned
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            w.q0[k] = v[k] & 0x0F0F0F0Fu;
            w.q0[4 + k] = (v[k] >> 4) & 0x0F0F0F0Fu;
        }
        if constexpr (QT == kTypeQ5_0 || QT == kTypeQ5_1) {
            constexpr int qh_off = QT == kTypeQ5_0 ? 2 : 4;
            const uint32_t qh = lds16(blk + qh_off) | (lds16(blk + qh_off + 2) << 16);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                w.q0[k] |= spread_bit4((qh >> (4 * k)) & 15u);
                w.q0[4 + k] |= spread_bit4((qh >> (16 + 4 * k)) & 15u);
            }
        }
    } else {  // Q8_0
        lds32_a2(blk + 2, w.q0);
    }
}

// Float contribution of one unit against one column; exact int32 block dots to `isum`
// (K4/K5/Q8_0: isum[0..1], one per 32; Q2_K, Q3_K, Q6_K: isum[0..3], one per 16).
template <int QT, int U>
__device__ __forceinline__ float dot_unit(const uint8_t *blk, const BlkHdr &h, const WBytes &w,
                                          const ActBlk &a0, const ActBlk &a1, int (&isum)[4]) {
    if constexpr (QT == kTypeQ4_K || QT == kTypeQ5_K) {
        int i0 = 0, i1 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            i0 = __dp4a(int(w.q0[k]), int(a0.q[k]), i0);
            if constexpr (QT == kTypeQ4_K) {
                i1 = dp4a_us(w.q1[k], a1.q[k], i1);
            } else {
                i1 = __dp4a(int(w.q1[k]), int(a1.q[k]), i1);
            }
        }
        if constexpr (QT == kTypeQ4_K) i1 >>= 4;  // exact: the sum is 16 x the nibble dot
        isum[0] = i0;
        isum[1] = i1;
        int sc0, sc1, m0, m1;
        scale_min_pair<U>(h, sc0, sc1, m0, m1);
        // d * sum_j d8_j * (sumi_j * sc_j) - dmin * sum_j m_j * (d8_j * sumq_j)
        // (vec_dot_q4_K_q8_1 structure, docs/llama-cpp-kernel-analysis.md:200-224)
        const float fd = a0.d * float(i0 * sc0) + a1.d * float(i1 * sc1);
        const float fm = a0.ds * float(m0) + a1.ds * float(m1);
        return h.d * fd - h.dmin * fm;
    } else if constexpr (QT == kTypeQ6_K) {
        constexpr int h6 = U >> 1, t = U & 1;
        int p00 = 0, p01 = 0, p10 = 0, p11 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            p00 = __dp4a(int(w.q0[k]), int(a0.q[k]), p00);
            p01 = __dp4a(int(w.q0[k + 4]), int(a0.q[k + 4]), p01);
            p10 = __dp4a(int(w.q1[k]), int(a1.q[k]), p10);
            p11 = __dp4a(int(w.q1[k + 4]), int(a1.q[k + 4]), p11);
        }
        // q - 32 through the activation sums: sum (q-32) a = sum q a - 32 sum a.
        p00 -= 32 * a0.slo;
        p01 -= 32 * a0.shi;
        p10 -= 32 * a1.slo;
        p11 -= 32 * a1.shi;
        isum[0] = p00;
        isum[1] = p01;
        isum[2] = p10;
        isum[3] = p11;
        constexpr int j0 = 4 * h6 + t, j1 = j0 + 2;
        const uint32_t sc0 = lds16(blk + 192 + 2 * j0);
        const uint32_t sc1 = lds16(blk + 192 + 2 * j1);
        const int s00 = int(int8_t(sc0 & 0xFF)), s01 = int(int8_t(sc0 >> 8));
        const int s10 = int(int8_t(sc1 & 0xFF)), s11 = int(int8_t(sc1 >> 8));
        return h.d * (a0.d * float(p00 * s00 + p01 * s01) + a1.d * float(p10 * s10 + p11 * s11));
    } else if constexpr (QT == kTypeIQ4_XS) {
        // d * sum_j d8_j * (ls_j - 32) * sum(level * q8) over groups j = 2U, 2U+1, with
        // ls_j = scales_l nibble j | (scales_h bits 2j, 2j+1) << 4
        int i0 = 0, i1 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            i0 = __dp4a(int(w.q0[k]), int(a0.q[k]), i0);
            i1 = __dp4a(int(w.q1[k]), int(a1.q[k]), i1);
        }
        isum[0] = i0;
        isum[1] = i1;
        const int ls0 = int(((h.s1 >> (8 * U)) & 15u) | (((h.s0 >> (4 * U)) & 3u) << 4)) - 32;
        const int ls1 = int(((h.s1 >> (8 * U + 4)) & 15u) | (((h.s0 >> (4 * U + 2)) & 3u) << 4)) - 32;
        return h.d * (a0.d * float(i0 * ls0) + a1.d * float(i1 * ls1));
    } else if constexpr (kIQLattice<QT> && !kSub16<QT>) {
        // one scale per sub-block: d * F * sum_j d8_j * M_j * sum(L q8)
        int i0 = 0, i1 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            i0 = __dp4a(int(w.q0[k]), int(a0.q[k]), i0);
            i1 = __dp4a(int(w.q1[k]), int(a1.q[k]), i1);
        }
        if constexpr (QT == kTypeIQ1_S) {
            // L = 8 grid +- 1: 8 sum(grid q8) plus or minus the block's sum of q8
            const uint32_t h0 = lds16(blk + 34 + 4 * U), h1 = lds16(blk + 36 + 4 * U);
            const int q0 = a0.slo + a0.shi, q1 = a1.slo + a1.shi;
            i0 = 8 * i0 + ((h0 & 0x8000u) ? -q0 : q0);
            i1 = 8 * i1 + ((h1 & 0x8000u) ? -q1 : q1);
        }
        isum[0] = i0;
        isum[1] = i1;
        const int m0 = iq_mult<QT>(blk, 2 * U), m1 = iq_mult<QT>(blk, 2 * U + 1);
        return h.d * kIQFactor<QT> * (a0.d * float(i0 * m0) + a1.d * float(i1 * m1));
    } else if constexpr (kIQLattice<QT>) {
        // one scale per 16 weights (two per sub-block)
        int p00 = 0, p01 = 0, p10 = 0, p11 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            p00 = __dp4a(int(w.q0[k]), int(a0.q[k]), p00);
            p01 = __dp4a(int(w.q0[k + 4]), int(a0.q[k + 4]), p01);
            p10 = __dp4a(int(w.q1[k]), int(a1.q[k]), p10);
            p11 = __dp4a(int(w.q1[k + 4]), int(a1.q[k + 4]), p11);
        }
        if constexpr (QT == kTypeIQ1_M) {
            // L = 8 grid +- 1 with a delta sign per 8 weights (bit 3 of the group's nibble):
            // 8 sum(grid q8) plus or minus each group's sum of q8
            const uint32_t nb = lds32_2(blk + 32 + 4 * U);  // nibbles of groups 8U..8U+7
            int g8[8];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                g8[g] = __dp4a(0x01010101, int(a0.q[2 * g]), __dp4a(0x01010101, int(a0.q[2 * g + 1]), 0));
                g8[4 + g] = __dp4a(0x01010101, int(a1.q[2 * g]), __dp4a(0x01010101, int(a1.q[2 * g + 1]), 0));
            }
#pragma unroll
            for (int g = 0; g < 8; ++g)
                if ((nb >> (4 * g + 3)) & 1u) g8[g] = -g8[g];
            p00 = 8 * p00 + g8[0] + g8[1];
            p01 = 8 * p01 + g8[2] + g8[3];
            p10 = 8 * p10 + g8[4] + g8[5];
            p11 = 8 * p11 + g8[6] + g8[7];
        }
        isum[0] = p00;
        isum[1] = p01;
        isum[2] = p10;
        isum[3] = p11;
        const int m00 = iq_mult<QT>(blk, 4 * U), m01 = iq_mult<QT>(blk, 4 * U + 1);
        const int m10 = iq_mult<QT>(blk, 4 * U + 2), m11 = iq_mult<QT>(blk, 4 * U + 3);
        return h.d * kIQFactor<QT> *
               (a0.d * float(p00 * m00 + p01 * m01) + a1.d * float(p10 * m10 + p11 * m11));
    } else if constexpr (QT == kTypeIQ4_NL) {
        int i0 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) i0 = __dp4a(int(w.q0[k]), int(a0.q[k]), i0);
        isum[0] = i0;
        return h.d * (a0.d * float(i0));
    } else if constexpr (QT == kTypeQ2_K || QT == kTypeQ3_K) {
        int p00 = 0, p01 = 0, p10 = 0, p11 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            p00 = __dp4a(int(w.q0[k]), int(a0.q[k]), p00);
            p01 = __dp4a(int(w.q0[k + 4]), int(a0.q[k + 4]), p01);
            p10 = __dp4a(int(w.q1[k]), int(a1.q[k]), p10);
            p11 = __dp4a(int(w.q1[k + 4]), int(a1.q[k + 4]), p11);
        }
        if constexpr (QT == kTypeQ3_K) {
            // q - 4 through the activation sums
            p00 -= 4 * a0.slo;
            p01 -= 4 * a0.shi;
            p10 -= 4 * a1.slo;
            p11 -= 4 * a1.shi;
        }
        isum[0] = p00;
        isum[1] = p01;
        isum[2] = p10;
        isum[3] = p11;
        if constexpr (QT == kTypeQ2_K) {
            // scale groups 4U..4U+3: low nibble scale, high nibble min
            // (vec_dot_q2_K_q8_1: d * sum sc * d8 * sumi - dmin * sum m * d8 * sumq)
            const uint32_t sw = lds16(blk + 4 * U) | (lds16(blk + 4 * U + 2) << 16);
            const int sc0 = sw & 15, sc1 = (sw >> 8) & 15, sc2 = (sw >> 16) & 15, sc3 = (sw >> 24) & 15;
            const int m0 = (sw >> 4) & 15, m1 = (sw >> 12) & 15, m2 = (sw >> 20) & 15, m3 = sw >> 28;
            const float fd = a0.d * float(p00 * sc0 + p01 * sc1) + a1.d * float(p10 * sc2 + p11 * sc3);
            const float fm = a0.d * float(m0 * a0.slo + m1 * a0.shi) + a1.d * float(m2 * a1.slo + m3 * a1.shi);
            return h.d * fd - h.dmin * fm;
        } else {
            // six-bit scales of groups 4U..4U+3: low nibbles from scales[4(U&1) ..] (high
            // nibbles for U >= 2), bits 4-5 from bits 2U of scales[8 .. 11]; minus 32
            const uint32_t lo = ((U & 1 ? h.s1 : h.s0) >> (U >= 2 ? 4 : 0)) & 0x0F0F0F0Fu;
            const uint32_t sc = lo | (((h.s2 >> (2 * U)) & 0x03030303u) << 4);
            const int sc0 = int(sc & 0xFF) - 32, sc1 = int((sc >> 8) & 0xFF) - 32;
            const int sc2 = int((sc >> 16) & 0xFF) - 32, sc3 = int(sc >> 24) - 32;
            return h.d * (a0.d * float(p00 * sc0 + p01 * sc1) + a1.d * float(p10 * sc2 + p11 * sc3));
        }
    } else if constexpr (kBasic<QT>) {
        // Q4_0 / Q5_0: d * d8 * sum((q - 8 | q - 16) q8), the offset through the block's
        // sum of q8; Q4_1 / Q5_1: d * d8 * sum(q q8) + m * d8 * sum(q8).
        int i0 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) i0 = __dp4a(int(w.q0[k]), int(a0.q[k]), i0);
        if constexpr (QT == kTypeQ4_0) i0 -= 8 * (a0.slo + a0.shi);
        if constexpr (QT == kTypeQ5_0) i0 -= 16 * (a0.slo + a0.shi);
        isum[0] = i0;
        if constexpr (QT == kTypeQ4_1 || QT == kTypeQ5_1) return h.d * (a0.d * float(i0)) + h.dmin * a0.ds;
        return h.d * (a0.d * float(i0));
    } else {
        int i0 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) i0 = __dp4a(int(w.q0[k]), int(a0.q[k]), i0);
        isum[0] = i0;
        return h.d * (a0.d * float(i0));
    }
}

template <int QT>
__device__ __forceinline__ void store_sums(int32_t *srow, int kb0, int kb1, const int (&isum)[4]) {
    if constexpr (kSub16<QT>) {
        srow[2 * kb0] = isum[0];
        srow[2 * kb0 + 1] = isum[1];
        srow[2 * kb1] = isum[2];
        srow[2 * kb1 + 1] = isum[3];
    } else if constexpr (kBlock32<QT>) {
        srow[kb0] = isum[0];
    } else {
        srow[kb0] = isum[0];
        srow[kb1] = isum[1];
    }
}

// Lanes per row (power of two) that keeps the most lanes busy: LB lanes split a row's
// nblk blocks, 32/LB lane groups take alternate rows of a tile of rpb rows.
__device__ __forceinline__ int choose_lanes_per_row(int nblk, int rpb) {
    int best = 32;
    float best_u = -1.f;
    for (int lb = 32; lb >= 1; lb >>= 1) {
        const int rg = 32 / lb;
        const int per_lane = (nblk + lb - 1) / lb;
        const float u = float(nblk) / float(lb * per_lane) * fminf(1.f, float(rpb) / float(rg));
        if (u > best_u + 1e-6f) {
            best_u = u;
            best = lb;
        }
    }
    return best;
}

// Per-tile context shared by the unit steps of one block.  A lane computes rows
// slot * RG + grp of the tile: every lane of the warp runs the same slot at the same time,
// so row ownership never splits a warp's instruction stream.  Slots past the tile's last
// row still compute (on stale stage bytes, inside the stage) and are simply not stored.
struct TileCtx {
    const uint8_t *lane_row0;  // stage row of slot 0 for this lane's group
    int slot_stride;           // bytes between consecutive slots (RG rows)
    int nrows, r0, rows, K, nkb, acb, RG, grp;
    const uint8_t *aq;
    const float *ad, *ads;
    const int2 *as;
    int32_t *sums;
};

// One compile-time unit U of block b for the NS slots and every column.
template <int QT, int NCOLS, int NS, int MODE, int U>
__device__ __forceinline__ void unit_step(const TileCtx &t, int b, const BlkHdr (&hdr)[NS],
                                          float (&acc)[NS][NCOLS]) {
    using TR = QTraits<QT>;
    int kb0, kb1;
    unit_kb<QT, U>(b, kb0, kb1);
    ActBlk a0, a1;
    if constexpr (NCOLS == 1) {
        const ActView v{t.aq, t.ad, t.ads, t.as};
        load_act<QT>(v, kb0, a0);
        if constexpr (!kBlock32<QT>) load_act<QT>(v, kb1, a1);
    }
    const uint8_t *blk0 = t.lane_row0 + b * TR::bytes;
#pragma unroll
    for (int sl = 0; sl < NS; ++sl) {
        const uint8_t *blk = blk0 + sl * t.slot_stride;
        WBytes wb;
        load_unit<QT, U>(blk, wb);
#pragma unroll
        for (int c = 0; c < NCOLS; ++c) {
            if constexpr (NCOLS > 1) {
                const ActView v{t.aq + c * t.acb, t.ad + c * t.nkb, t.ads + c * t.nkb,
                                t.as + c * t.nkb};
                load_act<QT>(v, kb0, a0);
                if constexpr (!kBlock32<QT>) load_act<QT>(v, kb1, a1);
            }
            int isum[4];
            acc[sl][c] += dot_unit<QT, U>(blk, hdr[sl], wb, a0, kBlock32<QT> ? a0 : a1, isum);
            if constexpr (MODE == kModeSums) {
                const int i = sl * t.RG + t.grp;
                if (i < t.rows) {
                    const int nsub = kSub16<QT> ? t.K / 16 : t.K / 32;
                    store_sums<QT>(t.sums + (size_t(c) * t.nrows + t.r0 + i) * nsub, kb0, kb1, isum);
                }
            }
        }
    }
}

// ---- the Q8_1 quantisation of one 32-value block by one warp ------------------------------
// Semantics of llama.cpp's CUDA quantize_q8_1: amax and sum by xor-butterfly warp
// reductions, d = amax / 127, q = roundf(x / d) (0 when amax == 0), both quotients the
// correctly rounded IEEE ones (q8_scale, quant_q8).
struct Q81Lane {
    int q;       // this lane's quant
    float d;     // fp32 scale (stored as fp16)
    float sum;   // block sum of x (stored as fp16)
};

__device__ __forceinline__ Q81Lane quantize_lane(float xi) {
    Q81Lane r;
    const float amax = warp_max(fabsf(xi));
    r.sum = warp_sum(xi);
    r.d = q8_scale(amax);
    const double rd64 = 1.0 / double(amax == 0.0f ? 1.0f : r.d);
    r.q = amax == 0.0f ? 0 : quant_q8(xi, float(rd64), rd64);
    return r;
}

// Packs lane quants into words: lanes 4w..4w+3 -> word w, returned on lane 4w.
__device__ __forceinline__ uint32_t pack_quants(int q) {
    const uint32_t b = uint32_t(q) & 0xFFu;
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, b, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, b, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, b, 3);
    return b | (b1 << 8) | (b2 << 16) | (b3 << 24);
}

// ---- fused Q8_1 staging from fp32 ------------------------------------------------------

// Quantises fp32 x (NCOLS columns of K) to Q8_1 straight into the swizzled shared layout,
// with d8, d8 * sum(q) and the half sums, by the arithmetic of quantize_q8_1 (d = amax/127
// by IEEE division, q = roundf(x / d) through quant_q8).  One 16-value chunk per thread
// and pass, two chunks in flight per thread; the two chunks of a Q8_1 block sit on
// adjacent lanes, which combine amax and the half sums.  Passes a warp has no chunk in
// are skipped whole (the shuffles stay warp-uniform).  x is 16-byte aligned.
template <int QT, int NCOLS>
__device__ __forceinline__ void stage_f32_q8_1(const float *__restrict__ x, int K, uint8_t *aq,
                                               float *ad, float *ads, int2 *as) {
    const int T = blockDim.x, tid = threadIdx.x;
    const int wbase = tid & ~31;
    const int nkb = K >> 5, nch = 2 * nkb, acb = act_col_bytes(nkb);
    const int total = NCOLS * nch;
    for (int base = 0; base < total; base += 2 * T) {
        float4 v[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int c = base + j * T + tid;
            if (c < total) {
                const int col = c / nch, cc = c - col * nch;
                const float4 *src = reinterpret_cast<const float4 *>(x + size_t(col) * K + cc * 16);
#pragma unroll
                for (int k = 0; k < 4; ++k) v[j][k] = __ldg(src + k);
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) v[j][k] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            if (base + j * T + wbase >= total) continue;  // whole warp past the end
            const int c = base + j * T + tid;
            float am = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                am = fmaxf(am, fabsf(v[j][k].x));
                am = fmaxf(am, fabsf(v[j][k].y));
                am = fmaxf(am, fabsf(v[j][k].z));
                am = fmaxf(am, fabsf(v[j][k].w));
            }
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
            const float d = q8_scale(am);
            const float dn = am == 0.0f ? 1.0f : d;  // all quants are 0 then; no 0/0
            const double rd64 = 1.0 / double(dn);
            const float rd = float(rd64);
            float e[16];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                e[4 * k] = v[j][k].x;
                e[4 * k + 1] = v[j][k].y;
                e[4 * k + 2] = v[j][k].z;
                e[4 * k + 3] = v[j][k].w;
            }
            uint32_t w[4];
            int s;
            quant16(e, am, rd, rd64, w, s);
            const int so = __shfl_xor_sync(0xffffffffu, s, 1);
            if (c < total) {
                const int col = c / nch, cc = c - col * nch;
                *reinterpret_cast<uint4 *>(aq + col * acb + act_chunk<QT>(cc) * 16) =
                    make_uint4(w[0], w[1], w[2], w[3]);
                if ((cc & 1) == 0) {
                    const int i = col * nkb + (cc >> 1);
                    const float dh = __half2float(__float2half_rn(d));
                    ad[i] = dh;
                    as[i] = make_int2(s, so);
                    ads[i] = dh * float(s + so);
                }
            }
        }
    }
}

// ---- the kernel --------------------------------------------------------------------------

// Host-side twin of choose_lanes_per_row (same arithmetic).
inline int host_lanes_per_row(int nblk, int rpb) {
    int best = 32;
    float best_u = -1.f;
    for (int lb = 32; lb >= 1; lb >>= 1) {
        const int rg = 32 / lb;
        const int per_lane = (nblk + lb - 1) / lb;
        const float r = float(rpb) / float(rg);
        const float u = float(nblk) / float(lb * per_lane) * (r < 1.f ? r : 1.f);
        if (u > best_u + 1e-6f) {
            best_u = u;
            best = lb;
        }
    }
    return best;
}

// LBT: lanes per row fixed at compile time (16 or 32), or 0 for the runtime choice.
template <int QT, int NCOLS, int RPB, int MODE, int LBT>
__global__ void __launch_bounds__(kMaxWarps * 32, NCOLS == 1 ? 2 : 1)
    mmvq_kernel(const __grid_constant__ MmvqArgs args) {
    using TR = QTraits<QT>;
    extern __shared__ __align__(16) uint8_t smem[];
    const int T = blockDim.x;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int nwarps = T >> 5;
    const int K = args.K, nstages = args.nstages;
    const int nkb = K >> 5;
    const int acb = act_col_bytes(nkb);
    const int nblk = K / TR::qk;
    const int row_bytes = nblk * TR::bytes;
    const MmvqSmem L = mmvq_smem_layout(QT, K, NCOLS, RPB, nwarps, nstages, MODE);
    uint8_t *aq = smem + L.aq;
    float *ad = reinterpret_cast<float *>(smem + L.ad);
    float *ads = reinterpret_cast<float *>(smem + L.ads);
    int2 *as = reinterpret_cast<int2 *>(smem + L.as);

    // Warp-tiles of RPB rows (of one segment) are dealt round-robin over all warps.
    const int ntiles = args.segTile[args.nseg];
    const int gwarp = blockIdx.x * nwarps + warp;
    const int wstride = gridDim.x * nwarps;
    const int my_tiles = gwarp < ntiles ? (ntiles - 1 - gwarp) / wstride + 1 : 0;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar) + warp * nstages;
    uint8_t *ring = smem + L.w + warp * nstages * L.stage;

    // Bulk copy of tile `tile` into stage `st` (lane 0 only).  The 16-byte aligned
    // interior of the row range goes through the copy engine; a range that does not start
    // or end on 16 bytes leaves at most 15 + 15 bytes for plain loads (below).
    auto issue = [&](int tile, int st) {
        if constexpr (MODE == kModeGLU) {
            // rows [r0, r0 + rows) of gate and up, 16-byte aligned rows (checked on the host)
            constexpr int HALF = RPB / 2;
            const int r0 = tile * HALF;
            const int rows = min(HALF, args.segRows[0] - r0);
            const uint32_t bytes = uint32_t(rows) * uint32_t(row_bytes);
            uint8_t *dst = ring + st * L.stage;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(&full[st], 2u * bytes);
            bulk_copy_g2s(dst, args.segW[0] + size_t(r0) * size_t(row_bytes), bytes, &full[st]);
            bulk_copy_g2s(dst + HALF * row_bytes, args.segW[1] + size_t(r0) * size_t(row_bytes), bytes,
                          &full[st]);
            return;
        }
        const int sg = mmvq_segment(args, tile);
        const int lt = tile - args.segTile[sg];
        const uint8_t *src = args.segW[sg] + size_t(lt) * RPB * size_t(row_bytes);
        const int rows = min(RPB, args.segRows[sg] - lt * RPB);
        const uintptr_t s = reinterpret_cast<uintptr_t>(src);
        const uintptr_t e = s + size_t(rows) * row_bytes;
        const uintptr_t s_al = (s + 15) & ~uintptr_t(15), e_al = e & ~uintptr_t(15);
        uint8_t *dst = ring + st * L.stage + int(s & 15);
        // Generic-proxy reads of this stage happen before the copy engine rewrites it.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (e_al > s_al) {
            mbar_arrive_expect_tx(&full[st], uint32_t(e_al - s_al));
            bulk_copy_g2s(dst + (s_al - s), reinterpret_cast<const void *>(s_al),
                          uint32_t(e_al - s_al), &full[st]);
        } else {
            mbar_arrive(&full[st]);
        }
    };

    // ---- 1. start streaming weights before waiting on the producer of x ------------
    if (lane == 0) {
        for (int st = 0; st < nstages; ++st) mbar_init(&full[st], 1);
        mbar_fence_init();
        for (int k = 0; k < my_tiles && k < nstages; ++k) issue(gwarp + k * wstride, k);
    }
    pdl_launch_dependents();
    pdl_wait();

    // ---- 2. stage the activation once per CTA ------------------------------------------
    if constexpr (MODE == kModeF32) {
        stage_f32_q8_1<QT, NCOLS>(static_cast<const float *>(args.x), K, aq, ad, ads, as);
    } else {
        // Q8_1 blocks, one per thread: 9 words ({d, s}, then 8 quant words) loaded together,
        // written to the swizzled layout with the block's d8, d8 * sum(q) and half sums.
        const uint32_t *xw = reinterpret_cast<const uint32_t *>(args.x);
        for (int c = 0; c < NCOLS; ++c) {
            uint8_t *aqc = aq + c * acb;
            for (int kb = tid; kb < nkb; kb += T) {
                const uint32_t *src = xw + (size_t(c) * nkb + kb) * 9;
                uint32_t v[9];
#pragma unroll
                for (int w = 0; w < 9; ++w) v[w] = __ldg(src + w);
                uint4 *d0 = reinterpret_cast<uint4 *>(aqc + act_chunk<QT>(2 * kb) * 16);
                uint4 *d1 = reinterpret_cast<uint4 *>(aqc + act_chunk<QT>(2 * kb + 1) * 16);
                *d0 = make_uint4(v[1], v[2], v[3], v[4]);
                *d1 = make_uint4(v[5], v[6], v[7], v[8]);
                int lo = 0, hi = 0;
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    lo = __dp4a(int(v[1 + w]), 0x01010101, lo);
                    hi = __dp4a(int(v[5 + w]), 0x01010101, hi);
                }
                const float d8 = h2f(v[0]);
                ad[c * nkb + kb] = d8;
                as[c * nkb + kb] = make_int2(lo, hi);
                ads[c * nkb + kb] = d8 * float(lo + hi);
            }
        }
    }
    __syncthreads();

    // ---- 3. lane -> (row group, blocks) mapping, fixed for all tiles -------------------
    // LB lanes split a row's blocks; the warp's RG = 32/LB lane groups take rows
    // slot * RG + grp.  With a compile-time LB the slot count NS is static.
    const int LB = LBT > 0 ? LBT : choose_lanes_per_row(nblk, RPB);
    const int RG = 32 / LB;
    const int bl = lane & (LB - 1);
    const int grp = lane / LB;
    constexpr int NS = LBT > 0 ? (RPB >= 32 / (LBT > 0 ? LBT : 32) ? RPB / (32 / (LBT > 0 ? LBT : 32)) : 1) : RPB;
    // Runtime-LB kernels walk all RPB slots and mask the ones past nslots.
    const int nslots = LBT > 0 ? NS : (RPB >= RG ? RPB / RG : 1);
    const bool grp_live = grp < RPB;  // groups beyond the tile's rows (RPB < RG) stay idle

    int st = 0;
    uint32_t phase = 0;
    for (int k = 0; k < my_tiles; ++k) {
        const int tile = gwarp + k * wstride;
        const int sg = mmvq_segment(args, tile);
        const int nrows = args.segRows[sg];
        constexpr int TROWS = MODE == kModeGLU ? RPB / 2 : RPB;  // output rows per tile
        const int r0 = (tile - args.segTile[sg]) * TROWS;
        const int rows = min(TROWS, nrows - r0);
        const uint8_t *src = args.segW[sg] + size_t(r0) * size_t(row_bytes);
        const uintptr_t s = MODE == kModeGLU ? 0 : reinterpret_cast<uintptr_t>(src);
        const uintptr_t e = MODE == kModeGLU ? 0 : s + size_t(rows) * row_bytes;
        uint8_t *wrow0 = ring + st * L.stage + int(s & 15);

        bool have_w = mbar_wait_bounded(&full[st], phase, args.wait_ns);
        if (!have_w) {
            // The copy did not land in time: one more bounded wait so that it is not still
            // writing this stage when the warp moves on; the tile is then skipped.
            (void)mbar_wait_bounded(&full[st], phase, args.wait_ns);
        }
        if ((s | e) & 15) {  // unaligned ends: plain loads of at most 30 bytes
            const uintptr_t s_al = (s + 15) & ~uintptr_t(15), e_al = e & ~uintptr_t(15);
            if (e_al > s_al) {
                const int nh = int(s_al - s), nt = int(e - e_al);
                for (int i = lane; i < nh + nt; i += 32) {
                    const size_t off = i < nh ? size_t(i) : size_t(e_al - s) + size_t(i - nh);
                    wrow0[off] = src[off];
                }
            } else {
                for (int i = lane; i < int(e - s); i += 32) wrow0[i] = src[i];
            }
            __syncwarp();
        }

        float acc[NS][NCOLS];
#pragma unroll
        for (int i = 0; i < NS; ++i)
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) acc[i][c] = 0.f;

        if (have_w && grp_live) {
            const TileCtx ctx{wrow0 + grp * row_bytes, RG * row_bytes, nrows, r0, rows, K, nkb,
                              acb, RG, grp, aq, ad, ads, as, args.sums};
            for (int b = bl; b < nblk; b += LB) {
                if (LBT > 0 || nslots == NS) {
                    // slots sl < NS are rows sl * RG + grp <= RPB - 1: inside the stage
                    BlkHdr hdr[NS];
#pragma unroll
                    for (int sl = 0; sl < NS; ++sl)
                        hdr[sl] = load_hdr<QT>(ctx.lane_row0 + sl * ctx.slot_stride + b * TR::bytes);
                    unit_step<QT, NCOLS, NS, MODE, 0>(ctx, b, hdr, acc);
                    if constexpr (Units<QT>::n == 4) {
                        unit_step<QT, NCOLS, NS, MODE, 1>(ctx, b, hdr, acc);
                        unit_step<QT, NCOLS, NS, MODE, 2>(ctx, b, hdr, acc);
                        unit_step<QT, NCOLS, NS, MODE, 3>(ctx, b, hdr, acc);
                    }
                } else {
                    // runtime LB with fewer slots than RPB: only slot 0 .. nslots-1 are rows
                    // of this lane; run them through the one-slot path.
                    for (int sl = 0; sl < nslots; ++sl) {
                        TileCtx c1 = ctx;
                        c1.lane_row0 = ctx.lane_row0 + sl * ctx.slot_stride;
                        c1.grp = grp + sl * RG;
                        const BlkHdr h1[1] = {load_hdr<QT>(c1.lane_row0 + b * TR::bytes)};
                        float a1[1][NCOLS];
#pragma unroll
                        for (int c = 0; c < NCOLS; ++c) a1[0][c] = 0.f;
                        unit_step<QT, NCOLS, 1, MODE, 0>(c1, b, h1, a1);
                        if constexpr (Units<QT>::n == 4) {
                            unit_step<QT, NCOLS, 1, MODE, 1>(c1, b, h1, a1);
                            unit_step<QT, NCOLS, 1, MODE, 2>(c1, b, h1, a1);
                            unit_step<QT, NCOLS, 1, MODE, 3>(c1, b, h1, a1);
                        }
#pragma unroll
                        for (int q = 0; q < NS; ++q)
                            if (q == sl)
#pragma unroll
                                for (int c = 0; c < NCOLS; ++c) acc[q][c] += a1[0][c];
                    }
                }
            }
        }

        // ---- 4. reduction over the LB lanes sharing a row, then store ------------------
        if constexpr (MODE == kModeGLU) {
            // slots [0, NS/2) hold gate rows, [NS/2, NS) the up rows of the same lanes
#pragma unroll
            for (int sl = 0; sl < NS / 2; ++sl) {
                float g = acc[sl][0], u = acc[sl + NS / 2][0];
#pragma unroll
                for (int o = LBT >> 1; o > 0; o >>= 1) {
                    g += __shfl_xor_sync(0xffffffffu, g, o);
                    u += __shfl_xor_sync(0xffffffffu, u, o);
                }
                const int i = sl * RG + grp;
                if (bl == 0 && grp_live && i < rows)
                    args.segY[0][r0 + i] = g / (1.0f + expf(-g)) * u;
            }
        } else if constexpr (MODE != kModeSums) {
#pragma unroll
            for (int sl = 0; sl < NS; ++sl) {
                if (LBT > 0 || sl < nslots || sl == 0) {  // uniform across the warp
                    const int i = sl * RG + grp;
#pragma unroll
                    for (int c = 0; c < NCOLS; ++c) {
                        float v = acc[sl][c];
                        if constexpr (LBT > 0) {
#pragma unroll
                            for (int o = LBT >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                        } else {
                            for (int o = LB >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                        }
                        if (bl == 0 && grp_live && sl < nslots && i < rows)
                            args.segY[sg][size_t(c) * nrows + r0 + i] = v;
                    }
                }
            }
        }
        __syncwarp();  // every lane is done with stage `st`
        if (lane == 0 && k + nstages < my_tiles) issue(tile + nstages * wstride, st);
        if (++st == nstages) {
            st = 0;
            phase ^= 1u;
        }
    }
}

// Host-side kernel table access, one instantiation file per type.
using MmvqKernelFn = void (*)(MmvqArgs);
MmvqKernelFn mmvq_kernel_q4k(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q5k(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q6k(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q80(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q40(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q41(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q50(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q51(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q2k(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_q3k(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq4nl(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq4xs(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq2xxs(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq2xs(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq2s(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq3xxs(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq3s(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq1s(int ncols, int rpb, int lbt, int mode);
MmvqKernelFn mmvq_kernel_iq1m(int ncols, int rpb, int lbt, int mode);
// Reads and clears the device status word of that type's translation unit (current device).
int mmvq_kernel_q4k_take_status();
int mmvq_kernel_q5k_take_status();
int mmvq_kernel_q6k_take_status();
int mmvq_kernel_q80_take_status();
int mmvq_kernel_q40_take_status();
int mmvq_kernel_q41_take_status();
int mmvq_kernel_q50_take_status();
int mmvq_kernel_q51_take_status();
int mmvq_kernel_q2k_take_status();
int mmvq_kernel_q3k_take_status();
int mmvq_kernel_iq4nl_take_status();
int mmvq_kernel_iq4xs_take_status();
int mmvq_kernel_iq2xxs_take_status();
int mmvq_kernel_iq2xs_take_status();
int mmvq_kernel_iq2s_take_status();
int mmvq_kernel_iq3xxs_take_status();
int mmvq_kernel_iq3s_take_status();
int mmvq_kernel_iq1s_take_status();
int mmvq_kernel_iq1m_take_status();

}  // namespace anvil

// Builds the [ncols 1..8] x [rpb 1,2,4,8] x [mode] x [lanes per row 16 / 32 / runtime]
// table for one type (compile-time lanes per row for 1, 2, 4 and 8 columns).  lbt is 16 or
// 32 for the compile-time variants, anything else for the runtime-LB kernel.
// ANVIL_MMVQ_TABLE_RT builds the runtime-LB kernels only (same results, a third of the code:
// the lattice I-quants, whose decode makes each instantiation large); it has no gate/up mode.
#define ANVIL_MMVQ_TABLE(FN, QT) ANVIL_MMVQ_TABLE_IMPL(FN, QT, true)
#define ANVIL_MMVQ_TABLE_RT(FN, QT) ANVIL_MMVQ_TABLE_IMPL(FN, QT, false)
#define ANVIL_MMVQ_TABLE_IMPL(FN, QT, COMPILE_LB)                                         \
    namespace anvil {                                                                     \
    template <int NC, int R, int LBT>                                                     \
    static MmvqKernelFn FN##_glu() {                                                      \
        if constexpr (NC == 1 && LBT > 0 && R >= 2 && (R / 2) % (32 / (LBT > 0 ? LBT : 32)) == 0) \
            return mmvq_kernel<QT, NC, R, kModeGLU, LBT>;                                 \
        return nullptr;                                                                   \
    }                                                                                     \
    template <int NC, int R, int LBT>                                                     \
    static MmvqKernelFn FN##_mode(int mode) {                                             \
        switch (mode) {                                                                   \
        case kModeQ81: return mmvq_kernel<QT, NC, R, kModeQ81, LBT>;                      \
        case kModeF32: return mmvq_kernel<QT, NC, R, kModeF32, LBT>;                      \
        case kModeSums: return mmvq_kernel<QT, NC, R, kModeSums, LBT>;                    \
        case kModeGLU: return FN##_glu<NC, R, LBT>();                                     \
        default: return nullptr;                                                          \
        }                                                                                 \
    }                                                                                     \
    template <int NC, int R>                                                              \
    static MmvqKernelFn FN##_lb(int lbt, int mode) {                                      \
        if constexpr (COMPILE_LB && (NC == 1 || NC == 2 || NC == 4 || NC == 8)) {         \
            if (lbt == 16) return FN##_mode<NC, R, 16>(mode);                             \
            if (lbt == 32) return FN##_mode<NC, R, 32>(mode);                             \
        }                                                                                 \
        return FN##_mode<NC, R, 0>(mode);                                                 \
    }                                                                                     \
    template <int NC>                                                                     \
    static MmvqKernelFn FN##_pick(int rpb, int lbt, int mode) {                           \
        switch (rpb) {                                                                    \
        case 1: return FN##_lb<NC, 1>(lbt, mode);                                         \
        case 2: return FN##_lb<NC, 2>(lbt, mode);                                         \
        case 4: return FN##_lb<NC, 4>(lbt, mode);                                         \
        case 8: return FN##_lb<NC, 8>(lbt, mode);                                         \
        default: return nullptr;                                                          \
        }                                                                                 \
    }                                                                                     \
    MmvqKernelFn FN(int ncols, int rpb, int lbt, int mode) {                              \
        switch (ncols) {                                                                  \
        case 1: return FN##_pick<1>(rpb, lbt, mode);                                      \
        case 2: return FN##_pick<2>(rpb, lbt, mode);                                      \
        case 3: return FN##_pick<3>(rpb, lbt, mode);                                      \
        case 4: return FN##_pick<4>(rpb, lbt, mode);                                      \
        case 5: return FN##_pick<5>(rpb, lbt, mode);                                      \
        case 6: return FN##_pick<6>(rpb, lbt, mode);                                      \
        case 7: return FN##_pick<7>(rpb, lbt, mode);                                      \
        case 8: return FN##_pick<8>(rpb, lbt, mode);                                      \
        default: return nullptr;                                                          \
        }                                                                                 \
    }                                                                                     \
    int FN##_take_status() {                                                              \
        int v = 0, z = 0;                                                                 \
        if (cudaMemcpyFromSymbol(&v, g_anvil_device_status, sizeof(int)) != cudaSuccess)  \
            return -1;                                                                    \
        if (cudaMemcpyToSymbol(g_anvil_device_status, &z, sizeof(int)) != cudaSuccess)    \
            return -1;                                                                    \
        return v;                                                                         \
    }                                                                                     \
    }
