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
//   2. After the wait the Q8_1 activation (NCOLS * K/32 blocks) is staged once per CTA:
//      quant words in a 16-byte-chunk XOR swizzle (bank-conflict-free per-unit reads),
//      fp32 scales, and int half-block sums of the quants (the Q4_K/Q5_K min term and the
//      Q6_K -32 offset use them).
//   3. Lanes walk the row's "units" (64 weights of a K-quant super-block, or one Q8_0
//      block) with stride 32, as the reference loop walks kbx with stride blocks_per_iter
//      (kernel_anvil/hip_codegen.py:266-285); each unit is decoded once per row and dotted
//      with __dp4a against every column.
//   4. Each row's partial sums are reduced with warp shuffles and lane 0 writes y.
//
// With SUMS=true the same kernel writes its exact int32 block dots instead of y (the
// parity probe behind anvil_mmvq_block_sums).
#pragma once

#include "anvil_common.cuh"

namespace anvil {

constexpr int kMaxWarps = 8;       // 256 threads: llama.cpp's MMVQ upper bound
constexpr int kMaxCols = 8;        // MMVQ_MAX_BATCH_SIZE
constexpr int kMaxSmem = 227 * 1024;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s bound on any mbarrier wait

struct MmvqSmem {
    int bar, w, stage, aq, ad, as, red, total;
};

__host__ __device__ inline int mmvq_type_bytes(int qt) {
    return qt == kTypeQ4_K ? 144 : qt == kTypeQ5_K ? 176 : qt == kTypeQ6_K ? 210 : 34;
}
__host__ __device__ inline int mmvq_type_qk(int qt) { return qt == kTypeQ8_0 ? 32 : 256; }

// Bytes of one column's swizzled activation quants: 2 chunks of 16 B per Q8_1 block,
// padded to whole 8-chunk groups so the XOR swizzle never leaves the column.
__host__ __device__ inline int act_col_bytes(int nkb) { return ((2 * nkb + 7) & ~7) * 16; }

// Dynamic shared memory layout; identical on host (launch size) and device.
// [nwarps x nstages mbarriers][nwarps x nstages weight stages][act quants][act scales][act sums]
__host__ __device__ inline MmvqSmem mmvq_smem_layout(int qt, int K, int ncols, int rpb,
                                                     int nwarps, int nstages) {
    const int row_bytes = (K / mmvq_type_qk(qt)) * mmvq_type_bytes(qt);
    const int nkb = K / 32;
    MmvqSmem L;
    L.bar = 0;
    L.w = (8 * nwarps * nstages + 15) & ~15;
    // +32 per stage: up to 15 bytes of head misalignment plus one word of funnel over-read.
    L.stage = ((rpb * row_bytes + 32) + 15) & ~15;
    L.aq = L.w + nwarps * nstages * L.stage;
    L.ad = L.aq + ncols * act_col_bytes(nkb);
    L.as = (L.ad + ncols * nkb * 4 + 15) & ~15;
    L.red = L.as + ncols * nkb * 8;
    L.total = L.red;
    return L;
}

// Swizzled position of 16-byte activation chunk `ci` (two chunks per Q8_1 block).  The XOR
// only flips bits 0-1 inside each aligned group of 8 chunks (the column is padded to whole
// groups), so chunks 4u..4u+3 read by consecutive threads land in distinct bank quads.
__device__ __forceinline__ int act_chunk(int ci) { return (ci & ~7) | ((ci & 7) ^ ((ci >> 3) & 3)); }

struct ActUnit {          // one column's activation operands for one unit
    uint32_t a0[8], a1[8];  // quant words of Q8_1 blocks kb0 and kb1 (a1 unused for Q8_0)
    float d0, d1;           // their fp16 scales, widened
    int s0lo, s0hi, s1lo, s1hi;  // sums of the first / last 16 quants of each block
};

struct WUnit {            // one row's decoded weight operands for one unit
    uint32_t q0[8], q1[8];  // weight bytes matching a0 / a1 (unsigned 0..63 or int8 for Q8_0)
    int sc[4];              // K4/K5: sc0, sc1, m0, m1.  Q6_K: scale of groups 0..3
    float d, dmin;
};

// Q8_1 blocks consumed by unit `ub` of super-block `b`.
template <int QT>
__device__ __forceinline__ void unit_blocks(int b, int ub, int &kb0, int &kb1) {
    if constexpr (QT == kTypeQ8_0) {
        kb0 = b;
        kb1 = b;
    } else if constexpr (QT == kTypeQ6_K) {
        // unit (h, t): sub-blocks 4h+t (low nibble, qh shift 2t) and 4h+2+t (high nibble).
        const int h = ub >> 1, t = ub & 1;
        kb0 = 8 * b + 4 * h + t;
        kb1 = kb0 + 2;
    } else {
        // unit p: sub-blocks 2p (low nibble) and 2p+1 (high nibble).
        kb0 = 8 * b + 2 * ub;
        kb1 = kb0 + 1;
    }
}

__device__ __forceinline__ void load_act_block(const uint8_t *aq, const float *ad,
                                               const int2 *as, int kb, uint32_t (&q)[8],
                                               float &d, int &slo, int &shi) {
    const uint4 c0 = *reinterpret_cast<const uint4 *>(aq + act_chunk(2 * kb) * 16);
    const uint4 c1 = *reinterpret_cast<const uint4 *>(aq + act_chunk(2 * kb + 1) * 16);
    q[0] = c0.x; q[1] = c0.y; q[2] = c0.z; q[3] = c0.w;
    q[4] = c1.x; q[5] = c1.y; q[6] = c1.z; q[7] = c1.w;
    d = ad[kb];
    const int2 s = as[kb];
    slo = s.x;
    shi = s.y;
}

template <int QT>
__device__ __forceinline__ ActUnit load_act(const uint8_t *aq, const float *ad, const int2 *as,
                                            int kb0, int kb1) {
    ActUnit a;
    load_act_block(aq, ad, as, kb0, a.a0, a.d0, a.s0lo, a.s0hi);
    if constexpr (QT != kTypeQ8_0) {
        load_act_block(aq, ad, as, kb1, a.a1, a.d1, a.s1lo, a.s1hi);
    }
    return a;
}

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

__device__ __forceinline__ uint32_t lds16_a2(const uint8_t *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}

// Six-bit scale/min pair of sub-blocks 2p and 2p+1 from the packed scales[12]
// (gguf-py quants.py:478-501, the Q4_K.get_scale_min unpacking): for j < 4
// sc = s[j] & 63, m = s[j+4] & 63; for j >= 4 sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4,
// m = (s[j+4] >> 4) | (s[j] >> 6) << 4.  Both bytes of a pair come out together.
__device__ __forceinline__ void unpack_scale_pair(uint32_t s0, uint32_t s1, uint32_t s2, int p,
                                                  int (&sc)[4]) {
    const uint32_t sh = (p & 1) * 16;
    const uint32_t b0 = (s0 >> sh) & 0xFFFFu, b1 = (s1 >> sh) & 0xFFFFu, b2 = (s2 >> sh) & 0xFFFFu;
    uint32_t scp, mp;
    if (p < 2) {
        scp = b0 & 0x3F3Fu;
        mp = b1 & 0x3F3Fu;
    } else {
        scp = (b2 & 0x0F0Fu) | ((b0 >> 2) & 0x3030u);
        mp = ((b2 >> 4) & 0x0F0Fu) | ((b1 >> 2) & 0x3030u);
    }
    sc[0] = scp & 0xFF;
    sc[1] = scp >> 8;
    sc[2] = mp & 0xFF;
    sc[3] = mp >> 8;
}

template <int QT>
__device__ __forceinline__ WUnit decode_unit(const uint8_t *blk, int ub) {
    WUnit w;
    if constexpr (QT == kTypeQ4_K || QT == kTypeQ5_K) {
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        const int qs_off = (QT == kTypeQ4_K ? 16 : 48) + 32 * ub;
        const uint4 qa = *reinterpret_cast<const uint4 *>(blk + qs_off);
        const uint4 qb = *reinterpret_cast<const uint4 *>(blk + qs_off + 16);
        const uint32_t v[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        if constexpr (QT == kTypeQ4_K) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                w.q0[k] = v[k] & 0x0F0F0F0Fu;
                w.q1[k] = (v[k] >> 4) & 0x0F0F0F0Fu;
            }
        } else {
            // fifth bit of weight e of sub-block j is bit j of qh[e] (gguf-py quants.py:540-547)
            const uint4 ha = *reinterpret_cast<const uint4 *>(blk + 16);
            const uint4 hb = *reinterpret_cast<const uint4 *>(blk + 32);
            const uint32_t qh[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
            const int j0 = 2 * ub;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                w.q0[k] = (v[k] & 0x0F0F0F0Fu) | (((qh[k] >> j0) & 0x01010101u) << 4);
                w.q1[k] = ((v[k] >> 4) & 0x0F0F0F0Fu) | (((qh[k] >> (j0 + 1)) & 0x01010101u) << 4);
            }
        }
        unpack_scale_pair(h.y, h.z, h.w, ub, w.sc);
        w.d = h2f(h.x);
        w.dmin = h2f(h.x >> 16);
    } else if constexpr (QT == kTypeQ6_K) {
        // unit (h, t): ql bytes [64h+32t, +32) hold sub-block 4h+t (low nibbles) and
        // 4h+2+t (high nibbles); qh bytes [32h, +32) hold their top two bits at shifts
        // 2t and 4+2t (gguf-py quants.py:563-569).
        const int h = ub >> 1, t = ub & 1;
        uint32_t ql[8], qh[8];
        lds32_a2(blk + 64 * h + 32 * t, ql);
        lds32_a2(blk + 128 + 32 * h, qh);
        const int s0 = 2 * t, s1 = 4 + 2 * t;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            w.q0[k] = (ql[k] & 0x0F0F0F0Fu) | (((qh[k] >> s0) & 0x03030303u) << 4);
            w.q1[k] = ((ql[k] >> 4) & 0x0F0F0F0Fu) | (((qh[k] >> s1) & 0x03030303u) << 4);
        }
        const int j0 = 4 * h + t, j1 = j0 + 2;
        const uint32_t sc0 = lds16_a2(blk + 192 + 2 * j0);
        const uint32_t sc1 = lds16_a2(blk + 192 + 2 * j1);
        w.sc[0] = int(int8_t(sc0 & 0xFF));
        w.sc[1] = int(int8_t(sc0 >> 8));
        w.sc[2] = int(int8_t(sc1 & 0xFF));
        w.sc[3] = int(int8_t(sc1 >> 8));
        w.d = h2f(lds16_a2(blk + 208));
        w.dmin = 0.f;
    } else {  // Q8_0
        lds32_a2(blk + 2, w.q0);
        w.d = h2f(lds16_a2(blk));
        w.dmin = 0.f;
    }
    return w;
}

// Float contribution of one decoded weight unit against one column; the exact int32
// block dots go to `isum` (K4/K5/Q8_0: isum[0..1] per 32; Q6_K: isum[0..3] per 16).
template <int QT>
__device__ __forceinline__ float dot_unit(const WUnit &w, const ActUnit &a, int (&isum)[4]) {
    if constexpr (QT == kTypeQ4_K || QT == kTypeQ5_K) {
        int i0 = 0, i1 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            i0 = __dp4a(int(w.q0[k]), int(a.a0[k]), i0);
            i1 = __dp4a(int(w.q1[k]), int(a.a1[k]), i1);
        }
        isum[0] = i0;
        isum[1] = i1;
        // llama.cpp vec_dot_q4_K_q8_1_impl_vmmq structure (docs/llama-cpp-kernel-analysis.md:200-224):
        // d * sum_j d8_j * (sumi_j * sc_j) - dmin * sum_j d8_j * (sumq_j * m_j)
        const float fd = a.d0 * float(i0 * w.sc[0]) + a.d1 * float(i1 * w.sc[1]);
        const float fm = a.d0 * float((a.s0lo + a.s0hi) * w.sc[2]) +
                         a.d1 * float((a.s1lo + a.s1hi) * w.sc[3]);
        return w.d * fd - w.dmin * fm;
    } else if constexpr (QT == kTypeQ6_K) {
        int p00 = 0, p01 = 0, p10 = 0, p11 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            p00 = __dp4a(int(w.q0[k]), int(a.a0[k]), p00);
            p01 = __dp4a(int(w.q0[k + 4]), int(a.a0[k + 4]), p01);
            p10 = __dp4a(int(w.q1[k]), int(a.a1[k]), p10);
            p11 = __dp4a(int(w.q1[k + 4]), int(a.a1[k + 4]), p11);
        }
        // q - 32 applied through the activation sums: sum (q-32) a = sum q a - 32 sum a.
        p00 -= 32 * a.s0lo;
        p01 -= 32 * a.s0hi;
        p10 -= 32 * a.s1lo;
        p11 -= 32 * a.s1hi;
        isum[0] = p00;
        isum[1] = p01;
        isum[2] = p10;
        isum[3] = p11;
        return w.d * (a.d0 * float(p00 * w.sc[0] + p01 * w.sc[1]) +
                      a.d1 * float(p10 * w.sc[2] + p11 * w.sc[3]));
    } else {
        int i0 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) i0 = __dp4a(int(w.q0[k]), int(a.a0[k]), i0);
        isum[0] = i0;
        return w.d * (a.d0 * float(i0));
    }
}

template <int QT>
__device__ __forceinline__ void store_sums(int32_t *srow, int kb0, int kb1, const int (&isum)[4]) {
    if constexpr (QT == kTypeQ6_K) {
        srow[2 * kb0] = isum[0];
        srow[2 * kb0 + 1] = isum[1];
        srow[2 * kb1] = isum[2];
        srow[2 * kb1 + 1] = isum[3];
    } else if constexpr (QT == kTypeQ8_0) {
        srow[kb0] = isum[0];
    } else {
        srow[kb0] = isum[0];
        srow[kb1] = isum[1];
    }
}

template <int QT, int NCOLS, int RPB, bool SUMS>
__global__ void __launch_bounds__(kMaxWarps * 32)
    mmvq_kernel(const uint8_t *__restrict__ W, const uint8_t *__restrict__ xq,
                float *__restrict__ y, int32_t *__restrict__ sums, int nrows, int K,
                int nstages) {
    using TR = QTraits<QT>;
    extern __shared__ __align__(16) uint8_t smem[];
    const int T = blockDim.x;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int nwarps = T >> 5;
    const int nkb = K >> 5;
    const int acb = act_col_bytes(nkb);
    const int nblk = K / TR::qk;
    const int row_bytes = nblk * TR::bytes;
    const MmvqSmem L = mmvq_smem_layout(QT, K, NCOLS, RPB, nwarps, nstages);
    uint8_t *aq = smem + L.aq;
    float *ad = reinterpret_cast<float *>(smem + L.ad);
    int2 *as = reinterpret_cast<int2 *>(smem + L.as);

    // Every warp is an independent consumer with its own ring of `nstages` row tiles.
    // Warp-tiles of RPB rows are dealt round-robin over all warps of the grid.
    const int ntiles = (nrows + RPB - 1) / RPB;
    const int gwarp = blockIdx.x * nwarps + warp;
    const int wstride = gridDim.x * nwarps;
    const int my_tiles = gwarp < ntiles ? (ntiles - 1 - gwarp) / wstride + 1 : 0;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar) + warp * nstages;
    uint8_t *ring = smem + L.w + warp * nstages * L.stage;

    // Bulk copy of tile `tile` into stage `st` (lane 0 only).  The 16-byte aligned
    // interior of the row range goes through the copy engine; a range that does not start
    // or end on 16 bytes leaves at most 15 + 15 bytes for plain loads (below).
    auto issue = [&](int tile, int st) {
        const uint8_t *src = W + size_t(tile) * RPB * size_t(row_bytes);
        const int rows = min(RPB, nrows - tile * RPB);
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

    // ---- 1. start streaming weights before waiting on the producer of xq -----------
    if (lane == 0) {
        for (int st = 0; st < nstages; ++st) mbar_init(&full[st], 1);
        mbar_fence_init();
        for (int k = 0; k < my_tiles && k < nstages; ++k) issue(gwarp + k * wstride, k);
    }
    pdl_launch_dependents();
    pdl_wait();

    // ---- 2. stage the Q8_1 activation once per CTA -----------------------------------
    {
        const uint32_t *xw = reinterpret_cast<const uint32_t *>(xq);
        const int nw = NCOLS * nkb * 9;
        for (int i = tid; i < nw; i += T) {
            const int blk = i / 9, w = i - blk * 9;  // blk = c * nkb + kb
            const uint32_t v = __ldg(xw + i);
            if (w == 0) {
                ad[blk] = h2f(v);
            } else {
                const int c = blk / nkb, kb = blk - c * nkb;
                const int ci = 2 * kb + ((w - 1) >> 2);
                *reinterpret_cast<uint32_t *>(aq + c * acb + act_chunk(ci) * 16 +
                                              ((w - 1) & 3) * 4) = v;
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < NCOLS * nkb * 2; i += T) {
        const int blk = i >> 1, half = i & 1;
        const int c = blk / nkb, kb = blk - c * nkb;
        const uint4 q =
            *reinterpret_cast<const uint4 *>(aq + c * acb + act_chunk(2 * kb + half) * 16);
        int sq = 0;
        sq = __dp4a(int(q.x), 0x01010101, sq);
        sq = __dp4a(int(q.y), 0x01010101, sq);
        sq = __dp4a(int(q.z), 0x01010101, sq);
        sq = __dp4a(int(q.w), 0x01010101, sq);
        reinterpret_cast<int *>(as)[i] = sq;
    }
    __syncthreads();

    // ---- 3. lane -> (row group, unit) mapping, fixed for all tiles -------------------
    // U units per row.  LPR lanes share a row (32, or the power of two >= U when a row
    // has fewer than 32 units); the warp's 32/LPR lane groups take alternate rows.
    const int U = nblk * TR::units;
    int LPR = 32;
    while (LPR > 1 && (LPR >> 1) >= U) LPR >>= 1;
    const int RG = 32 / LPR;
    const int ul = lane & (LPR - 1);
    const int grp = lane / LPR;
    unsigned rowmask = 0;
#pragma unroll
    for (int i = 0; i < RPB; ++i)
        if (i % RG == grp) rowmask |= 1u << i;

    for (int k = 0; k < my_tiles; ++k) {
        const int tile = gwarp + k * wstride;
        const int st = k % nstages;
        const int r0 = tile * RPB;
        const int rows = min(RPB, nrows - r0);
        const uint8_t *src = W + size_t(r0) * size_t(row_bytes);
        const uintptr_t s = reinterpret_cast<uintptr_t>(src);
        const uintptr_t e = s + size_t(rows) * row_bytes;
        uint8_t *wrow0 = ring + st * L.stage + int(s & 15);

        const bool have_w = mbar_wait_bounded(&full[st], (k / nstages) & 1, kWaitLimitNs);
        if (!have_w) {
            // The copy did not land in time: one more bounded wait so that it is not still
            // writing this stage when the warp moves on; the tile is then skipped.
            (void)mbar_wait_bounded(&full[st], (k / nstages) & 1, kWaitLimitNs);
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

        float acc[RPB][NCOLS];
#pragma unroll
        for (int i = 0; i < RPB; ++i)
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) acc[i][c] = 0.f;

        if (have_w) {
            for (int u = ul; u < U; u += LPR) {
                const int b = u / TR::units, ub = u - b * TR::units;
                int kb0, kb1;
                unit_blocks<QT>(b, ub, kb0, kb1);
                ActUnit a1;
                if constexpr (NCOLS == 1) a1 = load_act<QT>(aq, ad, as, kb0, kb1);
#pragma unroll
                for (int i = 0; i < RPB; ++i) {
                    if (((rowmask >> i) & 1u) && i < rows) {
                        const WUnit w =
                            decode_unit<QT>(wrow0 + i * row_bytes + b * TR::bytes, ub);
#pragma unroll
                        for (int c = 0; c < NCOLS; ++c) {
                            ActUnit a;
                            if constexpr (NCOLS == 1) {
                                a = a1;
                            } else {
                                a = load_act<QT>(aq + c * acb, ad + c * nkb, as + c * nkb, kb0,
                                                 kb1);
                            }
                            int isum[4];
                            acc[i][c] += dot_unit<QT>(w, a, isum);
                            if constexpr (SUMS) {
                                const int nsub = QT == kTypeQ6_K ? K / 16 : K / 32;
                                store_sums<QT>(sums + (size_t(c) * nrows + r0 + i) * nsub, kb0,
                                               kb1, isum);
                            }
                        }
                    }
                }
            }
        }

        // ---- 4. warp reduction and store (rows a lane group does not own add zeros) ---
#pragma unroll
        for (int i = 0; i < RPB; ++i)
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) {
                const float v = warp_sum(acc[i][c]);
                if constexpr (!SUMS) {
                    if (lane == 0 && i < rows) y[size_t(c) * nrows + r0 + i] = v;
                }
            }
        __syncwarp();  // every lane is done with stage `st`
        if (lane == 0 && k + nstages < my_tiles) issue(tile + nstages * wstride, st);
    }
}

// Host-side kernel table access, one instantiation file per type.
using MmvqKernelFn = void (*)(const uint8_t *, const uint8_t *, float *, int32_t *, int, int,
                              int);
MmvqKernelFn mmvq_kernel_q4k(int ncols, int rpb, bool sums);
MmvqKernelFn mmvq_kernel_q5k(int ncols, int rpb, bool sums);
MmvqKernelFn mmvq_kernel_q6k(int ncols, int rpb, bool sums);
MmvqKernelFn mmvq_kernel_q80(int ncols, int rpb, bool sums);
// Reads and clears the device status word of that type's translation unit (current device).
int mmvq_kernel_q4k_take_status();
int mmvq_kernel_q5k_take_status();
int mmvq_kernel_q6k_take_status();
int mmvq_kernel_q80_take_status();

}  // namespace anvil

// Builds the [ncols 1..8] x [rpb 1,2,4,8] x [sums] table for one type.
#define ANVIL_MMVQ_TABLE(FN, QT)                                                          \
    namespace anvil {                                                                     \
    template <int NC>                                                                     \
    static MmvqKernelFn FN##_pick(int rpb, bool sums) {                                   \
        switch (rpb) {                                                                    \
        case 1: return sums ? mmvq_kernel<QT, NC, 1, true> : mmvq_kernel<QT, NC, 1, false>; \
        case 2: return sums ? mmvq_kernel<QT, NC, 2, true> : mmvq_kernel<QT, NC, 2, false>; \
        case 4: return sums ? mmvq_kernel<QT, NC, 4, true> : mmvq_kernel<QT, NC, 4, false>; \
        case 8: return sums ? mmvq_kernel<QT, NC, 8, true> : mmvq_kernel<QT, NC, 8, false>; \
        default: return nullptr;                                                          \
        }                                                                                 \
    }                                                                                     \
    MmvqKernelFn FN(int ncols, int rpb, bool sums) {                                      \
        switch (ncols) {                                                                  \
        case 1: return FN##_pick<1>(rpb, sums);                                           \
        case 2: return FN##_pick<2>(rpb, sums);                                           \
        case 3: return FN##_pick<3>(rpb, sums);                                           \
        case 4: return FN##_pick<4>(rpb, sums);                                           \
        case 5: return FN##_pick<5>(rpb, sums);                                           \
        case 6: return FN##_pick<6>(rpb, sums);                                           \
        case 7: return FN##_pick<7>(rpb, sums);                                           \
        case 8: return FN##_pick<8>(rpb, sums);                                           \
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
