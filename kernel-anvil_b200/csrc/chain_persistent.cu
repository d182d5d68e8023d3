// chain_persistent.cu -- one cooperative launch runs a whole token's GEMV chain.
//
// A decode token is a fixed sequence of MMVQ GEMVs.  Launched one kernel per GEMV, each
// pays a start-up and drain cost of a few microseconds that the weight stream of a small
// GEMV cannot hide.  Here a persistent kernel walks the chain instead:
//
//   * Groups.  GEMVs that read the same activation form a group (q/k/v; gate/up; o; down;
//     lm_head).  At the start of a group every CTA quantises the group's fp32 input to
//     Q8_1 in shared memory, with the arithmetic of quantize_q8_1 (d = amax/127 by IEEE
//     division, q = roundf(x/d)), so the dots see exactly the quants a separate quantiser
//     would have written.  A group may wait for every group before it (the data flow of a
//     decoder layer: o-proj needs q/k/v done, gate/up need o-proj, ...): a grid barrier on
//     per-group arrival counters, spun by one thread per CTA with a 2 s bound.
//   * Weight rings.  Each warp owns a byte ring in shared memory and deals itself tiles
//     round-robin across the tiles of every group of the chain.  Lane 0 keeps the ring full
//     with bulk async copies (cp.async.bulk, completion on one of 8 mbarriers) and runs
//     ahead across group boundaries: while a CTA waits at a barrier or stages the next
//     activation, the copies for the next group's weights are already in flight, so HBM
//     keeps streaming through the whole token.  Tiles of different GEMVs differ in size;
//     a tile is placed at the ring head, or at offset 0 when it would cross the end.
//   * Dots.  The tile arithmetic is the MMVQ kernel's (unit_step, load_hdr; lane-per-block
//     decode with compile-time lanes per row), so for the same rows per tile and lanes per
//     row the outputs are bit-identical to anvil_mmvq's.
//   * Ranks.  With world > 1 each rank holds a row shard of every matrix and writes its
//     output rows into its own copy of the full output; at the end of a group the rank's
//     last CTA copies the rank's rows into every peer's copy (peer pointers over NVLink),
//     then counts the rank on every rank's group counter (one system-scope release per
//     rank and group).  The exchange is the all-gather of the row-sharded GEMV, inside the
//     kernel.
//
// Co-residency of all CTAs (required by the barriers) comes from the cooperative launch.
// Every wait is bounded; a wait that gives up raises a device status flag and the kernel
// runs on (its results are then wrong, never hung).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "anvil.h"
#include "anvil_host.h"
#include "mmvq.cuh"

namespace anvil {

constexpr int kPcMaxRanks = ANVIL_MAX_RANKS;
constexpr int kPcSlots = 8;  // tiles in flight per warp
constexpr int kStatusBarrierTimeout = 2;
constexpr uint64_t kBarrierLimitNs = 2000000000ull;

// Compile-time tile shapes: rows per tile x lanes per row.
enum PcVariant : int {
    kV1x32, kV2x32, kV4x32, kV8x32, kV2x16, kV4x16, kV8x16, kV4x8, kV8x8, kNumVariants
};
constexpr int kVarRpb[kNumVariants] = {1, 2, 4, 8, 2, 4, 8, 4, 8};
constexpr int kVarLb[kNumVariants] = {32, 32, 32, 32, 16, 16, 16, 8, 8};

struct PcGemv {
    const uint8_t *W;          // this rank's rows, GGUF blocks
    float *y[kPcMaxRanks];     // full output buffer (ncols x nrows_full) on each rank
    int type, variant, rpb;
    int nrows, row0, nrows_full;
    int row_bytes, alloc;      // alloc: ring bytes one tile takes
    int tile_base, ntiles;     // tiles of this GEMV within its group
};

struct PcGroup {
    const float *x;            // fp32 input, ncols x K
    int K, first, count, ntiles, rot, family;
    int wait_from, wait_to;    // wait on counters [wait_from, wait_to) before staging
};

struct PcArgs {
    const PcGroup *groups;
    const PcGemv *gemvs;
    uint32_t *const *counters;  // device array: counters[q] = rank q's arrival counters
    int ngroups, world, rank;
    int act_off, ring_off, ring_bytes;
    int first_wait_from;        // group 0 of launch e > 0 (world > 1): previous launch's tail
    uint32_t epoch;
};

// ---- synchronisation helpers ----------------------------------------------------------

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t *p, bool sys) {
    uint32_t v;
    if (sys)
        asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_relaxed_add(uint32_t *p, uint32_t v, bool sys) {
    if (sys)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
    else
        asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// True once any bounded wait of this translation unit has given up: later waits then
// end at once (barriers) or after 1 ms (weight copies), so a failed run finishes quickly.
__device__ __forceinline__ bool pc_failed() {
    return *reinterpret_cast<volatile int *>(&g_anvil_device_status) != 0;
}

// Thread 0 of a CTA: wait until counters [from, to) all reached `target` (wrap-safe).
// Relaxed polling; the fence after the last read orders what follows (acquire).
__device__ void pc_wait_counters(const PcArgs &a, int from, int to, uint32_t target) {
    const bool sys = a.world > 1;
    // one CTA count per group on one GPU; one rank count per group across GPUs
    const uint32_t *base = a.counters[a.rank] + (sys ? a.ngroups : 0);
    uint64_t t0 = 0;
    for (int g = from; g < to; ++g) {
        for (uint32_t it = 0;; ++it) {
            if (int32_t(ld_relaxed(base + g, sys) - target) >= 0) break;
            if ((it & 31u) == 31u) {
                if (pc_failed()) return;  // an earlier wait gave up: do not wait again
                const uint64_t now = global_timer_ns();
                if (t0 == 0) {
                    t0 = now;
                } else if (now - t0 > kBarrierLimitNs) {
                    atomicOr(&g_anvil_device_status, kStatusBarrierTimeout);
                    return;
                }
            }
        }
    }
    if (sys)
        asm volatile("fence.acq_rel.sys;" ::: "memory");
    else
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Copies this rank's output rows of the group's GEMVs from its own buffer into every peer's
// (16-byte stores where both sides allow them).  Whole CTA.
template <int NCOLS>
__device__ void pc_push_outputs(const PcArgs &a, const PcGroup &grp) {
    const int T = blockDim.x, tid = threadIdx.x;
    for (int m = grp.first; m < grp.first + grp.count; ++m) {
        const PcGemv *gm = a.gemvs + m;
        const int n = gm->nrows, r0 = gm->row0, nf = gm->nrows_full;
        for (int c = 0; c < NCOLS; ++c) {
            const float *src = gm->y[a.rank] + size_t(c) * nf + r0;
            for (int q = 0; q < a.world; ++q) {
                if (q == a.rank) continue;
                float *dst = gm->y[q] + size_t(c) * nf + r0;
                if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0 &&
                    (n & 3) == 0) {
                    const float4 *s4 = reinterpret_cast<const float4 *>(src);
                    float4 *d4 = reinterpret_cast<float4 *>(dst);
                    for (int i = tid; i < (n >> 2); i += T) d4[i] = s4[i];
                } else {
                    for (int i = tid; i < n; i += T) dst[i] = src[i];
                }
            }
        }
    }
}

// The CTA's arrival at the end of group g (whole CTA, after its barrier).  One GPU: thread 0
// publishes the CTA's outputs (release fence) and counts the CTA.  Several GPUs: the CTAs
// count themselves on this GPU; the last one (it sees every CTA's outputs through the
// acquire-release count) copies the rank's output rows to every peer, then one system-scope
// release and one count per rank on every rank's group counter.
template <int NCOLS>
__device__ void pc_arrive(const PcArgs &a, const PcGroup &grp, int g, int *s_last) {
    if (a.world == 1) {
        if (threadIdx.x == 0) {
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
            red_relaxed_add(a.counters[0] + g, 1u, false);
        }
        return;
    }
    if (threadIdx.x == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        const uint32_t old = atom_add_acq_rel_gpu(a.counters[a.rank] + g, 1u);
        *s_last = old + 1u == (a.epoch + 1u) * gridDim.x;
    }
    __syncthreads();
    if (*s_last) {
        pc_push_outputs<NCOLS>(a, grp);
        __syncthreads();
        if (threadIdx.x == 0) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            for (int q = 0; q < a.world; ++q) red_relaxed_add(a.counters[q] + a.ngroups + g, 1u, true);
        }
    }
}

// ---- tile arithmetic -------------------------------------------------------------------

// Dots of one staged tile (rows r0 .. r0 + rows - 1 of GEMV `gm`, a device descriptor) and
// the stores of its outputs to every rank's buffer.  Same lane mapping and reduction
// order as mmvq_kernel with LBT lanes per row.  Scalar arguments only, so the call keeps
// everything in registers.
template <int QT, int NCOLS, int RPB, int LBT>
__device__ __noinline__ void pc_tile(const PcGemv *__restrict__ gm, const uint8_t *wrow0, int r0,
                                     int rows, const uint8_t *aq, const float *ad,
                                     const float *ads, const int2 *as, int K, int rank) {
    using TR = QTraits<QT>;
    constexpr int RG = 32 / LBT;
    constexpr int NS = RPB >= RG ? RPB / RG : 1;
    const int lane = threadIdx.x & 31;
    const int bl = lane & (LBT - 1), grp = lane / LBT;
    const int nkb = K >> 5, acb = act_col_bytes(nkb);
    const int row_bytes = (K / TR::qk) * TR::bytes;
    const int nblk = K / TR::qk;
    float acc[NS][NCOLS];
#pragma unroll
    for (int i = 0; i < NS; ++i)
#pragma unroll
        for (int c = 0; c < NCOLS; ++c) acc[i][c] = 0.f;
    if (grp < RPB) {
        const TileCtx ctx{wrow0 + grp * row_bytes, RG * row_bytes, 0, r0, rows, K, nkb, acb, RG, grp,
                          aq, ad, ads, as, nullptr};
        for (int b = bl; b < nblk; b += LBT) {
            BlkHdr hdr[NS];
#pragma unroll
            for (int sl = 0; sl < NS; ++sl)
                hdr[sl] = load_hdr<QT>(ctx.lane_row0 + sl * ctx.slot_stride + b * TR::bytes);
            unit_step<QT, NCOLS, NS, kModeQ81, 0>(ctx, b, hdr, acc);
            if constexpr (Units<QT>::n == 4) {
                unit_step<QT, NCOLS, NS, kModeQ81, 1>(ctx, b, hdr, acc);
                unit_step<QT, NCOLS, NS, kModeQ81, 2>(ctx, b, hdr, acc);
                unit_step<QT, NCOLS, NS, kModeQ81, 3>(ctx, b, hdr, acc);
            }
        }
    }
    const int nfull = gm->nrows_full, row0 = gm->row0;
#pragma unroll
    for (int sl = 0; sl < NS; ++sl) {
        const int i = sl * RG + grp;
#pragma unroll
        for (int c = 0; c < NCOLS; ++c) {
            float v = acc[sl][c];
#pragma unroll
            for (int o = LBT >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (bl == 0 && grp < RPB && i < rows) {
                const size_t off = size_t(c) * nfull + row0 + r0 + i;
                gm->y[rank][off] = v;  // this rank's buffer; peers get the slice at group end
            }
        }
    }
}


#define ANVIL_PC_TILE_ARGS gm, wrow0, r0, rows, aq, ad, ads, as, K, rank

template <int QT, int NCOLS>
__device__ __forceinline__ void pc_tile_variant(int variant, const PcGemv *gm, const uint8_t *wrow0,
                                                int r0, int rows, const uint8_t *aq, const float *ad,
                                                const float *ads, const int2 *as, int K, int rank) {
    switch (variant) {
    case kV1x32: pc_tile<QT, NCOLS, 1, 32>(ANVIL_PC_TILE_ARGS); break;
    case kV2x32: pc_tile<QT, NCOLS, 2, 32>(ANVIL_PC_TILE_ARGS); break;
    case kV4x32: pc_tile<QT, NCOLS, 4, 32>(ANVIL_PC_TILE_ARGS); break;
    case kV8x32: pc_tile<QT, NCOLS, 8, 32>(ANVIL_PC_TILE_ARGS); break;
    case kV2x16: pc_tile<QT, NCOLS, 2, 16>(ANVIL_PC_TILE_ARGS); break;
    case kV4x16: pc_tile<QT, NCOLS, 4, 16>(ANVIL_PC_TILE_ARGS); break;
    case kV8x16: pc_tile<QT, NCOLS, 8, 16>(ANVIL_PC_TILE_ARGS); break;
    case kV4x8: pc_tile<QT, NCOLS, 4, 8>(ANVIL_PC_TILE_ARGS); break;
    case kV8x8: pc_tile<QT, NCOLS, 8, 8>(ANVIL_PC_TILE_ARGS); break;
    default: break;
    }
}

template <int NCOLS>
__device__ __forceinline__ void pc_tile_any(int type, int variant, const PcGemv *gm,
                                            const uint8_t *wrow0, int r0, int rows,
                                            const uint8_t *aq, const float *ad, const float *ads,
                                            const int2 *as, int K, int rank) {
    switch (type) {
    case kTypeQ4_K: pc_tile_variant<kTypeQ4_K, NCOLS>(variant, ANVIL_PC_TILE_ARGS); break;
    case kTypeQ5_K: pc_tile_variant<kTypeQ5_K, NCOLS>(variant, ANVIL_PC_TILE_ARGS); break;
    case kTypeQ6_K: pc_tile_variant<kTypeQ6_K, NCOLS>(variant, ANVIL_PC_TILE_ARGS); break;
    case kTypeQ8_0: pc_tile_variant<kTypeQ8_0, NCOLS>(variant, ANVIL_PC_TILE_ARGS); break;
    default: break;
    }
}

#undef ANVIL_PC_TILE_ARGS

// ---- the kernel ------------------------------------------------------------------------

// A warp's position in its tile sequence (group g, tile i of the group) with the current
// GEMV's descriptor fields held in registers; they are re-read only when the cursor
// crosses into another GEMV.
struct PcCursor {
    int g, i;
    int g_ntiles;              // tiles of group g
    int m, t_base, t_end;      // current GEMV index and its tile range in the group
    const uint8_t *W;
    int row_bytes, rpb, nrows, alloc, type, variant;
};

// Per-warp ring state (identical in every lane; lane 0 issues the copies).  Ring space is
// tracked two ways: cumulative byte counts (allocated incl. wrap padding / released) for
// the free-space test, and positions in the ring for the addresses.
struct PcRing {
    PcCursor pc;               // producer cursor, runs ahead of the consumer
    uint32_t p_total, c_total, p_pos, c_pos, issued, consumed;
};

// What every warp of the launch shares (pointers into this CTA's shared memory).
struct PcWarp {
    uint8_t *ring;
    uint64_t *bars;
    int *s_failed;
    int gw, nw, lane;
    uint32_t R;
};

__device__ __forceinline__ int pc_first(int rot, int gw, int nw) {
    int f = (gw - rot) % nw;
    return f < 0 ? f + nw : f;
}

// Loads the descriptor of the GEMV that holds tile c.i of group c.g.
__device__ __forceinline__ void pc_load_gemv(const PcArgs &a, PcCursor &c) {
    const PcGroup *gp = a.groups + c.g;
    const int count = gp->count;
    int m = gp->first;
    const PcGemv *gm = a.gemvs + m;
    for (int k = 0; k + 1 < count && c.i >= gm->tile_base + gm->ntiles; ++k) ++gm, ++m;
    c.m = m;
    c.t_base = gm->tile_base;
    c.t_end = gm->tile_base + gm->ntiles;
    c.W = gm->W;
    c.row_bytes = gm->row_bytes;
    c.rpb = gm->rpb;
    c.nrows = gm->nrows;
    c.alloc = gm->alloc;
    c.type = gm->type;
    c.variant = gm->variant;
}

// Moves `c` to the first group (from c.g on) that holds a tile of this warp
// (c.g == ngroups: none left) and loads that tile's GEMV.
__device__ __forceinline__ void pc_settle(const PcArgs &a, PcCursor &c, int gw, int nw) {
    while (c.g < a.ngroups) {
        c.g_ntiles = a.groups[c.g].ntiles;
        if (c.i < c.g_ntiles) {
            pc_load_gemv(a, c);
            return;
        }
        ++c.g;
        if (c.g < a.ngroups) c.i = pc_first(a.groups[c.g].rot, gw, nw);
    }
}

__device__ __forceinline__ void pc_advance(const PcArgs &a, PcCursor &c, int gw, int nw) {
    c.i += nw;
    if (c.i >= c.t_end) {
        if (c.i < c.g_ntiles) {
            pc_load_gemv(a, c);
        } else {
            ++c.g;
            if (c.g < a.ngroups) c.i = pc_first(a.groups[c.g].rot, gw, nw);
            pc_settle(a, c, gw, nw);
        }
    }
}

// Issues tiles while the ring and the mbarrier slots have room.
__device__ __forceinline__ void pc_produce(const PcArgs &a, PcRing &r, const PcWarp &w) {
    while (r.pc.g < a.ngroups && r.issued - r.consumed < uint32_t(kPcSlots)) {
        const uint32_t alloc = uint32_t(r.pc.alloc);
        const bool wrap = r.p_pos + alloc > w.R;
        const uint32_t need = (wrap ? w.R - r.p_pos : 0u) + alloc;
        // Live tiles hold p_total - c_total bytes; an empty ring takes any tile
        // (alloc <= R, checked on the host), whatever the wrap padding.
        if (r.issued != r.consumed && r.p_total - r.c_total + need > w.R) break;
        const uint32_t pos = wrap ? 0u : r.p_pos;
        if (w.lane == 0) {
            const int slot = int(r.issued % kPcSlots);
            const int r0 = (r.pc.i - r.pc.t_base) * r.pc.rpb;
            const int rows = min(r.pc.rpb, r.pc.nrows - r0);
            const uint8_t *src = r.pc.W + size_t(r0) * size_t(r.pc.row_bytes);
            const uintptr_t s = reinterpret_cast<uintptr_t>(src);
            const uintptr_t e = s + size_t(rows) * r.pc.row_bytes;
            const uintptr_t s_al = (s + 15) & ~uintptr_t(15), e_al = e & ~uintptr_t(15);
            uint8_t *dst = w.ring + pos + uint32_t(s & 15);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (e_al > s_al) {
                mbar_arrive_expect_tx(&w.bars[slot], uint32_t(e_al - s_al));
                bulk_copy_g2s(dst + (s_al - s), reinterpret_cast<const void *>(s_al),
                              uint32_t(e_al - s_al), &w.bars[slot]);
            } else {
                mbar_arrive(&w.bars[slot]);
            }
        }
        r.p_total += need;
        r.p_pos = pos + alloc;
        ++r.issued;
        pc_advance(a, r.pc, w.gw, w.nw);
    }
}


template <int NCOLS>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) pchain_kernel(const __grid_constant__ PcArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nwarps = blockDim.x >> 5;
    uint8_t *act_base = smem + a.act_off;
    // Set once a bounded wait of this CTA (or, at the launch start, of any kernel of this
    // library) has given up: later weight waits then use a 1 ms bound.
    __shared__ int s_failed, s_last;
    if (tid == 0) s_failed = 0;

    PcWarp w;
    w.ring = smem + a.ring_off + size_t(warp) * a.ring_bytes;
    w.bars = reinterpret_cast<uint64_t *>(smem) + warp * kPcSlots;
    w.s_failed = &s_failed;
    w.nw = gridDim.x * nwarps;
    w.gw = blockIdx.x * nwarps + warp;
    w.lane = lane;
    w.R = uint32_t(a.ring_bytes);

    PcRing r{};
    r.pc.g = 0;
    if (a.ngroups > 0) {
        r.pc.i = pc_first(a.groups[0].rot, w.gw, w.nw);
        pc_settle(a, r.pc, w.gw, w.nw);
    }

    if (lane == 0) {
        for (int s = 0; s < kPcSlots; ++s) mbar_init(&w.bars[s], 1);
        mbar_fence_init();
    }
    __syncwarp();

    pc_produce(a, r, w);  // the first weight tiles stream while the first activation is staged

    // The next group's descriptor is read one group ahead, off the barrier's critical path.
    PcGroup nx{};
    if (a.ngroups > 0) nx = a.groups[0];
    for (int g = 0; g < a.ngroups; ++g) {
        const PcGroup cur = nx;
        if (g + 1 < a.ngroups) nx = a.groups[g + 1];
        const int K = cur.K;
        // ---- 1. dependencies -------------------------------------------------------------
        if (tid == 0) {
            const uint32_t per_epoch = a.world > 1 ? uint32_t(a.world) : gridDim.x;
            if (g == 0) {
                if (pc_failed()) s_failed = 1;
                if (a.world > 1 && a.epoch > 0)
                    pc_wait_counters(a, a.first_wait_from, a.ngroups, a.epoch * per_epoch);
            } else if (cur.wait_to > cur.wait_from) {
                pc_wait_counters(a, cur.wait_from, cur.wait_to, (a.epoch + 1) * per_epoch);
            }
        }
        __syncthreads();
        // ---- 2. stage the group's activation (fused Q8_1 quantisation) ---------------------
        const int nkb = K >> 5;
        uint8_t *aq = act_base;
        float *ad = reinterpret_cast<float *>(aq + NCOLS * act_col_bytes(nkb));
        float *ads = ad + NCOLS * nkb;
        int2 *as = reinterpret_cast<int2 *>(
            (reinterpret_cast<uintptr_t>(ads + NCOLS * nkb) + 15) & ~uintptr_t(15));
        if (cur.family == 0)  // K-quant swizzle
            stage_f32_q8_1<kTypeQ4_K, NCOLS>(cur.x, K, aq, ad, ads, as);
        else                  // Q8_0 swizzle
            stage_f32_q8_1<kTypeQ8_0, NCOLS>(cur.x, K, aq, ad, ads, as);
        __syncthreads();

        // ---- 3. this warp's tiles of the group -------------------------------------------
        PcCursor cc{};
        cc.g = g;
        cc.i = pc_first(cur.rot, w.gw, w.nw);
        cc.g_ntiles = cur.ntiles;
        if (cc.i < cc.g_ntiles) pc_load_gemv(a, cc);
        for (; cc.i < cc.g_ntiles; cc.i += w.nw) {
            if (cc.i >= cc.t_end) pc_load_gemv(a, cc);
            if (r.issued == r.consumed) pc_produce(a, r, w);
            const uint32_t alloc = uint32_t(cc.alloc);
            const bool wrap = r.c_pos + alloc > w.R;
            const uint32_t pos = wrap ? 0u : r.c_pos;
            const int r0 = (cc.i - cc.t_base) * cc.rpb;
            const int rows = min(cc.rpb, cc.nrows - r0);
            const int slot = int(r.consumed % kPcSlots);
            const uint32_t parity = (r.consumed / kPcSlots) & 1u;
            const uint8_t *src = cc.W + size_t(r0) * size_t(cc.row_bytes);
            const uintptr_t s = reinterpret_cast<uintptr_t>(src);
            const uintptr_t e = s + size_t(rows) * cc.row_bytes;
            uint8_t *wrow0 = w.ring + pos + uint32_t(s & 15);
            bool have_w = mbar_try_wait(&w.bars[slot], parity);
            if (!have_w) {
                const uint64_t lim = *reinterpret_cast<volatile int *>(&s_failed) ? 1000000ull
                                                                                   : kWaitLimitNs;
                have_w = mbar_wait_bounded(&w.bars[slot], parity, lim);
                if (!have_w) {
                    s_failed = 1;
                    (void)mbar_wait_bounded(&w.bars[slot], parity, lim);
                }
            }
            if ((s | e) & 15) {  // unaligned ends: plain loads of at most 30 bytes
                const uintptr_t s_al = (s + 15) & ~uintptr_t(15), e_al = e & ~uintptr_t(15);
                if (e_al > s_al) {
                    const int nh = int(s_al - s), nt = int(e - e_al);
                    for (int k = lane; k < nh + nt; k += 32) {
                        const size_t off = k < nh ? size_t(k) : size_t(e_al - s) + size_t(k - nh);
                        wrow0[off] = src[off];
                    }
                } else {
                    for (int k = lane; k < int(e - s); k += 32) wrow0[k] = src[k];
                }
                __syncwarp();
            }
            if (have_w)
                pc_tile_any<NCOLS>(cc.type, cc.variant, a.gemvs + cc.m, wrow0, r0, rows, aq, ad, ads,
                                   as, K, a.rank);
            __syncwarp();  // every lane is done with the tile's ring bytes
            r.c_total += (wrap ? w.R - r.c_pos : 0u) + alloc;
            r.c_pos = pos + alloc;
            ++r.consumed;
            pc_produce(a, r, w);
        }
        // ---- 4. arrive -------------------------------------------------------------------
        __syncthreads();  // all warps done with this group's activation and outputs
        pc_arrive<NCOLS>(a, cur, g, &s_last);
    }
}

static int pc_take_status() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_anvil_device_status, sizeof(int)) != cudaSuccess) return -1;
    if (cudaMemcpyToSymbol(g_anvil_device_status, &z, sizeof(int)) != cudaSuccess) return -1;
    return v;
}

using PcKernel = void (*)(PcArgs);
static PcKernel pc_kernel_for(int ncols) {
    switch (ncols) {
    case 1: return pchain_kernel<1>;
    case 2: return pchain_kernel<2>;
    default: return nullptr;
    }
}

// Lanes-per-row utilisation of a (rows per tile, lanes per row) shape on rows of nblk blocks
// (the measure host_lanes_per_row maximises).
static float pc_util(int nblk, int rpb, int lb) {
    const int rg = 32 / lb;
    const int per_lane = (nblk + lb - 1) / lb;
    const float r = float(rpb) / float(rg);
    return float(nblk) / float(lb * per_lane) * (r < 1.f ? r : 1.f);
}

static int pc_variant(int rpb, int lb) {
    for (int v = 0; v < kNumVariants; ++v)
        if (kVarRpb[v] == rpb && kVarLb[v] == lb) return v;
    return -1;
}

}  // namespace anvil

using namespace anvil;

struct PcGemvHost {
    PcGemv d;
    int rpb_req, K, qk;
};

struct anvil_pchain {
    int world = 1, rank = 0, ncols = 0;
    std::vector<PcGroup> groups;
    std::vector<PcGemvHost> gemvs;
    uint32_t *counters[kPcMaxRanks] = {};
    uint32_t *own_counters = nullptr;
    PcGroup *d_groups = nullptr;
    PcGemv *d_gemvs = nullptr;
    uint32_t **d_counters = nullptr;
    PcKernel fn = nullptr;
    int grid = 0, nwarps = 0, smem = 0, ring_bytes = 0, act_off = 0, ring_off = 0;
    int first_wait_from = 0;
    uint32_t epoch = 0;
    bool ready = false;
};

extern "C" {

anvil_pchain *anvil_pchain_create(int world, int rank) {
    if (world < 1 || world > kPcMaxRanks || rank < 0 || rank >= world) {
        fail(ANVIL_ERR_INVALID, "world=%d rank=%d (world must be 1..%d)", world, rank, kPcMaxRanks);
        return nullptr;
    }
    anvil_pchain *c = new (std::nothrow) anvil_pchain();
    if (!c) {
        fail(ANVIL_ERR_INVALID, "out of host memory");
        return nullptr;
    }
    c->world = world;
    c->rank = rank;
    return c;
}

void anvil_pchain_destroy(anvil_pchain *c) {
    if (!c) return;
    if (c->d_groups) cudaFree(c->d_groups);
    if (c->d_gemvs) cudaFree(c->d_gemvs);
    if (c->d_counters) cudaFree(c->d_counters);
    if (c->own_counters) cudaFree(c->own_counters);
    delete c;
}

int anvil_pchain_add_group(anvil_pchain *c, const float *x, int K, int ncols, int wait_prev) {
    if (!c || !x) return fail(ANVIL_ERR_INVALID, "null argument");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (K <= 0 || K % 32 != 0) return fail(ANVIL_ERR_INVALID, "K=%d is not a positive multiple of 32", K);
    if (ncols != 1 && ncols != 2)
        return fail(ANVIL_ERR_UNSUPPORTED, "persistent chain supports ncols 1 and 2 (got %d)", ncols);
    if (c->ncols && ncols != c->ncols)
        return fail(ANVIL_ERR_INVALID, "all groups of a chain have the same ncols");
    if (reinterpret_cast<uintptr_t>(x) & 15) return fail(ANVIL_ERR_ALIGN, "x must be 16-byte aligned");
    c->ncols = ncols;
    PcGroup g{};
    g.x = x;
    g.K = K;
    g.first = int(c->gemvs.size());
    g.count = 0;
    g.family = -1;
    g.wait_from = g.wait_to = wait_prev ? 1 : 0;  // resolved at instantiation
    c->groups.push_back(g);
    return ANVIL_OK;
}

int anvil_pchain_add_gemv(anvil_pchain *c, int ggml_type, const void *W, int nrows, int row0,
                          int nrows_full, float *const *y, int rows_per_block) {
    if (!c || !W || !y) return fail(ANVIL_ERR_INVALID, "null argument");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (c->groups.empty()) return fail(ANVIL_ERR_INVALID, "add a group first");
    int qk, bb;
    if (int s = anvil_type_geometry(ggml_type, &qk, &bb)) return s;
    if (ggml_type != ANVIL_TYPE_Q8_0 && ggml_type != ANVIL_TYPE_Q4_K && ggml_type != ANVIL_TYPE_Q5_K &&
        ggml_type != ANVIL_TYPE_Q6_K)
        return fail(ANVIL_ERR_UNSUPPORTED, "the persistent chain takes Q8_0, Q4_K, Q5_K and Q6_K "
                                           "weights (type %d)", ggml_type);
    PcGroup &g = c->groups.back();
    if (g.K % qk) return fail(ANVIL_ERR_INVALID, "K=%d is not a multiple of the block size %d", g.K, qk);
    if (nrows < 1 || row0 < 0 || nrows_full < row0 + nrows)
        return fail(ANVIL_ERR_INVALID, "rows [%d, %d) outside a %d-row matrix", row0, row0 + nrows,
                    nrows_full);
    if (reinterpret_cast<uintptr_t>(W) & 15)
        return fail(ANVIL_ERR_ALIGN, "weights must be 16-byte aligned");
    for (int q = 0; q < c->world; ++q) {
        if (!y[q]) return fail(ANVIL_ERR_INVALID, "null output pointer for rank %d", q);
        if (reinterpret_cast<uintptr_t>(y[q]) & 3)
            return fail(ANVIL_ERR_ALIGN, "outputs must be 4-byte aligned");
    }
    const int family = ggml_type == ANVIL_TYPE_Q8_0 ? 1 : 0;
    if (g.family >= 0 && g.family != family) {
        // Q8_0 and the K-quants read the staged activation in different swizzles: continue
        // in a new group on the same input, restaged, with no barrier in between.
        PcGroup n{};
        n.x = g.x;
        n.K = g.K;
        n.first = int(c->gemvs.size());
        n.family = -1;
        n.wait_from = n.wait_to = 0;
        c->groups.push_back(n);
    }
    PcGroup &cur = c->groups.back();
    cur.family = family;
    cur.count += 1;
    PcGemvHost h{};
    h.d.W = static_cast<const uint8_t *>(W);
    for (int q = 0; q < c->world; ++q) h.d.y[q] = y[q];
    h.d.type = ggml_type;
    h.d.nrows = nrows;
    h.d.row0 = row0;
    h.d.nrows_full = nrows_full;
    h.d.row_bytes = (cur.K / qk) * bb;
    h.rpb_req = rows_per_block;
    h.K = cur.K;
    h.qk = qk;
    c->gemvs.push_back(h);
    return ANVIL_OK;
}

int anvil_pchain_set_counters(anvil_pchain *c, uint32_t *const *counters) {
    if (!c || !counters) return fail(ANVIL_ERR_INVALID, "null argument");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    for (int q = 0; q < c->world; ++q) {
        if (!counters[q] || (reinterpret_cast<uintptr_t>(counters[q]) & 3))
            return fail(ANVIL_ERR_INVALID, "counter array of rank %d is null or misaligned", q);
        c->counters[q] = counters[q];
    }
    return ANVIL_OK;
}

int anvil_pchain_instantiate(anvil_pchain *c, int nwarps, int ctas_per_sm) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (c->groups.empty()) return fail(ANVIL_ERR_INVALID, "empty chain");
    for (const PcGroup &g : c->groups)
        if (g.count == 0) return fail(ANVIL_ERR_INVALID, "a group has no GEMV");
    if (nwarps == 0) nwarps = 8;
    if (ctas_per_sm == 0) ctas_per_sm = 1;
    if (nwarps < 1 || nwarps > kMaxWarps) return fail(ANVIL_ERR_INVALID, "nwarps=%d", nwarps);
    if (ctas_per_sm < 1 || ctas_per_sm > 4) return fail(ANVIL_ERR_INVALID, "ctas_per_sm=%d", ctas_per_sm);
    if (c->world > 1)
        for (int q = 0; q < c->world; ++q)
            if (!c->counters[q]) return fail(ANVIL_ERR_INVALID, "world > 1 needs every rank's counters");
    int dev, nsm;
    if (int s = current_device(&dev)) return s;
    if (int s = sm_count(dev, &nsm)) return s;
    c->fn = pc_kernel_for(c->ncols);

    // Shared memory: [mbarriers][activation of the largest group][nwarps rings].
    int act = 0;
    for (const PcGroup &g : c->groups) {
        const int nkb = g.K / 32;
        const int b = c->ncols * act_col_bytes(nkb) + 2 * c->ncols * nkb * 4 + 16 + c->ncols * nkb * 8;
        act = std::max(act, b);
    }
    act = (act + 15) & ~15;
    const int bars = (nwarps * kPcSlots * 8 + 15) & ~15;
    const int budget = (228 * 1024) / ctas_per_sm - 1024;  // per CTA, less the runtime's reserve
    const int ring = ((std::min(budget, kMaxSmem) - bars - act) / nwarps) & ~15;
    if (ring < 4096) return fail(ANVIL_ERR_UNSUPPORTED, "no room for weight rings (%d B per warp)", ring);

    // Tile shape per GEMV: requested rows per tile (else the built-in default), the lanes per
    // row that keep the most lanes busy, and at most half a ring per tile.
    for (PcGemvHost &h : c->gemvs) {
        const int K = h.K;
        const int nblk = K / h.qk;
        int rpb = h.rpb_req > 0 ? h.rpb_req : (h.d.nrows < 2048 ? 1 : (K >= 8192 ? 2 : 4));
        rpb = rpb >= 8 ? 8 : rpb >= 4 ? 4 : rpb >= 2 ? 2 : 1;
        auto alloc_of = [&](int r) { return ((r * h.d.row_bytes + 32) + 15) & ~15; };
        while (rpb > 1 && alloc_of(rpb) > ring / 2) rpb >>= 1;
        if (alloc_of(rpb) > ring)
            return fail(ANVIL_ERR_UNSUPPORTED, "a %d-byte row does not fit a %d-byte ring",
                        h.d.row_bytes, ring);
        int best = -1;
        float bu = -1.f;
        for (int lb : {32, 16, 8}) {
            const int v = pc_variant(rpb, lb);
            if (v < 0) continue;
            const float u = pc_util(nblk, rpb, lb);
            if (u > bu + 1e-6f) {
                bu = u;
                best = v;
            }
        }
        if (best < 0) best = pc_variant(rpb, 32);
        h.d.variant = best;
        h.d.rpb = rpb;
        h.d.alloc = alloc_of(rpb);
    }

    // Tiles and barrier spans.
    std::vector<PcGemv> dg;
    dg.reserve(c->gemvs.size());
    for (const PcGemvHost &h : c->gemvs) dg.push_back(h.d);
    int last_wait = 0;
    for (size_t gi = 0; gi < c->groups.size(); ++gi) {
        PcGroup &g = c->groups[gi];
        int t = 0;
        for (int m = g.first; m < g.first + g.count; ++m) {
            dg[m].tile_base = t;
            dg[m].ntiles = (dg[m].nrows + dg[m].rpb - 1) / dg[m].rpb;
            t += dg[m].ntiles;
        }
        g.ntiles = t;
        const bool waits = gi > 0 && g.wait_to != 0;
        if (waits) {
            g.wait_from = last_wait;
            g.wait_to = int(gi);
            last_wait = int(gi);
        } else {
            g.wait_from = g.wait_to = 0;
        }
    }
    c->first_wait_from = last_wait;

    int occ = 0;
    const int threads = nwarps * 32;
    const int smem = bars + act + nwarps * ring;
    cudaError_t e = cudaFuncSetAttribute(c->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, c->fn, threads, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (occ < ctas_per_sm)
        return fail(ANVIL_ERR_UNSUPPORTED, "only %d CTAs of %d B fit per SM (asked %d)", occ, smem,
                    ctas_per_sm);
    c->grid = ctas_per_sm * nsm;
    c->nwarps = nwarps;
    c->smem = smem;
    c->ring_bytes = ring;
    c->act_off = bars;
    c->ring_off = bars + act;
    const int nw = c->grid * nwarps;
    long cum = 0;
    for (PcGroup &g : c->groups) {
        g.rot = int(cum % nw);
        cum += g.ntiles;
    }

    e = cudaMalloc(&c->d_groups, sizeof(PcGroup) * c->groups.size());
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(groups)");
    e = cudaMalloc(&c->d_gemvs, sizeof(PcGemv) * dg.size());
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(gemvs)");
    e = cudaMemcpy(c->d_groups, c->groups.data(), sizeof(PcGroup) * c->groups.size(),
                   cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(groups)");
    e = cudaMemcpy(c->d_gemvs, dg.data(), sizeof(PcGemv) * dg.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(gemvs)");
    for (size_t m = 0; m < dg.size(); ++m) c->gemvs[m].d = dg[m];
    if (c->world == 1 && !c->counters[0]) {
        e = cudaMalloc(&c->own_counters, 2 * sizeof(uint32_t) * c->groups.size());
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(counters)");
        e = cudaMemset(c->own_counters, 0, 2 * sizeof(uint32_t) * c->groups.size());
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(counters)");
        c->counters[0] = c->own_counters;
    }
    e = cudaMalloc(&c->d_counters, sizeof(uint32_t *) * c->world);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(counter table)");
    e = cudaMemcpy(c->d_counters, c->counters, sizeof(uint32_t *) * c->world, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(counter table)");
    c->ready = true;
    return ANVIL_OK;
}

int anvil_pchain_launch(anvil_pchain *c, anvil_stream_t stream) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (!c->ready) return fail(ANVIL_ERR_INVALID, "chain not instantiated");
    PcArgs a{};
    a.groups = c->d_groups;
    a.gemvs = c->d_gemvs;
    a.counters = c->d_counters;
    a.ngroups = int(c->groups.size());
    a.world = c->world;
    a.rank = c->rank;
    a.act_off = c->act_off;
    a.ring_off = c->ring_off;
    a.ring_bytes = c->ring_bytes;
    a.first_wait_from = c->first_wait_from;
    a.epoch = c->epoch;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(c->grid));
    cfg.blockDim = dim3(unsigned(c->nwarps * 32));
    cfg.dynamicSmemBytes = size_t(c->smem);
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, c->fn, a);
    if (e != cudaSuccess) return cuda_fail(e, "persistent chain launch");
    ++c->epoch;
    return ANVIL_OK;
}

int anvil_pchain_info(const anvil_pchain *c, int *grid, int *nwarps, int *ring_bytes,
                      int *smem_bytes, int *ngroups) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (grid) *grid = c->grid;
    if (nwarps) *nwarps = c->nwarps;
    if (ring_bytes) *ring_bytes = c->ring_bytes;
    if (smem_bytes) *smem_bytes = c->smem;
    if (ngroups) *ngroups = int(c->groups.size());
    return ANVIL_OK;
}

int anvil_pchain_gemv_shape(const anvil_pchain *c, int index, int *rows_per_block,
                            int *lanes_per_row) {
    if (!c || index < 0 || index >= int(c->gemvs.size()))
        return fail(ANVIL_ERR_INVALID, "bad GEMV index");
    if (!c->ready) return fail(ANVIL_ERR_INVALID, "chain not instantiated");
    if (rows_per_block) *rows_per_block = c->gemvs[index].d.rpb;
    if (lanes_per_row) *lanes_per_row = kVarLb[c->gemvs[index].d.variant];
    return ANVIL_OK;
}

int anvil_pchain_take_status(void) {
    const int v = pc_take_status();
    if (v < 0) return fail(ANVIL_ERR_CUDA, "reading device status failed");
    return v;
}

// ---- peer memory for the row-sharded chain -----------------------------------------------

int anvil_ipc_alloc(size_t bytes, void **ptr, void *handle) {
    if (!ptr || !handle || bytes == 0) return fail(ANVIL_ERR_INVALID, "null argument or zero size");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(peer buffer)");
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "cudaIpcGetMemHandle");
    }
    std::memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return ANVIL_OK;
}

int anvil_ipc_open(const void *handle, void **ptr) {
    if (!handle || !ptr) return fail(ANVIL_ERR_INVALID, "null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    return ANVIL_OK;
}

int anvil_ipc_close(void *ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
    return ANVIL_OK;
}

int anvil_ipc_free(void *ptr) {
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFree(peer buffer)");
    return ANVIL_OK;
}

}  // extern "C"
