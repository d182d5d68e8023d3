// chain_persistent.cu -- one cooperative launch runs a whole token's GEMV chain, on one GPU
// or row-sharded across several, with the decoder's data flow carried by flagged words.
//
// A decode token is a fixed sequence of MMVQ GEMVs.  Launched one kernel per GEMV, each
// pays a start-up and drain cost of a few microseconds that the weight stream of a small
// GEMV cannot hide.  Here a persistent kernel walks the chain instead:
//
//   * Groups.  GEMVs that read the same activation form a group (q/k/v; o; gate/up; down).
//     A group's input is either a fixed fp32 vector (the token's embedding) or the output
//     of an earlier GEMV of the chain ("chained": the attention output stands in as q's
//     output, the ffn input as o's, down's input as silu(gate) * up, the next layer's input
//     as down's).  Every CTA with work in the group quantises the input to Q8_1 in shared
//     memory itself, with the arithmetic of quantize_q8_1 (d = amax/127 by IEEE division,
//     q = roundf(x/d)).  Each warp stages its share of the next group right after its own
//     tiles of the current one, into the other of two activation buffers, so one CTA barrier
//     per group remains.  A chained input keeps d8 in fp32, and the group's results are
//     multiplied by a power of two, 2^-e with e the exponent of the input's largest
//     magnitude: values stay in range through hundreds of GEMVs, exactly (the quants are
//     those of the input itself).
//   * Flagged output words.  Every output value is written as one 8-byte word {fp32 value,
//     32-bit epoch}, the launch number, with a single 64-bit store, into each rank's copy of
//     the output (this GPU's, and the peers' over NVLink through CUDA IPC mappings).  A
//     consumer reads the words of its input and waits (bounded) only until each carries
//     the current epoch: a word is its own ready flag, so no fence, counter or grid barrier
//     sits between a producer and its consumers, and a group starts on each CTA as soon as
//     the values it reads have arrived.  Output buffers hold two epochs (launch parity), so
//     a rank one launch ahead never overwrites words a slower rank is still reading.
//     Chained sources are stored in a lane-blocked order (ll_pos) so that a warp's 16-byte
//     loads are contiguous and each lane still ends up with 16 consecutive values.
//   * Weight rings.  Each warp owns a byte ring in shared memory and deals itself tiles
//     round-robin across the tiles of every group of the chain.  Lane 0 keeps the ring full
//     with bulk async copies (cp.async.bulk, completion on one of 8 mbarriers) and runs
//     ahead across group boundaries: while a CTA waits for its next input, the copies for
//     the next groups' weights are already in flight.  A gate/up pair is one tile of h gate
//     rows and h up rows (two copies into one stage); its epilogue stores silu(g) * u.
//   * Dots.  The tile arithmetic is the MMVQ kernel's (unit_step, load_hdr; lane-per-block
//     decode with compile-time lanes per row), so for the same rows per tile and lanes per
//     row a fixed-input GEMV is bit-identical to anvil_mmvq's.
//
// Co-residency of all CTAs (consumers wait for other CTAs' words) comes from the cooperative
// launch.  Every wait is bounded; a wait that gives up raises a status flag of this
// translation unit (read by anvil_pchain_take_status), later waits of the launch then end
// at once, and the kernel runs to its end with wrong results, never hung.
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
constexpr int kPcSlots = 8;              // tiles in flight per warp
constexpr int kPcStaticPct = 100;        // default share of a group's tiles dealt round-robin
// Status flags: 1 (kStatusMbarTimeout) = a weight copy did not land in time, set by
// mbar_wait_bounded; 2 = an input word did not arrive in time.
constexpr int kStatusInputTimeout = 2;

// Compile-time tile shapes: rows per stage x lanes per row; the gate/up shapes stage h gate
// rows then h up rows (rows per stage 2h).
enum PcVariant : int {
    kV1x32, kV2x32, kV4x32, kV8x32, kV2x16, kV4x16, kV8x16, kV4x8, kV8x8,
    kG1x32, kG2x32, kG2x16, kG4x32, kG4x16, kG4x8, kNumVariants
};
constexpr int kVarRpb[kNumVariants] = {1, 2, 4, 8, 2, 4, 8, 4, 8, 2, 4, 4, 8, 8, 8};
constexpr int kVarLb[kNumVariants] = {32, 32, 32, 32, 16, 16, 16, 8, 8, 32, 32, 16, 32, 16, 8};
constexpr bool kVarGlu[kNumVariants] = {false, false, false, false, false, false, false, false,
                                        false, true,  true,  true,  true,  true,  true};

struct PcGemv {
    const uint8_t *W;          // this rank's rows (the gate rows of a gate/up pair)
    const uint8_t *W2;         // the up rows of a gate/up pair, else null
    uint64_t *y[kPcMaxRanks];  // each rank's output words: [2 parities][ncols][nrows_full]
    int type, variant;
    int rpb, trows;            // rows per stage; output rows per tile (rpb, or rpb/2 for a pair)
    int nrows, row0, nrows_full;
    int perm;                  // output stored in ll_pos order (a chained group reads it)
    int row_bytes, alloc;      // alloc: ring bytes one tile takes
    int tile_base, ntiles;     // tiles of this GEMV within its group
};

// Tiles of a group: tiles [0, spw * nw) are dealt round-robin over the nw warps of the grid
// (warp gw takes rot-shifted tiles gw - rot + k nw, k < spw); the rest are claimed one at a
// time from the group's counter by whichever warp has ring room first, so warps that start
// the group early (or run faster) take more of its tail.
struct PcGroup {
    const float *x;            // fixed fp32 input (ncols x K), or null
    const uint64_t *src;       // chained: this rank's output words of the source GEMV
    uint8_t *dump;             // optional: staged Q8_1 blocks written here (parity probe)
    int K, first, count, ntiles, rot, family;
    int spw;                   // round-robin tiles per warp
};

struct PcArgs {
    const PcGroup *groups;
    const PcGemv *gemvs;
    uint64_t *trace;            // optional: per CTA and group {start, staged, done, 1}
    int *claims;                // tile counters: [2 epoch parities][ngroups]
    uint64_t wait_ns;           // bound on every wait
    int ngroups, world, rank;
    int act_off[2], ring_off, ring_bytes;  // activation buffers of even / odd groups, rings
    uint32_t epoch;             // this launch's number: the flag of its words (never 0; its
                                // parity alternates from launch to launch)
};

// ---- flagged words -----------------------------------------------------------------------

// Position of value r of an n-value chained vector (n % 32 == 0) in its word array.  Values
// come in blocks of 512 (the last block holds t = n % 512 when that is not 0); within a block,
// value v = 16 l + 2 k + j (lane l, load k = 0..7, half j) sits at word k (t / 8) + 2 l + j, so
// the warp's k-th 16-byte load of the block is contiguous and lane l collects the 16
// consecutive values 16 l .. 16 l + 15.
__host__ __device__ __forceinline__ int ll_pos(int r, int n) {
    const int base = r & ~511;
    const int t = n - base < 512 ? n - base : 512;
    const int v = r & 511;
    return base + ((v & 15) >> 1) * (t >> 3) + ((v >> 4) << 1) + (v & 1);
}

__device__ __forceinline__ void st_word(uint64_t *p, float v, uint32_t epoch) {
    const uint64_t w = uint64_t(__float_as_uint(v)) | (uint64_t(epoch) << 32);
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ void ld_words2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// True once any bounded wait of this translation unit has given up: later waits then end at
// once (input words) or after 1 ms (weight copies), so a failed launch finishes quickly.
__device__ __forceinline__ bool pc_failed() {
    return *reinterpret_cast<volatile int *>(&g_anvil_device_status) != 0;
}

// A lane's 16 words of one 512-value block (p: the block start + 2 * lane; step = t / 8 for
// a block of t values): the warp's k-th 16-byte load is contiguous.
__device__ __forceinline__ void ll_issue(const uint64_t *p, int step, uint64_t (&w)[16]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) ld_words2(p + k * step, w[2 * k], w[2 * k + 1]);
}

// The values of the 16 words once all carry `epoch`: words that do not yet are re-read, with
// an exponential sleep between polls (64 ns doubling to 2 us) so that waiting warps leave L2
// to the producers, until they do or the bounded wait gives up (then the status flag is
// raised and the values are whatever was read).
__device__ __forceinline__ void ll_finish(const uint64_t *p, int step, uint32_t epoch,
                                          uint64_t wait_ns, uint64_t (&w)[16], float (&v)[16]) {
    uint32_t bad = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) bad |= uint32_t(uint32_t(w[i] >> 32) != epoch) << i;
    if (bad && !pc_failed()) {
        const uint64_t t0 = global_timer_ns();
        uint32_t nap = 64;
        while (bad) {
            __nanosleep(nap);
            nap = nap < 2048 ? 2 * nap : 2048;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                if (bad & (3u << (2 * k))) {
                    ld_words2(p + k * step, w[2 * k], w[2 * k + 1]);
                    bad &= ~(3u << (2 * k));
                    bad |= uint32_t(uint32_t(w[2 * k] >> 32) != epoch) << (2 * k);
                    bad |= uint32_t(uint32_t(w[2 * k + 1] >> 32) != epoch) << (2 * k + 1);
                }
            }
            if (bad && global_timer_ns() - t0 > wait_ns) {
                atomicOr(&g_anvil_device_status, kStatusInputTimeout);
                break;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(uint32_t(w[i]));
}

// 2^-e for a vector whose largest magnitude is m (e = the exponent of m); 2^127 for m == 0
// or subnormal m, 2^-126 from m >= 2^127 (infinities and NaN included).
__device__ __forceinline__ float pow2_scale(float m) {
    const int eb = int((__float_as_uint(m) >> 23) & 0xFF);
    const int E = min(max(254 - eb, 1), 254);
    return __uint_as_float(uint32_t(E) << 23);
}

// Where one staged activation lives in shared memory (one of the two buffers).
struct ActBuf {
    uint8_t *aq;
    float *ad, *ads;
    int2 *as;
};

__device__ __forceinline__ ActBuf act_buf(uint8_t *base, int K, int ncols) {
    const int nkb = K >> 5;
    ActBuf b;
    b.aq = base;
    b.ad = reinterpret_cast<float *>(base + ncols * act_col_bytes(nkb));
    b.ads = b.ad + ncols * nkb;
    b.as = reinterpret_cast<int2 *>((reinterpret_cast<uintptr_t>(b.ads + ncols * nkb) + 15) &
                                    ~uintptr_t(15));
    return b;
}

// Quantises this lane's 16 consecutive values (chunk cc of column col; the lane pair 2q, 2q+1
// holds one Q8_1 block) into the swizzled buffer, with the arithmetic of quantize_q8_1:
// d = amax / 127 (q8_scale), q = roundf(x / d) through quant_q8.  The stored d8 is
// rounded to fp16 (ROUND, as quantize_q8_1 stores it) or kept in fp32 (chained inputs).
// Returns the block's amax.  Whole warp (shuffles); `live` lanes store.
template <int QT, bool ROUND>
__device__ __forceinline__ float quant_chunk(const float (&v)[16], bool live, int col, int cc, int nkb,
                                             int acb, const ActBuf &b) {
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[i]));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    const float d = q8_scale(am);
    const float dn = am == 0.0f ? 1.0f : d;
    const double rd64 = 1.0 / double(dn);
    uint32_t w[4];
    int s;
    quant16(v, am, float(rd64), rd64, w, s);
    const int so = __shfl_xor_sync(0xffffffffu, s, 1);
    if (live) {
        *reinterpret_cast<uint4 *>(b.aq + col * acb + act_chunk<QT>(cc) * 16) =
            make_uint4(w[0], w[1], w[2], w[3]);
        if ((cc & 1) == 0) {
            const int i = col * nkb + (cc >> 1);
            const float dd = ROUND ? __half2float(__float2half_rn(d)) : d;
            b.ad[i] = dd;
            b.as[i] = make_int2(s, so);
            b.ads[i] = dd * float(s + so);
        }
    }
    return am;
}

// One warp's share of a chained group's staging: 512-value blocks warp, warp + nwarps, ...
// of the NCOLS columns of flagged words, read as they arrive, d8 kept in fp32; the warp's
// column maxima go to colmax[c].  Not inlined, and one block of words in flight per lane:
// the kernel body around it holds the registers its tile runs need.  (A second block in
// flight measured slower on the Llama-3-70B chain: 11.7 against 11.1 ms per token.)
template <int QT, int NCOLS>
__device__ __noinline__ void warp_stage_ll(const uint64_t *__restrict__ src, int K, uint32_t epoch,
                                           uint64_t wait_ns, uint32_t act_off, float *colmax) {
    extern __shared__ __align__(16) uint8_t smem[];
    const ActBuf b = act_buf(smem + act_off, K, NCOLS);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nkb = K >> 5, acb = act_col_bytes(nkb);
    const int nb = (K + 511) >> 9;
    const int total = NCOLS * nb;
    float cmax[NCOLS];
#pragma unroll
    for (int c = 0; c < NCOLS; ++c) cmax[c] = 0.f;
    for (int bi = warp; bi < total; bi += nw) {  // warp-uniform
        const int col = bi / nb, blk = bi - col * nb;
        const int t = min(512, K - blk * 512);
        const bool live = lane < (t >> 4);
        const uint64_t *p = src + size_t(col) * K + size_t(blk) * 512 + 2 * lane;
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        if (live) {
            uint64_t w[16];
            ll_issue(p, t >> 3, w);
            ll_finish(p, t >> 3, epoch, wait_ns, w, v);
        }
        const float am = quant_chunk<QT, false>(v, live, col, blk * 32 + lane, nkb, acb, b);
#pragma unroll
        for (int c = 0; c < NCOLS; ++c)
            if (c == col) cmax[c] = fmaxf(cmax[c], am);
    }
#pragma unroll
    for (int c = 0; c < NCOLS; ++c) {
        const float m = warp_max(cmax[c]);
        if (lane == 0) colmax[c] = m;
    }
}

// One warp's share of a fixed-input group's staging: the same blocks of fp32 values, d8
// rounded to fp16 as quantize_q8_1 stores it.
template <int QT, int NCOLS>
__device__ __noinline__ void warp_stage_f32(const float *__restrict__ x, int K, uint32_t act_off) {
    extern __shared__ __align__(16) uint8_t smem[];
    const ActBuf b = act_buf(smem + act_off, K, NCOLS);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nkb = K >> 5, acb = act_col_bytes(nkb);
    const int nb = (K + 511) >> 9;
    const int total = NCOLS * nb;
    for (int b0 = warp; b0 < total; b0 += 2 * nw) {
        float v[2][16];
        int col[2], blk[2];
        bool live[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int bi = min(b0 + j * nw, total - 1);
            col[j] = bi / nb;
            blk[j] = bi - col[j] * nb;
            live[j] = b0 + j * nw < total && lane < (min(512, K - blk[j] * 512) >> 4);
            const float4 *q = reinterpret_cast<const float4 *>(x + size_t(col[j]) * K + blk[j] * 512 +
                                                               16 * lane);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 f = live[j] ? __ldg(q + k) : make_float4(0.f, 0.f, 0.f, 0.f);
                v[j][4 * k] = f.x;
                v[j][4 * k + 1] = f.y;
                v[j][4 * k + 2] = f.z;
                v[j][4 * k + 3] = f.w;
            }
        }
        quant_chunk<QT, true>(v[0], live[0], col[0], blk[0] * 32 + lane, nkb, acb, b);
        if (b0 + nw < total) quant_chunk<QT, true>(v[1], live[1], col[1], blk[1] * 32 + lane, nkb, acb, b);
    }
}

// Writes the staged activation as {fp32 d8, 32 quants} blocks (parity probe).  Whole CTA.
template <int QT>
__device__ void dump_staged(uint8_t *out, int K, int ncols, const ActBuf &b) {
    const int nkb = K >> 5, acb = act_col_bytes(nkb);
    for (int i = threadIdx.x; i < ncols * nkb; i += blockDim.x) {
        const int c = i / nkb, kb = i - c * nkb;
        uint32_t *o = reinterpret_cast<uint32_t *>(out + size_t(i) * kQ8_1Bytes);
        o[0] = __float_as_uint(b.ad[i]);
        const uint4 u = *reinterpret_cast<const uint4 *>(b.aq + c * acb + act_chunk<QT>(2 * kb) * 16);
        const uint4 v = *reinterpret_cast<const uint4 *>(b.aq + c * acb + act_chunk<QT>(2 * kb + 1) * 16);
        o[1] = u.x; o[2] = u.y; o[3] = u.z; o[4] = u.w;
        o[5] = v.x; o[6] = v.y; o[7] = v.z; o[8] = v.w;
    }
}

// ---- tile arithmetic -------------------------------------------------------------------

// Where one GEMV's outputs go, held in registers per warp: the row offset of this rank's
// shard, the layout, and (set by pc_run, which knows the lanes per row) this lane's rank
// buffer: lane bl < world of a row's lanes stores to rank bl.
struct PcOut {
    uint64_t *const *ys;       // the GEMV descriptor's buffers, one per rank
    uint64_t *y;               // rank (bl < world ? bl : 0)'s buffer
    int nfull, row0, perm, world;
};

// Dots of one staged tile and the stores of its outputs, as flagged words, to every rank's
// buffer.  Plain: rows r0 .. r0 + rows - 1 of the GEMV.  Gate/up (GLU): the stage holds
// RPB/2 gate rows then RPB/2 up rows; slot s and slot s + NS/2 of a lane are gate and up row
// of the same output row, stored as silu(g) * u.  Same lane mapping and reduction order as
// mmvq_kernel with LBT lanes per row.  sc0 / sc1: the group's per-column input scale (1 for a
// fixed input).
template <int QT, int NCOLS, int RPB, int LBT, bool GLU>
__device__ __forceinline__ void pc_tile(const PcOut &o, uint32_t stage_off, int r0, int rows,
                                        uint32_t act_off, int K, uint32_t epoch, float sc0, float sc1) {
    extern __shared__ __align__(16) uint8_t smem[];
    const uint8_t *wrow0 = smem + stage_off;
    const ActBuf b = act_buf(smem + act_off, K, NCOLS);
    using TR = QTraits<QT>;
    constexpr int RG = 32 / LBT;
    constexpr int NS = RPB >= RG ? RPB / RG : 1;
    static_assert(!GLU || (NS % 2 == 0 && RPB % (2 * RG) == 0), "gate/up tile shape");
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
                          b.aq, b.ad, b.ads, b.as, nullptr};
        for (int blk = bl; blk < nblk; blk += LBT) {
            BlkHdr hdr[NS];
#pragma unroll
            for (int sl = 0; sl < NS; ++sl)
                hdr[sl] = load_hdr<QT>(ctx.lane_row0 + sl * ctx.slot_stride + blk * TR::bytes);
            unit_step<QT, NCOLS, NS, kModeQ81, 0>(ctx, blk, hdr, acc);
            if constexpr (Units<QT>::n == 4) {
                unit_step<QT, NCOLS, NS, kModeQ81, 1>(ctx, blk, hdr, acc);
                unit_step<QT, NCOLS, NS, kModeQ81, 2>(ctx, blk, hdr, acc);
                unit_step<QT, NCOLS, NS, kModeQ81, 3>(ctx, blk, hdr, acc);
            }
        }
    }
    const size_t par = size_t(epoch & 1u) * NCOLS;
    constexpr int NOUT = GLU ? NS / 2 : NS;
#pragma unroll
    for (int sl = 0; sl < NOUT; ++sl) {
        const int i = sl * RG + grp;
        const int row = o.row0 + r0 + i;
        const int pos = o.perm ? ll_pos(row, o.nfull) : row;
#pragma unroll
        for (int c = 0; c < NCOLS; ++c) {
            const float sc = c == 0 ? sc0 : sc1;
            float v = acc[sl][c];
#pragma unroll
            for (int k = LBT >> 1; k > 0; k >>= 1) v += __shfl_xor_sync(0xffffffffu, v, k);
            v *= sc;
            if constexpr (GLU) {
                float u = acc[sl + NS / 2][c];
#pragma unroll
                for (int k = LBT >> 1; k > 0; k >>= 1) u += __shfl_xor_sync(0xffffffffu, u, k);
                u *= sc;
                v = v / (1.0f + expf(-v)) * u;
            }
            if (bl < o.world && grp < RPB && i < rows) st_word(o.y + (par + c) * o.nfull + pos, v, epoch);
        }
    }
}

// ---- the kernel ------------------------------------------------------------------------

// A warp's position in its tile sequence (group g, tile i of the group) with the current
// GEMV's descriptor fields held in registers; they are re-read only when the cursor
// crosses into another GEMV.
struct PcCursor {
    int g, i;
    int g_ntiles;              // tiles of group g
    int k;                     // tiles this warp has taken of group g so far
    int m, t_base, t_end;      // current GEMV index and its tile range in the group
    const uint8_t *W, *W2;
    int row_bytes, rpb, trows, nrows, alloc, type, variant;
};

// Per-warp ring state (identical in every lane; lane 0 issues the copies).  Ring space is
// tracked two ways: cumulative byte counts (allocated incl. wrap padding / released) for
// the free-space test, and positions in the ring for the addresses.
struct PcRing {
    PcCursor pc;               // producer cursor, runs ahead of the consumer
    uint32_t p_total, c_total, p_pos, c_pos, issued, consumed;
};

struct PcWarp {
    uint8_t *ring;
    uint64_t *bars;
    int2 *tiles;               // per ring slot: {group, tile} of the copy issued into it
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
    c.W2 = gm->W2;
    c.row_bytes = gm->row_bytes;
    c.rpb = gm->rpb;
    c.trows = gm->trows;
    c.nrows = gm->nrows;
    c.alloc = gm->alloc;
    c.type = gm->type;
    c.variant = gm->variant;
}

// Moves the producer cursor to this warp's next tile: its round-robin tiles of group c.g
// first, then tiles claimed from the group's counter (lane 0 claims, every lane takes the
// result), then on to the next group once the group has none left (c.g == ngroups: the
// chain is done).  Loads the tile's GEMV when it differs from the current one.  Called by
// the whole warp.
__device__ __forceinline__ void pc_next(const PcArgs &a, PcCursor &c, const PcWarp &w) {
    while (c.g < a.ngroups) {
        const PcGroup *gp = a.groups + c.g;
        int i;
        if (c.k < gp->spw) {
            i = pc_first(gp->rot, w.gw, w.nw) + c.k * w.nw;
        } else {
            int t = 0;
            if (w.lane == 0) t = atomicAdd(a.claims + (a.epoch & 1u) * a.ngroups + c.g, 1);
            i = gp->spw * w.nw + __shfl_sync(0xffffffffu, t, 0);
        }
        ++c.k;
        if (i < gp->ntiles) {
            c.g_ntiles = gp->ntiles;
            c.i = i;
            if (i < c.t_base || i >= c.t_end) pc_load_gemv(a, c);
            return;
        }
        ++c.g;
        c.k = 0;
        c.t_base = c.t_end = 0;  // the next tile loads its GEMV
    }
}

// Issues tiles while the ring and the mbarrier slots have room, recording each slot's tile
// for the consumer.  The cursor holds the next tile, claimed as the previous one is issued.
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
            w.tiles[slot] = make_int2(r.pc.g, r.pc.i);
            const int r0 = (r.pc.i - r.pc.t_base) * r.pc.trows;
            const int rows = min(r.pc.trows, r.pc.nrows - r0);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (r.pc.W2) {
                // gate/up pair: whole 16-byte rows (checked on the host), gate rows then up rows
                const uint32_t bytes = uint32_t(rows) * uint32_t(r.pc.row_bytes);
                uint8_t *dst = w.ring + pos;
                mbar_arrive_expect_tx(&w.bars[slot], 2u * bytes);
                bulk_copy_g2s(dst, r.pc.W + size_t(r0) * size_t(r.pc.row_bytes), bytes, &w.bars[slot]);
                bulk_copy_g2s(dst + size_t(r.pc.trows) * r.pc.row_bytes,
                              r.pc.W2 + size_t(r0) * size_t(r.pc.row_bytes), bytes, &w.bars[slot]);
            } else {
                const uint8_t *src = r.pc.W + size_t(r0) * size_t(r.pc.row_bytes);
                const uintptr_t s = reinterpret_cast<uintptr_t>(src);
                const uintptr_t e = s + size_t(rows) * r.pc.row_bytes;
                const uintptr_t s_al = (s + 15) & ~uintptr_t(15), e_al = e & ~uintptr_t(15);
                uint8_t *dst = w.ring + pos + uint32_t(s & 15);
                if (e_al > s_al) {
                    mbar_arrive_expect_tx(&w.bars[slot], uint32_t(e_al - s_al));
                    bulk_copy_g2s(dst + (s_al - s), reinterpret_cast<const void *>(s_al),
                                  uint32_t(e_al - s_al), &w.bars[slot]);
                } else {
                    mbar_arrive(&w.bars[slot]);
                }
            }
        }
        r.p_total += need;
        r.p_pos = pos + alloc;
        ++r.issued;
        pc_next(a, r.pc, w);
    }
    __syncwarp();  // the slots' tile records are visible to every lane
}

// The tile at the head of this warp's ring ({ngroups, 0}: the chain has no tile left for
// it), issuing copies first if the ring is empty.  The ring state stays in shared memory.
__device__ __noinline__ int2 pc_head(const PcArgs &a, PcRing *rs, const PcWarp &w) {
    PcRing r = *rs;
    __syncwarp();
    if (r.issued == r.consumed) {
        pc_produce(a, r, w);
        if (w.lane == 0) *rs = r;
        __syncwarp();
    }
    return r.issued == r.consumed ? make_int2(a.ngroups, 0) : w.tiles[r.consumed % kPcSlots];
}

// Trace stamps of warp 0 (thread 0) per CTA and group: 0 its staging share starts, 1 it ends,
// 2 the CTA's barrier is passed (input staged), 3 its tiles are done.
__device__ __forceinline__ void pc_trace(const PcArgs &a, int g, int k) {
    if (a.trace && threadIdx.x == 0) a.trace[(size_t(blockIdx.x) * a.ngroups + g) * 4 + k] = global_timer_ns();
}

// This warp's tiles at the head of its ring while they belong to GEMV cc.m of group cc.g:
// wait for each tile's copy (bounded), fix up unaligned row ends, dot and store, refill the
// ring.  One call per run of tiles of one GEMV (the tile arithmetic is compiled into the
// loop).  The warp's ring state lives in shared memory between calls (rs): held in
// registers here, written back at the end, so the kernel body keeps no ring state across
// its other work.
template <int QT, int NCOLS, int RPB, int LBT, bool GLU>
__device__ __noinline__ void pc_run(const PcArgs &a, PcRing *rs, PcWarp w, PcCursor cc, PcOut o,
                                    uint32_t act_off, float sc0, float sc1, int *s_failed) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = w.lane;
    const int bl = lane & (LBT - 1);
    o.y = o.ys[bl < o.world ? bl : 0];
    PcRing r = *rs;
    __syncwarp();
    const int K = a.groups[cc.g].K;
    for (;;) {
        if (r.issued == r.consumed) pc_produce(a, r, w);
        if (r.issued == r.consumed) break;
        const int slot = int(r.consumed % kPcSlots);
        const int2 head = w.tiles[slot];
        if (head.x != cc.g || head.y < cc.t_base || head.y >= cc.t_end) break;
        cc.i = head.y;
        const uint32_t alloc = uint32_t(cc.alloc);
        const bool wrap = r.c_pos + alloc > w.R;
        const uint32_t pos = wrap ? 0u : r.c_pos;
        const int r0 = (cc.i - cc.t_base) * cc.trows;
        const int rows = min(cc.trows, cc.nrows - r0);
        const uint32_t parity = (r.consumed / kPcSlots) & 1u;
        const uint8_t *src = cc.W + size_t(r0) * size_t(cc.row_bytes);
        const uintptr_t s = GLU ? 0 : reinterpret_cast<uintptr_t>(src);
        const uintptr_t e = GLU ? 0 : s + size_t(rows) * cc.row_bytes;
        uint8_t *wrow0 = w.ring + pos + uint32_t(s & 15);
        bool have_w = mbar_try_wait(&w.bars[slot], parity);
        if (!have_w) {
            const uint64_t lim = *reinterpret_cast<volatile int *>(s_failed)
                                     ? (a.wait_ns < 1000000ull ? a.wait_ns : 1000000ull)
                                     : a.wait_ns;
            have_w = mbar_wait_bounded(&w.bars[slot], parity, lim);
            if (!have_w) {
                *s_failed = 1;
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
            pc_tile<QT, NCOLS, RPB, LBT, GLU>(o, uint32_t(wrow0 - smem), r0, rows, act_off, K, a.epoch,
                                              sc0, sc1);
        __syncwarp();  // every lane is done with the tile's ring bytes
        r.c_total += (wrap ? w.R - r.c_pos : 0u) + alloc;
        r.c_pos = pos + alloc;
        ++r.consumed;
        pc_produce(a, r, w);
    }
    if (lane == 0) *rs = r;
    __syncwarp();
}

#define ANVIL_PC_RUN_ARGS a, rs, w, cc, o, act_off, sc0, sc1, s_failed

template <int QT, int NCOLS>
__device__ __forceinline__ void pc_run_variant(const PcArgs &a, PcRing *rs, const PcWarp &w,
                                               const PcCursor &cc, const PcOut &o, uint32_t act_off,
                                               float sc0, float sc1, int *s_failed) {
    switch (cc.variant) {
    case kV1x32: pc_run<QT, NCOLS, 1, 32, false>(ANVIL_PC_RUN_ARGS); break;
    case kV2x32: pc_run<QT, NCOLS, 2, 32, false>(ANVIL_PC_RUN_ARGS); break;
    case kV4x32: pc_run<QT, NCOLS, 4, 32, false>(ANVIL_PC_RUN_ARGS); break;
    case kV8x32: pc_run<QT, NCOLS, 8, 32, false>(ANVIL_PC_RUN_ARGS); break;
    case kV2x16: pc_run<QT, NCOLS, 2, 16, false>(ANVIL_PC_RUN_ARGS); break;
    case kV4x16: pc_run<QT, NCOLS, 4, 16, false>(ANVIL_PC_RUN_ARGS); break;
    case kV8x16: pc_run<QT, NCOLS, 8, 16, false>(ANVIL_PC_RUN_ARGS); break;
    case kV4x8: pc_run<QT, NCOLS, 4, 8, false>(ANVIL_PC_RUN_ARGS); break;
    case kV8x8: pc_run<QT, NCOLS, 8, 8, false>(ANVIL_PC_RUN_ARGS); break;
    case kG1x32: pc_run<QT, NCOLS, 2, 32, true>(ANVIL_PC_RUN_ARGS); break;
    case kG2x32: pc_run<QT, NCOLS, 4, 32, true>(ANVIL_PC_RUN_ARGS); break;
    case kG2x16: pc_run<QT, NCOLS, 4, 16, true>(ANVIL_PC_RUN_ARGS); break;
    case kG4x32: pc_run<QT, NCOLS, 8, 32, true>(ANVIL_PC_RUN_ARGS); break;
    case kG4x16: pc_run<QT, NCOLS, 8, 16, true>(ANVIL_PC_RUN_ARGS); break;
    case kG4x8: pc_run<QT, NCOLS, 8, 8, true>(ANVIL_PC_RUN_ARGS); break;
    default: break;
    }
}

template <int NCOLS>
__device__ __forceinline__ void pc_run_any(const PcArgs &a, PcRing *rs, const PcWarp &w,
                                           const PcCursor &cc, const PcOut &o, uint32_t act_off,
                                           float sc0, float sc1, int *s_failed) {
    switch (cc.type) {
    case kTypeQ4_K: pc_run_variant<kTypeQ4_K, NCOLS>(ANVIL_PC_RUN_ARGS); break;
    case kTypeQ5_K: pc_run_variant<kTypeQ5_K, NCOLS>(ANVIL_PC_RUN_ARGS); break;
    case kTypeQ6_K: pc_run_variant<kTypeQ6_K, NCOLS>(ANVIL_PC_RUN_ARGS); break;
    case kTypeQ8_0: pc_run_variant<kTypeQ8_0, NCOLS>(ANVIL_PC_RUN_ARGS); break;
    default: break;
    }
}

#undef ANVIL_PC_RUN_ARGS

// This warp's share of group g's staging into activation buffer g & 1.
template <int NCOLS>
__device__ __forceinline__ void pc_stage_share(const PcArgs &a, int g, float (*s_max)[kMaxWarps][2]) {
    const int warp = threadIdx.x >> 5;
    const PcGroup *grp = a.groups + g;
    const uint32_t off = uint32_t(a.act_off[g & 1]);
    const int K = grp->K;
    if (grp->src) {
        const uint64_t *src = grp->src + size_t(a.epoch & 1u) * NCOLS * K;
        if (grp->family == 0)  // K-quant swizzle
            warp_stage_ll<kTypeQ4_K, NCOLS>(src, K, a.epoch, a.wait_ns, off, s_max[g & 1][warp]);
        else                   // Q8_0 swizzle
            warp_stage_ll<kTypeQ8_0, NCOLS>(src, K, a.epoch, a.wait_ns, off, s_max[g & 1][warp]);
    } else {
        if (grp->family == 0)
            warp_stage_f32<kTypeQ4_K, NCOLS>(grp->x, K, off);
        else
            warp_stage_f32<kTypeQ8_0, NCOLS>(grp->x, K, off);
    }
}

template <int NCOLS>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) pchain_kernel(const __grid_constant__ PcArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float s_max[2][kMaxWarps][2];  // per activation buffer, warp, column: input max
    __shared__ PcRing s_ring[kMaxWarps];      // each warp's ring state between tile runs
    __shared__ int2 s_tiles[kMaxWarps][kPcSlots];
    __shared__ int s_failed;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nwarps = blockDim.x >> 5;
    if (tid == 0) s_failed = pc_failed() ? 1 : 0;
    // The next launch's tile counters: nothing of this launch touches them, and the next
    // launch starts after this one has ended.
    if (blockIdx.x == 0)
        for (int g = tid; g < a.ngroups; g += blockDim.x) a.claims[((a.epoch + 1u) & 1u) * a.ngroups + g] = 0;

    PcWarp w;
    w.ring = smem + a.ring_off + size_t(warp) * a.ring_bytes;
    w.bars = reinterpret_cast<uint64_t *>(smem) + warp * kPcSlots;
    w.tiles = s_tiles[warp];
    w.nw = gridDim.x * nwarps;
    w.gw = blockIdx.x * nwarps + warp;
    w.lane = lane;
    w.R = uint32_t(a.ring_bytes);

    {
        PcRing r{};
        r.pc.g = 0;
        pc_next(a, r.pc, w);
        if (lane == 0) {
            for (int s = 0; s < kPcSlots; ++s) mbar_init(&w.bars[s], 1);
            mbar_fence_init();
        }
        __syncwarp();
        pc_produce(a, r, w);  // the first weight tiles stream while the first input is staged
        if (lane == 0) s_ring[warp] = r;
        __syncwarp();
    }

    if (a.ngroups > 0) {
        pc_trace(a, 0, 0);
        pc_stage_share<NCOLS>(a, 0, s_max);
        pc_trace(a, 0, 1);
    }
    for (int g = 0; g < a.ngroups; ++g) {
        const PcGroup cur = a.groups[g];
        const int K = cur.K;
        // ---- 1. the group's input is staged (every warp did its share) ----------------------
        // Also: every warp is done with group g - 1's tiles, so buffer (g + 1) & 1 is free.
        __syncthreads();
        pc_trace(a, g, 2);
        const uint32_t act_off = uint32_t(a.act_off[g & 1]);
        float sc[2] = {1.f, 1.f};
        if (cur.src) {
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) {
                float m = 0.f;
                for (int k = 0; k < nwarps; ++k) m = fmaxf(m, s_max[g & 1][k][c]);
                sc[c] = pow2_scale(m);
            }
        }
        if (cur.dump && blockIdx.x == 0) {
            const ActBuf b = act_buf(smem + act_off, K, NCOLS);
            if (cur.family == 0)
                dump_staged<kTypeQ4_K>(cur.dump, K, NCOLS, b);
            else
                dump_staged<kTypeQ8_0>(cur.dump, K, NCOLS, b);
        }

        // ---- 2. this warp's tiles of the group, one run per GEMV ----------------------------
        PcCursor cc{};
        cc.g = g;
        cc.g_ntiles = cur.ntiles;
        for (;;) {
            const int2 head = pc_head(a, &s_ring[warp], w);
            if (head.x != g) break;
            cc.i = head.y;
            pc_load_gemv(a, cc);
            const PcGemv *gm = a.gemvs + cc.m;
            PcOut o;
            o.ys = gm->y;
            o.y = nullptr;
            o.nfull = gm->nrows_full;
            o.row0 = gm->row0;
            o.perm = gm->perm;
            o.world = a.world;
            pc_run_any<NCOLS>(a, &s_ring[warp], w, cc, o, act_off, sc[0], sc[1], &s_failed);
        }
        pc_trace(a, g, 3);
        // ---- 3. this warp's share of the next group's input, into the other buffer ----------
        if (g + 1 < a.ngroups) {
            pc_trace(a, g + 1, 0);
            pc_stage_share<NCOLS>(a, g + 1, s_max);
            pc_trace(a, g + 1, 1);
        }
    }
}

// Current-epoch values of one output, in row order; NaN where a word does not carry `epoch`.
__global__ void pchain_read_kernel(const uint64_t *__restrict__ y, float *__restrict__ dst, int ncols,
                                   int n, int perm, uint32_t epoch) {
    const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= long(ncols) * n) return;
    const int c = int(i / n), r = int(i - long(c) * n);
    const int pos = perm ? ll_pos(r, n) : r;
    const uint64_t w = y[(size_t(epoch & 1u) * ncols + c) * n + pos];
    dst[i] = uint32_t(w >> 32) == epoch ? __uint_as_float(uint32_t(w)) : __uint_as_float(0x7fc00000u);
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

// Lanes-per-row utilisation of a (rows per stage, lanes per row) shape on rows of nblk blocks
// (the measure host_lanes_per_row maximises).
static float pc_util(int nblk, int rpb, int lb) {
    const int rg = 32 / lb;
    const int per_lane = (nblk + lb - 1) / lb;
    const float r = float(rpb) / float(rg);
    return float(nblk) / float(lb * per_lane) * (r < 1.f ? r : 1.f);
}

static int pc_variant(int rpb, int lb, bool glu) {
    for (int v = 0; v < kNumVariants; ++v)
        if (kVarRpb[v] == rpb && kVarLb[v] == lb && kVarGlu[v] == glu) return v;
    return -1;
}

}  // namespace anvil

using namespace anvil;

struct PcGemvHost {
    PcGemv d;
    int rpb_req, K, qk;
    bool own_y;
};

struct anvil_pchain {
    int world = 1, rank = 0, ncols = 0;
    std::vector<PcGroup> groups;
    std::vector<int> group_src;  // source GEMV of a chained group, -1 for a fixed input
    std::vector<PcGemvHost> gemvs;
    std::vector<void *> owned;   // device buffers this chain allocated
    PcGroup *d_groups = nullptr;
    PcGemv *d_gemvs = nullptr;
    uint64_t *trace = nullptr;
    int *claims = nullptr;       // tile counters, [2][groups]
    int static_pct = kPcStaticPct;
    PcKernel fn = nullptr;
    int grid = 0, nwarps = 0, smem = 0, ring_bytes = 0, ring_off = 0;
    int act_off[2] = {0, 0};
    uint32_t epoch = 0;
    bool ready = false;
};

namespace {

int pc_push_group(anvil_pchain *c, const float *x, int src, int K) {
    PcGroup g{};
    g.x = x;
    g.src = nullptr;  // resolved at instantiation (the source's buffer may be allocated then)
    g.K = K;
    g.first = int(c->gemvs.size());
    g.count = 0;
    g.family = -1;
    c->groups.push_back(g);
    c->group_src.push_back(src);
    return int(c->groups.size()) - 1;
}

int pc_add(anvil_pchain *c, int ggml_type, const void *W, const void *W2, int nrows, int row0,
           int nrows_full, uint64_t *const *y, int rows_per_block) {
    if (!c || !W) return fail(ANVIL_ERR_INVALID, "null argument");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (c->groups.empty()) return fail(ANVIL_ERR_INVALID, "add a group first");
    if (int(c->gemvs.size()) >= (1 << 20)) return fail(ANVIL_ERR_INVALID, "too many GEMVs");
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
    if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(W2)) & 15)
        return fail(ANVIL_ERR_ALIGN, "weights must be 16-byte aligned");
    const int row_bytes = (g.K / qk) * bb;
    if (W2 && row_bytes % 16)
        return fail(ANVIL_ERR_ALIGN, "gate/up rows must be a multiple of 16 bytes (%d)", row_bytes);
    if (y) {
        for (int q = 0; q < c->world; ++q) {
            if (!y[q]) return fail(ANVIL_ERR_INVALID, "null output pointer for rank %d", q);
            if (reinterpret_cast<uintptr_t>(y[q]) & 15)
                return fail(ANVIL_ERR_ALIGN, "output words must be 16-byte aligned");
        }
    } else if (c->world > 1) {
        return fail(ANVIL_ERR_INVALID, "world > 1 needs every rank's output buffer");
    }
    const int family = ggml_type == ANVIL_TYPE_Q8_0 ? 1 : 0;
    if (g.family >= 0 && g.family != family) {
        // Q8_0 and the K-quants read the staged activation in different swizzles: continue
        // in a new group on the same input, restaged.
        const PcGroup prev = g;
        pc_push_group(c, prev.x, c->group_src.back(), prev.K);
    }
    PcGroup &cur = c->groups.back();
    cur.family = family;
    cur.count += 1;
    PcGemvHost h{};
    h.d.W = static_cast<const uint8_t *>(W);
    h.d.W2 = static_cast<const uint8_t *>(W2);
    if (y)
        for (int q = 0; q < c->world; ++q) h.d.y[q] = y[q];
    h.own_y = y == nullptr;
    h.d.type = ggml_type;
    h.d.nrows = nrows;
    h.d.row0 = row0;
    h.d.nrows_full = nrows_full;
    h.d.row_bytes = row_bytes;
    h.rpb_req = rows_per_block;
    h.K = cur.K;
    h.qk = qk;
    c->gemvs.push_back(h);
    return int(c->gemvs.size()) - 1;
}

}  // namespace

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
    for (void *p : c->owned) cudaFree(p);
    delete c;
}

int anvil_pchain_add_group(anvil_pchain *c, const float *x, int K, int ncols) {
    if (!c || !x) return fail(ANVIL_ERR_INVALID, "null argument");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (K <= 0 || K % 32 != 0) return fail(ANVIL_ERR_INVALID, "K=%d is not a positive multiple of 32", K);
    if (ncols != 1 && ncols != 2)
        return fail(ANVIL_ERR_UNSUPPORTED, "persistent chain supports ncols 1 and 2 (got %d)", ncols);
    if (c->ncols && ncols != c->ncols)
        return fail(ANVIL_ERR_INVALID, "all groups of a chain have the same ncols");
    if (reinterpret_cast<uintptr_t>(x) & 15) return fail(ANVIL_ERR_ALIGN, "x must be 16-byte aligned");
    c->ncols = ncols;
    return pc_push_group(c, x, -1, K);
}

int anvil_pchain_add_group_chained(anvil_pchain *c, int src_gemv) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null argument");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (src_gemv < 0 || src_gemv >= int(c->gemvs.size()))
        return fail(ANVIL_ERR_INVALID, "source GEMV %d is not an earlier GEMV of the chain", src_gemv);
    const int K = c->gemvs[src_gemv].d.nrows_full;
    if (K % 32 != 0)
        return fail(ANVIL_ERR_INVALID, "a chained input needs a multiple of 32 values (source has %d)", K);
    c->gemvs[src_gemv].d.perm = 1;
    return pc_push_group(c, nullptr, src_gemv, K);
}

int anvil_pchain_add_gemv(anvil_pchain *c, int ggml_type, const void *W, int nrows, int row0,
                          int nrows_full, uint64_t *const *y, int rows_per_block) {
    return pc_add(c, ggml_type, W, nullptr, nrows, row0, nrows_full, y, rows_per_block);
}

int anvil_pchain_add_glu(anvil_pchain *c, int ggml_type, const void *W_gate, const void *W_up,
                         int nrows, int row0, int nrows_full, uint64_t *const *y,
                         int rows_per_block) {
    if (!W_up) return fail(ANVIL_ERR_INVALID, "null argument");
    return pc_add(c, ggml_type, W_gate, W_up, nrows, row0, nrows_full, y, rows_per_block);
}

int anvil_pchain_set_group_dump(anvil_pchain *c, int group, void *out) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (group < 0 || group >= int(c->groups.size())) return fail(ANVIL_ERR_INVALID, "bad group %d", group);
    if (reinterpret_cast<uintptr_t>(out) & 3) return fail(ANVIL_ERR_ALIGN, "dump buffer must be 4-byte aligned");
    c->groups[group].dump = static_cast<uint8_t *>(out);
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
    for (size_t gi = 0; gi < c->groups.size(); ++gi) {
        const int src = c->group_src[gi];
        if (src >= 0 && src >= c->groups[gi].first)
            return fail(ANVIL_ERR_INVALID, "group %zu reads GEMV %d, which is not before it", gi, src);
    }
    int dev, nsm;
    if (int s = current_device(&dev)) return s;
    if (int s = sm_count(dev, &nsm)) return s;
    c->fn = pc_kernel_for(c->ncols);

    // Shared memory: [mbarriers][activation buffer of even groups][of odd groups][nwarps rings].
    // Group g is staged into buffer g & 1 while group g - 1's tiles may still read the other.
    int act[2] = {0, 0};
    for (size_t gi = 0; gi < c->groups.size(); ++gi) {
        const int nkb = c->groups[gi].K / 32;
        const int b = c->ncols * act_col_bytes(nkb) + 2 * c->ncols * nkb * 4 + 16 + c->ncols * nkb * 8;
        act[gi & 1] = std::max(act[gi & 1], (b + 15) & ~15);
    }
    const int bars = (nwarps * kPcSlots * 8 + 15) & ~15;
    // Per CTA: the SM's 228 KB shared by ctas_per_sm CTAs less the runtime's 1 KB reserve each,
    // at most 227 KB per CTA, and the kernel's static shared memory comes out of both.
    cudaFuncAttributes fattr{};
    cudaError_t fe = cudaFuncGetAttributes(&fattr, reinterpret_cast<const void *>(c->fn));
    if (fe != cudaSuccess) return cuda_fail(fe, "cudaFuncGetAttributes");
    const int budget = std::min((228 * 1024) / ctas_per_sm - 1024, kMaxSmem) - int(fattr.sharedSizeBytes);
    const int ring = ((budget - bars - act[0] - act[1]) / nwarps) & ~15;
    if (ring < 4096) return fail(ANVIL_ERR_UNSUPPORTED, "no room for weight rings (%d B per warp)", ring);

    // Tile shape per GEMV: requested rows per tile (else the built-in default), the lanes per
    // row that keep the most lanes busy, and at most half a ring per tile.  A gate/up pair
    // stages h rows of each matrix (rows per stage 2h, h = 1, 2 or 4).
    for (PcGemvHost &h : c->gemvs) {
        const int K = h.K;
        const int nblk = K / h.qk;
        const bool glu = h.d.W2 != nullptr;
        int rpb = h.rpb_req > 0 ? h.rpb_req : (h.d.nrows < 2048 ? 1 : (K >= 8192 ? 2 : 4));
        rpb = rpb >= 8 ? 8 : rpb >= 4 ? 4 : rpb >= 2 ? 2 : 1;
        if (glu) rpb = std::max(2, std::min(8, 2 * rpb));
        auto alloc_of = [&](int r) { return ((r * h.d.row_bytes + 32) + 15) & ~15; };
        while (rpb > (glu ? 2 : 1) && alloc_of(rpb) > ring / 2) rpb >>= 1;
        if (alloc_of(rpb) > ring)
            return fail(ANVIL_ERR_UNSUPPORTED, "a %d-byte row does not fit a %d-byte ring",
                        h.d.row_bytes, ring);
        int best = -1;
        float bu = -1.f;
        for (int lb : {32, 16, 8}) {
            const int v = pc_variant(rpb, lb, glu);
            if (v < 0) continue;
            const float u = pc_util(nblk, rpb, lb);
            if (u > bu + 1e-6f) {
                bu = u;
                best = v;
            }
        }
        if (best < 0) best = pc_variant(rpb, 32, glu);
        h.d.variant = best;
        h.d.rpb = rpb;
        h.d.trows = glu ? rpb / 2 : rpb;
        h.d.alloc = alloc_of(rpb);
    }

    // Output buffers the chain owns (world 1, no buffer given): two parities, zeroed.
    for (PcGemvHost &h : c->gemvs) {
        if (!h.own_y || h.d.y[0]) continue;
        const size_t bytes = size_t(2) * c->ncols * h.d.nrows_full * sizeof(uint64_t);
        void *p = nullptr;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(outputs)");
        c->owned.push_back(p);
        e = cudaMemset(p, 0, bytes);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(outputs)");
        h.d.y[0] = static_cast<uint64_t *>(p);
    }

    // Tiles per group, chained sources.
    std::vector<PcGemv> dg;
    dg.reserve(c->gemvs.size());
    for (const PcGemvHost &h : c->gemvs) dg.push_back(h.d);
    for (size_t gi = 0; gi < c->groups.size(); ++gi) {
        PcGroup &g = c->groups[gi];
        int t = 0;
        for (int m = g.first; m < g.first + g.count; ++m) {
            dg[m].tile_base = t;
            dg[m].ntiles = (dg[m].nrows + dg[m].trows - 1) / dg[m].trows;
            t += dg[m].ntiles;
        }
        g.ntiles = t;
        const int src = c->group_src[gi];
        g.src = src >= 0 ? dg[src].y[c->rank] : nullptr;
    }

    int occ = 0;
    const int threads = nwarps * 32;
    const int smem = bars + act[0] + act[1] + nwarps * ring;
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
    c->act_off[0] = bars;
    c->act_off[1] = bars + act[0];
    c->ring_off = bars + act[0] + act[1];
    const int nw = c->grid * nwarps;
    long cum = 0;
    for (PcGroup &g : c->groups) {
        g.rot = int(cum % nw);
        cum += g.ntiles;
        g.spw = int((long(g.ntiles) * c->static_pct / 100) / nw);
    }
    e = cudaMalloc(&c->claims, sizeof(int) * 2 * c->groups.size());
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(claims)");
    c->owned.push_back(c->claims);
    e = cudaMemset(c->claims, 0, sizeof(int) * 2 * c->groups.size());
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(claims)");

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
    c->ready = true;
    return ANVIL_OK;
}

int anvil_pchain_set_static_share(anvil_pchain *c, int percent) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->ready) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (percent < 0 || percent > 100) return fail(ANVIL_ERR_INVALID, "static share %d%% outside 0..100", percent);
    c->static_pct = percent;
    return ANVIL_OK;
}

int anvil_pchain_set_trace(anvil_pchain *c, uint64_t *buf) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (reinterpret_cast<uintptr_t>(buf) & 7) return fail(ANVIL_ERR_ALIGN, "trace buffer must be 8-byte aligned");
    c->trace = buf;
    return ANVIL_OK;
}

int anvil_pchain_launch(anvil_pchain *c, anvil_stream_t stream) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (!c->ready) return fail(ANVIL_ERR_INVALID, "chain not instantiated");
    PcArgs a{};
    a.groups = c->d_groups;
    a.gemvs = c->d_gemvs;
    a.trace = c->trace;
    a.claims = c->claims;
    a.wait_ns = wait_limit_ns();
    a.ngroups = int(c->groups.size());
    a.world = c->world;
    a.rank = c->rank;
    a.act_off[0] = c->act_off[0];
    a.act_off[1] = c->act_off[1];
    a.ring_off = c->ring_off;
    a.ring_bytes = c->ring_bytes;
    a.epoch = c->epoch + 1;
    if (a.epoch == 0) a.epoch = 2;  // 0 is the flag of zeroed buffers; the parity alternates
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
    c->epoch = a.epoch;
    return ANVIL_OK;
}

int anvil_pchain_epoch(const anvil_pchain *c) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    return int(c->epoch & 0x7fffffffu);
}

int anvil_pchain_read_output(const anvil_pchain *c, int index, float *dst, anvil_stream_t stream) {
    if (!c || !dst) return fail(ANVIL_ERR_INVALID, "null argument");
    if (!c->ready) return fail(ANVIL_ERR_INVALID, "chain not instantiated");
    if (index < 0 || index >= int(c->gemvs.size())) return fail(ANVIL_ERR_INVALID, "bad GEMV index");
    if (c->epoch == 0) return fail(ANVIL_ERR_INVALID, "chain not launched yet");
    const PcGemv &d = c->gemvs[index].d;
    const long n = long(c->ncols) * d.nrows_full;
    const unsigned blocks = unsigned((n + 255) / 256);
    pchain_read_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        d.y[c->rank], dst, c->ncols, d.nrows_full, d.perm, c->epoch);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "read_output launch");
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
