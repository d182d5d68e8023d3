// Tensor-core MMVQ for 2..8 activation columns (the batched speculative-decode GEMV):
// Q4_K and Q5_K weights against Q8_1 activations through mma.sync m16n8k32 s8 x s8 -> s32.
//
// One MMA is one Q8_1 block (32 weights) of 16 weight rows against up to 8 columns, so its
// int32 results are exactly the block sums sum(q * q8) the dp4a kernel forms one row at a
// time (kModeSums output identical).  The per-block scales follow in a float epilogue with
// the dp4a kernel's formula (vec_dot_q4_K_q8_1 structure):
//   y[r][c] = sum_b d_b * sum_j d8_j[c] * sc_j * isum_j[r][c] - dmin_b * sum_j m_j * ds_j[c]
// with ds_j[c] = d8_j[c] * sum(q8) of the block.
//
// Work split: a CTA owns a tile of 16 rows (tiles dealt round-robin over the grid, across
// the launch's segments) and its warps split the tile's K-chunks (chunk c goes to warp
// c % nwarps); each warp streams its chunks, tile after tile, through its own ring of stages
// in shared memory, one bulk copy per row segment (16-byte aligned: Q4_K and Q5_K blocks are
// 144 and 176 bytes).  Row segments are padded by 16 bytes so the 8 rows a fragment load
// touches fall in distinct banks.  The warps' partial sums meet in shared memory and warp 0
// adds them in warp order (deterministic).  The activation is staged once per CTA as
// [block][column][8 words] with each lane's two B-fragment words adjacent (one 8-byte load),
// d8 and d8 * sum(q8) as [block][columns rounded up to even] (one 8-byte load per lane).
// Every mbarrier wait is bounded (status flag on expiry, the tile's outputs are not written).
#include <type_traits>

#include "mmvq.cuh"

namespace anvil {

constexpr int kMmaRows = 16;   // weight rows per CTA tile (the MMA's M)
// Warps per CTA.  16 (4 per scheduler) measured slower than 8 on Q4_K 12288 x 4096 at 8
// columns (17.6 against 15.2 us): a quarter of the K-chunk per warp adds per-chunk and
// per-tile work (35% more instructions) that the extra latency hiding does not repay.
constexpr int kMmaMaxWarps = 8;
constexpr int kChunkSbMax = 4; // at most 4 super-blocks (1024 weights) per staged K-chunk

// Super-blocks per K-chunk: enough chunks for every warp when K allows, at most kChunkSbMax.
__host__ __device__ inline int mma_chunk_sb(int K, int nwarps) {
    const int nsb = K / 256;
    int c = nsb / nwarps;
    c = c < 1 ? 1 : c > kChunkSbMax ? kChunkSbMax : c;
    return c;
}

struct MmaSmem {
    int bar, q, d8, ds, red, ring, seg, stage, total, ncp;
};

// [mbarriers][quants: nkb x ncols x 32 B][d8: nkb x ncp][d8 * sum q: nkb x ncp]
// [partials: 2 x nwarps x 32 lanes x 4][nwarps x nstages stages]; ncp = ncols rounded up to even
__host__ __device__ inline MmaSmem mma_smem_layout(int qt, int K, int ncols, int nwarps, int nstages) {
    const int nkb = K / 32;
    MmaSmem L;
    L.ncp = (ncols + 1) & ~1;
    L.bar = 0;
    L.q = (8 * nwarps * nstages + 15) & ~15;
    L.d8 = L.q + nkb * ncols * 32;
    L.ds = L.d8 + nkb * L.ncp * 4;
    L.red = (L.ds + nkb * L.ncp * 4 + 15) & ~15;
    L.ring = L.red + 2 * nwarps * 32 * 16;
    L.seg = mma_chunk_sb(K, nwarps) * mmvq_type_bytes(qt) + 16;
    L.stage = kMmaRows * L.seg;
    L.total = L.ring + nwarps * nstages * L.stage;
    return L;
}

__device__ __forceinline__ void mma_s8_16x8x32(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1, int (&d)[4]) {
    // not volatile: the instruction has no side effects, so the compiler may schedule it early
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Weights of sub-blocks 2U (lo) and 2U+1 (hi) of one super-block row at k = 4t..4t+3 (half
// 0) or 16+4t..16+4t+3 (half 1): four unsigned values per word.
template <int QT, int U>
__device__ __forceinline__ void mma_weights(const uint8_t *blk, int t, int half, uint32_t &lo,
                                            uint32_t &hi) {
    const int e = 16 * half + 4 * t;
    if constexpr (QT == kTypeQ4_K) {
        const uint32_t v = *reinterpret_cast<const uint32_t *>(blk + 16 + 32 * U + e);
        lo = v & 0x0F0F0F0Fu;
        hi = (v >> 4) & 0x0F0F0F0Fu;
    } else {  // Q5_K: fifth bit of weight e of sub-block j is bit j of qh[e]
        const uint32_t v = *reinterpret_cast<const uint32_t *>(blk + 48 + 32 * U + e);
        const uint32_t qh = *reinterpret_cast<const uint32_t *>(blk + 16 + e);
        lo = (v & 0x0F0F0F0Fu) | (((qh >> (2 * U)) & 0x01010101u) << 4);
        hi = ((v >> 4) & 0x0F0F0F0Fu) | (((qh >> (2 * U + 1)) & 0x01010101u) << 4);
    }
}

template <int QT, int NC, int MODE>
__global__ void __launch_bounds__(kMmaMaxWarps * 32, 1) mmvq_mma_kernel(const __grid_constant__ MmvqArgs args) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int TB = QTraits<QT>::bytes;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nwarps = blockDim.x >> 5;
    const int K = args.K, nst = args.nstages;
    const int nkb = K >> 5, nsb = K >> 8;
    const int row_bytes = nsb * TB;
    const MmaSmem L = mma_smem_layout(QT, K, NC, nwarps, nst);
    constexpr int NCP = (NC + 1) & ~1;
    const int csb = mma_chunk_sb(K, nwarps);
    const int nchunks = (nsb + csb - 1) / csb;
    const int cw = warp < nchunks ? (nchunks - 1 - warp) / nwarps + 1 : 0;  // chunks per tile
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar) + warp * nst;
    const uint32_t *sq = reinterpret_cast<const uint32_t *>(smem + L.q);
    float *sd8 = reinterpret_cast<float *>(smem + L.d8);
    float *sds = reinterpret_cast<float *>(smem + L.ds);
    float4 *red = reinterpret_cast<float4 *>(smem + L.red);
    uint8_t *ring = smem + L.ring + warp * nst * L.stage;

    const int ntiles = args.segTile[args.nseg];
    const int my_tiles = int(blockIdx.x) < ntiles ? (ntiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
    const int my_stages = my_tiles * cw;

    // Stage s of this warp: tile blockIdx.x + (s / cw) * gridDim.x, K-chunk warp + (s % cw) *
    // nwarps.  Lane r (< 16) copies row r's segment; lane 0 first expects the chunk's bytes.
    auto issue = [&](int s, int st) {
        const int tile = int(blockIdx.x) + (s / cw) * int(gridDim.x);
        const int c = warp + (s % cw) * nwarps;
        const int sg = mmvq_segment(args, tile);
        const int r0 = (tile - args.segTile[sg]) * kMmaRows;
        const int rows = min(kMmaRows, args.segRows[sg] - r0);
        const int nb = min(csb, nsb - c * csb);
        const uint32_t bytes = uint32_t(nb * TB);
        if (lane == 0) mbar_arrive_expect_tx(&full[st], bytes * uint32_t(rows));
        __syncwarp();
        if (lane < rows) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const uint8_t *src = args.segW[sg] + size_t(r0 + lane) * size_t(row_bytes) + size_t(c) * csb * TB;
            bulk_copy_g2s(ring + st * L.stage + lane * L.seg, src, bytes, &full[st]);
        }
    };

    // ---- 1. start streaming weights, then stage the activation ------------------------
    if (lane == 0) {
        for (int st = 0; st < nst; ++st) mbar_init(&full[st], 1);
        mbar_fence_init();
    }
    __syncwarp();
    for (int s = 0; s < my_stages && s < nst; ++s) issue(s, s);
    pdl_launch_dependents();
    pdl_wait();
    {
        // Q8_1 block (c, kb): 9 words {d, s}, quants; quant word w = t + 4h goes to slot 2t + h
        const uint32_t *xw = reinterpret_cast<const uint32_t *>(args.x);
        uint32_t *q = reinterpret_cast<uint32_t *>(smem + L.q);
        for (int i = tid; i < nkb * NCP; i += blockDim.x) {
            const int kb = i / NCP, c = i - kb * NCP;
            float d8 = 0.f, ds = 0.f;
            if (c < NC) {
                const uint32_t *src = xw + (size_t(c) * nkb + kb) * 9;
                uint32_t v[9];
#pragma unroll
                for (int w = 0; w < 9; ++w) v[w] = __ldg(src + w);
                uint32_t *dst = q + (kb * NC + c) * 8;
                int sum = 0;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    dst[2 * (w & 3) + (w >> 2)] = v[1 + w];
                    sum = __dp4a(int(v[1 + w]), 0x01010101, sum);
                }
                d8 = h2f(v[0]);
                ds = d8 * float(sum);
            }
            sd8[kb * NCP + c] = d8;  // columns NC..NCP-1 read as zero
            sds[kb * NCP + c] = ds;
        }
    }
    __syncthreads();

    // ---- 2. tiles: this warp's chunks, then the CTA's reduction ---------------------------
    const int g = lane >> 2, t = lane & 3;  // fragment row group and thread in group
    const bool tlive = 2 * t < NCP;         // lanes whose columns 2t, 2t+1 exist
    int st = 0;
    uint32_t phase = 0;
    bool ok = true;  // every copy of this warp landed (warp-uniform)
    for (int k = 0; k < my_tiles; ++k) {
        const int tile = int(blockIdx.x) + k * int(gridDim.x);
        const int sg = mmvq_segment(args, tile);
        const int nrows = args.segRows[sg];
        const int r0 = (tile - args.segTile[sg]) * kMmaRows;
        const int rows = min(kMmaRows, nrows - r0);
        float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [row g / g + 8][column 2t / 2t + 1]
        for (int i = 0; i < cw; ++i) {
            const int c = warp + i * nwarps;
            // a copy that did not land in time: one more bounded wait so no copy still
            // writes the stage, then the warp's results are dropped (the MMAs need every
            // lane, so the decision is the whole warp's)
            const bool got = mbar_wait_bounded(&full[st], phase, args.wait_ns);
            if (!got) (void)mbar_wait_bounded(&full[st], phase, args.wait_ns);
            if (!__all_sync(0xffffffffu, got)) ok = false;
            const int nb = min(csb, nsb - c * csb);
            const uint8_t *stage = ring + st * L.stage;
            for (int ib = 0; ok && ib < nb; ++ib) {
                const int b = c * csb + ib;
                const uint8_t *blk0 = stage + g * L.seg + ib * TB;        // row g
                const uint8_t *blk1 = stage + (g + 8) * L.seg + ib * TB;  // row g + 8
                const BlkHdr h0 = load_hdr<QT>(blk0), h1 = load_hdr<QT>(blk1);
                float fd[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, fm[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
                auto unit = [&](auto uc) {
                    constexpr int U = decltype(uc)::value;
                    uint32_t lo0, hi0, lo1, hi1, lo2, hi2, lo3, hi3;
                    mma_weights<QT, U>(blk0, t, 0, lo0, hi0);
                    mma_weights<QT, U>(blk1, t, 0, lo1, hi1);
                    mma_weights<QT, U>(blk0, t, 1, lo2, hi2);
                    mma_weights<QT, U>(blk1, t, 1, lo3, hi3);
                    int sc0[2], sc1[2], m0[2], m1[2];
                    scale_min_pair<U>(h0, sc0[0], sc1[0], m0[0], m1[0]);
                    scale_min_pair<U>(h1, sc0[1], sc1[1], m0[1], m1[1]);
#pragma unroll
                    // both MMAs of the unit first, then their epilogues: the second MMA
                    // runs while the first one's results are still on their way
                    int d[2][4];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {  // sub-block 2U + j
                        const int kb = 8 * b + 2 * U + j;
                        uint32_t b0 = 0, b1 = 0;
                        if (g < NC) {
                            const uint2 bw = *reinterpret_cast<const uint2 *>(sq + (kb * NC + g) * 8 + 2 * t);
                            b0 = bw.x;
                            b1 = bw.y;
                        }
                        if (j == 0) mma_s8_16x8x32(lo0, lo1, lo2, lo3, b0, b1, d[0]);
                        else mma_s8_16x8x32(hi0, hi1, hi2, hi3, b0, b1, d[1]);
                    }
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int kb = 8 * b + 2 * U + j;
                        float2 d8 = make_float2(0.f, 0.f), ds = make_float2(0.f, 0.f);
                        if (tlive) {
                            d8 = *reinterpret_cast<const float2 *>(sd8 + kb * NCP + 2 * t);
                            ds = *reinterpret_cast<const float2 *>(sds + kb * NCP + 2 * t);
                        }
                        const int s0 = j == 0 ? sc0[0] : sc1[0], s1 = j == 0 ? sc0[1] : sc1[1];
                        const float q0 = float(j == 0 ? m0[0] : m1[0]), q1 = float(j == 0 ? m0[1] : m1[1]);
                        fd[0][0] += d8.x * float(d[j][0] * s0);
                        fd[0][1] += d8.y * float(d[j][1] * s0);
                        fd[1][0] += d8.x * float(d[j][2] * s1);
                        fd[1][1] += d8.y * float(d[j][3] * s1);
                        fm[0][0] += ds.x * q0;
                        fm[0][1] += ds.y * q0;
                        fm[1][0] += ds.x * q1;
                        fm[1][1] += ds.y * q1;
                        if constexpr (MODE == kModeSums) {
                            const int nsub = K >> 5;
                            const int c0 = 2 * t, c1 = 2 * t + 1;
                            int32_t *out = args.sums;
                            if (g < rows) {
                                if (c0 < NC) out[(size_t(c0) * nrows + r0 + g) * nsub + kb] = d[j][0];
                                if (c1 < NC) out[(size_t(c1) * nrows + r0 + g) * nsub + kb] = d[j][1];
                            }
                            if (g + 8 < rows) {
                                if (c0 < NC) out[(size_t(c0) * nrows + r0 + g + 8) * nsub + kb] = d[j][2];
                                if (c1 < NC) out[(size_t(c1) * nrows + r0 + g + 8) * nsub + kb] = d[j][3];
                            }
                        }
                    }
                };
                unit(std::integral_constant<int, 0>{});
                unit(std::integral_constant<int, 1>{});
                unit(std::integral_constant<int, 2>{});
                unit(std::integral_constant<int, 3>{});
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    acc[0][cc] += h0.d * fd[0][cc] - h0.dmin * fm[0][cc];
                    acc[1][cc] += h1.d * fd[1][cc] - h1.dmin * fm[1][cc];
                }
            }
            __syncwarp();  // every lane is done with stage st
            const int s = k * cw + i;
            if (s + nst < my_stages) issue(s + nst, st);
            if (++st == nst) {
                st = 0;
                phase ^= 1u;
            }
        }
        if constexpr (MODE != kModeSums) {
            // partials of tile k in buffer k & 1 (the other buffer may still be read by warp 0
            // for tile k - 1 until the barrier below has been passed once more)
            float4 *rb = red + (k & 1) * nwarps * 32;
            rb[warp * 32 + lane] = make_float4(acc[0][0], acc[0][1], acc[1][0], acc[1][1]);
            const int bad = __syncthreads_or(ok ? 0 : 1);
            if (warp == 0 && !bad) {
                float4 v = rb[lane];
                for (int w = 1; w < nwarps; ++w) {
                    const float4 u = rb[w * 32 + lane];
                    v.x += u.x;
                    v.y += u.y;
                    v.z += u.z;
                    v.w += u.w;
                }
                float *y = args.segY[sg];
                const float vals[2][2] = {{v.x, v.y}, {v.z, v.w}};
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int row = g + 8 * rr;
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int col = 2 * t + cc;
                        if (row < rows && col < NC) y[size_t(col) * nrows + r0 + row] = vals[rr][cc];
                    }
                }
            }
        }
    }
}

template <int QT, int NC>
static MmvqKernelFn mma_pick_mode(int mode) {
    switch (mode) {
    case kModeQ81: return mmvq_mma_kernel<QT, NC, kModeQ81>;
    case kModeSums: return mmvq_mma_kernel<QT, NC, kModeSums>;
    default: return nullptr;
    }
}

template <int QT>
static MmvqKernelFn mma_pick(int ncols, int mode) {
    switch (ncols) {
    case 2: return mma_pick_mode<QT, 2>(mode);
    case 3: return mma_pick_mode<QT, 3>(mode);
    case 4: return mma_pick_mode<QT, 4>(mode);
    case 5: return mma_pick_mode<QT, 5>(mode);
    case 6: return mma_pick_mode<QT, 6>(mode);
    case 7: return mma_pick_mode<QT, 7>(mode);
    case 8: return mma_pick_mode<QT, 8>(mode);
    default: return nullptr;
    }
}

MmvqKernelFn mmvq_mma_kernel_for(int qt, int ncols, int mode) {
    switch (qt) {
    case kTypeQ4_K: return mma_pick<kTypeQ4_K>(ncols, mode);
    case kTypeQ5_K: return mma_pick<kTypeQ5_K>(ncols, mode);
    default: return nullptr;
    }
}

int mmvq_mma_max_warps() { return kMmaMaxWarps; }

int mmvq_mma_smem_bytes(int qt, int K, int ncols, int nwarps, int nstages) {
    return mma_smem_layout(qt, K, ncols, nwarps, nstages).total;
}

int mmvq_mma_take_status() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_anvil_device_status, sizeof(int)) != cudaSuccess) return -1;
    if (cudaMemcpyToSymbol(g_anvil_device_status, &z, sizeof(int)) != cudaSuccess) return -1;
    return v;
}

}  // namespace anvil
