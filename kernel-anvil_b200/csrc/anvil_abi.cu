// anvil_abi.cu -- extern "C" entry points of libanvil.so (declared in include/anvil.h):
// argument checks, launch planning, the Q8_1 quantiser kernel, programmatic dependent
// launch, and the CUDA-graph chain executor.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "anvil.h"
#include "anvil_host.h"
#include "mmvq.cuh"

namespace anvil {

// ---------------------------------------------------------------------------------
// Q8_1 quantiser.  One warp per 32-value block, one lane per value, the semantics of
// llama.cpp's CUDA quantize_q8_1: amax and sum by xor-butterfly warp reductions,
// d = amax / 127, q = roundf(x / d) (0 when amax == 0), block = {half(d), half(sum), q}.
// Both quotients are the correctly rounded IEEE ones (q8_scale, quant_q8; no fast-math),
// round-half-away-from-zero, fp16 round-to-nearest-even.
// ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    quantize_q8_1_kernel(const float *__restrict__ x, uint8_t *__restrict__ xq, int nblocks) {
    pdl_launch_dependents();
    pdl_wait();
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= nblocks) return;  // uniform per warp
    const float xi = x[size_t(gw) * 32 + lane];
    const float amax = warp_max(fabsf(xi));
    const float sum = warp_sum(xi);
    const float d = q8_scale(amax);
    const double rd64 = 1.0 / double(amax == 0.0f ? 1.0f : d);
    const int q = amax == 0.0f ? 0 : quant_q8(xi, float(rd64), rd64);
    // Pack four quants per lane group and store words (blocks are 4-byte aligned).
    const uint32_t b = uint32_t(q) & 0xFFu;
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, b, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, b, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, b, 3);
    uint32_t *blk = reinterpret_cast<uint32_t *>(xq + size_t(gw) * kQ8_1Bytes);
    if ((lane & 3) == 0) blk[1 + (lane >> 2)] = b | (b1 << 8) | (b2 << 16) | (b3 << 24);
    if (lane == 0) {
        const uint32_t hd = __half_as_ushort(__float2half_rn(d));
        const uint32_t hs = __half_as_ushort(__float2half_rn(sum));
        blk[0] = hd | (hs << 16);
    }
}

static int take_quantize_status() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_anvil_device_status, sizeof(int)) != cudaSuccess) return -1;
    if (cudaMemcpyToSymbol(g_anvil_device_status, &z, sizeof(int)) != cudaSuccess) return -1;
    return v;
}

// ---------------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------------
static thread_local std::string t_last_error;

int fail(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(ANVIL_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------------
// Per-device state: SM count, one-time function attributes, occupancy cache.
// ---------------------------------------------------------------------------------
constexpr int kMaxDevices = 64;

struct DeviceInfo {
    std::atomic<int> sm_count{0};
};
static DeviceInfo g_dev[kMaxDevices];

static std::atomic<unsigned long long> g_wait_limit_ns{kWaitLimitNs};

unsigned long long wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

static std::mutex g_cache_mu;
struct FnKey {
    const void *fn;
    int dev, threads, smem;
    bool operator==(const FnKey &o) const {
        return fn == o.fn && dev == o.dev && threads == o.threads && smem == o.smem;
    }
};
struct FnKeyHash {
    size_t operator()(const FnKey &k) const {
        return std::hash<const void *>()(k.fn) ^ (size_t(k.dev) << 48) ^ (size_t(k.threads) << 32) ^
               size_t(k.smem);
    }
};
static std::unordered_map<FnKey, int, FnKeyHash> g_occ_cache;
static std::unordered_map<uint64_t, bool> g_attr_set;  // (fn, dev) -> max smem attribute set

int current_device(int *dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= kMaxDevices) return fail(ANVIL_ERR_UNSUPPORTED, "device %d", *dev);
    return ANVIL_OK;
}

int sm_count(int dev, int *out) {
    int n = g_dev[dev].sm_count.load(std::memory_order_relaxed);
    if (n == 0) {
        cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
        g_dev[dev].sm_count.store(n, std::memory_order_relaxed);
    }
    *out = n;
    return ANVIL_OK;
}

// Lets `fn` use up to kMaxSmem of dynamic shared memory (once per device) and returns
// how many CTAs of `threads` x `smem` fit on one SM.
static int prepare_fn(const void *fn, int dev, int threads, int smem, int *occ) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    const uint64_t akey = reinterpret_cast<uint64_t>(fn) * 131u + uint64_t(dev);
    if (!g_attr_set.count(akey)) {
        cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
        g_attr_set[akey] = true;
    }
    FnKey k{fn, dev, threads, smem};
    auto it = g_occ_cache.find(k);
    if (it != g_occ_cache.end()) {
        *occ = it->second;
        return ANVIL_OK;
    }
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (n < 1) return fail(ANVIL_ERR_UNSUPPORTED, "kernel does not fit on an SM (%d B smem)", smem);
    g_occ_cache[k] = n;
    *occ = n;
    return ANVIL_OK;
}

// ---------------------------------------------------------------------------------
// Geometry and launch planning
// ---------------------------------------------------------------------------------
static bool supported_type(int t) {
    return t == kTypeQ4_K || t == kTypeQ5_K || t == kTypeQ6_K || t == kTypeQ8_0 || t == kTypeQ4_0 ||
           t == kTypeQ4_1 || t == kTypeQ5_0 || t == kTypeQ5_1 || t == kTypeQ2_K || t == kTypeQ3_K ||
           t == kTypeIQ4_NL || t == kTypeIQ4_XS || t == kTypeIQ2_XXS || t == kTypeIQ2_XS ||
           t == kTypeIQ2_S || t == kTypeIQ3_XXS || t == kTypeIQ3_S || t == kTypeIQ1_S ||
           t == kTypeIQ1_M;
}

static MmvqKernelFn kernel_for(int t, int ncols, int rpb, int lbt, int mode) {
    switch (t) {
    case kTypeQ4_K: return mmvq_kernel_q4k(ncols, rpb, lbt, mode);
    case kTypeQ5_K: return mmvq_kernel_q5k(ncols, rpb, lbt, mode);
    case kTypeQ6_K: return mmvq_kernel_q6k(ncols, rpb, lbt, mode);
    case kTypeQ8_0: return mmvq_kernel_q80(ncols, rpb, lbt, mode);
    case kTypeQ4_0: return mmvq_kernel_q40(ncols, rpb, lbt, mode);
    case kTypeQ4_1: return mmvq_kernel_q41(ncols, rpb, lbt, mode);
    case kTypeQ5_0: return mmvq_kernel_q50(ncols, rpb, lbt, mode);
    case kTypeQ5_1: return mmvq_kernel_q51(ncols, rpb, lbt, mode);
    case kTypeQ2_K: return mmvq_kernel_q2k(ncols, rpb, lbt, mode);
    case kTypeQ3_K: return mmvq_kernel_q3k(ncols, rpb, lbt, mode);
    case kTypeIQ4_NL: return mmvq_kernel_iq4nl(ncols, rpb, lbt, mode);
    case kTypeIQ4_XS: return mmvq_kernel_iq4xs(ncols, rpb, lbt, mode);
    case kTypeIQ2_XXS: return mmvq_kernel_iq2xxs(ncols, rpb, lbt, mode);
    case kTypeIQ2_XS: return mmvq_kernel_iq2xs(ncols, rpb, lbt, mode);
    case kTypeIQ2_S: return mmvq_kernel_iq2s(ncols, rpb, lbt, mode);
    case kTypeIQ3_XXS: return mmvq_kernel_iq3xxs(ncols, rpb, lbt, mode);
    case kTypeIQ3_S: return mmvq_kernel_iq3s(ncols, rpb, lbt, mode);
    case kTypeIQ1_S: return mmvq_kernel_iq1s(ncols, rpb, lbt, mode);
    case kTypeIQ1_M: return mmvq_kernel_iq1m(ncols, rpb, lbt, mode);
    default: return nullptr;
    }
}

// Built-in B200 default when neither the caller nor the smithy table chose, from the
// nwarps x rows_per_block sweep over the Qwen3-8B shapes: 4 warps with 4-row tiles (2 rows
// when K >= 8192); small N (< 2048 rows) prefers 8 warps of 1-row tiles so every warp has
// a row.
static void default_config(int t, int nrows, int K, int ncols, int *nw, int *rpb) {
    (void)t;
    if (nrows < 2048) {
        *nw = 8;
        *rpb = 1;
    } else {
        *nw = 4;
        // 4 or more columns: 2-row tiles keep two CTAs per SM beside the larger staged
        // activation (Q4_K 12288 x 4096 at 8 columns: 39.6 vs 50.7 us, measured)
        *rpb = (K >= 8192 || ncols >= 4) ? 2 : 4;
    }
}

struct Plan {
    MmvqKernelFn fn;
    int mode, nwarps, rpb, nstages, grid, smem;
    int occ, nsm;
    long ctas_needed;
    // Column chunks: when the staged activation of all ncols columns does not fit in shared
    // memory, the launch runs `chunk` columns at a time (fn and the fields above are the
    // chunk's plan) and `tail` plans the last ncols % chunk columns.  chunk 0: one launch.
    int ncols, chunk, type;
    bool cta_tiles = false;  // one tile per CTA (the tensor-core kernel), else one per warp
    std::shared_ptr<const Plan> tail;
};

// Grid of a plan when `share` kernels are meant to be resident on each SM at once (a chain
// under programmatic dependent launch: the next GEMV's CTAs fit beside the current one's
// and stream their first weight tiles while it runs).
static int grid_for(const Plan &p, int share) {
    const long per_sm = share > 1 ? std::max(1, p.occ / share) : p.occ;
    return int(std::min<long>(p.ctas_needed, per_sm * p.nsm));
}

static int round_rpb(int r) { return r >= 8 ? 8 : r >= 4 ? 4 : r >= 2 ? 2 : 1; }

// Tensor-core path (mmvq_mma.cu): Q4_K / Q5_K with 2..8 columns through mma.sync.
MmvqKernelFn mmvq_mma_kernel_for(int qt, int ncols, int mode);
int mmvq_mma_smem_bytes(int qt, int K, int ncols, int nwarps, int nstages);
int mmvq_mma_max_warps();
int mmvq_mma_take_status();
constexpr int kMmaTileRows = 16;
// Smallest column count that takes the tensor-core path (0: never).
// 4: at 2 columns the MMA tiles compute 8 columns' work and the dp4a kernels are faster
// (Q4_K 12288 x 4096: 13.4 against 8.2 us), from 4 on the MMA is (14.0 against 17.8 us).
static std::atomic<int> g_mma_min_cols{4};

static bool mma_eligible(int t, int ncols, int mode, int nwarps, int rpb) {
    const int m = g_mma_min_cols.load(std::memory_order_relaxed);
    return m > 0 && ncols >= m && ncols >= 2 && (t == kTypeQ4_K || t == kTypeQ5_K) &&
           (mode == kModeQ81 || mode == kModeSums) && nwarps == 0 && rpb == 0;
}

// Plan of the tensor-core kernel: 16-row CTA tiles whose K-chunks the CTA's warps share;
// warps per CTA up to 16 but no more than the K dimension's 256-weight super-blocks, the
// most of them (halving) whose rings of 3, else 2, chunk stages fit beside the staged
// activation.
static int plan_mma(int t, int nrows, int K, int ncols, int mode, Plan *p) {
    int nw = 0, ns = 0, smem = 0;
    int wmax = mmvq_mma_max_warps();
    while (wmax > 1 && wmax > K / 256) wmax >>= 1;
    for (int w = wmax; w >= 1 && !nw; w >>= 1)
        for (int st = 3; st >= 2 && !nw; --st) {
            const int b = mmvq_mma_smem_bytes(t, K, ncols, w, st);
            if (b <= kMaxSmem) {
                nw = w;
                ns = st;
                smem = b;
            }
        }
    if (!nw)
        return fail(ANVIL_ERR_UNSUPPORTED, "ncols_x=%d ncols_dst=%d does not fit in shared memory "
                                           "(tensor-core path)", K, ncols);
    int dev, nsm;
    if (int s = current_device(&dev)) return s;
    if (int s = sm_count(dev, &nsm)) return s;
    p->fn = mmvq_mma_kernel_for(t, ncols, mode);
    if (!p->fn) return fail(ANVIL_ERR_UNSUPPORTED, "no tensor-core kernel for ncols=%d", ncols);
    p->mode = mode;
    p->nwarps = nw;
    p->rpb = kMmaTileRows;
    p->nstages = ns;
    p->smem = smem;
    int occ = 0;
    if (int s = prepare_fn(reinterpret_cast<const void *>(p->fn), dev, nw * 32, smem, &occ)) return s;
    const long ntiles = (long(nrows) + kMmaTileRows - 1) / kMmaTileRows;
    p->ctas_needed = ntiles;  // one CTA per 16-row tile (persistent grid beyond the SMs)
    p->cta_tiles = true;
    p->occ = occ;
    p->nsm = nsm;
    p->grid = grid_for(*p, 1);
    return ANVIL_OK;
}

static int plan_one(int t, int nrows, int K, int ncols, int nwarps, int rpb, int mode,
                    Plan *p) {
    p->ncols = ncols;
    p->chunk = 0;
    p->type = t;
    p->cta_tiles = false;
    p->tail.reset();
    if (!supported_type(t)) return fail(ANVIL_ERR_UNSUPPORTED, "ggml type %d has no MMVQ kernel", t);
    if (nrows <= 0 || K <= 0) return fail(ANVIL_ERR_INVALID, "nrows=%d ncols_x=%d", nrows, K);
    const int qk = mmvq_type_qk(t);
    if (K % qk != 0)
        return fail(ANVIL_ERR_INVALID, "ncols_x=%d is not a multiple of the block size %d", K, qk);
    if (ncols < 1 || ncols > kMaxCols)
        return fail(ANVIL_ERR_INVALID, "ncols_dst=%d outside 1..%d", ncols, kMaxCols);
    if (mode == kModeGLU && ncols != 1)
        return fail(ANVIL_ERR_INVALID, "the gate/up epilogue takes one column, got %d", ncols);
    if (nwarps < 0 || rpb < 0)
        return fail(ANVIL_ERR_INVALID, "nwarps=%d rows_per_block=%d", nwarps, rpb);
    if (mma_eligible(t, ncols, mode, nwarps, rpb)) return plan_mma(t, nrows, K, ncols, mode, p);
    if (nwarps == 0 || rpb == 0) {
        int lnw = 0, lrpb = 0;
        if (anvil_smithy_lookup(t, nrows, K, &lnw, &lrpb) && lnw > 0 && lrpb > 0) {
            if (nwarps == 0) nwarps = lnw;
            if (rpb == 0) rpb = lrpb;
        }
        int dnw, drpb;
        default_config(t, nrows, K, ncols, &dnw, &drpb);
        if (nwarps == 0) nwarps = dnw;
        if (rpb == 0) rpb = drpb;
    }
    nwarps = std::min(std::max(nwarps, 1), kMaxWarps);
    rpb = round_rpb(rpb);
    // gate/up tiles hold rpb/2 rows of each matrix: at least one pair
    const int min_rpb = mode == kModeGLU ? 2 : 1;
    if (rpb < min_rpb) rpb = min_rpb;
    int dev;
    if (int s = current_device(&dev)) return s;
    int nsm;
    if (int s = sm_count(dev, &nsm)) return s;
    const int row_bytes = (K / qk) * mmvq_type_bytes(t);
    // Each warp owns a ring of stages of rpb rows: aim for ~12 KB of weights per warp ring
    // (2..8 stages); if the CTA does not fit in shared memory use fewer stages, then
    // smaller tiles, then fewer warps.
    for (;;) {
        const int tile = rpb * row_bytes;
        int ns = std::min(8, std::max(2, (12288 + tile - 1) / tile));
        MmvqSmem L = mmvq_smem_layout(t, K, ncols, rpb, nwarps, ns, mode);
        while (L.total > kMaxSmem && ns > 1)
            L = mmvq_smem_layout(t, K, ncols, rpb, nwarps, --ns, mode);
        if (L.total <= kMaxSmem) {
            p->nstages = ns;
            p->smem = L.total;
            break;
        }
        if (rpb > min_rpb) {
            rpb >>= 1;
        } else if (nwarps > 1) {
            nwarps >>= 1;
        } else {
            return fail(ANVIL_ERR_UNSUPPORTED, "ncols_x=%d ncols_dst=%d does not fit in shared memory",
                        K, ncols);
        }
    }
    // Lanes per row: the compile-time variants (16, 32) when the heuristic picks them.
    int lbt = host_lanes_per_row(K / qk, rpb);
    // gate/up pairing: lane group g owns gate row i and up row i, which needs a compile-time
    // lanes-per-row with rpb/2 a multiple of the 32/lbt row groups (32 lanes always are)
    if (mode == kModeGLU && !((lbt == 16 || lbt == 32) && (rpb / 2) % (32 / lbt) == 0)) lbt = 32;
    p->fn = kernel_for(t, ncols, rpb, lbt, mode);
    p->mode = mode;
    if (!p->fn) return fail(ANVIL_ERR_UNSUPPORTED, "no kernel for ncols=%d rpb=%d", ncols, rpb);
    p->nwarps = nwarps;
    p->rpb = rpb;
    int occ = 0;
    if (int s = prepare_fn(reinterpret_cast<const void *>(p->fn), dev, nwarps * 32, p->smem, &occ))
        return s;
    // Persistent grid: every warp takes warp-tiles of rpb rows (rpb/2 output rows for the
    // gate/up epilogue) round-robin.
    const int trows = mode == kModeGLU ? rpb / 2 : rpb;
    const long ntiles = (long(nrows) + trows - 1) / trows;
    p->ctas_needed = (ntiles + nwarps - 1) / nwarps;
    p->occ = occ;
    p->nsm = nsm;
    p->grid = grid_for(*p, 1);
    return ANVIL_OK;
}

// plan_one, or, when ncols columns of activation do not fit in shared memory, the largest
// column chunk that does (launched once per chunk; the weights are re-read per chunk).
static int plan_mmvq(int t, int nrows, int K, int ncols, int nwarps, int rpb, int mode,
                     Plan *p) {
    const int s = plan_one(t, nrows, K, ncols, nwarps, rpb, mode, p);
    if (s != ANVIL_ERR_UNSUPPORTED || ncols == 1 ||
        t_last_error.find("does not fit in shared memory") == std::string::npos)
        return s;
    const std::string why = t_last_error;
    for (int c = ncols - 1; c >= 1; --c) {
        Plan head;
        if (plan_one(t, nrows, K, c, nwarps, rpb, mode, &head) != ANVIL_OK) continue;
        if (ncols % c) {
            auto tail = std::make_shared<Plan>();
            if (plan_one(t, nrows, K, ncols % c, nwarps, rpb, mode, tail.get()) != ANVIL_OK) continue;
            head.tail = tail;
        }
        head.ncols = ncols;
        head.chunk = c;
        *p = head;
        t_last_error.clear();
        return ANVIL_OK;
    }
    t_last_error = why;
    return ANVIL_ERR_UNSUPPORTED;
}

// Segments of one launch: GEMVs of the plan's type that read the same activation.
struct Segs {
    int n;
    const void *W[kMaxSeg];
    float *y[kMaxSeg];
    int rows[kMaxSeg];
};

static int launch_segs_one(const Plan &p, const Segs &sg, const void *x, int32_t *sums, int K,
                           unsigned flags, cudaStream_t stream, int share) {
    MmvqArgs a;
    a.x = x;
    a.sums = sums;
    a.wait_ns = wait_limit_ns();
    a.K = K;
    a.nstages = p.nstages;
    a.nseg = sg.n;
    long tiles = 0;
    for (int i = 0; i < kMaxSeg; ++i) {
        const bool live = i < sg.n;
        a.segW[i] = live ? static_cast<const uint8_t *>(sg.W[i]) : nullptr;
        a.segY[i] = live ? sg.y[i] : nullptr;
        a.segRows[i] = live ? sg.rows[i] : 0;
        a.segTile[i] = int(tiles);
        if (live) tiles += (sg.rows[i] + p.rpb - 1) / p.rpb;
    }
    a.segTile[kMaxSeg] = int(tiles);
    if (sg.n < kMaxSeg) a.segTile[sg.n] = int(tiles);
    Plan q = p;
    q.ctas_needed = p.cta_tiles ? tiles : (tiles + p.nwarps - 1) / p.nwarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid_for(q, share));
    cfg.blockDim = dim3(p.nwarps * 32);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (flags & ANVIL_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, p.fn, a);
    if (e != cudaSuccess) return cuda_fail(e, "mmvq launch");
    return ANVIL_OK;
}

// One launch, or one per column chunk of the plan (columns are independent: chunk c0 reads
// activation columns c0.. and writes output columns c0..).
static int launch_mmvq_segs(const Plan &p, const Segs &sg, const void *x, int32_t *sums, int K,
                            unsigned flags, cudaStream_t stream, int share = 1) {
    if (p.chunk == 0) return launch_segs_one(p, sg, x, sums, K, flags, stream, share);
    const int nkb = K / 32;
    const bool sub16 = p.type == kTypeQ6_K || p.type == kTypeQ2_K || p.type == kTypeQ3_K ||
                       p.type == kTypeIQ2_XS || p.type == kTypeIQ2_S || p.type == kTypeIQ1_M;
    const int nsub = K / (sub16 ? 16 : 32);  // int32 sums per row and column (block-sum mode)
    for (int c0 = 0; c0 < p.ncols; c0 += p.chunk) {
        const Plan &q = p.ncols - c0 >= p.chunk ? p : *p.tail;
        Segs part = sg;
        for (int i = 0; i < sg.n; ++i) part.y[i] = sg.y[i] ? sg.y[i] + size_t(c0) * sg.rows[i] : nullptr;
        const void *xc = p.mode == kModeF32
                             ? static_cast<const void *>(static_cast<const float *>(x) + size_t(c0) * K)
                             : static_cast<const void *>(static_cast<const uint8_t *>(x) +
                                                         size_t(c0) * nkb * kQ8_1Bytes);
        int32_t *sc = sums ? sums + size_t(c0) * sg.rows[0] * nsub : nullptr;
        if (int s = launch_segs_one(q, part, xc, sc, K, flags, stream, share)) return s;
    }
    return ANVIL_OK;
}

static int launch_mmvq(const Plan &p, const void *W, const void *x, float *y, int32_t *sums,
                       int nrows, int K, unsigned flags, cudaStream_t stream, int share = 1) {
    Segs sg{};
    sg.n = 1;
    sg.W[0] = W;
    sg.y[0] = y;
    sg.rows[0] = nrows;
    return launch_mmvq_segs(p, sg, x, sums, K, flags, stream, share);
}

// Gate/up epilogue: y[r] = silu(W_gate[r] . x) * (W_up[r] . x), one column.  Tiles hold
// rpb/2 rows of each matrix, both copied whole (rows a multiple of 16 bytes).
static int launch_glu(const Plan &p, const void *Wg, const void *Wu, const void *xq, float *y,
                      int nrows, int K, unsigned flags, cudaStream_t stream, int share = 1) {
    MmvqArgs a = {};
    a.x = xq;
    a.sums = nullptr;
    a.wait_ns = wait_limit_ns();
    a.K = K;
    a.nstages = p.nstages;
    a.nseg = 1;
    a.segW[0] = static_cast<const uint8_t *>(Wg);
    a.segW[1] = static_cast<const uint8_t *>(Wu);
    a.segY[0] = y;
    a.segRows[0] = nrows;
    const int half = p.rpb / 2;
    const long tiles = (long(nrows) + half - 1) / half;
    a.segTile[0] = 0;
    for (int i = 1; i <= kMaxSeg; ++i) a.segTile[i] = int(tiles);
    Plan q = p;
    q.ctas_needed = p.cta_tiles ? tiles : (tiles + p.nwarps - 1) / p.nwarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid_for(q, share));
    cfg.blockDim = dim3(p.nwarps * 32);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (flags & ANVIL_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, p.fn, a);
    if (e != cudaSuccess) return cuda_fail(e, "mmvq gate/up launch");
    return ANVIL_OK;
}

static int check_glu_args(int t, const void *Wg, const void *Wu, const void *xq, const float *y,
                          int nrows, int K) {
    if (!Wg || !Wu || !xq || !y) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (!supported_type(t)) return fail(ANVIL_ERR_UNSUPPORTED, "ggml type %d has no MMVQ kernel", t);
    if (nrows <= 0 || K <= 0 || K % mmvq_type_qk(t))
        return fail(ANVIL_ERR_INVALID, "nrows=%d ncols_x=%d", nrows, K);
    if ((reinterpret_cast<uintptr_t>(Wg) | reinterpret_cast<uintptr_t>(Wu)) & 15)
        return fail(ANVIL_ERR_ALIGN, "weights must be 16-byte aligned");
    if ((long(K / mmvq_type_qk(t)) * mmvq_type_bytes(t)) % 16)
        return fail(ANVIL_ERR_ALIGN, "gate/up rows must be a multiple of 16 bytes (ncols_x=%d)", K);
    if ((reinterpret_cast<uintptr_t>(xq) | reinterpret_cast<uintptr_t>(y)) & 3)
        return fail(ANVIL_ERR_ALIGN, "activation and output must be 4-byte aligned");
    return ANVIL_OK;
}

static int check_mmvq_ptrs(int t, const void *W, const void *xq, const void *out) {
    if (!W || !xq || !out) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    (void)t;
    if (reinterpret_cast<uintptr_t>(W) & 15)
        return fail(ANVIL_ERR_ALIGN, "weights must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(xq) | reinterpret_cast<uintptr_t>(out)) & 3)
        return fail(ANVIL_ERR_ALIGN, "activation and output must be 4-byte aligned");
    return ANVIL_OK;
}

static int launch_quantize(const float *x, void *xq, int K, int ncols, unsigned flags,
                           cudaStream_t stream) {
    if (!x || !xq) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (K <= 0 || K % 32 != 0) return fail(ANVIL_ERR_INVALID, "K=%d is not a positive multiple of 32", K);
    if (ncols < 1) return fail(ANVIL_ERR_INVALID, "ncols=%d", ncols);
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(xq)) & 3)
        return fail(ANVIL_ERR_ALIGN, "x and xq must be 4-byte aligned");
    const long nblocks = long(K / 32) * ncols;
    if (nblocks > (1L << 26)) return fail(ANVIL_ERR_INVALID, "input too large");
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(256);
    cfg.gridDim = dim3(unsigned((nblocks + 7) / 8));
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (flags & ANVIL_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, quantize_q8_1_kernel, x, static_cast<uint8_t *>(xq),
                                       int(nblocks));
    if (e != cudaSuccess) return cuda_fail(e, "quantize_q8_1 launch");
    return ANVIL_OK;
}

}  // namespace anvil

using namespace anvil;

// ---------------------------------------------------------------------------------
// Chain executor
// ---------------------------------------------------------------------------------
struct ChainStep {
    bool quantize;
    bool fused;  // mmvq step reading fp32 x (fused quantisation, or quantise + mmvq)
    // quantize
    const float *x;
    void *xq;
    int K, ncols;
    // mmvq
    int type;
    const void *W;
    const void *W2;  // up matrix of a gate/up step (W is the gate)
    const void *xqin;
    float *y;
    int nrows, ncols_x, ncols_dst, nwarps, rpb;
    Plan plan;
    Segs segs;  // the GEMVs of an mmvq step (one, or several sharing the activation)
};

struct anvil_chain {
    std::vector<ChainStep> steps;
    int share = 1;  // kernels meant to be co-resident per SM (see grid_for)
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

extern "C" {

int anvil_abi_version(void) { return ANVIL_ABI_VERSION; }

int anvil_set_wait_limit_ns(unsigned long long ns) {
    if (ns > 60ull * 1000000000ull) return fail(ANVIL_ERR_INVALID, "wait limit %llu ns above 60 s", ns);
    g_wait_limit_ns.store(ns ? ns : kWaitLimitNs, std::memory_order_relaxed);
    return ANVIL_OK;
}

unsigned long long anvil_get_wait_limit_ns(void) { return wait_limit_ns(); }

int anvil_set_tensor_core_min_cols(int min_cols) {
    if (min_cols != 0 && (min_cols < 2 || min_cols > kMaxCols))
        return fail(ANVIL_ERR_INVALID, "tensor-core column threshold %d: 0 or 2..%d", min_cols, kMaxCols);
    g_mma_min_cols.store(min_cols, std::memory_order_relaxed);
    return ANVIL_OK;
}

int anvil_get_tensor_core_min_cols(void) { return g_mma_min_cols.load(std::memory_order_relaxed); }

const char *anvil_last_error(void) { return t_last_error.c_str(); }

int anvil_type_geometry(int ggml_type, int *qk, int *block_bytes) {
    int q = 0, b = 0;
    switch (ggml_type) {
    case ANVIL_TYPE_Q4_0: q = 32; b = 18; break;
    case ANVIL_TYPE_Q4_1: q = 32; b = 20; break;
    case ANVIL_TYPE_Q5_0: q = 32; b = 22; break;
    case ANVIL_TYPE_Q5_1: q = 32; b = 24; break;
    case ANVIL_TYPE_Q8_0: q = 32; b = 34; break;
    case ANVIL_TYPE_Q8_1: q = 32; b = 36; break;
    case ANVIL_TYPE_Q2_K: q = 256; b = 84; break;
    case ANVIL_TYPE_IQ4_NL: q = 32; b = 18; break;
    case ANVIL_TYPE_IQ4_XS: q = 256; b = 136; break;
    case ANVIL_TYPE_IQ2_XXS: q = 256; b = 66; break;
    case ANVIL_TYPE_IQ2_XS: q = 256; b = 74; break;
    case ANVIL_TYPE_IQ2_S: q = 256; b = 82; break;
    case ANVIL_TYPE_IQ3_XXS: q = 256; b = 98; break;
    case ANVIL_TYPE_IQ3_S: q = 256; b = 110; break;
    case ANVIL_TYPE_IQ1_S: q = 256; b = 50; break;
    case ANVIL_TYPE_IQ1_M: q = 256; b = 56; break;
    case ANVIL_TYPE_Q3_K: q = 256; b = 110; break;
    case ANVIL_TYPE_Q4_K: q = 256; b = 144; break;
    case ANVIL_TYPE_Q5_K: q = 256; b = 176; break;
    case ANVIL_TYPE_Q6_K: q = 256; b = 210; break;
    default: return fail(ANVIL_ERR_UNSUPPORTED, "ggml type %d has no block geometry here", ggml_type);
    }
    if (qk) *qk = q;
    if (block_bytes) *block_bytes = b;
    return ANVIL_OK;
}

int64_t anvil_row_bytes(int ggml_type, int K) {
    int qk, bb;
    if (int s = anvil_type_geometry(ggml_type, &qk, &bb)) return s;
    if (K <= 0 || K % qk) return fail(ANVIL_ERR_INVALID, "K=%d is not a multiple of %d", K, qk);
    return int64_t(K / qk) * bb;
}

int anvil_quantize_q8_1_ex(const float *x, void *xq, int K, int ncols, unsigned flags,
                           anvil_stream_t stream) {
    return launch_quantize(x, xq, K, ncols, flags, reinterpret_cast<cudaStream_t>(stream));
}

int anvil_quantize_q8_1(const float *x, void *xq, int K, int ncols, anvil_stream_t stream) {
    return anvil_quantize_q8_1_ex(x, xq, K, ncols, 0, stream);
}

int anvil_mmvq_plan(int ggml_type, int nrows, int ncols_x, int ncols_dst, int nwarps,
                    int rows_per_block, int *out_nwarps, int *out_rpb, int *out_grid,
                    int *out_smem_bytes) {
    Plan p;
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81, &p))
        return s;
    if (out_nwarps) *out_nwarps = p.nwarps;
    if (out_rpb) *out_rpb = p.rpb;
    if (out_grid) *out_grid = p.grid;
    if (out_smem_bytes) *out_smem_bytes = p.smem;
    return ANVIL_OK;
}

int anvil_mmvq_kernel_attributes(int ggml_type, int nrows, int ncols_x, int ncols_dst, int nwarps,
                                 int rows_per_block, int *regs_per_thread, int *local_bytes,
                                 int *max_threads_per_block) {
    Plan p;
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81, &p))
        return s;
    cudaFuncAttributes attr{};
    const cudaError_t e = cudaFuncGetAttributes(&attr, reinterpret_cast<const void *>(p.fn));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
    if (regs_per_thread) *regs_per_thread = attr.numRegs;
    if (local_bytes) *local_bytes = int(attr.localSizeBytes);
    if (max_threads_per_block) *max_threads_per_block = attr.maxThreadsPerBlock;
    return ANVIL_OK;
}

int anvil_mmvq_ex(int ggml_type, const void *W, const void *xq, float *y, int nrows,
                  int ncols_x, int ncols_dst, int nwarps, int rows_per_block, unsigned flags,
                  anvil_stream_t stream) {
    if (int s = check_mmvq_ptrs(ggml_type, W, xq, y)) return s;
    Plan p;
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81, &p))
        return s;
    return launch_mmvq(p, W, xq, y, nullptr, nrows, ncols_x, flags,
                       reinterpret_cast<cudaStream_t>(stream));
}

int anvil_mmvq(int ggml_type, const void *W, const void *xq, float *y, int nrows, int ncols_x,
               int ncols_dst, int nwarps, int rows_per_block, anvil_stream_t stream) {
    return anvil_mmvq_ex(ggml_type, W, xq, y, nrows, ncols_x, ncols_dst, nwarps, rows_per_block,
                         0, stream);
}

// Plans the fused fp32 path; returns false (with no error) when it cannot be used.
static bool plan_fused(int t, const float *x, int nrows, int K, int ncols, int nwarps, int rpb,
                       Plan *p) {
    if (reinterpret_cast<uintptr_t>(x) & 15) return false;
    const std::string saved = t_last_error;
    if (plan_mmvq(t, nrows, K, ncols, nwarps, rpb, kModeF32, p) != ANVIL_OK) {
        t_last_error = saved;
        return false;
    }
    return true;
}

int anvil_mmvq_f32_ex(int ggml_type, const void *W, const float *x, void *xq, float *y, int nrows,
                      int ncols_x, int ncols_dst, int nwarps, int rows_per_block, unsigned flags,
                      anvil_stream_t stream) {
    if (int s = check_mmvq_ptrs(ggml_type, W, xq, y)) return s;
    if (!x) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    Plan p;
    if (plan_fused(ggml_type, x, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, &p))
        return launch_mmvq(p, W, x, y, nullptr, nrows, ncols_x, flags, st);
    // Two launches: quantise into the caller's scratch, then the Q8_1 GEMV.  The GEMV's
    // only producer is that quantiser, which never writes W, so it may prefetch early.
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81, &p))
        return s;
    if (int s = launch_quantize(x, xq, ncols_x, ncols_dst, flags, st)) return s;
    return launch_mmvq(p, W, xq, y, nullptr, nrows, ncols_x, ANVIL_FLAG_PDL, st);
}

int anvil_mmvq_f32(int ggml_type, const void *W, const float *x, void *xq, float *y, int nrows,
                   int ncols_x, int ncols_dst, int nwarps, int rows_per_block,
                   anvil_stream_t stream) {
    return anvil_mmvq_f32_ex(ggml_type, W, x, xq, y, nrows, ncols_x, ncols_dst, nwarps,
                             rows_per_block, 0, stream);
}

// Checks and packs the segments of a grouped GEMV; *total = their rows together.
static int make_segs(int t, int nseg, const void *const *W, float *const *y, const int *nrows,
                     Segs *sg, int *total) {
    if (nseg < 1 || nseg > kMaxSeg) return fail(ANVIL_ERR_INVALID, "nseg=%d outside 1..%d", nseg, kMaxSeg);
    if (!W || !y || !nrows) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    sg->n = nseg;
    long sum = 0;
    for (int i = 0; i < nseg; ++i) {
        if (int s = check_mmvq_ptrs(t, W[i], W[i], y[i])) return s;
        if (nrows[i] <= 0) return fail(ANVIL_ERR_INVALID, "nrows[%d]=%d", i, nrows[i]);
        sg->W[i] = W[i];
        sg->y[i] = y[i];
        sg->rows[i] = nrows[i];
        sum += nrows[i];
    }
    if (sum > (1L << 30)) return fail(ANVIL_ERR_INVALID, "too many rows");
    *total = int(sum);
    return ANVIL_OK;
}

int anvil_mmvq_grouped(int ggml_type, int nseg, const void *const *W, const void *xq,
                       float *const *y, const int *nrows, int ncols_x, int ncols_dst, int nwarps,
                       int rows_per_block, unsigned flags, anvil_stream_t stream) {
    Segs sg;
    int total;
    if (int s = make_segs(ggml_type, nseg, W, y, nrows, &sg, &total)) return s;
    if (!xq) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (reinterpret_cast<uintptr_t>(xq) & 3) return fail(ANVIL_ERR_ALIGN, "xq must be 4-byte aligned");
    Plan p;
    if (int s = plan_mmvq(ggml_type, total, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81, &p))
        return s;
    return launch_mmvq_segs(p, sg, xq, nullptr, ncols_x, flags, reinterpret_cast<cudaStream_t>(stream));
}

int anvil_mmvq_grouped_f32(int ggml_type, int nseg, const void *const *W, const float *x,
                           void *xq, float *const *y, const int *nrows, int ncols_x, int ncols_dst,
                           int nwarps, int rows_per_block, unsigned flags, anvil_stream_t stream) {
    Segs sg;
    int total;
    if (int s = make_segs(ggml_type, nseg, W, y, nrows, &sg, &total)) return s;
    if (!x || !xq) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (reinterpret_cast<uintptr_t>(xq) & 3) return fail(ANVIL_ERR_ALIGN, "xq must be 4-byte aligned");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    Plan p;
    if (plan_fused(ggml_type, x, total, ncols_x, ncols_dst, nwarps, rows_per_block, &p))
        return launch_mmvq_segs(p, sg, x, nullptr, ncols_x, flags, st);
    if (int s = plan_mmvq(ggml_type, total, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81, &p))
        return s;
    if (int s = launch_quantize(x, xq, ncols_x, ncols_dst, flags, st)) return s;
    return launch_mmvq_segs(p, sg, xq, nullptr, ncols_x, ANVIL_FLAG_PDL, st);
}

int anvil_mmvq_glu(int ggml_type, const void *W_gate, const void *W_up, const void *xq, float *y,
                   int nrows, int ncols_x, int nwarps, int rows_per_block, unsigned flags,
                   anvil_stream_t stream) {
    if (int s = check_glu_args(ggml_type, W_gate, W_up, xq, y, nrows, ncols_x)) return s;
    Plan p;
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, 1, nwarps, rows_per_block, kModeGLU, &p))
        return s;
    return launch_glu(p, W_gate, W_up, xq, y, nrows, ncols_x, flags,
                      reinterpret_cast<cudaStream_t>(stream));
}

int anvil_mmvq_glu_f32(int ggml_type, const void *W_gate, const void *W_up, const float *x,
                       void *xq, float *y, int nrows, int ncols_x, int nwarps, int rows_per_block,
                       unsigned flags, anvil_stream_t stream) {
    if (!x) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (int s = check_glu_args(ggml_type, W_gate, W_up, xq, y, nrows, ncols_x)) return s;
    Plan p;
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, 1, nwarps, rows_per_block, kModeGLU, &p))
        return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (int s = launch_quantize(x, xq, ncols_x, 1, flags, st)) return s;
    return launch_glu(p, W_gate, W_up, xq, y, nrows, ncols_x, ANVIL_FLAG_PDL, st);
}

int anvil_mmvq_block_sums(int ggml_type, const void *W, const void *xq, int32_t *sums,
                          int nrows, int ncols_x, int ncols_dst, int nwarps, int rows_per_block,
                          anvil_stream_t stream) {
    if (int s = check_mmvq_ptrs(ggml_type, W, xq, sums)) return s;
    Plan p;
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, kModeSums, &p))
        return s;
    return launch_mmvq(p, W, xq, nullptr, sums, nrows, ncols_x, 0,
                       reinterpret_cast<cudaStream_t>(stream));
}

// Reads and clears the device status words (current device).  Returns the OR of all
// flags (0 = no bounded wait gave up) or a negative status.
int anvil_take_device_status(void) {
    int v = 0;
    int parts[21] = {take_quantize_status(), mmvq_mma_take_status(), mmvq_kernel_q4k_take_status(),
                    mmvq_kernel_q5k_take_status(), mmvq_kernel_q6k_take_status(),
                    mmvq_kernel_q80_take_status(), mmvq_kernel_q40_take_status(),
                    mmvq_kernel_q41_take_status(), mmvq_kernel_q50_take_status(),
                    mmvq_kernel_q51_take_status(), mmvq_kernel_q2k_take_status(),
                    mmvq_kernel_q3k_take_status(), mmvq_kernel_iq4nl_take_status(),
                    mmvq_kernel_iq4xs_take_status(), mmvq_kernel_iq2xxs_take_status(),
                    mmvq_kernel_iq2xs_take_status(), mmvq_kernel_iq2s_take_status(),
                    mmvq_kernel_iq3xxs_take_status(), mmvq_kernel_iq3s_take_status(),
                    mmvq_kernel_iq1s_take_status(), mmvq_kernel_iq1m_take_status()};
    for (int x : parts) {
        if (x < 0) return fail(ANVIL_ERR_CUDA, "reading device status failed");
        v |= x;
    }
    return v;
}

// ---- chain ------------------------------------------------------------------------

anvil_chain *anvil_chain_create(void) { return new (std::nothrow) anvil_chain(); }

void anvil_chain_destroy(anvil_chain *c) {
    if (!c) return;
    if (c->exec) cudaGraphExecDestroy(c->exec);
    if (c->graph) cudaGraphDestroy(c->graph);
    delete c;
}

int anvil_chain_num_steps(const anvil_chain *c) { return c ? int(c->steps.size()) : 0; }

int anvil_chain_set_coresident(anvil_chain *c, int kernels_per_sm) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (kernels_per_sm < 1 || kernels_per_sm > 4)
        return fail(ANVIL_ERR_INVALID, "kernels_per_sm=%d outside 1..4", kernels_per_sm);
    c->share = kernels_per_sm;
    return ANVIL_OK;
}

int anvil_chain_add_quantize(anvil_chain *c, const float *x, void *xq, int K, int ncols) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (!x || !xq || K <= 0 || K % 32 || ncols < 1)
        return fail(ANVIL_ERR_INVALID, "bad quantize step (K=%d ncols=%d)", K, ncols);
    ChainStep s = {};
    s.quantize = true;
    s.x = x;
    s.xq = xq;
    s.K = K;
    s.ncols = ncols;
    c->steps.push_back(s);
    return ANVIL_OK;
}

int anvil_chain_add_mmvq(anvil_chain *c, int ggml_type, const void *W, const void *xq, float *y,
                         int nrows, int ncols_x, int ncols_dst, int nwarps, int rows_per_block) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (int s = check_mmvq_ptrs(ggml_type, W, xq, y)) return s;
    ChainStep s = {};
    s.quantize = false;
    s.type = ggml_type;
    s.W = W;
    s.xqin = xq;
    s.y = y;
    s.nrows = nrows;
    s.ncols_x = ncols_x;
    s.ncols_dst = ncols_dst;
    s.nwarps = nwarps;
    s.rpb = rows_per_block;
    s.segs.n = 1;
    s.segs.W[0] = W;
    s.segs.y[0] = y;
    s.segs.rows[0] = nrows;
    if (int st = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81,
                           &s.plan))
        return st;
    c->steps.push_back(s);
    return ANVIL_OK;
}

int anvil_chain_add_mmvq_f32(anvil_chain *c, int ggml_type, const void *W, const float *x,
                             void *xq, float *y, int nrows, int ncols_x, int ncols_dst, int nwarps,
                             int rows_per_block) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (int s = check_mmvq_ptrs(ggml_type, W, xq, y)) return s;
    if (!x) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    ChainStep s = {};
    s.fused = true;
    s.type = ggml_type;
    s.W = W;
    s.x = x;
    s.xq = xq;
    s.xqin = xq;
    s.y = y;
    s.nrows = nrows;
    s.ncols_x = ncols_x;
    s.K = ncols_x;
    s.ncols = ncols_dst;
    s.ncols_dst = ncols_dst;
    s.nwarps = nwarps;
    s.rpb = rows_per_block;
    s.segs.n = 1;
    s.segs.W[0] = W;
    s.segs.y[0] = y;
    s.segs.rows[0] = nrows;
    if (!plan_fused(ggml_type, x, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, &s.plan)) {
        if (int st = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block,
                               kModeQ81, &s.plan))
            return st;
    }
    c->steps.push_back(s);
    return ANVIL_OK;
}

int anvil_chain_add_mmvq_grouped(anvil_chain *c, int ggml_type, int nseg, const void *const *W,
                                 const void *xq, float *const *y, const int *nrows, int ncols_x,
                                 int ncols_dst, int nwarps, int rows_per_block) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    ChainStep s = {};
    int total;
    if (int st = make_segs(ggml_type, nseg, W, y, nrows, &s.segs, &total)) return st;
    if (!xq) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (reinterpret_cast<uintptr_t>(xq) & 3) return fail(ANVIL_ERR_ALIGN, "xq must be 4-byte aligned");
    s.type = ggml_type;
    s.W = W[0];
    s.xqin = xq;
    s.y = y[0];
    s.nrows = total;
    s.ncols_x = ncols_x;
    s.ncols_dst = ncols_dst;
    s.nwarps = nwarps;
    s.rpb = rows_per_block;
    if (int st = plan_mmvq(ggml_type, total, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81,
                           &s.plan))
        return st;
    c->steps.push_back(s);
    return ANVIL_OK;
}

int anvil_chain_add_mmvq_grouped_f32(anvil_chain *c, int ggml_type, int nseg, const void *const *W,
                                     const float *x, void *xq, float *const *y, const int *nrows,
                                     int ncols_x, int ncols_dst, int nwarps, int rows_per_block) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    ChainStep s = {};
    int total;
    if (int st = make_segs(ggml_type, nseg, W, y, nrows, &s.segs, &total)) return st;
    if (!x || !xq) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (reinterpret_cast<uintptr_t>(xq) & 3) return fail(ANVIL_ERR_ALIGN, "xq must be 4-byte aligned");
    s.fused = true;
    s.type = ggml_type;
    s.W = W[0];
    s.x = x;
    s.xq = xq;
    s.xqin = xq;
    s.y = y[0];
    s.nrows = total;
    s.ncols_x = ncols_x;
    s.K = ncols_x;
    s.ncols = ncols_dst;
    s.ncols_dst = ncols_dst;
    s.nwarps = nwarps;
    s.rpb = rows_per_block;
    if (!plan_fused(ggml_type, x, total, ncols_x, ncols_dst, nwarps, rows_per_block, &s.plan)) {
        if (int st = plan_mmvq(ggml_type, total, ncols_x, ncols_dst, nwarps, rows_per_block,
                               kModeQ81, &s.plan))
            return st;
    }
    c->steps.push_back(s);
    return ANVIL_OK;
}

int anvil_chain_add_mmvq_glu(anvil_chain *c, int ggml_type, const void *W_gate, const void *W_up,
                             const void *xq, float *y, int nrows, int ncols_x, int nwarps,
                             int rows_per_block) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (int s = check_glu_args(ggml_type, W_gate, W_up, xq, y, nrows, ncols_x)) return s;
    ChainStep s = {};
    s.type = ggml_type;
    s.W = W_gate;
    s.W2 = W_up;
    s.xqin = xq;
    s.y = y;
    s.nrows = nrows;
    s.ncols_x = ncols_x;
    s.ncols_dst = 1;
    s.nwarps = nwarps;
    s.rpb = rows_per_block;
    if (int st = plan_mmvq(ggml_type, nrows, ncols_x, 1, nwarps, rows_per_block, kModeGLU, &s.plan))
        return st;
    c->steps.push_back(s);
    return ANVIL_OK;
}

static int run_steps(anvil_chain *c, bool use_pdl, cudaStream_t st) {
    for (size_t i = 0; i < c->steps.size(); ++i) {
        const ChainStep &s = c->steps[i];
        const unsigned flags = (use_pdl && i > 0) ? ANVIL_FLAG_PDL : 0u;
        int r;
        if (s.quantize) {
            r = launch_quantize(s.x, s.xq, s.K, s.ncols, flags, st);
        } else if (s.plan.mode == kModeGLU) {
            r = launch_glu(s.plan, s.W, s.W2, s.xqin, s.y, s.nrows, s.ncols_x, flags, st, c->share);
        } else if (s.fused && s.plan.mode == kModeF32) {
            r = launch_mmvq_segs(s.plan, s.segs, s.x, nullptr, s.ncols_x, flags, st, c->share);
        } else if (s.fused) {
            r = launch_quantize(s.x, s.xq, s.K, s.ncols, flags, st);
            if (!r) r = launch_mmvq_segs(s.plan, s.segs, s.xq, nullptr, s.ncols_x,
                                         use_pdl ? ANVIL_FLAG_PDL : 0u, st, c->share);
        } else {
            r = launch_mmvq_segs(s.plan, s.segs, s.xqin, nullptr, s.ncols_x, flags, st, c->share);
        }
        if (r) return r;
    }
    return ANVIL_OK;
}

int anvil_chain_instantiate(anvil_chain *c, int use_pdl, anvil_stream_t stream) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    if (c->exec) return fail(ANVIL_ERR_INVALID, "chain already instantiated");
    if (c->steps.empty()) return fail(ANVIL_ERR_INVALID, "empty chain");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (!st) return fail(ANVIL_ERR_INVALID, "graph capture needs a non-default stream");
    cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamBeginCapture");
    const int r = run_steps(c, use_pdl != 0, st);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(st, &g);
    if (r) {
        if (g) cudaGraphDestroy(g);
        return r;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        return cuda_fail(e, "cudaGraphInstantiate");
    }
    c->graph = g;
    c->exec = ex;
    return ANVIL_OK;
}

int anvil_chain_launch(anvil_chain *c, anvil_stream_t stream) {
    if (!c) return fail(ANVIL_ERR_INVALID, "null chain");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (c->exec) {
        cudaError_t e = cudaGraphLaunch(c->exec, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGraphLaunch");
        return ANVIL_OK;
    }
    return run_steps(c, false, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------------
// Allocation-free fp32 GEMV (anvil_mmvq_f32_noalloc).  Same result as anvil_mmvq_f32's
// two-launch path -- quantise x to Q8_1, then the Q8_1 GEMV -- but the Q8_1 intermediate
// lives in the file-scope device buffer below instead of caller scratch, so the call
// allocates no device memory and needs none from the caller.  It serves callers that may
// not allocate while decoding: hosts that reserve their whole device budget before the
// first token (llama.cpp's ggml allocator sizes its compute buffers up front, and a later
// cudaMalloc can fail or fragment what is left), and hosts on a latency-critical path,
// where cudaFree would synchronise the whole device.
//
// Set-up: the first call in each CUDA context (one per device unless a context is reset),
// with that device current, looks the buffer's device address up with cudaGetSymbolAddress
// and keeps it, keyed by the context's unique id; make that first call outside any stream
// capture.  After cudaDeviceReset the next call finds a new context id and looks the address
// up again.  Nothing in the buffer has to start at zero: the quantiser writes every byte the
// GEMV then reads.  All calls on one device share the buffer, so calls whose launches
// overlap (different streams without ordering between them, or several host threads) race
// on it: order them on one stream or with events.
// ---------------------------------------------------------------------------------
namespace anvil {

// 1 MiB = ncols * (K/32) * 36 bytes of Q8_1 blocks: K up to 932,064 for one column,
// 116,480 for eight.
constexpr size_t kStaticXqBytes = size_t(1) << 20;
static __device__ __align__(256) uint8_t g_static_xq[kStaticXqBytes];

struct StaticXqEntry {
    unsigned long long ctx_id;  // 0: not looked up yet
    void *addr;
};
static StaticXqEntry g_static_xq_addr[kMaxDevices];  // device address of g_static_xq, per device
static std::mutex g_static_xq_mu;

// Unique id of the calling thread's current context (driver API cuCtxGetCurrent + cuCtxGetId,
// reached through the runtime's entry-point table, so no link against libcuda).
static int current_context_id(unsigned long long *id) {
    using GetCurrent = CUresult (*)(CUcontext *);
    using GetId = CUresult (*)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    if (!get_current || !get_id) {
        void *a = nullptr, *b = nullptr;
        cudaDriverEntryPointQueryResult qa, qb;
        cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa);
        if (e == cudaSuccess) e = cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDriverEntryPoint");
        if (qa != cudaDriverEntryPointSuccess || qb != cudaDriverEntryPointSuccess || !a || !b)
            return fail(ANVIL_ERR_UNSUPPORTED, "driver lacks cuCtxGetCurrent / cuCtxGetId");
        get_current = reinterpret_cast<GetCurrent>(a);
        get_id = reinterpret_cast<GetId>(b);
    }
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx)
        return fail(ANVIL_ERR_CUDA, "no current CUDA context");
    if (get_id(ctx, id) != CUDA_SUCCESS) return fail(ANVIL_ERR_CUDA, "cuCtxGetId failed");
    return ANVIL_OK;
}

// Device address of g_static_xq on `dev` (which must be the current device), looked up once
// per context.
static int static_xq_addr(int dev, void **out) {
    std::lock_guard<std::mutex> lock(g_static_xq_mu);
    // a runtime call first, so the device's primary context exists and is current
    void *ptr = nullptr;
    unsigned long long id = 0;
    if (!g_static_xq_addr[dev].ctx_id) {
        const cudaError_t e = cudaGetSymbolAddress((void **)&ptr, g_static_xq);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_static_xq)");
        if (int s = current_context_id(&id)) return s;
        g_static_xq_addr[dev] = {id, ptr};
    } else {
        if (int s = current_context_id(&id)) return s;
        if (id != g_static_xq_addr[dev].ctx_id) {  // the context was reset: look up again
            const cudaError_t e = cudaGetSymbolAddress((void **)&ptr, g_static_xq);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_static_xq)");
            g_static_xq_addr[dev] = {id, ptr};
        }
    }
    *out = g_static_xq_addr[dev].addr;
    return ANVIL_OK;
}

}  // namespace anvil

extern "C" int anvil_mmvq_f32_noalloc(int ggml_type, const void *W, const float *x, float *y,
                                      int nrows, int ncols_x, int ncols_dst, int nwarps,
                                      int rows_per_block, anvil_stream_t stream) {
    if (!x) return fail(ANVIL_ERR_INVALID, "null pointer argument");
    if (ncols_x <= 0 || ncols_x % 32 != 0)
        return fail(ANVIL_ERR_INVALID, "K=%d is not a positive multiple of 32", ncols_x);
    if (ncols_dst < 1) return fail(ANVIL_ERR_INVALID, "ncols=%d", ncols_dst);
    const size_t need = size_t(ncols_dst) * size_t(ncols_x / 32) * kQ8_1Bytes;
    if (need > kStaticXqBytes)
        return fail(ANVIL_ERR_INVALID,
                    "anvil_mmvq_f32_noalloc: the Q8_1 activation needs %zu bytes (%d columns of "
                    "K=%d), more than its %zu-byte static buffer; use anvil_mmvq_f32 with caller "
                    "scratch", need, ncols_dst, ncols_x, kStaticXqBytes);
    int dev;
    if (int s = current_device(&dev)) return s;
    void *xq = nullptr;
    if (int s = static_xq_addr(dev, &xq)) return s;
    if (int s = check_mmvq_ptrs(ggml_type, W, xq, y)) return s;
    Plan p;
    if (int s = plan_mmvq(ggml_type, nrows, ncols_x, ncols_dst, nwarps, rows_per_block, kModeQ81, &p))
        return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (int s = launch_quantize(x, xq, ncols_x, ncols_dst, 0, st)) return s;
    return launch_mmvq(p, W, xq, y, nullptr, nrows, ncols_x, ANVIL_FLAG_PDL, st);
}
