// anvil_common.cuh -- GGUF block geometry, PTX helpers and status plumbing shared by
// the sm_100a kernels of libanvil.so.
//
// Block layouts are the GGUF/ggml ones (byte offsets within one block):
//   Q2_K ( 84 B / 256 weights): scales[16] @0 (low nibble scale, high nibble min of each
//                                16 weights), qs[64] @16 (2-bit), d f16 @80, dmin f16 @82
//   Q3_K (110 B / 256 weights): hmask[32] @0, qs[64] @32 (2-bit), scales[12] @96 (16 6-bit
//                                scales, minus 32), d f16 @108; q = low 2 bits - 4 unless
//                                the weight's hmask bit is set
//   Q4_K (144 B / 256 weights): d f16 @0, dmin f16 @2, scales[12] @4, qs[128] @16
//   Q5_K (176 B / 256 weights): d @0, dmin @2, scales[12] @4, qh[32] @16, qs[128] @48
//   Q6_K (210 B / 256 weights): ql[128] @0, qh[64] @128, scales int8[16] @192, d f16 @208
//   Q4_0 ( 18 B /  32 weights): d f16 @0, qs[16] @2 (nibbles; weight e < 16 = low nibble
//                                of qs[e], e >= 16 = high nibble of qs[e-16]; q - 8)
//   Q4_1 ( 20 B /  32 weights): d f16 @0, m f16 @2, qs[16] @4 (x = d q + m)
//   Q5_0 ( 22 B /  32 weights): d f16 @0, qh u32 @2 (bit e = bit 4 of weight e), qs[16] @6; q - 16
//   Q5_1 ( 24 B /  32 weights): d f16 @0, m f16 @2, qh u32 @4, qs[16] @8 (x = d q + m)
//   Q8_0 ( 34 B /  32 weights): d f16 @0, qs int8[32] @2
//   IQ4_NL ( 18 B /  32 weights): d f16 @0, qs[16] @2 (nibbles in Q4_0 order) indexing the
//                                  16 non-linear int8 levels kIQ4Levels0..3
//   IQ4_XS (136 B / 256 weights): d f16 @0, scales_h u16 @2, scales_l[4] @4, qs[128] @8;
//                                  8 groups of 32 (qs bytes 16j..16j+15, low then high
//                                  nibbles), 6-bit group scale minus 32
//   Q8_1 ( 36 B /  32 values ): d f16 @0, s f16 @2, qs int8[32] @4   (GPU layout)
// (gguf-py quants.py:396-401, 504-523, 527-549, 554-572, Q2_K / Q3_K / IQ4_NL / IQ4_XS
//  dequantize_blocks;
//  kernel_anvil/hip_codegen.py:84-85, 101-102, 385-396.)
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace anvil {

constexpr int kTypeQ4_0 = 2;
constexpr int kTypeQ4_1 = 3;
constexpr int kTypeQ5_0 = 6;
constexpr int kTypeQ5_1 = 7;
constexpr int kTypeQ8_0 = 8;
constexpr int kTypeQ8_1 = 9;
constexpr int kTypeQ2_K = 10;
constexpr int kTypeQ3_K = 11;
constexpr int kTypeQ4_K = 12;
constexpr int kTypeQ5_K = 13;
constexpr int kTypeQ6_K = 14;
constexpr int kTypeIQ2_XXS = 16;
constexpr int kTypeIQ2_XS = 17;
constexpr int kTypeIQ3_XXS = 18;
constexpr int kTypeIQ1_S = 19;
constexpr int kTypeIQ4_NL = 20;
constexpr int kTypeIQ3_S = 21;
constexpr int kTypeIQ2_S = 22;
constexpr int kTypeIQ4_XS = 23;
constexpr int kTypeIQ1_M = 29;

constexpr int kQK_K = 256;
constexpr int kQK8_1 = 32;
constexpr int kQ8_1Bytes = 36;

// Per-type geometry.  A "unit" is the slice of one weight block that one thread
// handles per visit: 64 weights (two Q8_1 blocks) for the K-quants, one 32-weight
// block for Q8_0.
template <int QT> struct QTraits;
template <> struct QTraits<kTypeQ4_K> {
    static constexpr int qk = 256, bytes = 144, units = 4, sub = 32;
};
template <> struct QTraits<kTypeQ5_K> {
    static constexpr int qk = 256, bytes = 176, units = 4, sub = 32;
};
template <> struct QTraits<kTypeQ6_K> {
    static constexpr int qk = 256, bytes = 210, units = 4, sub = 16;
};
template <> struct QTraits<kTypeQ2_K> {
    static constexpr int qk = 256, bytes = 84, units = 4, sub = 16;
};
template <> struct QTraits<kTypeQ3_K> {
    static constexpr int qk = 256, bytes = 110, units = 4, sub = 16;
};
template <> struct QTraits<kTypeQ4_0> {
    static constexpr int qk = 32, bytes = 18, units = 1, sub = 32;
};
template <> struct QTraits<kTypeQ4_1> {
    static constexpr int qk = 32, bytes = 20, units = 1, sub = 32;
};
template <> struct QTraits<kTypeQ5_0> {
    static constexpr int qk = 32, bytes = 22, units = 1, sub = 32;
};
template <> struct QTraits<kTypeQ5_1> {
    static constexpr int qk = 32, bytes = 24, units = 1, sub = 32;
};
template <> struct QTraits<kTypeIQ4_NL> {
    static constexpr int qk = 32, bytes = 18, units = 1, sub = 32;
};
template <> struct QTraits<kTypeIQ4_XS> {
    static constexpr int qk = 256, bytes = 136, units = 4, sub = 32;
};
template <> struct QTraits<kTypeIQ2_XXS> {
    static constexpr int qk = 256, bytes = 66, units = 4, sub = 32;
};
template <> struct QTraits<kTypeIQ2_XS> {
    static constexpr int qk = 256, bytes = 74, units = 4, sub = 16;
};
template <> struct QTraits<kTypeIQ2_S> {
    static constexpr int qk = 256, bytes = 82, units = 4, sub = 16;
};
template <> struct QTraits<kTypeIQ3_XXS> {
    static constexpr int qk = 256, bytes = 98, units = 4, sub = 32;
};
template <> struct QTraits<kTypeIQ3_S> {
    static constexpr int qk = 256, bytes = 110, units = 4, sub = 32;
};
template <> struct QTraits<kTypeIQ1_S> {
    static constexpr int qk = 256, bytes = 50, units = 4, sub = 32;
};
template <> struct QTraits<kTypeIQ1_M> {
    static constexpr int qk = 256, bytes = 56, units = 4, sub = 16;
};
template <> struct QTraits<kTypeQ8_0> {
    static constexpr int qk = 32, bytes = 34, units = 1, sub = 32;
};

// Device status word: bit flags set by kernels whose bounded waits gave up.  One copy per
// translation unit and device (no relocatable device code); the host reads and clears
// all of them through anvil_take_device_status().
constexpr int kStatusMbarTimeout = 1;
static __device__ int g_anvil_device_status;

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// ---- PTX wrappers --------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Makes the initialised barrier visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Gives up after `limit_ns` of wall time, sets the
// device status flag and returns false; the caller then skips the data it guarded.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) {
            atomicOr(&g_anvil_device_status, kStatusMbarTimeout);
            return false;
        }
    }
}

// Bulk (non-tensor) async copy global -> shared, completion signalled on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.  Only this CTA's shared memory is
// written (no cluster-wide delivery).
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes,
                                              uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Programmatic dependent launch controls (no-ops when launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace anvil
