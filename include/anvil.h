/*
 * anvil.h -- C ABI of libanvil.so, the B200 (sm_100a) MMVQ quantized GEMV library.
 *
 * libanvil.so replaces two things the reference (apollosenvy/kernel-anvil) drives:
 *
 *   1. llama.cpp's MMVQ device path: `quantize_q8_1` followed by
 *      `mul_mat_vec_q<type, ncols_dst>` (reached from
 *      `mul_mat_vec_q_switch_ncols_dst`, patched by patches/mmvq-smithy.patch:28-34;
 *      the reference's own kernel ABI is the generated
 *      `mmvq_<qt>_n<N>_k<K>_w<nw>_r<rpb>(weights, input_q8, output, stride_row)`,
 *      kernel_anvil/hip_codegen.py:244-251, 408-415, launched with grid
 *      (ceil(N/rpb)) and block (32, nwarps), kernel_anvil/autoforge.py:137-141).
 *   2. The smithy runtime config loader, patches/smithy-config.h:30-331
 *      (`smithy_get_bucket`, `smithy_set_model`, `smithy_load_configs`,
 *      `smithy_try_load`, `smithy_lookup`).
 *
 * Conventions shared by every entry point:
 *   - Return value: 0 (ANVIL_OK) on success, a negative anvil_status on failure.
 *     `anvil_last_error()` returns a message for the calling thread's last failure.
 *   - Device pointers are caller-owned.  Kernels write only their output buffers.
 *     Nothing in the launch path allocates device memory.
 *   - Every launch is asynchronous on the given stream (NULL = legacy default stream).
 *   - Weight matrices are raw GGUF blocks, row-major: row r of a matrix with K columns
 *     starts at byte r * (K / qk) * block_bytes.  Activation columns are contiguous:
 *     column c of a K-long input starts at element c * K (fp32) or at byte
 *     c * (K / 32) * 36 (Q8_1).  Output column c starts at element c * nrows.
 *   - ggml type ids follow ggml.h (kernel_anvil/codegen.py:22-31):
 *     Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q2_K = 10, Q3_K = 11, Q4_K = 12,
 *     Q5_K = 13, Q6_K = 14, IQ4_NL = 20, IQ4_XS = 23 (the persistent chain takes Q8_0,
 *     Q4_K, Q5_K and Q6_K).
 *   - Thread-safe: the smithy table is guarded by a reader/writer lock; the launch
 *     entry points keep no mutable shared state besides one-time function attributes.
 */
#ifndef ANVIL_H
#define ANVIL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t / CUstream, declared without the CUDA headers. */
typedef struct CUstream_st *anvil_stream_t;

#define ANVIL_ABI_VERSION 2

enum anvil_status {
    ANVIL_OK = 0,
    ANVIL_ERR_INVALID = -1,     /* bad argument: sizes, type, null pointer      */
    ANVIL_ERR_UNSUPPORTED = -2, /* valid request this build does not implement   */
    ANVIL_ERR_CUDA = -3,        /* a CUDA runtime call failed                    */
    ANVIL_ERR_ALIGN = -4,       /* a pointer is not aligned as required          */
    ANVIL_ERR_TIMEOUT = -5      /* a bounded device-side wait gave up            */
};

enum anvil_ggml_type {
    ANVIL_TYPE_Q4_0 = 2,
    ANVIL_TYPE_Q4_1 = 3,
    ANVIL_TYPE_Q5_0 = 6,
    ANVIL_TYPE_Q5_1 = 7,
    ANVIL_TYPE_Q8_0 = 8,
    ANVIL_TYPE_Q8_1 = 9,
    ANVIL_TYPE_Q2_K = 10,
    ANVIL_TYPE_Q3_K = 11,
    ANVIL_TYPE_Q4_K = 12,
    ANVIL_TYPE_Q5_K = 13,
    ANVIL_TYPE_Q6_K = 14,
    ANVIL_TYPE_IQ2_XXS = 16,
    ANVIL_TYPE_IQ2_XS = 17,
    ANVIL_TYPE_IQ3_XXS = 18,
    ANVIL_TYPE_IQ1_S = 19,
    ANVIL_TYPE_IQ4_NL = 20,
    ANVIL_TYPE_IQ3_S = 21,
    ANVIL_TYPE_IQ2_S = 22,
    ANVIL_TYPE_IQ4_XS = 23,
    ANVIL_TYPE_IQ1_M = 29
};

/* Launch flags for anvil_mmvq_ex / anvil_quantize_q8_1_ex. */
enum anvil_flags {
    /* Launch with programmatic dependent launch.  The kernel starts streaming its
     * weight tile before it waits for the preceding kernel in the stream, so the
     * weights must not be written by that kernel (true for model weights).
     * Activations and outputs are only touched after the wait. */
    ANVIL_FLAG_PDL = 1u << 0
};

/* ---- library ------------------------------------------------------------ */

int anvil_abi_version(void);
const char *anvil_last_error(void);

/* GGUF block geometry of a ggml type: values per block (qk) and bytes per block.
 * Mirrors QUANT_TYPES qk/block_size, kernel_anvil/hip_codegen.py:75-102. */
int anvil_type_geometry(int ggml_type, int *qk, int *block_bytes);

/* Bytes of one weight row of K columns, or a negative status. */
int64_t anvil_row_bytes(int ggml_type, int K);

/* ---- Q8_1 activation quantiser ------------------------------------------ */

/* Replaces llama.cpp `quantize_q8_1` (layout kernel_anvil/hip_codegen.py:392-396,
 * 36-byte block kernel_anvil/hip_codegen.py:101-102).
 * x: ncols columns of K fp32 values.  xq: ncols * (K/32) blocks of
 * {half d, half s, int8 qs[32]}.  Per 32-value block: d = max|x| / 127 (fp32),
 * qs = roundf(x / d) (0 when max|x| == 0), stored d = fp16(d), s = fp16(sum x)
 * with the sum taken in xor-butterfly order (offsets 16, 8, 4, 2, 1).
 * K % 32 == 0, x 4-byte aligned, xq 4-byte aligned. */
int anvil_quantize_q8_1(const float *x, void *xq, int K, int ncols, anvil_stream_t stream);
int anvil_quantize_q8_1_ex(const float *x, void *xq, int K, int ncols, unsigned flags,
                           anvil_stream_t stream);

/* ---- MMVQ quantized GEMV -------------------------------------------------- */

/* y[c][r] = sum_k W[r][k] * xq[c][k] for r < nrows, c < ncols_dst.
 * Replaces llama.cpp `mul_mat_vec_q<type, ncols_dst>` as launched by
 * `mul_mat_vec_q_switch_ncols_dst` (docs/llama-cpp-kernel-analysis.md:16-24, 128-148)
 * and the reference's generated kernels (kernel_anvil/hip_codegen.py:179-334).
 * ncols_x is K (the weight row length); ncols_dst is 1..8 activation columns.
 * nwarps (warps per CTA, 1..32) and rows_per_block (rows per CTA) keep their smithy
 * meaning; 0 selects the smithy table entry for (type, nrows, ncols_x), else the
 * built-in default.  rows_per_block is rounded down to 1, 2, 4 or 8 and reduced
 * further when the tile would not fit in shared memory.  When ncols_dst columns of
 * activation do not fit (K = 28672 with 6-8 columns), the call launches the columns in
 * chunks that do, each chunk reading the weights again.
 * Requirements: K % qk == 0; W 16-byte aligned; xq 4-byte aligned; y 4-byte aligned. */
int anvil_mmvq(int ggml_type, const void *W, const void *xq, float *y, int nrows, int ncols_x,
               int ncols_dst, int nwarps, int rows_per_block, anvil_stream_t stream);
int anvil_mmvq_ex(int ggml_type, const void *W, const void *xq, float *y, int nrows,
                  int ncols_x, int ncols_dst, int nwarps, int rows_per_block, unsigned flags,
                  anvil_stream_t stream);

/* GEMV from fp32 activations: y = W . dequant(Q8_1(x)), bit-identical to calling
 * anvil_quantize_q8_1 then anvil_mmvq.  When x is 16-byte aligned and the launch fits,
 * one kernel quantises x in its prologue (every CTA, from registers into shared memory)
 * and xq is not touched; otherwise the two launches run and xq receives the Q8_1 blocks.  xq is scratch of
 * ncols * (K/32) * 36 bytes whose contents are unspecified afterwards.
 * anvil_mmvq_f32_ex takes anvil_flags (ANVIL_FLAG_PDL). */
int anvil_mmvq_f32(int ggml_type, const void *W, const float *x, void *xq, float *y, int nrows,
                   int ncols_x, int ncols_dst, int nwarps, int rows_per_block,
                   anvil_stream_t stream);
int anvil_mmvq_f32_ex(int ggml_type, const void *W, const float *x, void *xq, float *y,
                      int nrows, int ncols_x, int ncols_dst, int nwarps, int rows_per_block,
                      unsigned flags, anvil_stream_t stream);

/* anvil_mmvq_f32 without caller scratch and without any device allocation: the Q8_1
 * intermediate lives in a 1 MiB static device buffer inside libanvil.  No counterpart in
 * the reference.  For hosts that may not allocate device memory while decoding (a
 * device budget reserved before the first token; cudaFree synchronising the device).
 * Limit: ncols_dst * (ncols_x/32) * 36 <= 1048576 bytes (K <= 932064 for one column,
 * 116480 for eight), else ANVIL_ERR_INVALID and nothing is launched.  Set-up: the first
 * call in each CUDA context (that device current) looks the buffer's address up with
 * cudaGetSymbolAddress and keeps it keyed by the context's id, so a call after
 * cudaDeviceReset looks it up again; make the first call outside any stream capture.  The
 * buffer needs no zeroing.  All calls on a device share it: calls whose launches overlap
 * (unordered streams, several threads) race, so order them. */
int anvil_mmvq_f32_noalloc(int ggml_type, const void *W, const float *x, float *y, int nrows,
                           int ncols_x, int ncols_dst, int nwarps, int rows_per_block,
                           anvil_stream_t stream);

/* Several GEMVs of one weight type that read the same activation (attention q/k/v,
 * ffn gate/up) in one launch: segment s multiplies W[s] (nrows[s] rows of ncols_x
 * columns) into y[s] (ncols_dst x nrows[s]), for s < nseg (1..4).  Each output equals
 * anvil_mmvq's for that matrix alone.  Replaces a run of mul_mat_vec_q launches on one
 * input (docs/decode-pipeline-breakdown.md:20-21; the fused gate/up of the reference's
 * profile, docs/vulkan-vs-rocm-analysis.md:103-106).  _f32: fp32 x as anvil_mmvq_f32
 * (quantised in the kernel when it fits, else into xq). */
int anvil_mmvq_grouped(int ggml_type, int nseg, const void *const *W, const void *xq,
                       float *const *y, const int *nrows, int ncols_x, int ncols_dst, int nwarps,
                       int rows_per_block, unsigned flags, anvil_stream_t stream);
int anvil_mmvq_grouped_f32(int ggml_type, int nseg, const void *const *W, const float *x,
                           void *xq, float *const *y, const int *nrows, int ncols_x, int ncols_dst,
                           int nwarps, int rows_per_block, unsigned flags, anvil_stream_t stream);

/* Gate/up GEMV pair with the SwiGLU product in the epilogue, one activation column:
 * y[r] = silu(g) * u with g = W_gate[r] . dequant(xq), u = W_up[r] . dequant(xq) and
 * silu(g) = g / (1 + exp(-g)), r < nrows.  g and u are each what anvil_mmvq computes for
 * its matrix alone with the same lanes per row; neither is written out.  Replaces the
 * llama.cpp decode sequence mul_mat_vec_q(gate), mul_mat_vec_q(up), GLU: the
 * "Q4_K fused (gate+SiLU)" MMVQ variant of docs/decode-pipeline-breakdown.md:40, the fused
 * gate+up launch of docs/vulkan-vs-rocm-analysis.md:103-106 and its GLU op (:135).  Both
 * matrices have ggml_type and nrows x ncols_x values; their rows must be a multiple of 16
 * bytes (Q4_K, Q5_K always; Q8_0, Q4_0 .. Q5_1, IQ4_NL when ncols_x % 256 == 0; IQ4_XS
 * when ncols_x % 512 == 0; Q2_K when ncols_x % 1024 == 0; Q3_K, Q6_K when
 * ncols_x % 2048 == 0), else ANVIL_ERR_ALIGN.
 * rows_per_block counts gate and up rows together (at least 2).  _f32: fp32 x quantised
 * into the scratch xq first (two launches, the second under ANVIL_FLAG_PDL). */
int anvil_mmvq_glu(int ggml_type, const void *W_gate, const void *W_up, const void *xq, float *y,
                   int nrows, int ncols_x, int nwarps, int rows_per_block, unsigned flags,
                   anvil_stream_t stream);
int anvil_mmvq_glu_f32(int ggml_type, const void *W_gate, const void *W_up, const float *x,
                       void *xq, float *y, int nrows, int ncols_x, int nwarps, int rows_per_block,
                       unsigned flags, anvil_stream_t stream);

/* Reads and clears the device status words of the current device: the OR of
 * anvil_device_status flags set by kernels whose bounded waits gave up (0 = none),
 * or a negative anvil_status.  Synchronous. */
enum anvil_device_status { ANVIL_DEVICE_MBAR_TIMEOUT = 1 };
int anvil_take_device_status(void);

/* Parity probe: runs the production MMVQ kernel with its integer block sums written
 * out instead of y.  sums[(c * nrows + r) * nsub + s] is the exact int32 dot of
 * sub-block s of row r with column c, where a sub-block is 32 weights (one Q8_1
 * block) for Q4_K, Q5_K, Q8_0, Q4_0 .. Q5_1, IQ4_NL and IQ4_XS (the int8 level times q8),
 * and 16 weights (one scale group) for Q2_K,
 * Q3_K and Q6_K, so nsub = K/32 or K/16.  For Q2_K/Q4_K/Q5_K and the _1 types the weight
 * operand is the unsigned quant (the min term is separate); for Q3_K it is q with its
 * offset of -4; for Q6_K q - 32; for Q4_0 / Q5_0 q - 8 / q - 16; for Q8_0 the int8 quant. */
int anvil_mmvq_block_sums(int ggml_type, const void *W, const void *xq, int32_t *sums,
                          int nrows, int ncols_x, int ncols_dst, int nwarps, int rows_per_block,
                          anvil_stream_t stream);

/* Launch geometry that anvil_mmvq would use: resolved nwarps, rows_per_block,
 * grid size and dynamic shared memory bytes. */
int anvil_mmvq_plan(int ggml_type, int nrows, int ncols_x, int ncols_dst, int nwarps,
                    int rows_per_block, int *out_nwarps, int *out_rpb, int *out_grid,
                    int *out_smem_bytes);

/* Compiled resources of the kernel anvil_mmvq would launch for this shape
 * (cudaFuncGetAttributes): registers per thread, local memory per thread (register spills),
 * maximum threads per block.  Replaces the reference's VGPR / LDS / scratch estimates
 * (kernel_anvil/profile.py:7-34, 86) with the real numbers. */
int anvil_mmvq_kernel_attributes(int ggml_type, int nrows, int ncols_x, int ncols_dst, int nwarps,
                                 int rows_per_block, int *regs_per_thread, int *local_bytes,
                                 int *max_threads_per_block);

/* ---- GEMV chain executor (native CUDA-graph runtime) ---------------------- */

/* A chain is an ordered list of quantize / MMVQ steps on fixed device buffers,
 * captured once into a CUDA graph (with programmatic dependent launch between
 * steps) and replayed per token.  It stands in for llama.cpp's per-token sequence
 * of quantize_q8_1 + mul_mat_vec_q launches (docs/decode-pipeline-breakdown.md:20-21). */
typedef struct anvil_chain anvil_chain;

anvil_chain *anvil_chain_create(void);
void anvil_chain_destroy(anvil_chain *chain);
int anvil_chain_add_quantize(anvil_chain *chain, const float *x, void *xq, int K, int ncols);
int anvil_chain_add_mmvq(anvil_chain *chain, int ggml_type, const void *W, const void *xq,
                         float *y, int nrows, int ncols_x, int ncols_dst, int nwarps,
                         int rows_per_block);
/* A GEMV step reading fp32 x (anvil_mmvq_f32 semantics: fused quantisation when it fits). */
int anvil_chain_add_mmvq_f32(anvil_chain *chain, int ggml_type, const void *W, const float *x,
                             void *xq, float *y, int nrows, int ncols_x, int ncols_dst,
                             int nwarps, int rows_per_block);
/* Grouped GEMV steps: anvil_mmvq_grouped (Q8_1 input from an earlier quantize step) and
 * anvil_mmvq_grouped_f32 semantics. */
int anvil_chain_add_mmvq_grouped(anvil_chain *chain, int ggml_type, int nseg, const void *const *W,
                                 const void *xq, float *const *y, const int *nrows, int ncols_x,
                                 int ncols_dst, int nwarps, int rows_per_block);
int anvil_chain_add_mmvq_grouped_f32(anvil_chain *chain, int ggml_type, int nseg, const void *const *W,
                                     const float *x, void *xq, float *const *y, const int *nrows,
                                     int ncols_x, int ncols_dst, int nwarps, int rows_per_block);
/* Gate/up step: anvil_mmvq_glu's launch as a chain step (reads xq, writes y). */
int anvil_chain_add_mmvq_glu(anvil_chain *chain, int ggml_type, const void *W_gate,
                             const void *W_up, const void *xq, float *y, int nrows, int ncols_x,
                             int nwarps, int rows_per_block);
/* Sizes every GEMV grid so that `kernels_per_sm` consecutive GEMVs (1..4) fit on each SM
 * together: with programmatic dependent launch the next GEMV's CTAs are then resident
 * while the current one runs and stream their first weight tiles early.  Default 1 (each
 * GEMV takes every resident slot).  Call before instantiation. */
int anvil_chain_set_coresident(anvil_chain *chain, int kernels_per_sm);
/* use_pdl: launch every step after the first with ANVIL_FLAG_PDL. */
int anvil_chain_instantiate(anvil_chain *chain, int use_pdl, anvil_stream_t stream);
/* Replays the graph (or, before instantiation, launches the steps one by one). */
int anvil_chain_launch(anvil_chain *chain, anvil_stream_t stream);
int anvil_chain_num_steps(const anvil_chain *chain);

/* ---- persistent chain: one cooperative launch per token ------------------ */

/* The per-token GEMV sequence of a decoder run by one persistent kernel, on one GPU or
 * row-sharded across several.  No counterpart kernel in the reference (its chain is a
 * stream of separate quantize_q8_1 + mul_mat_vec_q launches,
 * docs/decode-pipeline-breakdown.md:20-21); each GEMV computes what anvil_mmvq computes for
 * its rows, on the input its group stages.
 *
 * Groups: GEMVs added after a group read that group's input, which every CTA quantises to
 * Q8_1 itself with the arithmetic of anvil_quantize_q8_1.  anvil_pchain_add_group: a fixed
 * fp32 input x (ncols x K, 16-byte aligned).  anvil_pchain_add_group_chained: the output of
 * an earlier GEMV of the chain (K = its nrows_full, a multiple of 32), quantised to the Q8_1
 * quants of anvil_quantize_q8_1 with d8 kept in fp32 (not rounded to fp16), and the group's
 * results multiplied by 2^-e, e the exponent of the input column's largest magnitude (so
 * values stay in range along a chain of any length).  A chained group waits, per value and
 * bounded, only for the words it reads; there is no grid barrier.
 *
 * Outputs: every value is one 8-byte word {fp32 value (low half), uint32 epoch (high half)}
 * written with one 64-bit store; the epoch is the launch number (1, 2, ...).  A GEMV's buffer
 * holds two epochs: words [(epoch & 1) * ncols + c] * nrows_full + pos, pos = the row, or for
 * a chained source the row's position in 512-value blocks (anvil_pchain_read_output returns
 * rows in order).  y[q] = rank q's buffer for this GEMV (2 * ncols * nrows_full words,
 * zeroed, 16-byte aligned; a peer mapping from anvil_ipc_open for q != rank); with world = 1
 * y may be NULL and the chain allocates it.  Ranks: world > 1 row-shards every matrix; rank
 * r passes its rows [row0, row0 + nrows) of an nrows_full-row matrix, and writes each of its
 * output rows into every rank's buffer.  Every rank builds the same chain and launches it the
 * same number of times.
 *
 * Every wait in the kernel is bounded (anvil_set_wait_limit_ns, default 2 s); one that gives
 * up sets a flag read by anvil_pchain_take_status (2 = an input word did not arrive, 1 = a
 * weight copy did not land), later waits of the launch end at once, and the launch's
 * outputs are then wrong. */
#define ANVIL_MAX_RANKS 8
typedef struct anvil_pchain anvil_pchain;

anvil_pchain *anvil_pchain_create(int world, int rank);
void anvil_pchain_destroy(anvil_pchain *chain);
/* Both return the new group's index (>= 0) or a negative status.  A GEMV whose weight family
 * differs from the group's (Q8_0 against the K-quants) continues in a new group on the same
 * input. */
int anvil_pchain_add_group(anvil_pchain *chain, const float *x, int K, int ncols);
int anvil_pchain_add_group_chained(anvil_pchain *chain, int src_gemv);
/* A GEMV of the current group; returns its index (>= 0) or a negative status.
 * rows_per_block: rows per weight tile (0 = built-in default); lanes per row are chosen to
 * keep the most lanes busy (read back with anvil_pchain_gemv_shape). */
int anvil_pchain_add_gemv(anvil_pchain *chain, int ggml_type, const void *W, int nrows, int row0,
                          int nrows_full, uint64_t *const *y, int rows_per_block);
/* A gate/up pair of the current group (anvil_mmvq_glu's arithmetic): output row r is
 * silu(W_gate[r] . x) * (W_up[r] . x); both matrices hold the same rows, which must be a
 * multiple of 16 bytes.  rows_per_block counts rows of one matrix.  Returns the index. */
int anvil_pchain_add_glu(anvil_pchain *chain, int ggml_type, const void *W_gate, const void *W_up,
                         int nrows, int row0, int nrows_full, uint64_t *const *y,
                         int rows_per_block);
/* Parity probe: the staged activation of group `group` ({fp32 d8, 32 quants} per 32 values,
 * ncols * K/32 blocks of 36 bytes) is written to `out` by the first CTA. */
int anvil_pchain_set_group_dump(anvil_pchain *chain, int group, void *out);
/* Load balance (before anvil_pchain_instantiate): `percent` of each group's tiles (rounded
 * down to whole tiles per warp) are dealt round-robin over the grid's warps; the rest are
 * claimed one at a time, from a per-group counter, by whichever warp has room for its next
 * weight copy first.  Default 100 (only the tiles left over after whole rounds are
 * claimed); 0 claims every tile.  The outputs do not depend on it. */
int anvil_pchain_set_static_share(anvil_pchain *chain, int percent);
/* nwarps per CTA (0 = 8), CTAs per SM (0 = 1); allocates the device descriptors. */
int anvil_pchain_instantiate(anvil_pchain *chain, int nwarps, int ctas_per_sm);
/* Optional timestamps: buf holds grid * ngroups * 4 words; for each CTA and group,
 * %globaltimer when its warp 0 starts and ends its share of the group's staging, when the
 * CTA's barrier after the staging is passed, and when warp 0's tiles of the group are done. */
int anvil_pchain_set_trace(anvil_pchain *chain, uint64_t *buf);
/* One token: a cooperative launch on `stream`.  Not for stream capture. */
int anvil_pchain_launch(anvil_pchain *chain, anvil_stream_t stream);
/* Epoch of the last launch (0 before the first). */
int anvil_pchain_epoch(const anvil_pchain *chain);
/* The last launch's output of GEMV `index` on this rank, ncols x nrows_full fp32 in row
 * order, into dst (device); NaN where a word does not carry the last epoch. */
int anvil_pchain_read_output(const anvil_pchain *chain, int index, float *dst,
                             anvil_stream_t stream);
int anvil_pchain_info(const anvil_pchain *chain, int *grid, int *nwarps, int *ring_bytes,
                      int *smem_bytes, int *ngroups);
int anvil_pchain_gemv_shape(const anvil_pchain *chain, int index, int *rows_per_block,
                            int *lanes_per_row);
/* Reads and clears the persistent kernel's device status flags (current device). */
int anvil_pchain_take_status(void);

/* Bound on every device-side wait (mbarrier waits of the MMVQ kernels, the persistent
 * chain's input and weight waits) of launches made from now on; 0 restores the default 2 s.
 * At most 60 s.  No counterpart in the reference (its kernels have no waits). */
int anvil_set_wait_limit_ns(unsigned long long ns);
unsigned long long anvil_get_wait_limit_ns(void);
/* Tensor-core path of the batched GEMV: Q4_K and Q5_K launches with at least `min_cols`
 * activation columns (2..8) and no explicit nwarps / rows_per_block run as mma.sync
 * m16n8k32 int8 tiles of 16 rows (same block sums, y within fp32 rounding of the dp4a
 * kernels).  0 turns it off; default 4 (at 2 and 3 columns the dp4a kernels are faster).
 * Process-wide. */
int anvil_set_tensor_core_min_cols(int min_cols);
int anvil_get_tensor_core_min_cols(void);

/* Device buffers shared between the ranks' processes (CUDA IPC): allocate (zeroed) and
 * export a 64-byte handle; open a peer's handle into this process; close; free. */
int anvil_ipc_alloc(size_t bytes, void **ptr, void *handle);
int anvil_ipc_open(const void *handle, void **ptr);
int anvil_ipc_close(void *ptr);
int anvil_ipc_free(void *ptr);

/* ---- smithy runtime config (replaces patches/smithy-config.h) ------------ */

/* patches/smithy-config.h:44-50: <=128 -> 0, <=1024 -> 1, <=4096 -> 2, <=16384 -> 3, else 4. */
int anvil_smithy_bucket(int dim);

/* patches/smithy-config.h:70-87: remember the model path (its stem selects
 * ~/.cache/smithy/<stem>.json), clear the table and the load flags. */
void anvil_smithy_set_model(const char *path);

/* patches/smithy-config.h:89-266: parse one JSON file into the table.  Returns the
 * number of cells loaded (> 0 means the table is now active), 0 when the file
 * parsed but held no valid cell, or a negative status when unreadable / over 1 MiB. */
int anvil_smithy_load(const char *path);

/* patches/smithy-config.h:268-317: lazy load, first success wins:
 * $SMITHY_CONFIG, then $HOME/.cache/smithy/<stem>.json (stem from
 * anvil_smithy_set_model or $SMITHY_MODEL), then $HOME/.cache/smithy/default.json.
 * Returns 1 when a table is active afterwards, else 0. */
int anvil_smithy_try_load(void);

/* patches/smithy-config.h:319-331: {nwarps, rows_per_block} for
 * [type][bucket(nrows)][bucket(ncols)]; {0, 0} means "no override".
 * Triggers the lazy load.  Returns 1 when an override was found, else 0. */
int anvil_smithy_lookup(int ggml_type, int nrows, int ncols, int *nwarps, int *rows_per_block);

/* Clears the table, the model path and the load flags (test helper). */
void anvil_smithy_reset(void);

#ifdef __cplusplus
}
#endif

#endif /* ANVIL_H */
