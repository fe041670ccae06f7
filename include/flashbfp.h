/*
 * flashbfp.h — C ABI of libflashbfp.so, the B200 (sm_100a) OABF weight-streaming library.
 *
 * OABF (outlier-aware block floating point) packs a weight matrix W[N_out, K_in] as
 * 16-element blocks along K: one int8 shared exponent, one 16-bit sign word and two
 * 32-bit words of 4-bit mantissas per block (11 bytes per 16 weights), plus the
 * values above an adaptive threshold as a COO list. Block b = n * (Kpad/16) + kb covers
 * W[n, 16*kb : 16*kb + 16]. Packed arrays use exactly the byte layout of the reference
 * compressor (Ragu-123/FlashBFP flash_bfp/compressor.py:109-117).
 *
 * Conventions for every entry point:
 *   - all pointers are DEVICE pointers unless stated otherwise; sizes are element counts;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - the return value is an fbfp_status; FBFP_OK is 0. On error, fbfp_last_error()
 *     returns a message for the calling thread. Nothing falls back to the CPU;
 *   - calls only enqueue work on `stream` (no host synchronisation) unless stated.
 */
#ifndef FLASHBFP_H
#define FLASHBFP_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum fbfp_status {
  FBFP_OK = 0,
  FBFP_ERR_ARG = 1,          /* invalid argument (null pointer, bad size, bad dtype)        */
  FBFP_ERR_UNSUPPORTED = 2,  /* valid but unsupported configuration (e.g. block size != 16)  */
  FBFP_ERR_CUDA = 3,         /* a CUDA runtime call or kernel launch failed                  */
  FBFP_ERR_ALIGN = 4,        /* pointer alignment requirement not met                        */
  FBFP_ERR_TIMEOUT = 5       /* a bounded device-side wait gave up                           */
};

enum fbfp_dtype { FBFP_F32 = 0, FBFP_BF16 = 1, FBFP_F16 = 2 };

/* Library identity. */
int fbfp_abi_version(void);
const char* fbfp_status_string(int status);
const char* fbfp_last_error(void);

/* ------------------------------------------------------------------------------------
 * Dequantisation (bit-exact).
 * Replaces the dequantisation in _cpu_fallback_gemm (flash_bfp/triton_kernel.py:94-125)
 * and in oabf_gemm_kernel (triton_kernel.py:68-80): w = (sign ? -1 : +1) * fl(m/15) * 2^e.
 * Writes out[n * ldo + k] for n < n_out, k < k_in (the [:C_orig, :R_orig] crop). For
 * out_dtype FBFP_BF16 the fp32 value is rounded to bf16, which equals both reference
 * paths. sign=1 with m=0 gives -0.0 exactly as the reference formula does.
 * ---------------------------------------------------------------------------------- */
int fbfp_dequant(const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                 int64_t n_out, int64_t k_in, int64_t kpad,
                 int out_dtype, void* out, int64_t ldo, void* stream);

/* Write outliers into a dequantised matrix: out[c * ldo + r] = (float)value for every
 * COO entry with r = g % kpad < k_in and c = g / kpad < n_out, g = block_idx*16 + offset.
 * Follows the outlier re-insertion of flash_bfp main.py:100-113 and the index
 * derivation of OABFLinear.load_from_weight (triton_kernel.py:261-277). `value_f16`
 * holds IEEE half bit patterns. */
int fbfp_scatter_outliers(const int32_t* block_idx, const int32_t* offset, const uint16_t* value_f16,
                          int64_t count, int64_t kpad, int64_t n_out, int64_t k_in,
                          int out_dtype, void* out, int64_t ldo, void* stream);

/* ------------------------------------------------------------------------------------
 * Outlier layout for the fused GEMV/GEMM (built once at load time).
 * Replaces the (r, c, v) cache of OABFLinear.load_from_weight (triton_kernel.py:254-291).
 * Entries are grouped by (128-row group, 256-column stage); each entry is one uint32:
 * bits 0-15 fp16 value, bits 16-23 column within the stage, bits 24-30 row within the
 * group. `seg_ptr` (the outlier index, fbfp_outlier_tiles_index_words(npad, kpad) int32
 * words) holds the n_groups * n_stages + 1 segment pointers (group-major; n_groups =
 * ceil(npad/128), n_stages = ceil(kpad/256)), padded to a multiple of 4 words, followed by
 * one 68-word block per segment: 136 uint16 row starts relative to the segment start (entry
 * 128 = segment size). The COO list must be in ascending flat-index order, as the
 * compressor emits it. `entries` must have room for count rounded up to a multiple of 4
 * (the GEMV kernels copy whole 16-byte groups of it).
 * fbfp_outlier_tiles_scratch_bytes gives the scratch size the build needs.
 * ---------------------------------------------------------------------------------- */
int64_t fbfp_outlier_tiles_index_words(int64_t npad, int64_t kpad);
int64_t fbfp_outlier_tiles_scratch_bytes(int64_t npad, int64_t kpad);
int fbfp_outlier_tiles_build(const int32_t* block_idx, const int32_t* offset, const uint16_t* value_f16,
                             int64_t count, int64_t kpad, int64_t npad, int64_t n_out, int64_t k_in,
                             uint32_t* entries, int32_t* seg_ptr, void* scratch, void* stream);

/* ------------------------------------------------------------------------------------
 * Fused dequant-GEMV for decode, 1 <= M <= 16 tokens.
 * Replaces oabf_gemm (triton_kernel.py:130-195) for small M and, when `entries` is
 * non-null, the outlier SpMV (triton_kernel.py:339-356) and bias add (:358-362) of
 * OABFLinear.forward:  y[m, n] = sum_k x[m, k] * W_full[n, k] + bias[n], fp32 accumulate.
 *   x: [M, K] row-major (leading dim ldx), dtype x_dtype (FBFP_BF16, FBFP_F32 or FBFP_F16;
 *      fp32/fp16 activations are rounded to bf16 for the tensor-core product);
 *   y: [M, n_out] row-major (leading dim ldy), dtype y_dtype (any fbfp_dtype);
 *   bias: optional [n_out] of dtype bias_dtype (NULL for none);
 *   workspace: fbfp_gemv_workspace_bytes(M, npad) bytes of ZERO-initialised device memory
 *      (error word, arrival counters, fp32 partial sums). The kernel returns it to zero
 *      before it exits, so it can be reused by later calls on the same stream, also for
 *      smaller matrices; concurrent calls must use distinct workspaces.
 * Matrices with kpad a multiple of 256 (16 blocks per row stage) and 16-byte aligned
 * packed arrays run on the persistent tcgen05 kernel; other shapes on the mma.sync kernel.
 * ---------------------------------------------------------------------------------- */
int64_t fbfp_gemv_workspace_bytes(int64_t m, int64_t npad);
/* Synchronises `stream` and reports FBFP_ERR_TIMEOUT if a kernel that used `workspace`
 * gave up a bounded device-side wait since the last check (then clears the record).
 * workspace NULL: the built-in scratch of fbfp_gemv_noalloc on the current device. */
int fbfp_gemv_check(void* workspace, void* stream);
int fbfp_gemv(const void* x, int x_dtype, int64_t m, int64_t ldx,
              const int8_t* exponents, const int16_t* signs, const int32_t* payload,
              int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
              const uint32_t* entries, const int32_t* seg_ptr,
              const void* bias, int bias_dtype,
              void* y, int y_dtype, int64_t ldy,
              void* workspace, void* stream);

/* Same as fbfp_gemv for weights already resident: the packed arrays, `entries` and `seg_ptr`
 * must not have been written by the kernel that immediately precedes this call in `stream`
 * (any other kernel in between, e.g. fbfp_stream_fence, suffices). The tcgen05 kernel is launched
 * with programmatic stream serialisation and then fetches its first weight stages while the
 * previous kernel finishes (fbfp_gemv also overlaps that kernel's tail, but reads no global
 * memory until it has completed). No counterpart in the reference. */
int fbfp_gemv_resident(const void* x, int x_dtype, int64_t m, int64_t ldx,
                       const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                       int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                       const uint32_t* entries, const int32_t* seg_ptr,
                       const void* bias, int bias_dtype,
                       void* y, int y_dtype, int64_t ldy,
                       void* workspace, void* stream);
/* Row-parallel tensor-parallel GEMV with the exchange fused in: every rank of the all-reduce
 * handle (fbfp_allreduce_create, all peers opened) calls it on its K slice of the matrix (same
 * n_out, m and unit split on every rank), and every rank gets
 *   y[m, n] = bias[n] + sum over ranks r (in rank order) of that rank's x_r @ W_r^T,
 * identical bits on all ranks. The epilogue that finishes a row pushes the row's fp32 partials
 * into every peer's exchange buffer over NVLink and sums the peers' partials as they arrive, so
 * the exchange overlaps the rest of the GEMV and costs no separate launch. Replaces, for the
 * row-parallel (o, down) shards, packed GEMV + dist.all_reduce of the partial outputs + bias.
 * Requires the tensor-core GEMV (x bf16, 16-byte aligned operands, kpad a multiple of 256, k_in
 * and ldx multiples of 8) and m * n_out <= the handle's max_elems. resident: as
 * fbfp_gemv_resident. A wait that gave up (a peer that never arrives within the handle's timeout,
 * fbfp_allreduce_set_timeout) is reported by fbfp_gemv_check on the workspace; the handle is
 * unusable after that. The handle's
 * call counter is shared with fbfp_allreduce_sum_f32, so both may be mixed on one stream, in the
 * same order on every rank. No counterpart in the reference (single-GPU only). */
int fbfp_gemv_allreduce(const void* x, int x_dtype, int64_t m, int64_t ldx,
                        const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                        int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                        const uint32_t* entries, const int32_t* seg_ptr,
                        const void* bias, int bias_dtype,
                        void* y, int y_dtype, int64_t ldy,
                        void* workspace, void* allreduce, int resident, void* stream);
/* ------------------------------------------------------------------------------------
 * Stage records: the decode GEMV's own device layout of a packed matrix and its outliers, built
 * once at load time from the reference arrays and the outlier layout above (kpad a multiple of
 * 256). A table of int64 byte offsets (one per record plus the end, padded to 256 bytes), then
 * one record per (128-row group g, 256-column stage st), index g * (kpad / 256) + st: every
 * weight as the 5-bit value 16 + s*m (80 bits per 16-weight block, as the reference's signs +
 * nibbles), each block's exponent biased by 134, then the record's outliers (136 uint16 row
 * starts and the uint32 entries of fbfp_outlier_tiles_build). So 11 bytes per 16 weights plus
 * 4 per outlier, and one bulk copy brings a record's weights and outliers together.
 * fbfp_records_bytes(npad, kpad, outliers) is the size to allocate (outliers = the COO count; an
 * upper bound on what the build writes) and fbfp_records_scratch_bytes the scratch the build
 * needs; both return -1 unless kpad is a multiple of 256. `records` must be 256-byte aligned.
 * Exponents above 120 (the compressor emits at most -3) cannot be biased into a byte:
 * `bad_exponents` (optional device int32, caller zeroes it) counts such blocks. Replaces the
 * GPU-side widening of the packed arrays and the outlier cache of OABFLinear.load_from_weight
 * (flash_bfp/triton_kernel.py:232-291).
 * ---------------------------------------------------------------------------------- */
int64_t fbfp_records_bytes(int64_t npad, int64_t kpad, int64_t outliers);
int64_t fbfp_records_scratch_bytes(int64_t npad, int64_t kpad);
int fbfp_records_build(const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                       int64_t npad, int64_t kpad, const uint32_t* entries, const int32_t* seg_ptr,
                       int64_t outliers, void* records, int32_t* bad_exponents, void* scratch,
                       void* stream);

/* Decode GEMV on stage records: the same product as fbfp_gemv (y = x W_full^T + bias, fp32
 * accumulate, the records' outliers included) for bf16 x (16-byte aligned, ldx and k_in
 * multiples of 8) and 1 <= m <= 16. Replaces oabf_gemm (triton_kernel.py:130-195, the
 * oabf_gemm_kernel tiles of :22-86) and the outlier SpMV (:339-356) and bias add (:358-362) of
 * OABFLinear.forward. `workspace` as for fbfp_gemv.
 * allreduce: NULL, or an all-reduce handle whose peers are all open to fuse the row-parallel
 * exchange into the kernel as fbfp_gemv_allreduce does (y = bias + sum over ranks, in rank
 * order, of the ranks' partial products; same bits on every rank).
 * flags: FBFP_GEMV_RESIDENT as fbfp_gemv_resident (the records were not written by the kernel
 * just before this call in `stream`, so the first records are fetched while that kernel
 * finishes); FBFP_GEMV_DENSE_ONLY leaves the outliers out (the dense part, as oabf_gemm).
 * One token (m = 1) runs on the CUDA cores (fp32 FMAs), more on the tensor cores (tcgen05, one
 * M=128 x N=16 x K=16 MMA per 16-weight block column); FBFP_GEMV_TENSOR_CORES sends one token to
 * the tensor cores too. */
enum { FBFP_GEMV_RESIDENT = 1, FBFP_GEMV_DENSE_ONLY = 4, FBFP_GEMV_TENSOR_CORES = 8 };
int fbfp_gemv_records(const void* x, int64_t m, int64_t ldx, const void* records,
                      int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                      const void* bias, int bias_dtype, void* y, int y_dtype, int64_t ldy,
                      void* workspace, void* allreduce, int flags, void* stream);

/* Launches an empty kernel on `stream`: placed after the kernels that write a matrix's packed
 * arrays, it makes the matrix resident for fbfp_gemv_resident. No counterpart in the reference. */
int fbfp_stream_fence(void* stream);

/* ------------------------------------------------------------------------------------
 * Fused dequant-GEMM for prefill (many tokens), tcgen05 tensor cores.
 * Replaces oabf_gemm (triton_kernel.py:130-195, the oabf_gemm_kernel tiles of :22-86) at
 * prefill sizes and, when `entries` is non-null, the outlier SpMV (triton_kernel.py:339-356)
 * and bias add (:358-362) of OABFLinear.forward; same result as fbfp_gemv:
 *   y[m, n] = sum_k x[m, k] * W_full[n, k] + bias[n], fp32 accumulate, any m >= 1.
 * Requirements: x bf16 (16-byte aligned, ldx and k_in multiples of 8); kpad a multiple of
 * 256; 16-byte aligned packed arrays. Outlier values enter the tensor-core product rounded to
 * bf16 (as the reference's bf16 index_add rounds them).
 * workspace: at least 256 bytes of zero-initialised device memory (its first word records a
 * bounded device-side wait that gave up; fbfp_gemv_check reads and clears it); the workspace
 * of fbfp_gemv serves. Tiles of 128 output rows x 256 tokens; no cross-CTA reduction.
 * ---------------------------------------------------------------------------------- */
int fbfp_gemm_prefill(const void* x, int x_dtype, int64_t m, int64_t ldx,
                      const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                      int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                      const uint32_t* entries, const int32_t* seg_ptr,
                      const void* bias, int bias_dtype,
                      void* y, int y_dtype, int64_t ldy,
                      void* workspace, void* stream);

/* ------------------------------------------------------------------------------------
 * Two-pass prefill for many tokens (bf16 in; bf16 or fp32 out): the packed matrix is expanded into a bf16
 * scratch holding 15 x its dequantised values, then a cuBLASLt bf16 GEMM (fp32 accumulation,
 * alpha = 1/15, bias in its epilogue) gives
 *   y[m, n] = sum_k x[m, k] * W_full[n, k] + bias[n]
 * as fbfp_gemm_prefill does, with the same bf16 operand: dense elements s * m * 2^e exactly and
 * outliers bf16(15 v) (the reference's oabf_gemm, triton_kernel.py:130-195, rounds the
 * dequantised weight s * fl(m / 15) * 2^e to the activation dtype instead). The outliers come
 * as the tile-grouped index of fbfp_outlier_tiles_build (entries, seg_ptr, built for npad rows;
 * written inside the expansion) or, with entries or seg_ptr null, as the COO list of the
 * compressor (block_idx, offset, fp16 value bits; count may be 0; a separate scatter).
 * Requirements: x bf16, y and bias (optional) both bf16 or both fp32 (y_dtype), all 16-byte
 * aligned with 16-byte row strides (ldx a multiple of 8); scratch
 * 256-byte aligned, at least fbfp_gemm_expanded_scratch_bytes(n_out, kpad) bytes (the expanded
 * matrix, n_out x kpad bf16, then the GEMM's workspace). No counterpart in the reference.
 * ---------------------------------------------------------------------------------- */
int64_t fbfp_gemm_expanded_scratch_bytes(int64_t n_out, int64_t kpad);
int fbfp_gemm_expanded(const void* x, int64_t m, int64_t ldx, const int8_t* exponents,
                       const int16_t* signs, const int32_t* payload, int64_t n_out, int64_t k_in,
                       int64_t kpad, const int32_t* block_idx, const int32_t* offset,
                       const uint16_t* value_f16, int64_t count, const uint32_t* entries,
                       const int32_t* seg_ptr, int64_t npad, const void* bias, void* y,
                       int y_dtype, int64_t ldy, void* scratch, int64_t scratch_bytes, void* stream);

/* The expansion alone: out[n * ldo + k] = bf16 of 15 x the dequantised W_full[n, k] for
 * n < n_out, k < k_in (dense s * m * 2^e exactly, outliers bf16(15 v)); ldo a multiple of 8,
 * out 16-byte aligned. */
int fbfp_expand_x15(const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                    int64_t n_out, int64_t k_in, int64_t kpad, const int32_t* block_idx,
                    const int32_t* offset, const uint16_t* value_f16, int64_t count,
                    const uint32_t* entries, const int32_t* seg_ptr, int64_t npad,
                    void* out, int64_t ldo, void* stream);

/* ------------------------------------------------------------------------------------
 * Tensor-parallel exchange: one-shot fp32 sum all-reduce over NVLink peer memory (plain peer
 * stores and loads, bounded waits). Replaces the collective of the row-parallel linears (the
 * reference has no multi-GPU path; this is the exchange of the sharded o/down projections).
 * One handle per rank and device: fbfp_allreduce_create allocates the rank's buffer and writes
 * its CUDA IPC handle (fbfp_allreduce_ipc_handle_bytes() bytes) to ipc_handle_out; exchange
 * the handles between ranks (any host channel) and call fbfp_allreduce_open_peer for every
 * other rank. fbfp_allreduce_sum_f32 then replaces y[0..n) (n <= max_elems) on every rank with
 * the sum over ranks, in rank order (bit-identical on every rank); all ranks must make the same
 * calls in the same order. A wait that gives up (a rank that never arrives within the handle's
 * timeout: two seconds unless fbfp_allreduce_set_timeout changed it, between 1 us and 60 s) is
 * reported by fbfp_allreduce_check as FBFP_ERR_TIMEOUT. Graph-capturable.
 * ---------------------------------------------------------------------------------- */
int64_t fbfp_allreduce_ipc_handle_bytes(void);
int fbfp_allreduce_create(int world, int rank, int64_t max_elems, void** handle,
                          void* ipc_handle_out);
int fbfp_allreduce_open_peer(void* handle, int peer, const void* ipc_handle);
int fbfp_allreduce_sum_f32(void* handle, float* y, int64_t n, void* stream);
int fbfp_allreduce_set_timeout(void* handle, int64_t timeout_us);
int fbfp_allreduce_check(void* handle, void* stream);
int fbfp_allreduce_destroy(void* handle);

/* fbfp_gemv without a caller workspace. No counterpart in the reference: it exists for
 * callers that cannot allocate device memory — a plugin inside a host application that owns
 * all GPU memory through its own pool and forbids stray cudaMalloc calls, or a thin
 * foreign-language binding with no device allocator to hand over a workspace.
 * Same arguments and results as fbfp_gemv, minus `workspace`: the scratch lives in an 8 MiB
 * array compiled into the library (every GPU that loads the library holds it until exit).
 * Returns FBFP_ERR_ARG when fbfp_gemv_workspace_bytes(m, npad) exceeds 8 MiB (about 130,000
 * padded rows at m = 16); every argument is checked before anything is enqueued. Allocates
 * nothing; each call clears the part of the array it uses except its error word: a bounded
 * device-side wait that gave up stays recorded there until fbfp_gemv_check(NULL, stream)
 * reports it (FBFP_ERR_TIMEOUT) and clears it. The first call on a device (and the first after
 * the device's context changes) looks up the array's device address (cudaGetSymbolAddress):
 * make that first call outside any stream capture. All calls on a device share the one
 * array, so calls that overlap on the GPU (other streams, other host threads) race and
 * corrupt each other's results: serialise them. */
int fbfp_gemv_noalloc(const void* x, int x_dtype, int64_t m, int64_t ldx,
                      const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                      int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                      const uint32_t* entries, const int32_t* seg_ptr,
                      const void* bias, int bias_dtype,
                      void* y, int y_dtype, int64_t ldy, void* stream);

/* ------------------------------------------------------------------------------------
 * GPU compressor. Replaces OABFCompressor.compute_dynamic_threshold and
 * compress_matrix (flash_bfp/compressor.py:11-117) with identical output bytes.
 * w: [n_out, k_in] row-major (leading dim ldw) of dtype w_dtype (FBFP_F32 / FBFP_BF16);
 * all arithmetic follows the reference's dtype-following torch semantics.
 *
 * Step 1, fbfp_compress_threshold: kurtosis-adaptive threshold written to *thr_out
 *   (device float). scratch: fbfp_compress_scratch_bytes(...) bytes.
 * Step 2, fbfp_compress_pack: packed exponents/signs/payload for the padded
 *   [npad, kpad] matrix, the outlier bitmask per block (scratch) and per-row outlier
 *   counts; then the exclusive scan of the row counts into row_offsets[npad + 1]
 *   (row_offsets[npad] = total outlier count).
 * Step 3, fbfp_compress_outliers: the COO list in ascending flat-index order
 *   (block_idx, offset, fp16 value) into arrays of row_offsets[npad] entries.
 * `thr` points to the device float threshold used by steps 2 and 3.
 * ---------------------------------------------------------------------------------- */
int64_t fbfp_compress_scratch_bytes(int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad);
int fbfp_compress_threshold(const void* w, int w_dtype, int64_t n_out, int64_t k_in, int64_t ldw,
                            float* thr_out, void* scratch, void* stream);
int fbfp_compress_pack(const void* w, int w_dtype, int64_t n_out, int64_t k_in, int64_t ldw,
                       int64_t kpad, int64_t npad, const float* thr,
                       int8_t* exponents, int16_t* signs, int32_t* payload,
                       int32_t* row_offsets, void* scratch, void* stream);
int fbfp_compress_outliers(const void* w, int w_dtype, int64_t n_out, int64_t k_in, int64_t ldw,
                           int64_t kpad, int64_t npad, const int32_t* row_offsets,
                           int32_t* block_idx, int32_t* offset, uint16_t* value_f16,
                           void* scratch, void* stream);

/* ------------------------------------------------------------------------------------
 * Gemma-3 decoding around the OABF linears (csrc/decode.cu; no counterpart in the reference,
 * which runs these parts through Hugging Face modules). bf16 activations in rows: m tokens, row r
 * at position *pos + r (a prompt chunk, or m = 1 per decoded token); token ids (int64) and the
 * position (int32) are read from device memory, so a token step replays from one CUDA graph.
 * RMSNorm: bf16(x * rsqrt(mean(x^2) + eps) * (1 + w)), fp32 inside. 1 <= m <= 65535.
 *
 * fbfp_embed: out[r] = bf16(table[tok[r]] * bf16(scale)); an id outside [0, vocab) sets *err = 1.
 * fbfp_rmsnorm: y[r] = RMSNorm(x[r]; w) over `hidden` (<= 12000) values.
 * fbfp_post_residual_norm: h = bf16(resid[r] + RMSNorm(y[r]; w_post)); resid[r] = h; x_next[r] =
 *   RMSNorm(h; w_pre) (the post-norm, residual add and next pre-norm between a layer's halves).
 * fbfp_qk_rope_cache: on each fused q|k|v row (nh + 2 nkv heads of hd), RMSNorm of every q and
 *   k head, the rotary embedding with the bf16 cos/sin rows at the row's position (tables
 *   [max_ctx][hd]), q to q_out [m][nh][hd], k and v appended to the caches [nkv][max_ctx][hd];
 *   a position outside [0, max_ctx) sets *err = 2 and writes nothing for that row.
 * fbfp_decode_attention: per row and q head (GQA: kv head = head / (nh / nkv)),
 *   softmax(q k^T * scaling) v over cache positions [lo, p] in fp32, p the row's position and
 *   lo = p - window + 1 when window > 0, else 0 (causal); hd a multiple of 8 up to 256,
 *   max_ctx + 8 hd <= 10000, q and caches 16-byte aligned.
 * fbfp_geglu: out[r][i] = bf16(bf16(gelu_tanh(gate[r][i])) * up[r][i]) for rows [gate | up].
 * fbfp_advance_position: *pos += m.
 *
 * One new token per sequence (a batch of b sequences; b = 1 for a single one): row r is sequence
 * r at its own position pos[r], with its own caches at k_cache + r * seq_stride (elements; at
 * least nkv * max_ctx * hd apart).
 * fbfp_decode_attention_step: fbfp_qk_rope_cache followed by fbfp_decode_attention for such rows
 *   in one launch (the q/k norm, rotation and cache append folded into the attention, which is
 *   split over positions in ranges of 64 and merged by the last CTA of each head and row); out
 *   [b][nh][hd] (hd a multiple of 16 up to 256). `scratch`:
 *   fbfp_decode_attention_step_scratch_bytes(b, nh, hd, max_ctx) bytes,
 *   16-byte aligned and zeroed once before the first call (every call leaves its counters at
 *   zero). A position outside [0, max_ctx) sets *err = 2 and skips that row.
 * fbfp_advance_positions: pos[r] += 1 for r < b (1 <= b <= 1024).
 * ---------------------------------------------------------------------------------- */
int fbfp_embed(const int64_t* tok, int64_t m, const void* table, int64_t vocab, int64_t hidden,
               float scale, void* out, int32_t* err, void* stream);
int fbfp_rmsnorm(const void* x, int64_t m, const void* w, float eps, int64_t hidden, void* y,
                 void* stream);
int fbfp_post_residual_norm(const void* y, int64_t m, const void* w_post, void* resid,
                            const void* w_pre, float eps, int64_t hidden, void* x_next, void* stream);
int fbfp_qk_rope_cache(const void* qkv, int64_t m, int64_t nh, int64_t nkv, int64_t hd,
                       const void* q_norm_w, const void* k_norm_w, float eps, const void* cos_table,
                       const void* sin_table, const int32_t* pos, int64_t max_ctx, void* q_out,
                       void* k_cache, void* v_cache, int32_t* err, void* stream);
int fbfp_decode_attention(const void* q, int64_t m, const void* k_cache, const void* v_cache,
                          int64_t nh, int64_t nkv, int64_t hd, int64_t max_ctx, const int32_t* pos,
                          int64_t window, float scaling, void* out, void* stream);
int fbfp_geglu(const void* gate_up, int64_t m, int64_t inter, void* out, void* stream);
int fbfp_advance_position(int32_t* pos, int64_t m, void* stream);
int64_t fbfp_decode_attention_step_scratch_bytes(int64_t b, int64_t nh, int64_t hd, int64_t max_ctx);
int fbfp_decode_attention_step(const void* qkv, int64_t b, int64_t nh, int64_t nkv, int64_t hd,
                               const void* q_norm_w, const void* k_norm_w, float eps,
                               const void* cos_table, const void* sin_table, const int32_t* pos,
                               int64_t max_ctx, void* k_cache, void* v_cache, int64_t seq_stride,
                               int64_t window, float scaling, void* scratch, void* out, int32_t* err,
                               void* stream);
int fbfp_advance_positions(int32_t* pos, int64_t b, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FLASHBFP_H */
