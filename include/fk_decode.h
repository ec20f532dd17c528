/*
 * fk_decode.h -- C-ABI of the B200 (sm_100a) GQA decode-attention library.
 *
 * One query token per sequence; each query head qh attends to KV head
 * qh / G (G = q_heads / kv_heads, GQA).  out[b, qh, :] =
 *     sum_t softmax_t(q.k_t / sqrt(D) [with sink]) * v_t
 * with the sink formula of the reference's torch oracle
 * (fskernels/tilelang/tilelang_gqa_decode.py:198-203):
 *     M   = max(max_t x_t, s_aux[qh])
 *     out = sum_t e^(x_t - M) v_t / (sum_t e^(x_t - M) + e^(s_aux[qh] - M)).
 * A sequence of length 0 yields an all-zero output row (the oracle masks
 * every weight to 0, tilelang_gqa_decode.py:205).
 *
 * Conventions shared by every entry point
 *  - All pointers are device pointers except `stream` (a cudaStream_t passed
 *    as void*; NULL = legacy default stream).  Strides are in ELEMENTS.
 *  - head_dim D is 128, or 64 with f16/bf16 KV (the reference's Triton
 *    kernels take any power of two, triton_gqa_decode.py:136-152; its native
 *    kernel only 128, flash_decode_cuda.cu:168-189).  q_heads % kv_heads
 *    == 0; any group size G = q_heads / kv_heads.  Shapes below write D
 *    as 128.
 *  - The innermost (head_dim) stride of every tensor is 1; K/V base pointers
 *    and their strides in bytes must be multiples of 16 (TMA rule).
 *  - Nothing is synchronised with the host and nothing is allocated: the
 *    call enqueues one kernel on `stream` and returns.  It is safe to capture
 *    in a CUDA graph once `workspace` exists.
 *  - The workspace also carries per-(sequence, KV head) arrival counters
 *    that each launch leaves at zero; calls sharing a workspace must be
 *    stream-ordered, and a new workspace must start zeroed.
 *  - `workspace` is caller-owned device memory of at least
 *    fk_decode_workspace_bytes_gqa(...) bytes.  Its first int32 is a sticky
 *    status word (FK_STATUS_*) that kernels OR into; the caller clears it.
 *  - Return value: FK_OK or an FK_ERR_* code; fk_last_error() describes it.
 */
#ifndef FK_DECODE_H_
#define FK_DECODE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define FK_DTYPE_F16 0
#define FK_DTYPE_BF16 1
#define FK_DTYPE_E4M3 2 /* float8_e4m3fn */

/* return codes */
#define FK_OK 0
#define FK_ERR_INVALID_ARG 1
#define FK_ERR_UNSUPPORTED 2
#define FK_ERR_WORKSPACE 3
#define FK_ERR_CUDA 4
#define FK_ERR_TENSOR_MAP 5

/* bits of the device status word (first int32 of the workspace) */
#define FK_STATUS_BAD_PAGE 1 /* block-table entry outside [0, num_pages): page skipped, its tokens masked */
#define FK_STATUS_TIMEOUT 2  /* a pipeline wait ran past its bound and the CTA gave up */

/* Library version, e.g. 100 for 0.1.0. */
int fk_version(void);

/* Human-readable description of the last error returned on this thread. */
const char* fk_last_error(void);

/*
 * Bytes of workspace an entry point needs for `batch` sequences, `q_heads`
 * query heads and `kv_heads` KV heads with KV element type `kv_dtype`, on
 * `device`.  Any GQA group size q_heads / kv_heads is accepted, as the
 * reference's Triton kernels accept any (they pad the group to BLOCK_H =
 * max(16, next_pow2(G)), fskernels/triton/triton_gqa_decode.py:132): a group
 * of more than 8 query heads is processed in chunks of at most 8, which
 * needs more workspace.  Returns 0 on error (see fk_last_error()).
 */
size_t fk_decode_workspace_bytes_gqa(int device, int batch, int q_heads, int kv_heads, int kv_dtype);

/* The same for group sizes q_heads / kv_heads <= 8. */
size_t fk_decode_workspace_bytes(int device, int batch, int kv_heads, int kv_dtype);

/*
 * Contiguous varlen decode with optional attention sinks.
 * Replaces the reference's native boundary
 *   launch_flash_decode_gqa(q, k, v, cu_seqlens, s_aux, out, b, q_heads,
 *       kv_heads, group_size, max_seqlen, d, has_sink, strides...)
 *   (fskernels/cuda/flash_decode_cuda.cu:168-189, bound by
 *    fskernels/cuda/flash_decode_api.cpp:4-8,10-48)
 * and the Triton wrapper flash_decode_gqa_varlen
 *   (fskernels/triton/triton_gqa_decode.py:126-155).
 * group_size is derived, max_seqlen is not needed (no host sync).
 *   q    [batch, q_heads, 128]            strides (sq_b, sq_h, 1)
 *   k, v [total_tokens, kv_heads, 128]    strides (s*_t, s*_h, 1)
 *   cu_seqlens_k [batch + 1] int32, sequence b owns rows
 *                cu_seqlens_k[b] .. cu_seqlens_k[b+1]-1
 *   s_aux [q_heads] fp32 or NULL
 *   out  [batch, q_heads, 128]            strides (so_b, so_h, 1)
 *   dtype: FK_DTYPE_F16 or FK_DTYPE_BF16 for q, k, v and out.
 */
int fk_flash_decode_gqa_varlen(const void* q, const void* k_varlen, const void* v_varlen,
                               const int32_t* cu_seqlens_k, const float* s_aux, void* out,
                               int batch, int q_heads, int kv_heads, int head_dim,
                               int64_t total_tokens, int dtype,
                               int64_t sq_b, int64_t sq_h,
                               int64_t sk_t, int64_t sk_h,
                               int64_t sv_t, int64_t sv_h,
                               int64_t so_b, int64_t so_h,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * HF dense-cache decode (BHSD cache), fp16/bf16 or FP8 e4m3 KV.
 * Replaces flash_decode_gqa_hf_dense_optimized + its two Triton kernels
 *   (fskernels/triton/triton_gqa_decode_hf.py:146-211, :18-99, :103-137)
 * and flash_decode_gqa_hf_fp8 + kernels
 *   (fskernels/triton/triton_gqa_decode_hf_fp8.py:164-227, :19-110, :113-148).
 * Sequence b attends to cache rows start_k_offsets[b] .. cache_lens[b]-1
 * (start_k_offsets may be NULL = all zeros), as the reference kernel does
 * (triton_gqa_decode_hf.py:44-50).
 *   q       [batch, q_heads, 128]          q_dtype F16/BF16/E4M3 (E4M3: times *scale_q)
 *   k_cache [batch, kv_heads, max_seqlen, 128] strides (sk_b, sk_h, sk_s, 1)
 *   v_cache likewise;  kv_dtype F16/BF16 (then == q_dtype) or E4M3
 *   scale_q/scale_k/scale_v: fp32 device scalars for E4M3 tensors (NULL = 1)
 *   out     [batch, q_heads, 128]          out_dtype F16/BF16
 */
int fk_flash_decode_gqa_hf_dense(const void* q, const void* k_cache, const void* v_cache,
                                 const int32_t* cache_lens, const int32_t* start_k_offsets,
                                 const float* s_aux, void* out,
                                 int batch, int q_heads, int kv_heads, int head_dim,
                                 int64_t max_seqlen, int q_dtype, int kv_dtype, int out_dtype,
                                 const float* scale_q, const float* scale_k, const float* scale_v,
                                 int64_t sq_b, int64_t sq_h,
                                 int64_t sk_b, int64_t sk_h, int64_t sk_s,
                                 int64_t sv_b, int64_t sv_h, int64_t sv_s,
                                 int64_t so_b, int64_t so_h,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Paged decode over 16-token pages through a block table, fp16/bf16 or
 * FP8 e4m3 KV, optional sinks.
 * Replaces paged_flash_decode + _paged_flash_decode_kernel
 *   (fskernels/paged_attn/triton_paged_attn.py:96-125, :19-93).
 *   k_pool, v_pool [num_pages, kv_heads, 16, 128]  strides (s*_p, s*_h, s*_s, 1)
 *   block_table [batch, max_blocks] int32 (row stride bt_b; -1 = unused)
 *   seq_lens [batch] int32
 * page_size must be 16.  Entries outside [0, num_pages) reached by a
 * sequence set FK_STATUS_BAD_PAGE and their tokens are masked out.
 * For the same logical KV and lengths the result is bit-identical to
 * fk_flash_decode_gqa_varlen / fk_flash_decode_gqa_hf_dense.
 */
int fk_paged_flash_decode(const void* q, const void* k_pool, const void* v_pool,
                          const int32_t* block_table, const int32_t* seq_lens,
                          const float* s_aux, void* out,
                          int batch, int q_heads, int kv_heads, int head_dim,
                          int64_t num_pages, int page_size, int max_blocks,
                          int q_dtype, int kv_dtype, int out_dtype,
                          const float* scale_q, const float* scale_k, const float* scale_v,
                          int64_t sq_b, int64_t sq_h,
                          int64_t sk_p, int64_t sk_h, int64_t sk_s,
                          int64_t sv_p, int64_t sv_h, int64_t sv_s,
                          int64_t bt_b,
                          int64_t so_b, int64_t so_h,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * Paged KV append: write one new token's K and V for every sequence into its
 * page, at position positions[b] (page block_table[b, pos / 16], slot
 * pos % 16), then add 1 to positions[b] when `increment` is non-zero.
 * Replaces PagedKVCache.append_kv (fskernels/paged_attn/paged_kv_cache.py:109-132)
 * driven per sequence and per layer by the paged HF adapter
 * (benchmarks/run_hf_triton_fp8_paged.py:38-43), and the per-step
 * quantize_to_fp8 of K/V in the FP8 adapter (triton_gqa_decode_hf_fp8.py:268-269):
 * for an e4m3 pool the values are stored as e4m3(clamp(x / scale, +-448))
 * with the pool's fixed per-tensor scales (device scalars).
 *   k_new, v_new [batch, kv_heads, 128] f16/bf16  strides (s*n_b, s*n_h, 1)
 *   k_pool, v_pool [num_pages, kv_heads, 16, 128]  pool_dtype = in_dtype or E4M3
 *   block_table [batch, max_blocks] int32 (row stride bt_b)
 * Pages must already be allocated; an entry outside [0, num_pages) skips the
 * sequence and sets FK_STATUS_BAD_PAGE in *status (when non-null).
 */
int fk_paged_kv_append(const void* k_new, const void* v_new, int in_dtype, void* k_pool, void* v_pool,
                       int pool_dtype, const int32_t* block_table, int32_t* positions, int increment,
                       const float* scale_k, const float* scale_v, int* status, int batch, int kv_heads,
                       int head_dim, int64_t num_pages, int max_blocks, int64_t skn_b, int64_t skn_h,
                       int64_t svn_b, int64_t svn_h, int64_t sk_p, int64_t sk_h, int64_t sk_s,
                       int64_t sv_p, int64_t sv_h, int64_t sv_s, int64_t bt_b, void* stream);

/*
 * Measurement hooks (no reference counterpart: the reference times with
 * torch.profiler / triton.testing.do_bench, benchmarks/benchmark.py:87-91).
 * fk_profile_begin(n) records CUDA events on the launching stream just before
 * and just after the decode kernel of the next n decode calls made from any
 * thread; fk_profile_end() stops recording, waits for the events and returns
 * the summed kernel milliseconds and the number of calls recorded.
 */
int fk_profile_begin(int max_launches);
int fk_profile_end(float* kernel_ms, int* launches);

/*
 * Allocation-free varlen decode (no counterpart in the reference).
 * Same arguments and result as fk_flash_decode_gqa_varlen, without the
 * workspace: for callers that cannot allocate device memory -- a plugin whose
 * host framework owns every allocation, or a process where cudaMalloc is not
 * allowed once serving starts -- the scratch comes from a fixed array inside
 * the library (fk_noalloc_scratch_bytes() bytes, 8 MiB, held on every GPU that
 * loads the library until exit).  It holds
 *   batch * kv_heads * ceil(G / 8) + (resident CTAs, 148 on a B200)
 *     <= (fk_noalloc_scratch_bytes() - 1280) / 8324  (= 1007 segments),
 * G = q_heads / kv_heads: about 850 sequence-head pairs for G <= 8, half that
 * for 8 < G <= 16.  Larger calls return FK_ERR_WORKSPACE and queue nothing.
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture.  Each call clears the scratch's
 * arrival counters on `stream`; the status word collects FK_STATUS_* bits
 * until fk_noalloc_read_status clears it.  All calls share the one array, so
 * calls that overlap on the GPU (different streams, or different threads)
 * race: serialise them.  Nothing is allocated: no cudaMalloc/cudaFree.
 */
int fk_flash_decode_gqa_varlen_noalloc(const void* q, const void* k_varlen, const void* v_varlen,
                                       const int32_t* cu_seqlens_k, const float* s_aux, void* out,
                                       int batch, int q_heads, int kv_heads, int head_dim,
                                       int64_t total_tokens, int dtype,
                                       int64_t sq_b, int64_t sq_h,
                                       int64_t sk_t, int64_t sk_h,
                                       int64_t sv_t, int64_t sv_h,
                                       int64_t so_b, int64_t so_h, void* stream);

/* Bytes of the fixed scratch used by fk_flash_decode_gqa_varlen_noalloc. */
size_t fk_noalloc_scratch_bytes(void);

/*
 * Status of the allocation-free entry point on `device` (no counterpart in
 * the reference): the OR of FK_STATUS_* bits (FK_STATUS_TIMEOUT when a
 * bounded wait ran out and the output is incomplete) set by its calls since
 * the last clear.  Waits for the device to finish its work (keep it off the
 * hot path); clear != 0 then zeroes the word.
 */
int fk_noalloc_read_status(int device, int* status, int clear);

/* Size of the persistent decode grid (resident CTAs) on `device` for this
 * KV element type and KV head count. */
int fk_decode_num_ctas(int device, int kv_dtype, int kv_heads);

/*
 * Diagnostics for tests of the bounded waits (no counterpart in the
 * reference).  wait_ns bounds every mbarrier wait of later launches (default
 * 4 s, range [1 ms, 60 s]); inject = 1 makes each CTA's producer publish
 * nothing for its first pipeline stage, so its consumers' wait runs out, the
 * kernel sets FK_STATUS_TIMEOUT and returns (no fault; before exiting, each
 * CTA waits, bounded, for the copies it issued to land).  Clear the workspace after a timeout: arrival counters of split
 * items may be left mid-count.  inject = 0 restores normal operation.
 */
int fk_debug_configure(unsigned long long wait_ns, int inject);

#ifdef __cplusplus
}
#endif

#endif /* FK_DECODE_H_ */
