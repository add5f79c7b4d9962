/*
 * nvfp4kv -- C ABI of the B200 (sm_100a) NVFP4 paged KV-cache library.
 *
 * Pool layout (one row per token, 288 bytes, rows 16-byte aligned):
 *   bytes [0, 256)   : 512 e2m1 codes, byte i = code[2i] | code[2i+1] << 4
 *   bytes [256, 288) : 32 e4m3 block scales, scale g covers elements [16g, 16g + 16)
 * A paged pool is [num_pages, page_size, 288]; token slot = page * page_size + offset.
 * Reference layout: nvfp4-kv/glm53_nvfp4_runtime.py:4-6, :26, :37-65 and
 * nvfp4-kv/patch_nvfp4_kv.py:29-53 (Plaaasma/glm53-flash-dual-dgx-spark).
 *
 * Conventions:
 *   - every pointer is a device pointer unless stated otherwise; the caller owns all memory;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream);
 *   - functions return NVFP4KV_OK or an NVFP4KV_E* code and never synchronize;
 *     nvfp4kv_last_error() gives a message for the calling thread's last failure;
 *   - `err_flag` (may be NULL) is a device int32 the kernels OR NVFP4KV_DEVERR_* bits into
 *     when they meet out-of-range slots / indices / pages or a wait that timed out.  Bad
 *     entries are masked, never dereferenced.
 */
#ifndef NVFP4KV_H_
#define NVFP4KV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4KV_ROW_BYTES 288
#define NVFP4KV_DS_BYTES 656
#define NVFP4KV_LATENT 512
#define NVFP4KV_ROPE 64
#define NVFP4KV_INDEX_DIM 128       /* indexer key dims */
#define NVFP4KV_INDEX_ROW_BYTES 72  /* NVFP4 indexer key row: 64 B codes + 8 e4m3 scales */

/* host-side return codes */
#define NVFP4KV_OK 0
#define NVFP4KV_EINVAL 1     /* bad argument (shape, alignment, dtype) */
#define NVFP4KV_EWORKSPACE 2 /* workspace too small */
#define NVFP4KV_ECUDA 3      /* a CUDA runtime call failed */

/* device-side error bits (OR-ed into *err_flag) */
#define NVFP4KV_DEVERR_TIMEOUT 1    /* a bounded wait gave up */
#define NVFP4KV_DEVERR_BAD_SLOT 2   /* append slot >= pool_rows (row skipped) */
#define NVFP4KV_DEVERR_BAD_INDEX 4  /* sparse index < -1 or >= pool_rows (masked) */
#define NVFP4KV_DEVERR_BAD_PAGE 8   /* page id < 0 or >= num_pages (masked) */
#define NVFP4KV_DEVERR_SEQ_LEN 16   /* seq_len beyond the table / top-k width (clamped) */
#define NVFP4KV_DEVERR_CAPACITY 32  /* more distinct rows than the scratch holds (truncated) */

/* input element types */
#define NVFP4KV_DTYPE_BF16 0
#define NVFP4KV_DTYPE_F16 1
/* index element types */
#define NVFP4KV_INDEX_I64 0
#define NVFP4KV_INDEX_I32 1

typedef struct CUstream_st* nvfp4kv_stream_t;

/* Library version (major * 10000 + minor * 100 + patch). */
int nvfp4kv_version(void);

/* Message describing the calling thread's last non-OK return ("" if none). */
const char* nvfp4kv_last_error(void);

/*
 * Quantize-on-append.  Replaces _quant_kernel + write_nvfp4
 * (nvfp4-kv/glm53_nvfp4_runtime.py:37-76), which the write seam calls from
 * do_kv_cache_update (nvfp4-kv/patch_nvfp4_kv.py:67-72).
 *
 * kv_c: [num_tokens, >=512] bf16/fp16 with row stride `src_stride` elements (inner dim
 * contiguous); token t is quantised into pool row slot[t].  slot < 0 skips the token (as
 * the reference does); slot >= pool_rows skips it and sets NVFP4KV_DEVERR_BAD_SLOT.
 * Bit-exact with the reference: per-16 scale = e4m3_rne(max(amax/6, 1e-8)), code by the
 * reference's `<` threshold ladder on x / scale (ties go up), sign = (x / scale < 0).
 * num_tokens == 0 is a no-op.
 */
int nvfp4kv_append(const void* kv_c, int kv_dtype, int64_t num_tokens, int64_t src_stride,
                   uint8_t* pool, int64_t pool_rows, const void* slot_mapping, int slot_dtype,
                   int32_t* err_flag, nvfp4kv_stream_t stream);

/*
 * 656-byte fp8_ds_mla gather.  Replaces _gather_kernel + _gather
 * (nvfp4-kv/glm53_nvfp4_runtime.py:87-131); build_scratch (:143-182) calls it.
 * out: [num_rows, 656] bytes; row r is pool row clamp(idx[r], 0, pool_rows-1) re-encoded
 * as 512 e4m3 bytes (per-128 scale = max(amax/448, 1e-12), stored as fp32 at 512+4j)
 * followed by 128 zero bytes.  Byte-identical to the reference.
 */
int nvfp4kv_gather_ds656(const uint8_t* pool, int64_t pool_rows, const int32_t* idx,
                         int64_t num_rows, uint8_t* out, nvfp4kv_stream_t stream);

/*
 * Division used by the 656-byte row encoders (nvfp4kv_gather_ds656, nvfp4kv_dedup_gather_ds656)
 * for the reference's two fp32 quotients, gscale = max(amax / 448, 1e-12) and 1 / gscale
 * (nvfp4-kv/glm53_nvfp4_runtime.py:113-116):
 *   NVFP4KV_DIV_IEEE   (default) exact division: the reference's kernel as run on the CPU
 *                      (the Triton interpreter computes in IEEE fp32);
 *   NVFP4KV_DIV_TRITON the reference's kernel as Triton compiles it for the GPU, whose fp32 `/`
 *                      is the approximate div.full.f32: rows byte-identical to it.
 * The two differ in the last bit of about half of the fp32 scales and, where a value lands on
 * an e4m3 rounding tie, in that e4m3 byte.  Process-wide; set it once before launching.  The
 * append (nvfp4kv_append) gives the same bytes under both (no input can sit between the two
 * quotients' roundings there), so it has no mode.  No counterpart in the reference.
 */
#define NVFP4KV_DIV_IEEE 0
#define NVFP4KV_DIV_TRITON 1
int nvfp4kv_set_gather_division(int mode);
int nvfp4kv_get_gather_division(void);

/*
 * Sync-free deduplicating gather: the T > _SYNC_FREE_T branch of build_scratch
 * (nvfp4-kv/glm53_nvfp4_runtime.py:177-182: torch.unique(flat, return_inverse=True) then
 * _gather into a zeroed [ceil(S/64), 64, 656] scratch) without the host synchronisation
 * torch.unique needs for its data-dependent size.  All outputs are written on the device, in
 * stream order, by fixed-size launches (CUDA-graph capturable):
 *   tables[j]  = position of entries[j] among the distinct entries in ascending order (the
 *                inverse of torch.unique), int32;
 *   scratch    = row u (656 B) is the _gather_kernel row of distinct entry u (-1 reads row 0)
 *                for u < *n_unique, and zeros up to the next multiple of 64 rows;
 *   *n_unique  = number of distinct entries (device int32).
 * entries: num_entries int32 pool rows, -1 padded.  Entries < -1 or >= pool_rows set
 * NVFP4KV_DEVERR_BAD_INDEX and count as -1 (the reference keeps each such value distinct and
 * gathers its clamped row).  scratch holds scratch_rows rows (16-byte aligned); with more
 * distinct entries than that, the first scratch_rows rows are written and
 * NVFP4KV_DEVERR_CAPACITY is set.  workspace: nvfp4kv_dedup_workspace_ints() int32 values,
 * no initial contents needed.  pool_rows < 2^31 - 1.
 */
int nvfp4kv_dedup_gather_ds656(const uint8_t* pool, int64_t pool_rows, const int32_t* entries,
                               int64_t num_entries, int32_t* workspace, int64_t workspace_ints,
                               int32_t* tables, uint8_t* scratch, int64_t scratch_rows,
                               int32_t* n_unique, int32_t* err_flag, nvfp4kv_stream_t stream);

/* int32 workspace size of nvfp4kv_dedup_gather_ds656 (pool_rows + 1 marks, one value per
 * 4096 marks, min(num_entries, pool_rows + 1) distinct values). */
int nvfp4kv_dedup_workspace_ints(int64_t pool_rows, int64_t num_entries, int64_t* ints);

/*
 * Dequantise pool rows to bf16: out[r, :] = decode(pool[rows[r]]) for 0 <= rows[r] <
 * pool_rows, zeros otherwise (NVFP4KV_DEVERR_BAD_INDEX for rows < -1 or >= pool_rows).
 * The values (code x block scale) are exact in bf16.  The reference has no standalone
 * equivalent; it is the decode half of _gather_kernel (:99-108) without the fp8 re-encode.
 */
int nvfp4kv_dequant_bf16(const uint8_t* pool, int64_t pool_rows, const void* rows,
                         int rows_dtype, int64_t num_rows, void* out,
                         int32_t* err_flag, nvfp4kv_stream_t stream);

/*
 * Fused NVFP4 gather + dequant + MLA decode attention (tcgen05, split-K + LSE combine).
 * Replaces build_scratch + trtllm_batch_decode_with_kv_cache_mla at the read seam
 * (nvfp4-kv/patch_nvfp4_kv.py:84-118; call signature of the consumer:
 * flashinfer mla/_core.py:598-620, as called in nvfp4-kv/test_kernel_equiv.py:34-39).
 * It reads the 288-byte pool directly; no scratch rows are materialised.
 *
 * q: bf16 [batch, q_len, num_heads, head_dim_qk] with element strides
 *    (q_stride_b, q_stride_q, q_stride_h) and a contiguous last dim.  Only the first
 *    kv_lora_rank (512) dims take part: the 288-byte rows carry no rope part (the reference
 *    drops k_pe, patch_nvfp4_kv.py:70), so the trailing rope dims of q multiply zeros.
 * Dense mode (sparse_topk == 0): tables [batch, >= ceil(max_seq_len/page_size)] page ids
 *    (row stride tables_stride), seq_lens[b] = context length.  With q_len > 1 query
 *    token i sees tokens t < seq_len - (q_len - 1 - i) (causal MTP).
 * Sparse mode (sparse_topk > 0, q_len must be 1): tables [batch, >= sparse_topk] physical
 *    pool rows, -1 padded; seq_lens[b] = number of leading entries to use.
 * out: bf16 [batch, q_len, num_heads, 512], 16-byte aligned, with strides (out_stride_b,
 *    out_stride_q, out_stride_h), multiples of 8 elements:
 *    softmax(bmm1_scale * q.k) . v * bmm2_scale, k = v = dequantised rows.
 *    A query row with no visible token is written as zeros.
 * workspace: device scratch of at least nvfp4kv_mla_decode_workspace_size() bytes, 256-B
 *    aligned.  No allocation and no host synchronisation happen inside the call.
 */
int nvfp4kv_mla_decode(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                       const uint8_t* pool, int64_t pool_rows,
                       const int32_t* tables, int64_t tables_stride,
                       const int32_t* seq_lens,
                       int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank,
                       int sparse_topk, int page_size, int max_seq_len,
                       float bmm1_scale, float bmm2_scale,
                       void* out, int64_t out_stride_b, int64_t out_stride_q, int64_t out_stride_h,
                       void* workspace, size_t workspace_bytes,
                       int32_t* err_flag, nvfp4kv_stream_t stream);

/*
 * nvfp4kv_mla_decode that also writes lse [batch, q_len, num_heads] float32 (contiguous): the
 * natural-log sum over the visible tokens of exp(bmm1_scale * q.k), -inf for a row with no
 * visible token.  With it, results over disjoint token ranges of one sequence (computed on
 * different GPUs) merge exactly: out = sum_r exp(lse_r - lse) out_r, lse = log sum_r exp(lse_r).
 * No counterpart in the reference (its consumer returns no LSE); used by the multi-GPU
 * sequence partition.
 */
int nvfp4kv_mla_decode_lse(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                           const uint8_t* pool, int64_t pool_rows,
                           const int32_t* tables, int64_t tables_stride,
                           const int32_t* seq_lens,
                           int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank,
                           int sparse_topk, int page_size, int max_seq_len,
                           float bmm1_scale, float bmm2_scale,
                           void* out, int64_t out_stride_b, int64_t out_stride_q, int64_t out_stride_h,
                           float* lse, void* workspace, size_t workspace_bytes,
                           int32_t* err_flag, nvfp4kv_stream_t stream);

/* Workspace bytes nvfp4kv_mla_decode needs for this shape on the current device. */
int nvfp4kv_mla_decode_workspace_size(int batch, int q_len, int num_heads, int max_seq_len,
                                      int sparse_topk, size_t* bytes);

/* Split plan of nvfp4kv_mla_decode for this shape on the current device: token splits per
 * 64-row query group, and kernel launches per call (Q preparation + attention, + split
 * combine when splits > 1).  No counterpart in the reference; for schedulers and benchmarks. */
int nvfp4kv_mla_decode_plan(int batch, int q_len, int num_heads, int max_seq_len,
                            int sparse_topk, int* splits, int* launches);

/* Measurement hook, no counterpart in the reference: the calling thread's next
 * nvfp4kv_mla_decode (or _static) call records the CUDA events `start` and `stop`
 * (cudaEvent_t) on its stream immediately before and after its attention kernel, then the
 * hook clears itself.  Both NULL clears it. */
int nvfp4kv_set_kernel_events(void* start, void* stop);

/* Failure-detection self-test, no counterpart in the reference: one thread waits, with the
 * bounded wait every kernel of this library uses, on an mbarrier that nothing arrives on.
 * The wait gives up after its time limit (2 s) and ORs NVFP4KV_DEVERR_TIMEOUT into *err_flag;
 * the kernel then returns normally, so the CUDA context stays usable. */
int nvfp4kv_selftest_bounded_wait(int32_t* err_flag, nvfp4kv_stream_t stream);

/*
 * Rope side-pool.  No counterpart in the reference: its model is NoPE, its write seam drops
 * k_pe (nvfp4-kv/patch_nvfp4_kv.py:70) and its 656-byte rows carry zero rope bytes
 * (nvfp4-kv/glm53_nvfp4_runtime.py:121-122).  For MLA models whose keys carry a 64-d rope part
 * the library keeps it beside the 288-byte pool in a pool of its own: [pool_rows, 64] bf16
 * (128-byte rows, 16-byte aligned) addressed by the same token slots.  The 288-byte layout is
 * unchanged, so every entry point above works on the same pool with or without it.
 */

/* k_pe [num_tokens, >= 64] bf16, row stride src_stride elements (inner dim contiguous) ->
 * rope_pool[slot[t]].  slot < 0 skips the token; slot >= pool_rows skips it and sets
 * NVFP4KV_DEVERR_BAD_SLOT (as nvfp4kv_append).  Call it beside nvfp4kv_append at the write seam. */
int nvfp4kv_append_rope(const void* k_pe, int64_t num_tokens, int64_t src_stride, void* rope_pool,
                        int64_t pool_rows, const void* slot_mapping, int slot_dtype,
                        int32_t* err_flag, nvfp4kv_stream_t stream);

/* nvfp4kv_gather_ds656 whose rows carry the rope part: bytes [528, 656) of row r are the 64
 * bf16 of rope_pool[clamp(idx[r], 0, pool_rows - 1)] (the fp8_ds_mla format's rope field)
 * instead of zeros; bytes [0, 528) as nvfp4kv_gather_ds656, division mode included. */
int nvfp4kv_gather_ds656_rope(const uint8_t* pool, const void* rope_pool, int64_t pool_rows,
                              const int32_t* idx, int64_t num_rows, uint8_t* out,
                              nvfp4kv_stream_t stream);

/* nvfp4kv_mla_decode with the rope part: q's dims [512, 576) (head_dim_qk >= 576) meet the
 * rope rows, score = bmm1_scale * (q_nope . k + q_rope . k_rope); V is the latent as before.
 * The rope scores are computed in fp32 by a kernel before the attention and added to its
 * scores, so the workspace (nvfp4kv_mla_decode_rope_workspace_size) adds a 16 KB rope image
 * per 64-row query group and 4 bytes per (query row, context position): 512 B per context
 * token of a 64-head group (268 MB for batch 16 at 32K tokens).  Same errors as
 * nvfp4kv_mla_decode, plus EINVAL for a null or unaligned rope pool. */
int nvfp4kv_mla_decode_rope(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                            const uint8_t* pool, int64_t pool_rows, const void* rope_pool,
                            const int32_t* tables, int64_t tables_stride,
                            const int32_t* seq_lens,
                            int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank,
                            int sparse_topk, int page_size, int max_seq_len,
                            float bmm1_scale, float bmm2_scale,
                            void* out, int64_t out_stride_b, int64_t out_stride_q, int64_t out_stride_h,
                            void* workspace, size_t workspace_bytes,
                            int32_t* err_flag, nvfp4kv_stream_t stream);

/* Workspace bytes nvfp4kv_mla_decode_rope needs for this shape on the current device. */
int nvfp4kv_mla_decode_rope_workspace_size(int batch, int q_len, int num_heads, int max_seq_len,
                                           int sparse_topk, size_t* bytes);

/*
 * Indexer K-pool: the keys of the sparse-attention (DSA) lightning indexer whose top-k rows the
 * sparse decode reads.  The reference keeps them an fp8 pool ("stays fp8", nvfp4-kv/PLAN.md:29;
 * "FP4 indexer keys need sm_100", README.md:321) and takes its top-k from vLLM's indexer
 * (topk_indices_buffer, vllm-0.22 flashinfer_mla_sparse.py:327-337).  Here the 128-d keys are
 * NVFP4, 72-byte rows [num_pages, page_size, 72] (bytes [0, 64) codes, byte i = code[2i] |
 * code[2i+1] << 4; bytes [64, 72) e4m3 scales, scale g for elements [16g, 16g + 16)),
 * addressed by the same token slots as the 288-byte pool and quantised by the same rule.
 */

/* k [num_tokens, >= 128] bf16, row stride src_stride elements -> index_pool[slot[t]];
 * slot < 0 skips, slot >= pool_rows skips and sets NVFP4KV_DEVERR_BAD_SLOT. */
int nvfp4kv_index_append(const void* k, int64_t num_tokens, int64_t src_stride, uint8_t* index_pool,
                         int64_t pool_rows, const void* slot_mapping, int slot_dtype,
                         int32_t* err_flag, nvfp4kv_stream_t stream);

/*
 * Top-k selection by the DSA indexer rule (DeepSeek-V3.2's, as vLLM 0.22 states it):
 *   score[b, s] = sum_h weights[b, h] * max(q[b, h, :] . k[s, :], 0)
 * over the visible positions s < seq_lens[b] of entry b (a page-table entry, as in dense
 * decode), k the exactly dequantised keys, fp32 accumulation.  out_rows[b, :] receives the pool
 * rows of the topk highest-scoring positions in ascending position order (ties at the
 * threshold go to the lower positions), -1 after out_count[b] = min(seq_lens[b], topk) and for
 * a position on a missing page: exactly the sparse tables and seq_lens nvfp4kv_mla_decode takes.
 * q: bf16 [batch, 64 heads, 128] with element strides (q_stride_b, q_stride_h), 16-byte
 * aligned; weights fp32 [batch, 64], row stride weights_stride; workspace: the scores,
 * nvfp4kv_index_topk_workspace_size() bytes, 16-byte aligned.  index_pool 16-byte aligned and
 * page_size a power of two in [2, 4096] dividing pool_rows: the scoring kernel copies whole
 * pages (or 128-row runs of them) with 16-byte bulk copies, and two 72-byte rows are the
 * smallest run that is a multiple of 16 bytes.
 */
int nvfp4kv_index_topk(const void* q, int64_t q_stride_b, int64_t q_stride_h, const float* weights,
                       int64_t weights_stride, const uint8_t* index_pool, int64_t pool_rows,
                       const int32_t* tables, int64_t tables_stride, const int32_t* seq_lens,
                       int batch, int num_heads, int page_size, int max_seq_len, int topk,
                       int32_t* out_rows, int32_t* out_count, void* workspace, size_t workspace_bytes,
                       int32_t* err_flag, nvfp4kv_stream_t stream);

/* Workspace bytes of nvfp4kv_index_topk: 4 per (entry, position up to max_seq_len rounded to 128). */
int nvfp4kv_index_topk_workspace_size(int batch, int max_seq_len, size_t* bytes);

/* Capacity of the device scratch array behind nvfp4kv_mla_decode_static. */
#define NVFP4KV_STATIC_SCRATCH_BYTES 33554432u

/*
 * nvfp4kv_mla_decode without a workspace argument: its workspace (split-K partials, prepared
 * Q) goes to a file-scope device array of NVFP4KV_STATIC_SCRATCH_BYTES (32 MiB, reserved per
 * device when the module loads), so the call allocates nothing.  No counterpart in the
 * reference (its decode takes a workspace buffer); it is for callers that cannot allocate
 * device memory per call.
 * Same arguments, semantics and errors as nvfp4kv_mla_decode, plus:
 *   - NVFP4KV_EWORKSPACE if nvfp4kv_mla_decode_workspace_size() of the shape exceeds the
 *     scratch (on a 148-SM device: calls with more than 453 query groups of 64 rows,
 *     e.g. batch > 453 at 64 heads and q_len 1);
 *   - argument errors (EINVAL) are reported before the capacity check (EWORKSPACE);
 *   - the first call on a device looks up the scratch address with that device current and
 *     keeps it for the life of the process; make it before any stream capture begins, and do
 *     not use the library on a device after a cudaDeviceReset (the array may move);
 *   - one scratch per device: calls whose kernels overlap on a device race on it.
 */
int nvfp4kv_mla_decode_static(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                              const uint8_t* pool, int64_t pool_rows,
                              const int32_t* tables, int64_t tables_stride,
                              const int32_t* seq_lens,
                              int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank,
                              int sparse_topk, int page_size, int max_seq_len,
                              float bmm1_scale, float bmm2_scale,
                              void* out, int64_t out_stride_b, int64_t out_stride_q, int64_t out_stride_h,
                              int32_t* err_flag, nvfp4kv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4KV_H_ */
