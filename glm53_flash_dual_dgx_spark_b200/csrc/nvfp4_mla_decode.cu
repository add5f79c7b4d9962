// nvfp4kv_mla_decode: argument checks, the split plan and the split combine around the fused
// NVFP4 decode kernel (nvfp4_mla_decode_fp4.cu).
//
// Replaces, at the reference's read seam (nvfp4-kv/patch_nvfp4_kv.py:84-118), the pair
//   build_scratch(...)                         -> 656-byte fp8 scratch (glm53_nvfp4_runtime.py:143-182)
//   trtllm_batch_decode_with_kv_cache_mla(...) -> attention over that scratch
// with kernels that read the 288-byte pool rows directly.
//
// Work unit: query group (b, g) of up to 64 query rows (MTP token i, head h) of batch entry b,
// which all share the latent rows, x token split s.  The plan spreads one call over the SMs:
// splits = min(SMs / units, 64, tiles), so a small batch still fills the GPU; each split
// writes unnormalised partial O plus (max, sum) per row and combine_kernel merges them with
// log-sum-exp weights.
#include <math.h>

#include "abi_common.h"
#include "common.cuh"
#include "decode_shared.h"

namespace nvfp4kv {
namespace {

constexpr int kTile = kDecTile;         // tokens per tile
constexpr int kNQ = kDecRows;           // query rows per work unit
constexpr int kMaxSplits = kDecMaxSplits;

// Merge split partials: out = sum_s w_s O_s / sum_s w_s l_s * bmm2_scale with
// w_s = 2^(m_s - max m).  One block per query row (spread over every SM), one float4 of
// latent dims per thread; the loads of all splits are independent so they overlap.
__global__ void __launch_bounds__(128)
combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits,
               int batch, int groups, int q_len, int num_heads, float bmm2_scale,
               __nv_bfloat16* __restrict__ out, int64_t o_sb, int64_t o_sq, int64_t o_sh,
               float* __restrict__ lse) {
    __shared__ float wts[kMaxSplits];
    griddep_wait();   // a programmatic dependent of the attention kernel that writes the partials
    const int n = blockIdx.x % kNQ;
    const int bg = blockIdx.x / kNQ;
    const int g = bg % groups, b = bg / groups;
    const int r = g * kNQ + n;
    if (r >= q_len * num_heads) return;
    const int64_t unit_row = (static_cast<int64_t>(b) * groups + g) * kNQ + n;
    const int64_t split_rows = static_cast<int64_t>(batch) * groups * kNQ;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        float m[2], l[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int s = lane + 32 * k;
            m[k] = -INFINITY;
            l[k] = 0.0f;
            if (s < splits) {
                const float2 ml = *reinterpret_cast<const float2*>(part_ml + (s * split_rows + unit_row) * 2);
                m[k] = ml.x;
                l[k] = ml.y;
            }
        }
        float M = fmaxf(l[0] > 0.0f ? m[0] : -INFINITY, l[1] > 0.0f ? m[1] : -INFINITY);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
        float w[2], Ls = 0.0f;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            w[k] = l[k] > 0.0f ? exp2f(m[k] - M) : 0.0f;
            Ls += w[k] * l[k];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xFFFFFFFFu, Ls, o);
        const float inv = Ls > 0.0f ? bmm2_scale / Ls : 0.0f;
        // log-sum-exp of the row's scores over all splits: sum 2^x = 2^M Ls (x in log2 units)
        if (lse && lane == 0)
            lse[static_cast<int64_t>(b) * q_len * num_heads + r] =
                Ls > 0.0f ? 0.69314718055994531f * (M + log2f(Ls)) : -INFINITY;
#pragma unroll
        for (int k = 0; k < 2; ++k)
            if (lane + 32 * k < splits) wts[lane + 32 * k] = w[k] * inv;
    }
    __syncthreads();
    const float* base = part_o + unit_row * kLatent + 4 * threadIdx.x;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
    for (int s = 0; s < splits; ++s) {
        const float wgt = wts[s];
        if (wgt != 0.0f) {   // an empty split never wrote its O rows
            const float4 v = __ldg(reinterpret_cast<const float4*>(base + s * split_rows * kLatent));
            acc.x = fmaf(wgt, v.x, acc.x);
            acc.y = fmaf(wgt, v.y, acc.y);
            acc.z = fmaf(wgt, v.z, acc.z);
            acc.w = fmaf(wgt, v.w, acc.w);
        }
    }
    const int qi = r / num_heads, h = r % num_heads;
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + b * o_sb + qi * o_sq + h * o_sh + 4 * threadIdx.x) = pk;
}

}  // namespace

DecodePlan make_decode_plan(int batch, int q_len, int num_heads, int max_seq_len, int sparse_topk) {
    DecodePlan pl{};
    pl.groups = (q_len * num_heads + kNQ - 1) / kNQ;
    const int ctx = sparse_topk > 0 ? sparse_topk : max_seq_len;
    const int tiles = ctx > 0 ? (ctx + kTile - 1) / kTile : 1;
    const int units = batch * pl.groups;
    const int sms = device_sm_count();
    int want = units >= sms ? 1 : sms / units;
    want = want < 1 ? 1 : (want > kMaxSplits ? kMaxSplits : want);
    want = want > tiles ? tiles : want;
    // the fewest splits with the same longest split: ceil(T / ceil(T / want)) (e.g. 64 tiles
    // over at most 9 splits: 8 splits of 8, not 9 splits of 7-8), so fewer partials to merge
    const int longest = (tiles + want - 1) / want;
    want = (tiles + longest - 1) / longest;
    pl.tiles_total = tiles;
    pl.splits = want < 1 ? 1 : want;   // split sizes differ by at most one tile
    pl.part_bytes = pl.splits > 1
                        ? static_cast<size_t>(pl.splits) * units * kNQ * (kLatent + 2) * sizeof(float)
                        : 0;
    pl.qimg_bytes = static_cast<size_t>(units) * kQImageBytes;
    pl.ws_bytes = pl.part_bytes + pl.qimg_bytes;
    return pl;
}

namespace {

// One thread waits on an mbarrier whose single expected arrival never comes.
__global__ void bounded_wait_selftest_kernel(int32_t* err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    abort_flag = 0;
    mbar_fence_init();
    mbar_wait(b, 0, &abort_flag, err);   // returns false after NVFP4KV_WAIT_TIMEOUT_NS
}

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_selftest_bounded_wait(int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (!err_flag) return fail(NVFP4KV_EINVAL, "selftest_bounded_wait: null error word");
    bounded_wait_selftest_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(err_flag);
    return check_launch("nvfp4kv_selftest_bounded_wait");
}

extern "C" int nvfp4kv_mla_decode_workspace_size(int batch, int q_len, int num_heads,
                                                 int max_seq_len, int sparse_topk, size_t* bytes) {
    using namespace nvfp4kv;
    if (!bytes) return fail(NVFP4KV_EINVAL, "workspace_size: null output");
    if (batch < 0 || q_len < 1 || num_heads < 1 || max_seq_len < 0 || sparse_topk < 0)
        return fail(NVFP4KV_EINVAL, "workspace_size: bad shape");
    *bytes = batch == 0 ? 0 : make_decode_plan(batch, q_len, num_heads, max_seq_len, sparse_topk).ws_bytes;
    return NVFP4KV_OK;
}

extern "C" int nvfp4kv_mla_decode_plan(int batch, int q_len, int num_heads, int max_seq_len,
                                       int sparse_topk, int* splits, int* launches) {
    using namespace nvfp4kv;
    if (!splits || !launches) return fail(NVFP4KV_EINVAL, "mla_decode_plan: null output");
    if (batch < 0 || q_len < 1 || num_heads < 1 || max_seq_len < 0 || sparse_topk < 0)
        return fail(NVFP4KV_EINVAL, "mla_decode_plan: bad shape");
    if (batch == 0) {
        *splits = 0;
        *launches = 0;
        return NVFP4KV_OK;
    }
    const DecodePlan pl = make_decode_plan(batch, q_len, num_heads, max_seq_len, sparse_topk);
    *splits = pl.splits;
    *launches = 2 + (pl.splits > 1 ? 1 : 0);   // Q preparation + attention (+ split combine)
    return NVFP4KV_OK;
}

namespace nvfp4kv {

int check_decode_args(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                      const uint8_t* pool, int64_t pool_rows, const int32_t* tables, const int32_t* seq_lens,
                      int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank, int sparse_topk,
                      int page_size, int max_seq_len, const void* out, int64_t out_stride_b,
                      int64_t out_stride_q, int64_t out_stride_h, int* page_shift_out) {
    if (batch < 0) return fail(NVFP4KV_EINVAL, "mla_decode: batch < 0");
    if (!q || !pool || !tables || !seq_lens || !out)
        return fail(NVFP4KV_EINVAL, "mla_decode: null pointer");
    if (kv_lora_rank != NVFP4KV_LATENT)
        return fail(NVFP4KV_EINVAL, "mla_decode: kv_lora_rank must be 512 (got %d)", kv_lora_rank);
    if (head_dim_qk < NVFP4KV_LATENT)
        return fail(NVFP4KV_EINVAL, "mla_decode: head_dim_qk %d < 512", head_dim_qk);
    if (q_len < 1 || num_heads < 1) return fail(NVFP4KV_EINVAL, "mla_decode: q_len and num_heads must be >= 1");
    if (sparse_topk < 0) return fail(NVFP4KV_EINVAL, "mla_decode: sparse_topk < 0");
    if (sparse_topk > 0 && q_len != 1)
        return fail(NVFP4KV_EINVAL, "mla_decode: sparse mode needs q_len == 1 (got %d)", q_len);
    if (max_seq_len < 0) return fail(NVFP4KV_EINVAL, "mla_decode: max_seq_len < 0");
    if (pool_rows <= 0) return fail(NVFP4KV_EINVAL, "mla_decode: empty pool");
    int page_shift = 0;
    if (sparse_topk == 0) {
        if (page_size <= 0 || (page_size & (page_size - 1)) != 0 || page_size > 4096)
            return fail(NVFP4KV_EINVAL, "mla_decode: page_size must be a power of two <= 4096 (got %d)", page_size);
        while ((1 << page_shift) < page_size) ++page_shift;
        if (pool_rows % page_size != 0)
            return fail(NVFP4KV_EINVAL, "mla_decode: pool_rows %lld not a multiple of page_size %d",
                        (long long)pool_rows, page_size);
    }
    if (reinterpret_cast<uintptr_t>(pool) % 16 || reinterpret_cast<uintptr_t>(q) % 16 ||
        q_stride_b % 8 || q_stride_q % 8 || q_stride_h % 8)
        return fail(NVFP4KV_EINVAL, "mla_decode: pool/q must be 16-byte aligned and q strides multiples of 8");
    if (reinterpret_cast<uintptr_t>(out) % 16 || out_stride_b % 8 || out_stride_q % 8 || out_stride_h % 8)
        return fail(NVFP4KV_EINVAL, "mla_decode: out must be 16-byte aligned and its strides multiples of 8");
    if (page_shift_out) *page_shift_out = page_shift;
    return NVFP4KV_OK;
}

namespace {

int decode_impl(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                const uint8_t* pool, int64_t pool_rows, const int32_t* tables, int64_t tables_stride,
                const int32_t* seq_lens, int batch, int q_len, int num_heads, int head_dim_qk,
                int kv_lora_rank, int sparse_topk, int page_size, int max_seq_len, float bmm1_scale,
                float bmm2_scale, void* out, int64_t out_stride_b, int64_t out_stride_q,
                int64_t out_stride_h, float* lse, void* workspace, size_t workspace_bytes,
                int32_t* err_flag, nvfp4kv_stream_t stream, const void* rope_pool = nullptr) {
    if (batch < 0) return fail(NVFP4KV_EINVAL, "mla_decode: batch < 0");
    if (batch == 0) return NVFP4KV_OK;
    if (rope_pool && (head_dim_qk < NVFP4KV_LATENT + NVFP4KV_ROPE || reinterpret_cast<uintptr_t>(rope_pool) % 16))
        return fail(NVFP4KV_EINVAL, "mla_decode_rope: head_dim_qk must be >= 576 and the rope pool 16-byte aligned");
    int page_shift = 0;
    int rc = check_decode_args(q, q_stride_b, q_stride_q, q_stride_h, pool, pool_rows, tables, seq_lens, batch,
                               q_len, num_heads, head_dim_qk, kv_lora_rank, sparse_topk, page_size, max_seq_len,
                               out, out_stride_b, out_stride_q, out_stride_h, &page_shift);
    if (rc != NVFP4KV_OK) return rc;
    const DecodePlan pl = make_decode_plan(batch, q_len, num_heads, max_seq_len, sparse_topk);
    const size_t need = pl.ws_bytes + (rope_pool ? rope_q_bytes(pl, batch) + rope_logit_bytes(pl, batch) : 0);
    if (!workspace || workspace_bytes < need)
        return fail(NVFP4KV_EWORKSPACE, "mla_decode: workspace %zu bytes < %zu required", workspace_bytes, need);
    if (reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(NVFP4KV_EINVAL, "mla_decode: workspace must be 256-byte aligned");
    const size_t part_o_bytes = static_cast<size_t>(pl.splits) * batch * pl.groups * kNQ * kLatent * sizeof(float);
    float* part_o = pl.splits > 1 ? static_cast<float*>(workspace) : nullptr;
    float* part_ml = pl.splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + part_o_bytes) : nullptr;

    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    {
        DecodeArgs a{};
        a.q = q; a.q_sb = q_stride_b; a.q_sq = q_stride_q; a.q_sh = q_stride_h;
        a.pool = pool; a.pool_rows = pool_rows;
        a.tables = tables; a.tables_stride = tables_stride; a.seq_lens = seq_lens;
        a.batch = batch; a.q_len = q_len; a.num_heads = num_heads;
        a.sparse_topk = sparse_topk; a.page_size = page_size; a.page_shift = page_shift;
        a.max_seq_len = max_seq_len;
        a.bmm1_scale = bmm1_scale; a.bmm2_scale = bmm2_scale;
        a.out = out; a.o_sb = out_stride_b; a.o_sq = out_stride_q; a.o_sh = out_stride_h;
        a.part_o = part_o; a.part_ml = part_ml; a.err = err_flag; a.lse = lse;
        a.qimg = static_cast<uint8_t*>(workspace) + pl.part_bytes;
        if (rope_pool) {
            a.rope_pool = static_cast<const uint16_t*>(rope_pool);
            a.rope_q = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + pl.ws_bytes);
            a.rope_logits = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + pl.ws_bytes +
                                                     rope_q_bytes(pl, batch));
        }
        if ((rc = launch_decode_fp4(a, pl, st)) != NVFP4KV_OK) return rc;
    }
    if (pl.splits > 1) {
        const cudaError_t le = launch_dependent(
            combine_kernel, dim3(batch * pl.groups * kNQ), dim3(128), 0, st, part_o, part_ml, pl.splits, batch,
            pl.groups, q_len, num_heads, bmm2_scale, static_cast<__nv_bfloat16*>(out), out_stride_b, out_stride_q,
            out_stride_h, lse);
        if (le != cudaSuccess)
            return fail(NVFP4KV_ECUDA, "nvfp4kv_mla_decode combine launch failed: %s", cudaGetErrorString(le));
        if ((rc = check_launch("nvfp4kv_mla_decode combine")) != NVFP4KV_OK) return rc;
    }
    return NVFP4KV_OK;
}

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_mla_decode(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                                  const uint8_t* pool, int64_t pool_rows,
                                  const int32_t* tables, int64_t tables_stride,
                                  const int32_t* seq_lens,
                                  int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank,
                                  int sparse_topk, int page_size, int max_seq_len,
                                  float bmm1_scale, float bmm2_scale,
                                  void* out, int64_t out_stride_b, int64_t out_stride_q, int64_t out_stride_h,
                                  void* workspace, size_t workspace_bytes,
                                  int32_t* err_flag, nvfp4kv_stream_t stream) {
    return nvfp4kv::decode_impl(q, q_stride_b, q_stride_q, q_stride_h, pool, pool_rows, tables, tables_stride,
                                seq_lens, batch, q_len, num_heads, head_dim_qk, kv_lora_rank, sparse_topk,
                                page_size, max_seq_len, bmm1_scale, bmm2_scale, out, out_stride_b,
                                out_stride_q, out_stride_h, nullptr, workspace, workspace_bytes, err_flag,
                                stream);
}

extern "C" int nvfp4kv_mla_decode_rope(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                                       const uint8_t* pool, int64_t pool_rows, const void* rope_pool,
                                       const int32_t* tables, int64_t tables_stride,
                                       const int32_t* seq_lens,
                                       int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank,
                                       int sparse_topk, int page_size, int max_seq_len,
                                       float bmm1_scale, float bmm2_scale,
                                       void* out, int64_t out_stride_b, int64_t out_stride_q, int64_t out_stride_h,
                                       void* workspace, size_t workspace_bytes,
                                       int32_t* err_flag, nvfp4kv_stream_t stream) {
    if (!rope_pool && batch > 0) return nvfp4kv::fail(NVFP4KV_EINVAL, "mla_decode_rope: null rope pool");
    return nvfp4kv::decode_impl(q, q_stride_b, q_stride_q, q_stride_h, pool, pool_rows, tables, tables_stride,
                                seq_lens, batch, q_len, num_heads, head_dim_qk, kv_lora_rank, sparse_topk,
                                page_size, max_seq_len, bmm1_scale, bmm2_scale, out, out_stride_b,
                                out_stride_q, out_stride_h, nullptr, workspace, workspace_bytes, err_flag,
                                stream, rope_pool);
}

extern "C" int nvfp4kv_mla_decode_rope_workspace_size(int batch, int q_len, int num_heads, int max_seq_len,
                                                      int sparse_topk, size_t* bytes) {
    using namespace nvfp4kv;
    if (!bytes) return fail(NVFP4KV_EINVAL, "rope_workspace_size: null output");
    if (batch < 0 || q_len < 1 || num_heads < 1 || max_seq_len < 0 || sparse_topk < 0)
        return fail(NVFP4KV_EINVAL, "rope_workspace_size: bad shape");
    if (batch == 0) {
        *bytes = 0;
        return NVFP4KV_OK;
    }
    const DecodePlan pl = make_decode_plan(batch, q_len, num_heads, max_seq_len, sparse_topk);
    *bytes = pl.ws_bytes + rope_q_bytes(pl, batch) + rope_logit_bytes(pl, batch);
    return NVFP4KV_OK;
}

extern "C" int nvfp4kv_mla_decode_lse(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                                      const uint8_t* pool, int64_t pool_rows,
                                      const int32_t* tables, int64_t tables_stride,
                                      const int32_t* seq_lens,
                                      int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank,
                                      int sparse_topk, int page_size, int max_seq_len,
                                      float bmm1_scale, float bmm2_scale,
                                      void* out, int64_t out_stride_b, int64_t out_stride_q, int64_t out_stride_h,
                                      float* lse, void* workspace, size_t workspace_bytes,
                                      int32_t* err_flag, nvfp4kv_stream_t stream) {
    if (!lse) return nvfp4kv::fail(NVFP4KV_EINVAL, "mla_decode_lse: null lse");
    return nvfp4kv::decode_impl(q, q_stride_b, q_stride_q, q_stride_h, pool, pool_rows, tables, tables_stride,
                                seq_lens, batch, q_len, num_heads, head_dim_qk, kv_lora_rank, sparse_topk,
                                page_size, max_seq_len, bmm1_scale, bmm2_scale, out, out_stride_b,
                                out_stride_q, out_stride_h, lse, workspace, workspace_bytes, err_flag, stream);
}
