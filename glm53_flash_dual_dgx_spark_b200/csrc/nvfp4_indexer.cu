// Indexer K-pool (DSA top-k selection) over NVFP4 indexer keys.
//
// The reference's sparse MLA layers read the top-2048 rows a lightning indexer picks
// (topk_indices_buffer at vllm-0.22 flashinfer_mla_sparse.py:327-337); its indexer keys stay an
// fp8 pool ("Indexer kpool: separate pool ... stays fp8", nvfp4-kv/PLAN.md:29) because FP4
// indexer keys need sm_100 (README.md:321).  This file is that sm_100 step: 128-d indexer keys
// in NVFP4 (72 bytes a token, against 132 for fp8 + an fp32 scale), and the selection the
// sparse decode consumes, with the scoring rule of DeepSeek-V3.2's indexer as vLLM 0.22 states
// it (model_executor/models/deepseek_v2.py:604-735, layers/sparse_attn_indexer.py):
//
//   score[b, s] = sum_h w[b, h] * max(q[b, h, :] . k[s, :], 0)
//
// for every visible position s < seq_len[b], then the topk largest.
//
// Kernels:
//   index_score_kernel  one block per (query, 128-position tile): keys dequantised exactly
//                       to bf16 in shared memory (code x e4m3 scale has at most 5
//                       significant bits), K . Q^T on the tensor cores (wmma bf16, fp32
//                       accumulation), then the ReLU-weighted head sum per position.
//   index_topk_kernel   one block per query: a 4-pass 8-bit radix select of the k-th largest
//                       score, then the selected positions written in ascending order (ties
//                       at the threshold go to the lowest positions), mapped to pool rows.
#include <mma.h>

#include "abi_common.h"
#include "common.cuh"

namespace nvfp4kv {
namespace {

constexpr int kITile = 128;                         // positions per score block
constexpr int kIHeads = 64;                         // indexer heads
constexpr int kIDim = NVFP4KV_INDEX_DIM;            // 128
constexpr int kIRow = NVFP4KV_INDEX_ROW_BYTES;      // 72
constexpr int kScoreSmem = kIHeads * kIDim * 2 + kITile * kIDim * 2 + kITile * kIHeads * 4;   // 81920

struct ScoreParams {
    const __nv_bfloat16* q;       // [batch][heads][128], row strides below
    int64_t q_sb, q_sh;
    const float* w;               // [batch][heads]
    int64_t w_sb;
    const uint8_t* pool;          // [rows][72]
    int64_t pool_rows, num_pages;
    const int32_t* tables;        // [batch][>= pages] page ids
    int64_t tables_stride;
    const int32_t* seq_lens;
    int page_shift, max_seq_len, tiles;
    float* scores;                // [batch][tiles * 128]
};

__device__ __forceinline__ int clamp_len(const int32_t* seq_lens, int b, int max_len, int32_t* err) {
    int L = __ldg(seq_lens + b);
    if (L > max_len) {
        if (threadIdx.x == 0) set_error(err, NVFP4KV_DEVERR_SEQ_LEN);
        L = max_len;
    }
    return L < 0 ? 0 : L;
}

// Pool row of visible position pos of entry b, or -1 (page missing / out of the pool).
__device__ __forceinline__ int64_t index_row(const int32_t* tables, int64_t stride, int b, int pos, int shift,
                                             int64_t num_pages) {
    const int pg = __ldg(tables + b * stride + (pos >> shift));
    if (pg < 0 || pg >= num_pages) return -1;
    return (static_cast<int64_t>(pg) << shift) | (pos & ((1 << shift) - 1));
}

__device__ __forceinline__ float e2m1_val(uint32_t c) {
    const uint32_t mag = c & 7u, e = mag >> 1, m = mag & 1u;
    const float v = e == 0 ? 0.5f * m : __uint_as_float(((126u + e) << 23) | (m << 22));
    return (c & 8u) ? -v : v;
}

__global__ void __launch_bounds__(256) index_score_kernel(const ScoreParams p, int32_t* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem);              // [64 heads][128]
    __nv_bfloat16* ks = qs + kIHeads * kIDim;                                 // [128 positions][128]
    float* ss = reinterpret_cast<float*>(ks + kITile * kIDim);                // [128 positions][64 heads]
    __shared__ float ws[kIHeads];
    const int b = blockIdx.x / p.tiles, tile = blockIdx.x % p.tiles;
    const int L = clamp_len(p.seq_lens, b, p.max_seq_len, err);
    if (tile * kITile >= L) return;                  // the whole block: nothing visible here
    const int tid = threadIdx.x;
    for (int i = tid; i < kIHeads * kIDim / 8; i += blockDim.x) {
        const int h = i >> 4, c = i & 15;
        reinterpret_cast<uint4*>(qs)[i] = ldg_nc_v4(p.q + b * p.q_sb + h * p.q_sh + 8 * c);
    }
    if (tid < kIHeads) ws[tid] = __ldg(p.w + b * p.w_sb + tid);
    // keys: thread (position tid >> 1, half tid & 1) dequantises 64 elements = 4 blocks
    const int tok = tid >> 1, half = tid & 1;
    const int pos = tile * kITile + tok;
    const int64_t row = pos < L ? index_row(p.tables, p.tables_stride, b, pos, p.page_shift, p.num_pages) : -1;
    uint32_t* kdst = reinterpret_cast<uint32_t*>(ks + tok * kIDim + 64 * half);
    if (row >= 0 && row < p.pool_rows) {
        const uint8_t* src = p.pool + row * kIRow;
        const uint32_t sw = *reinterpret_cast<const uint32_t*>(src + 64 + 4 * half);   // 4 scale bytes
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
            const uint2 cw = *reinterpret_cast<const uint2*>(src + 32 * half + 8 * blk);
            const float s = e4m3_to_f32(static_cast<uint8_t>(sw >> (8 * blk)));
            const uint32_t w2[2] = {cw.x, cw.y};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t byte = (w2[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                // code x scale is exact in bf16 (at most 5 significant bits)
                const __nv_bfloat162 v = __floats2bfloat162_rn(e2m1_val(byte & 15u) * s, e2m1_val(byte >> 4) * s);
                kdst[8 * blk + j] = *reinterpret_cast<const uint32_t*>(&v);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) kdst[j] = 0u;
    }
    __syncthreads();
    // warp w: positions 16w .. 16w+15 against all 64 heads
    const int warp = tid >> 5;
    using namespace nvcuda;
    wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc[4];
#pragma unroll
    for (int n = 0; n < 4; ++n) wmma::fill_fragment(acc[n], 0.0f);
#pragma unroll
    for (int kk = 0; kk < kIDim / 16; ++kk) {
        wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::row_major> a;
        wmma::load_matrix_sync(a, ks + 16 * warp * kIDim + 16 * kk, kIDim);
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::col_major> bq;
            wmma::load_matrix_sync(bq, qs + 16 * n * kIDim + 16 * kk, kIDim);
            wmma::mma_sync(acc[n], a, bq, acc[n]);
        }
    }
#pragma unroll
    for (int n = 0; n < 4; ++n)
        wmma::store_matrix_sync(ss + 16 * warp * kIHeads + 16 * n, acc[n], kIHeads, wmma::mem_row_major);
    __syncwarp();
    // thread (position tid >> 1, heads 32 half .. +32): the ReLU-weighted sum, halves combined
    float sum = 0.0f;
#pragma unroll 8
    for (int h = 0; h < 32; ++h) sum = fmaf(ws[32 * half + h], fmaxf(ss[tok * kIHeads + 32 * half + h], 0.0f), sum);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    if (half == 0 && pos < L)
        p.scores[static_cast<int64_t>(b) * p.tiles * kITile + pos] = row >= 0 ? sum : -INFINITY;
}

// ------------------------------------------------------------------ top-k selection
constexpr int kKThreads = 1024;

// Order-preserving map of an fp32 score to an unsigned key (larger score -> larger key).
__device__ __forceinline__ uint32_t score_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive scan of one value per thread (1024 threads); `total` gets the sum.
__device__ __forceinline__ int block_scan_1024(int v, int* warp_sums, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    total = warp_sums[31];
    const int before = warp == 0 ? 0 : warp_sums[warp - 1];
    __syncthreads();
    return before + x - v;
}

struct TopkParams {
    const float* scores;          // [batch][ld]
    int64_t ld;
    const int32_t* tables;
    int64_t tables_stride;
    const int32_t* seq_lens;
    int64_t num_pages;
    int page_shift, max_seq_len, topk;
    int32_t* out_rows;            // [batch][topk]: pool rows of the selected positions, ascending; -1 after
    int32_t* out_count;           // [batch]: min(seq_len, topk)
};

__global__ void __launch_bounds__(kKThreads) index_topk_kernel(const TopkParams p, int32_t* err) {
    __shared__ int hist[32][257];                   // per-warp 256-bin histograms (+1 pad)
    __shared__ int warp_sums[32];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_remaining;
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = clamp_len(p.seq_lens, b, p.max_seq_len, err);
    const int k = n < p.topk ? n : p.topk;
    const float* sc = p.scores + static_cast<int64_t>(b) * p.ld;
    int32_t* out = p.out_rows + static_cast<int64_t>(b) * p.topk;
    if (tid == 0) p.out_count[b] = k;
    uint32_t thr = 0;
    int need_eq = 0;                                // positions with key == thr to take
    if (k < n) {
        if (tid == 0) {
            s_prefix = 0u;
            s_mask = 0u;
            s_remaining = k;
        }
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = tid; i < 32 * 257; i += kKThreads) (&hist[0][0])[i] = 0;
            __syncthreads();
            const uint32_t prefix = s_prefix, mask = s_mask;
            for (int pos = tid; pos < n; pos += kKThreads) {
                const uint32_t u = score_key(sc[pos]);
                if ((u & mask) == prefix) atomicAdd(&hist[warp][(u >> shift) & 255u], 1);
            }
            __syncthreads();
            if (warp == 0) {
                // bins 255 .. 0 in chunks of 32 from the top; find where the running count
                // from the top reaches `remaining`
                const int remaining = s_remaining;
                int above = 0, found = -1, above_found = 0;
                for (int base = 224; base >= 0 && found < 0; base -= 32) {
                    const int bin = base + (31 - lane);      // lane 0 takes the highest bin
                    int c = 0;
                    for (int w = 0; w < 32; ++w) c += hist[w][bin];
                    int incl = c;                            // inclusive prefix over lanes 0..lane
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                        if (lane >= o) incl += y;
                    }
                    const bool hit = above + incl >= remaining;
                    const unsigned ballot = __ballot_sync(0xFFFFFFFFu, hit);
                    if (ballot) {
                        const int first = __ffs(ballot) - 1;
                        const int excl = __shfl_sync(0xFFFFFFFFu, incl - c, first);
                        found = base + (31 - first);
                        above_found = above + excl;
                    } else {
                        above += __shfl_sync(0xFFFFFFFFu, incl, 31);
                    }
                }
                if (lane == 0) {
                    s_prefix |= static_cast<uint32_t>(found) << shift;
                    s_mask |= 255u << shift;
                    s_remaining = remaining - above_found;
                }
            }
            __syncthreads();
        }
        thr = s_prefix;
        need_eq = s_remaining;
    }
    // selection in ascending position order: thread tid owns positions [tid c, tid c + c)
    const int chunk = (n + kKThreads - 1) / kKThreads;
    const int lo = tid * chunk, hi = min(n, lo + chunk);
    int eq = 0;
    if (k < n)
        for (int pos = lo; pos < hi; ++pos) eq += score_key(sc[pos]) == thr;
    int eq_total;
    const int eq_base = block_scan_1024(eq, warp_sums, eq_total);
    int sel = 0;
    for (int pos = lo, r = eq_base; pos < hi; ++pos) {
        if (k >= n) { ++sel; continue; }
        const uint32_t u = score_key(sc[pos]);
        if (u > thr) ++sel;
        else if (u == thr) sel += (r++ < need_eq);
    }
    int sel_total;
    int o = block_scan_1024(sel, warp_sums, sel_total);
    for (int pos = lo, r = eq_base; pos < hi; ++pos) {
        bool take = k >= n;
        if (!take) {
            const uint32_t u = score_key(sc[pos]);
            take = u > thr || (u == thr && r++ < need_eq);
        }
        if (take) {
            const int64_t row = index_row(p.tables, p.tables_stride, b, pos, p.page_shift, p.num_pages);
            out[o++] = row >= 0 ? static_cast<int32_t>(row) : -1;
        }
    }
    for (int j = k + tid; j < p.topk; j += kKThreads) out[j] = -1;
}

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_index_topk_workspace_size(int batch, int max_seq_len, size_t* bytes) {
    using namespace nvfp4kv;
    if (!bytes) return fail(NVFP4KV_EINVAL, "index_topk_workspace_size: null output");
    if (batch < 0 || max_seq_len < 0) return fail(NVFP4KV_EINVAL, "index_topk_workspace_size: bad shape");
    const int64_t tiles = (static_cast<int64_t>(max_seq_len) + kITile - 1) / kITile;
    *bytes = static_cast<size_t>(batch) * static_cast<size_t>(tiles) * kITile * sizeof(float);
    return NVFP4KV_OK;
}

extern "C" int nvfp4kv_index_topk(const void* q, int64_t q_stride_b, int64_t q_stride_h, const float* weights,
                                  int64_t weights_stride, const uint8_t* index_pool, int64_t pool_rows,
                                  const int32_t* tables, int64_t tables_stride, const int32_t* seq_lens,
                                  int batch, int num_heads, int page_size, int max_seq_len, int topk,
                                  int32_t* out_rows, int32_t* out_count, void* workspace, size_t workspace_bytes,
                                  int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (batch < 0) return fail(NVFP4KV_EINVAL, "index_topk: batch < 0");
    if (batch == 0) return NVFP4KV_OK;
    if (!q || !weights || !index_pool || !tables || !seq_lens || !out_rows || !out_count)
        return fail(NVFP4KV_EINVAL, "index_topk: null pointer");
    if (num_heads != kIHeads) return fail(NVFP4KV_EINVAL, "index_topk: num_heads must be 64 (got %d)", num_heads);
    if (topk < 1 || max_seq_len < 0) return fail(NVFP4KV_EINVAL, "index_topk: bad topk / max_seq_len");
    if (pool_rows <= 0) return fail(NVFP4KV_EINVAL, "index_topk: empty index pool");
    if (page_size <= 0 || (page_size & (page_size - 1)) || page_size > 4096 || pool_rows % page_size)
        return fail(NVFP4KV_EINVAL, "index_topk: page_size must be a power of two <= 4096 dividing pool_rows");
    if (reinterpret_cast<uintptr_t>(q) % 16 || q_stride_b % 8 || q_stride_h % 8 ||
        reinterpret_cast<uintptr_t>(index_pool) % 8)
        return fail(NVFP4KV_EINVAL, "index_topk: q must be 16-byte aligned with strides multiples of 8, "
                                    "the index pool 8-byte aligned");
    size_t need = 0;
    nvfp4kv_index_topk_workspace_size(batch, max_seq_len, &need);
    if (need > 0 && (!workspace || workspace_bytes < need))
        return fail(NVFP4KV_EWORKSPACE, "index_topk: workspace %zu bytes < %zu required", workspace_bytes, need);
    if (reinterpret_cast<uintptr_t>(workspace) % 16)
        return fail(NVFP4KV_EINVAL, "index_topk: workspace must be 16-byte aligned");
    int shift = 0;
    while ((1 << shift) < page_size) ++shift;
    const int tiles = (max_seq_len + kITile - 1) / kITile;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (tiles > 0) {
        static int attr_done[64] = {0};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaGetDevice failed");
        if (dev < 0 || dev >= 64 || !attr_done[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(index_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       kScoreSmem);
            if (e != cudaSuccess) return fail(NVFP4KV_ECUDA, "index_topk: smem attribute: %s", cudaGetErrorString(e));
            if (dev >= 0 && dev < 64) attr_done[dev] = 1;
        }
        ScoreParams sp{};
        sp.q = static_cast<const __nv_bfloat16*>(q); sp.q_sb = q_stride_b; sp.q_sh = q_stride_h;
        sp.w = weights; sp.w_sb = weights_stride;
        sp.pool = index_pool; sp.pool_rows = pool_rows; sp.num_pages = pool_rows / page_size;
        sp.tables = tables; sp.tables_stride = tables_stride; sp.seq_lens = seq_lens;
        sp.page_shift = shift; sp.max_seq_len = max_seq_len; sp.tiles = tiles;
        sp.scores = static_cast<float*>(workspace);
        index_score_kernel<<<static_cast<unsigned>(static_cast<int64_t>(batch) * tiles), 256, kScoreSmem, st>>>(
            sp, err_flag);
        int rc = check_launch("nvfp4kv_index_topk (scores)");
        if (rc != NVFP4KV_OK) return rc;
    }
    TopkParams tp{};
    tp.scores = static_cast<const float*>(workspace); tp.ld = static_cast<int64_t>(tiles) * kITile;
    tp.tables = tables; tp.tables_stride = tables_stride; tp.seq_lens = seq_lens;
    tp.num_pages = pool_rows / page_size; tp.page_shift = shift; tp.max_seq_len = max_seq_len; tp.topk = topk;
    tp.out_rows = out_rows; tp.out_count = out_count;
    index_topk_kernel<<<static_cast<unsigned>(batch), kKThreads, 0, st>>>(tp, err_flag);
    return check_launch("nvfp4kv_index_topk (selection)");
}
