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
//   index_score_kernel  one block per (query, run of 8 128-position tiles): keys dequantised exactly
//                       to fp16 in shared memory by the hardware conversions (code x e4m3
//                       scale has at most 5 significant bits), q in fp16 after an exact
//                       power-of-two scale per head (folded into the head's weight), K . Q^T on
//                       the tensor cores (mma.sync m16n8k16 fp16, fp32 accumulation; a warp
//                       takes 32 positions x 32 heads and keeps its q fragments in registers for
//                       the run), then the ReLU-weighted head sum per position from the
//                       accumulators.
//   index_topk_kernel   one thread-block cluster of 8 CTAs per query, each CTA an eighth of
//                       the positions: an 8-pass 4-bit radix select of the k-th largest score
//                       (digit counts exchanged through distributed shared memory), then the
//                       selected positions written in ascending order (ties at the threshold
//                       go to the lowest positions), mapped to pool rows.
#include "abi_common.h"
#include "common.cuh"

namespace nvfp4kv {
namespace {

constexpr int kITile = 128;                         // positions per score block
constexpr int kIHeads = 64;                         // indexer heads
constexpr int kIDim = NVFP4KV_INDEX_DIM;            // 128
constexpr int kIRow = NVFP4KV_INDEX_ROW_BYTES;      // 72
// Shared-memory row strides padded by 16 bytes: rows 256 bytes apart would put every row of a
// 16 x 16 fragment load in the same banks.
constexpr int kQLd = kIDim + 8;                     // fp16 elements
constexpr int kKLd = kIDim + 8;
constexpr int kScoreSmem = kIHeads * kQLd * 2 + kITile * kKLd * 2;   // 52224

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

// One thread's share of a key tile: position tid >> 1, half tid & 1 (64 elements = 4 blocks):
// 32 code bytes and 4 scale bytes, loaded ahead of their use.
struct KeyPart {
    uint2 c[4];
    uint32_t s;
    bool ok;
};

__device__ __forceinline__ KeyPart load_key_part(const ScoreParams& p, int b, int pos, int L, int half) {
    KeyPart k{};
    const int64_t row = pos < L ? index_row(p.tables, p.tables_stride, b, pos, p.page_shift, p.num_pages) : -1;
    k.ok = row >= 0;
    if (k.ok) {
        const uint8_t* src = p.pool + row * kIRow;
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) k.c[blk] = *reinterpret_cast<const uint2*>(src + 32 * half + 8 * blk);
        k.s = *reinterpret_cast<const uint32_t*>(src + 64 + 4 * half);
    }
    return k;
}

// Dequantise a key part into the fp16 tile row with the hardware conversions (e2m1 pair ->
// f16x2, e4m3 pair -> f16x2, one f16x2 multiply): code x scale is exact in fp16 (at most 5
// significant bits, magnitudes 2^-10 .. 2688), zeros for a masked position.
__device__ __forceinline__ void store_key_part(const KeyPart& k, uint32_t* dst) {
    if (!k.ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) dst[j] = 0u;
        return;
    }
    const uint32_t s01 = e4m3x2_to_f16x2(static_cast<uint16_t>(k.s & 0xFFFFu));
    const uint32_t s23 = e4m3x2_to_f16x2(static_cast<uint16_t>(k.s >> 16));
    const uint32_t sb[4] = {(s01 & 0xFFFFu) * 0x10001u, (s01 >> 16) * 0x10001u, (s23 & 0xFFFFu) * 0x10001u,
                            (s23 >> 16) * 0x10001u};
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const uint32_t w2[2] = {k.c[blk].x, k.c[blk].y};
#pragma unroll
        for (int j = 0; j < 8; ++j)
            dst[8 * blk + j] = hmul2_u32(e2m1x2_to_f16x2((w2[j >> 2] >> (8 * (j & 3))) & 0xFFu), sb[blk]);
    }
}

// Tensor-core fragments of mma.sync m16n8k16 (fp16 in, fp32 accumulation): A 16 x 16 row-major
// from four 8 x 8 shared-memory matrices, B 16 x 8 (k x n) from two, stored n-major.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Block = (entry b, a run of kTilesPerBlock position tiles): the entry's q and weights are
// loaded once, and each tile's key bytes are loaded a tile ahead of their dequantisation.
constexpr int kTilesPerBlock = 8;

__global__ void __launch_bounds__(256) index_score_kernel(const ScoreParams p, int32_t* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __half* qs = reinterpret_cast<__half*>(smem);                            // [64 heads][kQLd] fp16
    __half* ks = qs + kIHeads * kQLd;                                        // [128 positions][kKLd] fp16
    __shared__ float ws[kIHeads];
    __shared__ float red[2 * kITile];                // per head half: the tile's partial sums
    __shared__ uint8_t tile_ok[kITile];              // position on a page of the pool
    const int runs = (p.tiles + kTilesPerBlock - 1) / kTilesPerBlock;
    const int b = blockIdx.x / runs, run = blockIdx.x % runs;
    const int L = clamp_len(p.seq_lens, b, p.max_seq_len, err);
    const int t0 = run * kTilesPerBlock;
    const int t1 = min(min(t0 + kTilesPerBlock, p.tiles), (L + kITile - 1) / kITile);
    if (t0 >= t1) return;                            // the whole block: nothing visible here
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    {
        // q in fp16 for the fp16 tensor-core product: head h is scaled by 2^(10 - e_h), e_h =
        // floor(log2 max|q_h|), which is exact and keeps the head inside fp16's range, and its
        // weight by 2^(e_h - 10) (max(c x, 0) = c max(x, 0) for c > 0).  Four threads per head,
        // 32 dims each.
        const int h = tid >> 2, c0 = 32 * (tid & 3);
        const __nv_bfloat16* src = p.q + b * p.q_sb + h * p.q_sh + c0;
        uint4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = ldg_nc_v4(src + 8 * j);
        float x[32];
        float am = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                x[8 * j + 2 * t] = __uint_as_float(w4[t] << 16);
                x[8 * j + 2 * t + 1] = __uint_as_float(w4[t] & 0xFFFF0000u);
            }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) am = fmaxf(am, fabsf(x[j]));
        am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, 2));
        const int eb = static_cast<int>((__float_as_uint(am) >> 23) & 0xFFu);   // biased exponent
        const int e = (eb > 0 && eb < 255) ? eb - 127 : 0;
        const int sh = max(-100, min(100, 10 - e));
        const float mul = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);   // 2^sh
        uint32_t* dst = reinterpret_cast<uint32_t*>(qs + h * kQLd + c0);
#pragma unroll
        for (int j = 0; j < 16; ++j) dst[j] = pack_half2(x[2 * j] * mul, x[2 * j + 1] * mul);
        if ((tid & 3) == 0) ws[h] = __ldg(p.w + b * p.w_sb + h) * __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
    }
    const int tok = tid >> 1, half = tid & 1;
    uint32_t* kdst = reinterpret_cast<uint32_t*>(ks + tok * kKLd + 64 * half);
    KeyPart next = load_key_part(p, b, t0 * kITile + tok, L, half);
    __syncthreads();                                 // q and the weights are in shared memory
    // Warp w: positions 32 (w & 3) .. +31 (two m-tiles of 16) x heads 32 (w >> 2) .. +31 (four
    // n-tiles of 8): the key tile is read twice per tile in all (not once per warp), and the
    // warp's q fragments (B of m16n8k16, all 128 dims) and weights stay in registers for the run.
    const int pb = warp & 3, hq = warp >> 2;
    uint32_t qf[kIDim / 16][4][2];
#pragma unroll
    for (int kk = 0; kk < kIDim / 16; ++kk)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
            ldsm_x2(smem_u32(qs + (32 * hq + 8 * nt + (lane & 7)) * kQLd + 16 * kk + 8 * ((lane >> 3) & 1)),
                    qf[kk][nt]);
    float wv[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
        wv[nt][0] = ws[32 * hq + 8 * nt + 2 * (lane & 3)];
        wv[nt][1] = ws[32 * hq + 8 * nt + 2 * (lane & 3) + 1];
    }
#pragma unroll 1
    for (int tile = t0; tile < t1; ++tile) {
        const KeyPart cur = next;
        __syncthreads();                             // the previous tile's keys and sums are consumed
        store_key_part(cur, kdst);
        if (half == 0) tile_ok[tok] = cur.ok;
        if (tile + 1 < t1) next = load_key_part(p, b, (tile + 1) * kITile + tok, L, half);
        __syncthreads();
        // thread l of the warp ends with positions 32 pb + 16 mt + l/4 (+8) x heads
        // 32 hq + 8 nt + 2 (l % 4) (+1); the ReLU-weighted sum over its heads, then the quad's
        float acc[2][4][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[mt][nt][j] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < kIDim / 16; ++kk) {
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                uint32_t af[4];
                ldsm_x4(smem_u32(ks + (32 * pb + 16 * mt + (lane & 15)) * kKLd + 16 * kk + 8 * (lane >> 4)), af);
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) mma_16816(acc[mt][nt], af, qf[kk][nt]);
            }
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            float lo = 0.0f, hi = 0.0f;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                lo = fmaf(wv[nt][0], fmaxf(acc[mt][nt][0], 0.0f), fmaf(wv[nt][1], fmaxf(acc[mt][nt][1], 0.0f), lo));
                hi = fmaf(wv[nt][0], fmaxf(acc[mt][nt][2], 0.0f), fmaf(wv[nt][1], fmaxf(acc[mt][nt][3], 0.0f), hi));
            }
            lo += __shfl_xor_sync(0xFFFFFFFFu, lo, 1);
            lo += __shfl_xor_sync(0xFFFFFFFFu, lo, 2);
            hi += __shfl_xor_sync(0xFFFFFFFFu, hi, 1);
            hi += __shfl_xor_sync(0xFFFFFFFFu, hi, 2);
            if ((lane & 3) == 0) {
                red[hq * kITile + 32 * pb + 16 * mt + (lane >> 2)] = lo;
                red[hq * kITile + 32 * pb + 16 * mt + (lane >> 2) + 8] = hi;
            }
        }
        __syncthreads();
        if (tid < kITile) {
            const float sum = red[tid] + red[kITile + tid];
            const int pos = tile * kITile + tid;
            if (pos < L) p.scores[static_cast<int64_t>(b) * p.tiles * kITile + pos] = tile_ok[tid] ? sum : -INFINITY;
        }
    }
}

// ------------------------------------------------------------------ top-k selection
constexpr int kKThreads = 512;

// Order-preserving map of an fp32 score to an unsigned key (larger score -> larger key).
__device__ __forceinline__ uint32_t score_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
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
    int staged;                   // every CTA's chunk fits kStageMax keys: staged in shared memory
};

// One query per cluster of kCl CTAs, CTA r taking positions [r c, (r + 1) c) of the query's
// n scores (c = ceil(n / kCl), a multiple of kKThreads).  A radix select with 4-bit digits,
// most significant first, finds the k-th largest key: each thread counts the 16 digits of its
// candidates in registers (shared-memory atomics serialise on the few bins the scores crowd
// into), a CTA's warps reduce them, and every CTA reads all kCl CTAs' counts of the pass
// through distributed shared memory after one cluster barrier (the counts are double-buffered
// by pass, so a CTA overwrites a buffer only two passes after it was written, when every peer
// has read it) and picks the same digit.  Then every position above the threshold and the
// first need_eq ties, in ascending position order, go out: a CTA's output offset is the count
// taken by the CTAs before it (from their (above, tie) counts, after one more cluster barrier),
// and within a CTA coalesced rounds of kKThreads positions place them by ballot prefix counts.
// A last cluster barrier keeps every CTA alive until its peers' remote reads are done.  A
// CTA's keys are staged once in shared memory when its chunk fits (kStageMax keys: 128K-token
// contexts and somewhat beyond), so the eight passes and the selection read them there; a
// longer chunk is read from the score buffer on every pass.
constexpr int kCl = 8;
constexpr int kStageMax = 40960;                    // keys a CTA stages (160 KB)

__global__ void __launch_bounds__(kKThreads) index_topk_kernel(const TopkParams p, int32_t* err) {
    extern __shared__ __align__(16) uint32_t skeys[];  // [chunk] when staged
    __shared__ int hist[kKThreads / 32][17];        // per-warp counts of the 16 digits
    __shared__ int cta_cnt[2][16];                  // this CTA's digit counts, by pass parity
    __shared__ int s_part[kCl][16];                 // the peers' counts of the pass
    __shared__ int s_tot[16];                       // the cluster's counts of the pass
    __shared__ int sel[2];                          // this CTA's (above, tie) counts
    __shared__ int s_before[2];                     // the same, summed over the CTAs before it
    constexpr int kWarps = kKThreads / 32;
    const int rank = static_cast<int>(cluster_rank());
    const int b = blockIdx.x / kCl, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = clamp_len(p.seq_lens, b, p.max_seq_len, rank == 0 ? err : nullptr);
    const int k = n < p.topk ? n : p.topk;
    const int chunk = ((n + kCl - 1) / kCl + kKThreads - 1) / kKThreads * kKThreads;
    const int lo = min(n, rank * chunk), hi = min(n, lo + chunk);
    const float* sc = p.scores + static_cast<int64_t>(b) * p.ld;
    int32_t* out = p.out_rows + static_cast<int64_t>(b) * p.topk;
    if (tid == 0 && rank == 0) p.out_count[b] = k;
    const bool all = k >= n;                        // the same in every CTA of the cluster
    const bool staged = p.staged != 0;              // chunk <= kStageMax for every query of the call
    if (staged) {
        for (int pos = lo + tid; pos < hi; pos += kKThreads) skeys[pos - lo] = score_key(sc[pos]);
        __syncthreads();
    }
    auto key = [&](int pos) -> uint32_t { return staged ? skeys[pos - lo] : score_key(sc[pos]); };
    uint32_t prefix = 0u, mask = 0u;
    int remaining = k;
    if (!all) {
        for (int pass = 0; pass < 8; ++pass) {
            const int shift = 28 - 4 * pass;
            // the 16 counts as 8-bit fields of two 64-bit registers, drained into integers
            // every 255 keys a thread sees (once per pass for a staged chunk: <= 80 keys)
            int c[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) c[j] = 0;
            for (int base = lo + tid; base < hi; base += 255 * kKThreads) {
                uint64_t c_lo = 0, c_hi = 0;
                const int lim = min(hi, base + 255 * kKThreads);
                for (int pos = base; pos < lim; pos += kKThreads) {
                    const uint32_t u = key(pos);
                    if ((u & mask) == prefix) {
                        const uint32_t d = (u >> shift) & 15u;
                        const uint64_t one = 1ull << (8 * (d & 7u));
                        if (d < 8) c_lo += one;
                        else c_hi += one;
                    }
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) c[j] += static_cast<int>(((j < 8 ? c_lo : c_hi) >> (8 * (j & 7))) & 0xFFu);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) c[j] = __reduce_add_sync(0xFFFFFFFFu, c[j]);
            if (lane == 0)
#pragma unroll
                for (int j = 0; j < 16; ++j) hist[warp][j] = c[j];
            __syncthreads();
            if (tid < 16) {
                int t = 0;
                for (int w = 0; w < kWarps; ++w) t += hist[w][tid];
                cta_cnt[pass & 1][tid] = t;
            }
            cluster_sync();                         // every CTA's counts of this pass are out
            if (tid < 16 * kCl) {                   // one remote load per thread, all in flight
                const int r = tid >> 4, j = tid & 15;
                s_part[r][j] = ld_cluster_s32(cluster_map(smem_u32(&cta_cnt[pass & 1][j]), static_cast<uint32_t>(r)));
            }
            __syncthreads();
            if (tid < 16) {
                int t = 0;
#pragma unroll
                for (int r = 0; r < kCl; ++r) t += s_part[r][tid];
                s_tot[tid] = t;
            }
            __syncthreads();
            // the digit at which the count from the top reaches the number still wanted (every
            // thread computes it from the same totals)
            int above = 0, digit = 0;
            for (int dg = 15; dg >= 0; --dg) {
                const int t = s_tot[dg];
                if (above + t >= remaining) {
                    digit = dg;
                    break;
                }
                above += t;
            }
            prefix |= static_cast<uint32_t>(digit) << shift;
            mask |= 15u << shift;
            remaining -= above;
        }
    }
    const uint32_t thr = prefix;
    const int need_eq = all ? 0 : remaining;        // ties (key == thr) to take, lowest positions first
    // Selection: warp w walks the contiguous positions [lo + w wc, lo + (w + 1) wc) of this
    // CTA's chunk (wc = chunk / kWarps, a multiple of 32) in rounds of 32: a first walk counts
    // the positions above the threshold and the ties, whose sums over the warps and then over
    // the CTAs before this one (after a cluster barrier) give each warp its offsets, and a
    // second walk writes them in ascending order (ballot prefix counts within a round).
    const int wc = chunk / kWarps;
    const int wlo = min(hi, lo + warp * wc), whi = min(hi, wlo + wc);
    const unsigned below = (1u << lane) - 1u;
    int w_gt = 0, w_eq = 0;
    if (!all)
        for (int base = wlo; base < whi; base += 32) {
            const int pos = base + lane;
            const uint32_t u = pos < whi ? key(pos) : 0u;
            w_gt += __popc(__ballot_sync(0xFFFFFFFFu, pos < whi && u > thr));
            w_eq += __popc(__ballot_sync(0xFFFFFFFFu, pos < whi && u == thr));
        }
    if (lane == 0) {
        hist[warp][2] = w_gt;
        hist[warp][3] = w_eq;
    }
    __syncthreads();
    if (tid < 2) {
        int t = 0;
        for (int w = 0; w < kWarps; ++w) t += hist[w][2 + tid];
        sel[tid] = t;
    }
    cluster_sync();                                 // every CTA's (above, tie) counts are out
    if (tid < 2) {
        const uint32_t a = smem_u32(&sel[tid]);
        int t = 0;
        for (int r = 0; r < rank; ++r) t += ld_cluster_s32(cluster_map(a, static_cast<uint32_t>(r)));
        s_before[tid] = t;
    }
    __syncthreads();
    int gt_off = 0, eq_off = 0;
    for (int w = 0; w < warp; ++w) {
        gt_off += hist[w][2];
        eq_off += hist[w][3];
    }
    int eq_before = s_before[1] + eq_off;                       // ties before this warp's range
    int out_before = all ? wlo : s_before[0] + gt_off + min(eq_before, need_eq);
    for (int base = wlo; base < whi; base += 32) {
        const int pos = base + lane;
        const bool in = pos < whi;
        const uint32_t u = in ? key(pos) : 0u;
        const bool eq = in && !all && u == thr;
        const unsigned beq = __ballot_sync(0xFFFFFFFFu, eq);
        const bool take = (all && in) || (in && !all && u > thr) || (eq && eq_before + __popc(beq & below) < need_eq);
        const unsigned btk = __ballot_sync(0xFFFFFFFFu, take);
        const int slot = out_before + __popc(btk & below);
        if (take && slot < p.topk) {   // exactly k are taken; the bound only guards the row
            const int64_t row = index_row(p.tables, p.tables_stride, b, pos, p.page_shift, p.num_pages);
            out[slot] = row >= 0 ? static_cast<int32_t>(row) : -1;
        }
        eq_before += __popc(beq);
        out_before += __popc(btk);
    }
    if (rank == kCl - 1)
        for (int j = k + tid; j < p.topk; j += kKThreads) out[j] = -1;
    cluster_sync();                                 // no CTA exits while a peer reads its counts
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
        const int64_t runs = (tiles + kTilesPerBlock - 1) / kTilesPerBlock;
        index_score_kernel<<<static_cast<unsigned>(static_cast<int64_t>(batch) * runs), 256, kScoreSmem, st>>>(
            sp, err_flag);
        int rc = check_launch("nvfp4kv_index_topk (scores)");
        if (rc != NVFP4KV_OK) return rc;
    }
    TopkParams tp{};
    tp.scores = static_cast<const float*>(workspace); tp.ld = static_cast<int64_t>(tiles) * kITile;
    tp.tables = tables; tp.tables_stride = tables_stride; tp.seq_lens = seq_lens;
    tp.num_pages = pool_rows / page_size; tp.page_shift = shift; tp.max_seq_len = max_seq_len; tp.topk = topk;
    tp.out_rows = out_rows; tp.out_count = out_count;
    // chunk per CTA for the longest query: ceil(max_seq_len / kCl) rounded up to kKThreads
    const int64_t chunk = ((static_cast<int64_t>(max_seq_len) + kCl - 1) / kCl + kKThreads - 1) / kKThreads * kKThreads;
    tp.staged = chunk <= kStageMax ? 1 : 0;
    const size_t stage_bytes = tp.staged ? static_cast<size_t>(chunk) * 4 : 0;
    {
        static int topk_attr_done[64] = {0};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaGetDevice failed");
        if (dev < 0 || dev >= 64 || !topk_attr_done[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(index_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       kStageMax * 4);
            if (e != cudaSuccess) return fail(NVFP4KV_ECUDA, "index_topk: smem attribute: %s", cudaGetErrorString(e));
            if (dev >= 0 && dev < 64) topk_attr_done[dev] = 1;
        }
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(batch) * kCl);
    cfg.blockDim = dim3(kKThreads);
    cfg.dynamicSmemBytes = stage_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, index_topk_kernel, tp, err_flag);
    if (le != cudaSuccess) return fail(NVFP4KV_ECUDA, "index_topk: selection launch: %s", cudaGetErrorString(le));
    return check_launch("nvfp4kv_index_topk (selection)");
}
