// Fused NVFP4 gather + dequant + MLA decode attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces, at the reference's read seam (nvfp4-kv/patch_nvfp4_kv.py:84-118), the pair
//   build_scratch(...)                       -> 656-byte fp8 scratch (glm53_nvfp4_runtime.py:143-182)
//   trtllm_batch_decode_with_kv_cache_mla(...) -> attention over that scratch
// with one kernel that reads the 288-byte pool rows directly.
//
// Work unit (one CTA, one per SM): query group (b, g) x token split s.  A query group is up
// to 64 query rows (MTP token i, head h) of batch entry b; they all share the latent rows.
//
// With only 64 query rows the tensor core is used in its M=64 ("rows on M") form: one MMA
// instruction costs about the same for any N up to 128, so the shapes are chosen to put as
// many tokens or latent dims as possible on N.
//
//   TMEM (512 columns, M=64 layout: row r -> lane r%16 + 32*(r/16) + {0 | 16}).  An MMA that
//   reads A from TMEM keeps A and D at lane offset 0; only SMEM-operand MMAs use offset 16.
//     lanes +0 : columns [0,256) Q (fp16 A operand of QK, 64 rows x 512),
//                columns [256,384) S (fp32, 64 rows x 128 tokens)
//     lanes +16: columns [0,512) O (fp32, 64 rows x 512)
//   SMEM: fp16 KV tile [128 tokens x 512] (128B-swizzled, 8 d-blocks), P [64 rows x 128
//         tokens] fp16, a 2-slot ring of raw 288-byte rows (one 128-token tile per slot).
//
// Per 128-token tile:
//   producers (4 warps, thread = token): cp.async.bulk the raw row of tile i+1 into the ring
//     (one tile ahead; completion counted in bytes on an mbarrier), then dequantise tile i
//     from the ring with cvt.rn.f16x2.e2m1x2 x e4m3 scale (exact in fp16) into the KV tile,
//     one 128-d chunk at a time (kv_full[c] / kv_empty[c]), and publish a validity mask.
//   MMA thread: S = Q K^T    M=64 N=128 K=512, A = Q from TMEM, B = KV tile (K-major);
//               O += P V     M=64 N=256 (d half) K=128, A = P (K-major), B = KV tile (MN-major).
//   softmax (4 warps): lanes 0-15 own the S/P row of query row 16w + lane (row max / exp /
//     row sum are thread-local over the tile's 128 columns); lanes 16-31 own the O row.  O is
//     rescaled only when some row max grows by more than 2^8 (a vote over the 128 threads).
// Splits write unnormalised partial O plus (max, sum) per row; a combine kernel merges them
// with log-sum-exp weights.  Every wait is bounded (common.cuh).
#include <math.h>

#include "abi_common.h"
#include "common.cuh"
#include "decode_shared.h"

namespace nvfp4kv {
namespace {

constexpr int kTile = 128;        // tokens per tile
constexpr int kNQ = 64;           // query rows per CTA (MMA M)
constexpr int kSoftmaxWarps = 4;  // warps 0-3: TMEM lane quadrants 0-3
constexpr int kMmaWarp = 4;
constexpr int kProducerWarps = 4;  // warps 5-8, thread = token of the tile
constexpr int kThreads = (kSoftmaxWarps + 1 + kProducerWarps) * 32;
constexpr int kMaxSplits = 64;
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when a row max grows by > 2^8

// Shared memory map, offsets from a 1024-byte aligned base.
constexpr int SM_KV = 0;                          // 8 d-blocks x [128 tokens x 128 B], fp16
constexpr int SM_P = SM_KV + 8 * kTile * 128;     // 2 token-blocks x [64 rows x 128 B], fp16
constexpr int SM_STAGE = SM_P + 2 * kNQ * 128;    // 2 slots x [128 rows x 288 B] raw pool rows
constexpr int kSlotBytes = kTile * kRowBytes;
constexpr int SM_QSCALE = SM_STAGE + 2 * kSlotBytes;  // 64 floats: log2e * bmm1_scale * 2^e_row
constexpr int SM_LIMIT = SM_QSCALE + 64 * 4;      // 64 ints: visible token bound per row
constexpr int SM_ALPHA = SM_LIMIT + 64 * 4;       // 64 floats: per-tile rescale factors
constexpr int SM_MROW = SM_ALPHA + 64 * 4;        // 64 floats: final row max (log2 units)
constexpr int SM_LSUM = SM_MROW + 64 * 4;         // 64 floats: final row sums
constexpr int SM_ROWOFF = SM_LSUM + 64 * 4;       // 64 int64: output row offsets (elements)
constexpr int SM_MASK = SM_ROWOFF + 64 * 8;       // 2 tiles x 4 words: valid-token bitmask
constexpr int kMaxIdx = 1024;                     // staged page ids (dense) / row indices (sparse)
constexpr int SM_IDX = SM_MASK + 2 * 4 * 4;       // kMaxIdx int32 for this CTA's token range
constexpr int SM_FLAGS = SM_IDX + kMaxIdx * 4;    // [1] abort, [2] tmem base
constexpr int SM_BARS = SM_FLAGS + 64;
enum { B_KV_FULL = 0, B_KV_EMPTY = 4, B_S_FULL = 8, B_P_FULL = 9, B_PV_DONE = 10, B_FINAL = 11,
       B_STAGE = 12, B_Q = 14, kNumBars = 15 };
constexpr int SM_END = SM_BARS + kNumBars * 8;
constexpr int kSmemBytes = SM_END + 1024;         // slack for aligning the base
static_assert(kSmemBytes <= 232448, "shared memory budget");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kHalfB = 16u << 16;   // lane offset of the second M=64 accumulator tile
constexpr uint32_t kTmemQ = 0;           // lanes 0..15 of each quadrant, columns [0, 256)
constexpr uint32_t kTmemS = 256;         // lanes 0..15, columns [256, 384)
constexpr uint32_t kTmemO = kHalfB;      // lanes 16..31, columns [0, 512): d = column

struct DecodeParams {
    const __nv_bfloat16* q;
    int64_t q_sb, q_sq, q_sh;
    const uint8_t* pool;
    int64_t pool_rows;
    const int32_t* tables;
    int64_t tables_stride;
    const int32_t* seq_lens;
    int batch, q_len, num_heads, groups, splits;
    int sparse, topk;
    int page_shift;
    int64_t num_pages;
    int max_seq_len, tiles_total;   // tiles of the planned context, spread over the splits
    float scale_log2, bmm2_scale;
    __nv_bfloat16* out;
    int64_t o_sb, o_sq, o_sh;
    float* part_o;   // [splits][batch][groups][64][512]
    float* part_ml;  // [splits][batch][groups][64][2]
    int32_t* err;
};

// Pool row of token position t (within batch entry b), or -1 when the token is masked.
// Page ids (dense) or row indices (sparse) of the CTA's token range come from shared memory
// when they were staged there (`sidx`, first entry `idx_base`), else from global memory.
template <bool kSparse>
__device__ __forceinline__ int64_t row_of(const DecodeParams& p, const int* sidx, bool staged,
                                          int idx_base, int b, int t, int end, bool report) {
    if (t >= end) return -1;
    if constexpr (kSparse) {
        const int32_t idx = staged ? sidx[t - idx_base] : __ldg(p.tables + b * p.tables_stride + t);
        if (idx < 0 || idx >= p.pool_rows) {
            if (report && idx != -1) set_error(p.err, NVFP4KV_DEVERR_BAD_INDEX);
            return -1;
        }
        return idx;
    } else {
        const int pi = t >> p.page_shift;
        const int32_t pg = staged ? sidx[pi - idx_base] : __ldg(p.tables + b * p.tables_stride + pi);
        if (pg < 0 || pg >= p.num_pages) {
            if (report) set_error(p.err, NVFP4KV_DEVERR_BAD_PAGE);
            return -1;
        }
        return (static_cast<int64_t>(pg) << p.page_shift) | (t & ((1 << p.page_shift) - 1));
    }
}

template <bool kSparse>
__global__ void __launch_bounds__(kThreads, 1) mla_decode_kernel(const DecodeParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int s = blockIdx.x % p.splits;
    const int bg = blockIdx.x / p.splits;
    const int g = bg % p.groups;
    const int b = bg / p.groups;

    // Context length of this batch entry and this CTA's token range [start, end).
    int L = __ldg(p.seq_lens + b);
    const int cap = kSparse ? p.topk : p.max_seq_len;
    if (L > cap) {
        if (threadIdx.x == 0) set_error(p.err, NVFP4KV_DEVERR_SEQ_LEN);
        L = cap;
    }
    if (L < 0) L = 0;
    // split s covers tiles [s T / splits, (s + 1) T / splits) of the planned context
    const int start = static_cast<int>((static_cast<int64_t>(s) * p.tiles_total) / p.splits) * kTile;
    const int end = min(static_cast<int>((static_cast<int64_t>(s + 1) * p.tiles_total) / p.splits) * kTile, L);
    const int n_tiles = end > start ? (end - start + kTile - 1) / kTile : 0;
    const int rows_total = p.q_len * p.num_heads;
    const int rows_here = min(kNQ, rows_total - g * kNQ);

    float* qscale = reinterpret_cast<float*>(smem + SM_QSCALE);
    int* limit = reinterpret_cast<int*>(smem + SM_LIMIT);
    float* alpha = reinterpret_cast<float*>(smem + SM_ALPHA);
    float* mrow = reinterpret_cast<float*>(smem + SM_MROW);
    float* lsum = reinterpret_cast<float*>(smem + SM_LSUM);
    int64_t* rowoff = reinterpret_cast<int64_t*>(smem + SM_ROWOFF);
    uint32_t* mask = reinterpret_cast<uint32_t*>(smem + SM_MASK);
    int* sidx = reinterpret_cast<int*>(smem + SM_IDX);
    volatile int* flags = reinterpret_cast<volatile int*>(smem + SM_FLAGS);
    volatile int* abort_flag = flags + 1;
    auto bar = [&](int i) -> uint32_t { return sbase + SM_BARS + 8 * i; };

    if (threadIdx.x == 0) {
        for (int c = 0; c < 4; ++c) {
            mbar_init(bar(B_KV_FULL + c), kProducerWarps);
            mbar_init(bar(B_KV_EMPTY + c), 1);
        }
        mbar_init(bar(B_S_FULL), 1);
        mbar_init(bar(B_P_FULL), kSoftmaxWarps);
        mbar_init(bar(B_PV_DONE), 1);
        mbar_init(bar(B_FINAL), 1);
        mbar_init(bar(B_STAGE + 0), kProducerWarps * 32);
        mbar_init(bar(B_STAGE + 1), kProducerWarps * 32);
        mbar_init(bar(B_Q), 1);
        flags[1] = 0;
        mbar_fence_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(sbase + SM_FLAGS + 8, kTmemCols);
        tmem_relinquish();
    }

    // ---- stage this CTA's page ids (dense) / row indices (sparse) in shared memory
    int idx_base, idx_count;
    if constexpr (kSparse) {
        idx_base = start;
        idx_count = end > start ? end - start : 0;
    } else {
        idx_base = start >> p.page_shift;
        idx_count = end > start ? ((end - 1) >> p.page_shift) - idx_base + 1 : 0;
    }
    const bool staged = idx_count <= kMaxIdx;
    if (staged)
        for (int k = threadIdx.x; k < idx_count; k += kThreads)
            sidx[k] = __ldg(p.tables + b * p.tables_stride + idx_base + k);
    tc_fence_before();
    __syncthreads();   // barrier inits, TMEM address and staged ids visible
    tc_fence_after();

    // ---- Q rows (bf16, 1 KB each) are bulk-copied into the (still unused) KV tile region
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar(B_Q), static_cast<uint32_t>(rows_here) * 1024u);
        for (int n = 0; n < rows_here; ++n) {
            const int r = g * kNQ + n;
            const int qi = r / p.num_heads, h = r % p.num_heads;
            bulk_copy_g2s(sbase + SM_KV + n * 1024, p.q + b * p.q_sb + qi * p.q_sq + h * p.q_sh, 1024, bar(B_Q));
        }
    }

    // ---- producers: copy the raw rows of tile 0 into ring slot 0
    const bool producer = warp > kMmaWarp;
    const int ptl = 32 * (warp - kMmaWarp - 1) + lane;   // producer's token within the tile
    bool pvalid = false;                                  // producer's token of the current tile
    if (producer) {
        if (n_tiles > 0) {
            const int64_t row = row_of<kSparse>(p, sidx, staged, idx_base, b, start + ptl, end, true);
            pvalid = row >= 0;
            if (pvalid) {
                mbar_arrive_expect_tx(bar(B_STAGE + 0), kRowBytes);
                bulk_copy_g2s(sbase + SM_STAGE + ptl * kRowBytes, p.pool + row * kRowBytes, kRowBytes,
                              bar(B_STAGE + 0));
            } else {
                mbar_arrive(bar(B_STAGE + 0));
            }
        }
    } else if (warp < kSoftmaxWarps) {
        // ---- Q -> fp16 in TMEM: thread (w, l < 16) converts row 16w + l with a per-row power
        // of two that keeps it inside fp16 range exactly, and stores it into its own TMEM lane.
        // All 32 lanes take part in the (warp-collective) TMEM stores; lanes 16-31 store zeros
        // into O columns, which the first PV MMA overwrites.
        const int n = 16 * warp + (lane & 15);
        const bool mine = lane < 16 && n < rows_here;
        mbar_wait(bar(B_Q), 0, abort_flag, p.err);
        const uint4* src = reinterpret_cast<const uint4*>(smem + SM_KV + n * 1024);
        float amax = 0.0f;
        if (mine) {
#pragma unroll 4
            for (int k = 0; k < 64; ++k) {
                const uint4 u = src[k];
                const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(w4[j] << 16)),
                                             fabsf(__uint_as_float(w4[j] & 0xFFFF0000u))));
            }
        }
        const int e = (amax > 0.0f && amax <= 3.0e38f) ? ilogbf(amax) - 14 : 0;
        const float mul = mine ? ldexpf(1.0f, -e) : 0.0f;
        if (lane < 16) {
            const int r = g * kNQ + n;
            const bool real = n < rows_here;
            const int qi = real ? r / p.num_heads : 0;
            const int h = real ? r % p.num_heads : 0;
            qscale[n] = real ? p.scale_log2 * ldexpf(1.0f, e) : 0.0f;
            limit[n] = real ? (kSparse ? L : L - (p.q_len - 1 - qi)) : -1;
            rowoff[n] = real ? b * p.o_sb + qi * p.o_sq + h * p.o_sh : 0;
        }
        const uint32_t tq = *reinterpret_cast<volatile uint32_t*>(smem + SM_FLAGS + 8) + kTmemQ +
                            (static_cast<uint32_t>(32 * warp) << 16);
#pragma unroll 1
        for (int cb = 0; cb < 8; ++cb) {             // 8 x 32 columns = 512 fp16
            uint32_t hv[32];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint4 u = mine ? src[cb * 8 + k] : make_uint4(0, 0, 0, 0);
                const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    hv[4 * k + j] = pack_half2(__uint_as_float(w4[j] << 16) * mul,
                                               __uint_as_float(w4[j] & 0xFFFF0000u) * mul);
            }
            tmem_st32(tq + 32 * cb, hv);
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();   // Q is in TMEM; the KV region is free for the producers
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + SM_FLAGS + 8);

    if (producer) {
        // ================================================================ producers
        uint8_t* kv = smem + SM_KV + ptl * 128;
        const int pw = warp - kMmaWarp - 1;
        for (int i = 0; i < n_tiles; ++i) {
            // Copy tile i+1 into the other slot (it held tile i-1, already dequantised).
            bool nvalid = false;
            if (i + 1 < n_tiles) {
                const int sl = (i + 1) & 1;
                const int64_t row = row_of<kSparse>(p, sidx, staged, idx_base, b,
                                                    start + (i + 1) * kTile + ptl, end, true);
                nvalid = row >= 0;
                fence_proxy_async_smem();   // my reads of this slot precede the async overwrite
                if (nvalid) {
                    mbar_arrive_expect_tx(bar(B_STAGE + sl), kRowBytes);
                    bulk_copy_g2s(sbase + SM_STAGE + sl * kSlotBytes + ptl * kRowBytes,
                                  p.pool + row * kRowBytes, kRowBytes, bar(B_STAGE + sl));
                } else {
                    mbar_arrive(bar(B_STAGE + sl));
                }
            }
            // Tile i: wait for its raw rows, publish the validity mask, dequantise.
            mbar_wait(bar(B_STAGE + (i & 1)), (i >> 1) & 1, abort_flag, p.err);
            const uint32_t vb = __ballot_sync(0xFFFFFFFFu, pvalid);
            if (lane == 0) mask[(i & 1) * 4 + pw] = vb;
            const uint8_t* raw = smem + SM_STAGE + (i & 1) * kSlotBytes + ptl * kRowBytes;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint4 code[4];
                uint2 scl;
                if (pvalid) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) code[k] = *reinterpret_cast<const uint4*>(raw + 64 * c + 16 * k);
                    scl = *reinterpret_cast<const uint2*>(raw + 256 + 8 * c);
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k) code[k] = make_uint4(0, 0, 0, 0);
                    scl = make_uint2(0, 0);
                }
                mbar_wait(bar(B_KV_EMPTY + c), (i & 1) ^ 1, abort_flag, p.err);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint32_t sw = half ? scl.y : scl.x;
                    const uint32_t s01 = e4m3x2_to_f16x2(static_cast<uint16_t>(sw & 0xFFFFu));
                    const uint32_t s23 = e4m3x2_to_f16x2(static_cast<uint16_t>(sw >> 16));
                    const uint32_t S[4] = {__byte_perm(s01, 0, 0x1010), __byte_perm(s01, 0, 0x3232),
                                           __byte_perm(s23, 0, 0x1010), __byte_perm(s23, 0, 0x3232)};
                    const uint4 u0 = code[2 * half], u1 = code[2 * half + 1];
                    const uint32_t cw[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                    uint8_t* dst = kv + (2 * c + half) * (kTile * 128);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        uint32_t hv[4];
                        e2m1x8_to_f16x2x4(cw[k], hv);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) hv[q4] = hmul2_u32(hv[q4], S[k >> 1]);
                        *reinterpret_cast<uint4*>(dst + ((k ^ (ptl & 7)) << 4)) =
                            make_uint4(hv[0], hv[1], hv[2], hv[3]);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_KV_FULL + c));
            }
            pvalid = nvalid;
        }
    } else if (warp == kMmaWarp) {
        // ================================================================ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_f16_f32(kNQ, kTile, false, false);  // A TMEM, B K-major
            constexpr uint32_t idesc_pv = idesc_f16_f32(kNQ, 256, false, true);     // A K-major, B MN-major
            const uint32_t tQ = tmem + kTmemQ, tS = tmem + kTmemS, tO = tmem + kTmemO;
            const uint64_t kv_k = smem_desc_sw128(sbase + SM_KV, 16, 1024);            // K-major
            const uint64_t kv_mn = smem_desc_sw128(sbase + SM_KV, kTile * 128, 1024);  // MN-major
            const uint64_t p_k = smem_desc_sw128(sbase + SM_P, 16, 1024);              // K-major
            // Loops stay rolled: unrolled, the compiler hoists every loop-invariant descriptor
            // out of the tile loop into registers and spills; an MMA takes ~50-90 ns, so the
            // few integer adds per issue are free.
            for (int i = 0; i < n_tiles; ++i) {
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    mbar_wait(bar(B_KV_FULL + c), i & 1, abort_flag, p.err);
                    tc_fence_after();
#pragma unroll 1
                    for (int ks = 0; ks < 8; ++ks) {
                        const int kk = 8 * c + ks;                     // 16-d step 0..31
                        const uint64_t bd = kv_k + ((((kk >> 2) * (kTile * 128)) + (kk & 3) * 32) >> 4);
                        tc_mma_f16_ts(tS, tQ + 8 * kk, bd, idesc_qk, kk != 0);
                    }
                }
                tc_commit(bar(B_S_FULL));
                mbar_wait(bar(B_P_FULL), i & 1, abort_flag, p.err);
                tc_fence_after();
#pragma unroll 1
                for (int hf = 0; hf < 2; ++hf) {
#pragma unroll 1
                    for (int ks = 0; ks < 8; ++ks) {                   // 16 tokens per step
                        const uint64_t ad = p_k + ((((ks >> 2) * (kNQ * 128)) + (ks & 3) * 32) >> 4);
                        const uint64_t bd = kv_mn + ((4 * hf * (kTile * 128) + ks * 2048) >> 4);
                        tc_mma_f16(tO + 256 * hf, ad, bd, idesc_pv, (i > 0 || ks > 0) ? 1u : 0u);
                    }
                    tc_commit(bar(B_KV_EMPTY + 2 * hf));
                    tc_commit(bar(B_KV_EMPTY + 2 * hf + 1));
                }
                tc_commit(bar(B_PV_DONE));
            }
            // Drain: nothing may still write TMEM or read shared memory at teardown.
            tc_commit(bar(B_FINAL));
            int no_abort = 0;
            mbar_wait(bar(B_FINAL), 0, &no_abort, p.err);
        }
        __syncwarp();
    } else {
        // ================================================================ softmax
        // Lanes 0-15 own the S/P row of query row 16w + lane (their TMEM lane holds S);
        // lanes 16-31 own the O row 16w + lane - 16 (their TMEM lane holds O).
        const int w = warp;
        const uint32_t lane_base = static_cast<uint32_t>(32 * w) << 16;
        const int orow = 16 * w + (lane & 15);
        const bool srow = lane < 16;
        const float qs = qscale[orow];
        const int lim = limit[orow];
        float m = -INFINITY, l = 0.0f;          // running row max (log2 units) / row sum
        for (int i = 0; i < n_tiles; ++i) {
            const int t0 = start + i * kTile;
            mbar_wait(bar(B_S_FULL), i & 1, abort_flag, p.err);
            tc_fence_after();
            // the producers published tile i's mask before their last kv_full arrive
            mbar_wait(bar(B_KV_FULL + 3), i & 1, abort_flag, p.err);
            const uint32_t* mk = mask + (i & 1) * 4;
            const int ncol = srow ? min(max(lim - t0, 0), kTile) : 0;   // causal MTP bound
            // pass 1: tile max of this row
            float tmax = -INFINITY;
#pragma unroll 1
            for (int cb = 0; cb < 4; ++cb) {
                uint32_t sr[32];
                // lanes 0-15 of the quadrant hold S; lanes 16-31 read O columns and ignore them
                tmem_ld32(tmem + kTmemS + lane_base + 32 * cb, sr);
                tmem_wait_ld();
                const uint32_t mw = mk[cb];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const bool ok = ((mw >> j) & 1u) && (32 * cb + j < ncol);
                    tmax = fmaxf(tmax, ok ? __uint_as_float(sr[j]) : -INFINITY);
                }
            }
            tmax *= qs;   // qs > 0 for real rows; padding rows have ncol = 0 (tmax = -inf)
            float a = 1.0f;
            bool grow = false;
            if (srow && tmax > m + kRescaleLog2) {
                a = (m == -INFINITY) ? 0.0f : ex2_approx(m - tmax);
                m = tmax;
                grow = true;
            }
            l *= a;
            if (srow) alpha[orow] = a;
            const bool any_grow = named_bar_red_or(1, kSoftmaxWarps * 32, grow);   // also orders alpha
            if (i > 0) {   // PV(i-1) must be done before O is rescaled or P overwritten
                mbar_wait(bar(B_PV_DONE), (i - 1) & 1, abort_flag, p.err);
                tc_fence_after();
            }
            if (any_grow && i > 0) {
                // Lanes 16-31 scale their O row; the collective load/store also covers lanes
                // 0-15 (Q and S), which write back exactly the bits they read.
                const float ar = alpha[orow];
                const uint32_t to = tmem + lane_base;
#pragma unroll 1
                for (int cc = 0; cc < 16; ++cc) {
                    uint32_t ob[32];
                    tmem_ld32(to + 32 * cc, ob);
                    tmem_wait_ld();
                    if (!srow) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) ob[j] = __float_as_uint(__uint_as_float(ob[j]) * ar);
                    }
                    tmem_st32(to + 32 * cc, ob);
                }
                tmem_wait_st();
            }
            // pass 2: p = 2^(s * qs - m) -> P row in shared memory, row sum
            const float negm = (m == -INFINITY) ? 0.0f : -m;
            uint8_t* prow = smem + SM_P + orow * 128;
#pragma unroll 1
            for (int cb = 0; cb < 4; ++cb) {
                uint32_t sr[32];
                tmem_ld32(tmem + kTmemS + lane_base + 32 * cb, sr);
                tmem_wait_ld();
                const uint32_t mw = mk[cb];
                uint32_t ph[16];
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const bool ok0 = ((mw >> j) & 1u) && (32 * cb + j < ncol);
                    const bool ok1 = ((mw >> (j + 1)) & 1u) && (32 * cb + j + 1 < ncol);
                    const float p0 = ok0 ? ex2_approx(fmaf(__uint_as_float(sr[j]), qs, negm)) : 0.0f;
                    const float p1 = ok1 ? ex2_approx(fmaf(__uint_as_float(sr[j + 1]), qs, negm)) : 0.0f;
                    l += p0 + p1;
                    ph[j >> 1] = pack_half2(p0, p1);
                }
                if (srow) {
                    // token block cb >> 1 (64 tokens), 16-byte chunks (cb & 1) * 4 + k of the row
                    uint8_t* dst = prow + (cb >> 1) * (kNQ * 128);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int chunk = (cb & 1) * 4 + k;
                        *reinterpret_cast<uint4*>(dst + ((chunk ^ (orow & 7)) << 4)) =
                            make_uint4(ph[4 * k], ph[4 * k + 1], ph[4 * k + 2], ph[4 * k + 3]);
                    }
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_P_FULL));
        }
        if (n_tiles > 0) {
            mbar_wait(bar(B_PV_DONE), (n_tiles - 1) & 1, abort_flag, p.err);
            tc_fence_after();
        }
        // ---- epilogue: lanes 16-31 write their O row (512 columns of their TMEM lane)
        if (srow) {
            mrow[orow] = m;
            lsum[orow] = l;
        }
        named_bar_sync(1, kSoftmaxWarps * 32);
        const bool mine = !srow && orow < rows_here;
        const uint32_t to = tmem + lane_base;   // quadrant base: lanes 16-31 read their O row (kTmemO)
        if (p.splits == 1) {
            const float lr = lsum[orow];
            const float inv = (n_tiles > 0 && lr > 0.0f) ? p.bmm2_scale / lr : 0.0f;
            __nv_bfloat16* dst = p.out + (mine ? rowoff[orow] : 0);
#pragma unroll 1
            for (int cc = 0; cc < 16; ++cc) {
                uint32_t ob[32];
                if (n_tiles > 0) {
                    tmem_ld32(to + 32 * cc, ob);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) ob[j] = 0u;
                }
                if (mine) {
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        uint4 v;
                        v.x = pack_bf16x2(__uint_as_float(ob[j]) * inv, __uint_as_float(ob[j + 1]) * inv);
                        v.y = pack_bf16x2(__uint_as_float(ob[j + 2]) * inv, __uint_as_float(ob[j + 3]) * inv);
                        v.z = pack_bf16x2(__uint_as_float(ob[j + 4]) * inv, __uint_as_float(ob[j + 5]) * inv);
                        v.w = pack_bf16x2(__uint_as_float(ob[j + 6]) * inv, __uint_as_float(ob[j + 7]) * inv);
                        *reinterpret_cast<uint4*>(dst + 32 * cc + j) = v;
                    }
                }
            }
        } else {
            const int64_t unit = (static_cast<int64_t>(s) * p.batch + b) * p.groups + g;
            float* po = p.part_o + unit * (kNQ * kLatent) + orow * kLatent;
            if (n_tiles > 0) {
#pragma unroll 1
                for (int cc = 0; cc < 16; ++cc) {
                    uint32_t ob[32];
                    tmem_ld32(to + 32 * cc, ob);
                    tmem_wait_ld();
                    if (mine) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<uint4*>(po + 32 * cc + j) = make_uint4(ob[j], ob[j + 1], ob[j + 2], ob[j + 3]);
                    }
                }
            }
            if (srow) {
                float* ml = p.part_ml + unit * (kNQ * 2) + 2 * orow;
                ml[0] = n_tiles > 0 ? m : -INFINITY;
                ml[1] = n_tiles > 0 ? l : 0.0f;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Merge split partials: out = sum_s w_s O_s / sum_s w_s l_s * bmm2_scale with
// w_s = 2^(m_s - max m).  One block per query row (spread over every SM), one float4 of
// latent dims per thread; the loads of all splits are independent so they overlap.
__global__ void __launch_bounds__(128)
combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits,
               int batch, int groups, int q_len, int num_heads, float bmm2_scale,
               __nv_bfloat16* __restrict__ out, int64_t o_sb, int64_t o_sq, int64_t o_sh) {
    __shared__ float wts[kMaxSplits];
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

using Plan = DecodePlan;

template <bool kSparse>
int ensure_smem_attr() {
    static int done[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaGetDevice failed");
    if (dev >= 0 && dev < 64 && done[dev]) return NVFP4KV_OK;
    cudaError_t e = cudaFuncSetAttribute(mla_decode_kernel<kSparse>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess)
        return fail(NVFP4KV_ECUDA, "cudaFuncSetAttribute(max dynamic smem %d): %s", kSmemBytes,
                    cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) done[dev] = 1;
    return NVFP4KV_OK;
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
    pl.tiles_total = tiles;
    pl.splits = want < 1 ? 1 : want;   // split sizes differ by at most one tile
    pl.part_bytes = pl.splits > 1
                        ? static_cast<size_t>(pl.splits) * units * kNQ * (kLatent + 2) * sizeof(float)
                        : 0;
    pl.qimg_bytes = sparse_topk > 0 ? 0 : static_cast<size_t>(units) * kQImageBytes;
    pl.ws_bytes = pl.part_bytes + pl.qimg_bytes;
    return pl;
}

}  // namespace nvfp4kv

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
    *launches = 1 + (pl.splits > 1 ? 1 : 0) + (sparse_topk > 0 ? 0 : 1);   // (Q prep) + attention + (combine)
    return NVFP4KV_OK;
}

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
    using namespace nvfp4kv;
    if (batch < 0) return fail(NVFP4KV_EINVAL, "mla_decode: batch < 0");
    if (batch == 0) return NVFP4KV_OK;
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
    const Plan pl = make_decode_plan(batch, q_len, num_heads, max_seq_len, sparse_topk);
    if (pl.ws_bytes > 0) {
        if (!workspace || workspace_bytes < pl.ws_bytes)
            return fail(NVFP4KV_EWORKSPACE, "mla_decode: workspace %zu bytes < %zu required",
                        workspace_bytes, pl.ws_bytes);
        if (reinterpret_cast<uintptr_t>(workspace) % 256)
            return fail(NVFP4KV_EINVAL, "mla_decode: workspace must be 256-byte aligned");
    }
    DecodeParams prm{};
    prm.q = static_cast<const __nv_bfloat16*>(q);
    prm.q_sb = q_stride_b; prm.q_sq = q_stride_q; prm.q_sh = q_stride_h;
    prm.pool = pool; prm.pool_rows = pool_rows;
    prm.tables = tables; prm.tables_stride = tables_stride;
    prm.seq_lens = seq_lens;
    prm.batch = batch; prm.q_len = q_len; prm.num_heads = num_heads;
    prm.groups = pl.groups; prm.splits = pl.splits;
    prm.sparse = sparse_topk > 0; prm.topk = sparse_topk;
    prm.page_shift = page_shift;
    prm.num_pages = sparse_topk > 0 ? 0 : pool_rows / page_size;
    prm.max_seq_len = sparse_topk > 0 ? sparse_topk : max_seq_len;
    prm.tiles_total = pl.tiles_total;
    prm.scale_log2 = bmm1_scale * 1.4426950408889634f;
    prm.bmm2_scale = bmm2_scale;
    prm.out = static_cast<__nv_bfloat16*>(out);
    prm.o_sb = out_stride_b; prm.o_sq = out_stride_q; prm.o_sh = out_stride_h;
    size_t part_o_bytes = static_cast<size_t>(pl.splits) * batch * pl.groups * kNQ * kLatent * sizeof(float);
    prm.part_o = pl.splits > 1 ? static_cast<float*>(workspace) : nullptr;
    prm.part_ml = pl.splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + part_o_bytes) : nullptr;
    prm.err = err_flag;

    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(batch * pl.groups * pl.splits));
    int rc;
    if (sparse_topk > 0) {
        if ((rc = ensure_smem_attr<true>()) != NVFP4KV_OK) return rc;
        cudaEvent_t ev0, ev1;
        take_kernel_events(&ev0, &ev1);
        if (ev0 && cudaEventRecord(ev0, st) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaEventRecord failed");
        mla_decode_kernel<true><<<grid, kThreads, kSmemBytes, st>>>(prm);
        if ((rc = check_launch("nvfp4kv_mla_decode")) != NVFP4KV_OK) return rc;
        if (ev1 && cudaEventRecord(ev1, st) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaEventRecord failed");
    } else {
        DecodeArgs a{};
        a.q = q; a.q_sb = q_stride_b; a.q_sq = q_stride_q; a.q_sh = q_stride_h;
        a.pool = pool; a.pool_rows = pool_rows;
        a.tables = tables; a.tables_stride = tables_stride; a.seq_lens = seq_lens;
        a.batch = batch; a.q_len = q_len; a.num_heads = num_heads;
        a.sparse_topk = 0; a.page_size = page_size; a.page_shift = page_shift; a.max_seq_len = max_seq_len;
        a.bmm1_scale = bmm1_scale; a.bmm2_scale = bmm2_scale;
        a.out = out; a.o_sb = out_stride_b; a.o_sq = out_stride_q; a.o_sh = out_stride_h;
        a.part_o = prm.part_o; a.part_ml = prm.part_ml; a.err = err_flag;
        a.qimg = static_cast<uint8_t*>(workspace) + pl.part_bytes;
        if ((rc = launch_decode_fp4_dense(a, pl, st)) != NVFP4KV_OK) return rc;
    }
    if (pl.splits > 1) {
        combine_kernel<<<batch * pl.groups * kNQ, 128, 0, st>>>(prm.part_o, prm.part_ml, pl.splits, batch,
                                                          pl.groups, q_len, num_heads, bmm2_scale,
                                                          prm.out, out_stride_b, out_stride_q, out_stride_h);
        if ((rc = check_launch("nvfp4kv_mla_decode combine")) != NVFP4KV_OK) return rc;
    }
    return NVFP4KV_OK;
}
