// Fused NVFP4 gather + dequant + MLA decode attention for sm_100a (tcgen05 + TMEM).
//
// Replaces, at the reference's read seam (nvfp4-kv/patch_nvfp4_kv.py:84-118), the pair
//   build_scratch(...)                       -> 656-byte fp8 scratch (glm53_nvfp4_runtime.py:143-182)
//   trtllm_batch_decode_with_kv_cache_mla(...) -> attention over that scratch
// with one kernel that reads the 288-byte pool rows directly.
//
// Work unit (one CTA, one per SM): query group (b, g) x token split s.  A query group is up
// to 64 query rows (MTP token i, head h) of batch entry b; they all share the latent rows.
//
// Per 128-token tile:
//   producers (8 warps)  : load raw rows (16-byte ld.global.nc), dequantise with
//                          cvt.rn.f16x2.e2m1x2 x e4m3 scale (exact in fp16) into a
//                          128B-swizzled fp16 tile [128 tokens x 512] in shared memory,
//                          one 128-d chunk at a time (kv_full[c] / kv_empty[c]).
//   MMA thread (1 lane)  : S^T[tok, row] = K . Q^T   M=128 (tokens) N=64 (rows) K=512,
//                          A = KV tile (K-major), B = Q (K-major), D in TMEM columns [0,64);
//                          O^T[d, row] += V^T . P^T  M=128 (d chunk) N=64 K=128 (tokens),
//                          A = the same KV tile read MN-major, B = P (MN-major),
//                          D in TMEM columns [256, 512) (4 chunks x 64).
//   softmax (4 warps)    : thread = token lane; row maxima / sums over tokens by a
//                          shuffle reduce-scatter, lazy rescaling of O (only when a row max
//                          grows by more than 2^8), P written as fp16 to shared memory.
// Splits write unnormalised partial O plus (max, sum) per row; a combine kernel merges them
// with log-sum-exp weights.  Every wait is bounded (common.cuh).
#include <math.h>

#include "abi_common.h"
#include "common.cuh"

namespace nvfp4kv {
namespace {

constexpr int kTile = 128;        // tokens per tile
constexpr int kNQ = 64;           // query rows per CTA (MMA N)
constexpr int kSoftmaxWarps = 4;  // warps 0-3: TMEM lanes 0-127
constexpr int kMmaWarp = 4;
constexpr int kProducerWarps = 8;  // warps 5-12
constexpr int kThreads = (kSoftmaxWarps + 1 + kProducerWarps) * 32;
constexpr int kMaxSplits = 64;
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when a row max grows by > 2^8

// Shared memory map, offsets from a 1024-byte aligned base.
constexpr int SM_Q = 0;                          // 8 d-blocks x [64 rows x 128 B], fp16
constexpr int SM_KV = SM_Q + 8 * kNQ * 128;      // 8 d-blocks x [128 tokens x 128 B], fp16
constexpr int SM_P = SM_KV + 8 * kTile * 128;    // [128 tokens x 64 rows] fp16, 128 B/token
constexpr int SM_RED = SM_P + kTile * 128;       // 4 warps x 64 floats
constexpr int SM_MROW = SM_RED + 4 * 64 * 4;     // 64 floats: running row max (log2 units)
constexpr int SM_ALPHA = SM_MROW + 64 * 4;       // 64 floats: per-tile rescale factors
constexpr int SM_QSCALE = SM_ALPHA + 64 * 4;     // 64 floats: log2e * bmm1_scale * 2^e_row
constexpr int SM_LIMIT = SM_QSCALE + 64 * 4;     // 64 ints: visible token bound per row
constexpr int SM_LSUM = SM_LIMIT + 64 * 4;       // 64 floats: final row sums
constexpr int SM_ROWOFF = SM_LSUM + 64 * 4;      // 64 int64: output row offsets (elements)
constexpr int SM_COEF = SM_ROWOFF + 64 * 8;      // 64 x {qscale, -row max}: p = 2^(s*qs - m)
constexpr int SM_FLAGS = SM_COEF + 64 * 8;       // [0] rescale tile tag, [1] abort, [2] tmem base
constexpr int SM_BARS = SM_FLAGS + 64;
enum { B_KV_FULL = 0, B_KV_EMPTY = 4, B_S_FULL = 8, B_P_FULL = 9, B_PV_DONE = 10, B_FINAL = 11,
       kNumBars = 12 };
constexpr int SM_END = SM_BARS + kNumBars * 8;
constexpr int kSmemBytes = SM_END + 1024;        // slack for aligning the base

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;     // S^T: columns [0, 64)
constexpr uint32_t kTmemO = 256;   // O^T: columns [256, 512)

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
    int max_seq_len, tokens_per_split;
    float scale_log2, bmm2_scale;
    __nv_bfloat16* out;
    int64_t o_sb, o_sq, o_sh;
    float* part_o;   // [splits][batch][groups][64][512]
    float* part_ml;  // [splits][batch][groups][64][2]
    int32_t* err;
};

__device__ __forceinline__ float fmax_op(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ float fadd_op(float a, float b) { return a + b; }

// Reduce 64 per-thread values over the 32 lanes of a warp, scattering the results: lane l
// ends with the reductions of entries 2l and 2l+1.  62 shuffles instead of 64 x 5.
template <bool kMax>
__device__ __forceinline__ void reduce_scatter64(float (&v)[64], int lane, float& r0, float& r1) {
    auto op = [](float a, float b) { return kMax ? fmax_op(a, b) : fadd_op(a, b); };
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        const bool up = lane & 16;
        const float send = up ? v[k] : v[k + 32];
        const float keep = up ? v[k + 32] : v[k];
        v[k] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 16));
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const bool up = lane & 8;
        const float send = up ? v[k] : v[k + 16];
        const float keep = up ? v[k + 16] : v[k];
        v[k] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 8));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const bool up = lane & 4;
        const float send = up ? v[k] : v[k + 8];
        const float keep = up ? v[k + 8] : v[k];
        v[k] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 4));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool up = lane & 2;
        const float send = up ? v[k] : v[k + 4];
        const float keep = up ? v[k + 4] : v[k];
        v[k] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 2));
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const bool up = lane & 1;
        const float send = up ? v[k] : v[k + 2];
        const float keep = up ? v[k + 2] : v[k];
        v[k] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 1));
    }
    r0 = v[0];
    r1 = v[1];
}

// Pool row of token position t (within batch entry b), or -1 when the token is masked.
template <bool kSparse>
__device__ __forceinline__ int64_t token_row(const DecodeParams& p, int b, int t, int end,
                                             bool report) {
    if (t >= end) return -1;
    if constexpr (kSparse) {
        const int32_t idx = __ldg(p.tables + b * p.tables_stride + t);
        if (idx < 0 || idx >= p.pool_rows) {
            if (report && idx != -1) set_error(p.err, NVFP4KV_DEVERR_BAD_INDEX);
            return -1;
        }
        return idx;
    } else {
        const int32_t pg = __ldg(p.tables + b * p.tables_stride + (t >> p.page_shift));
        if (pg < 0 || pg >= p.num_pages) {
            if (report) set_error(p.err, NVFP4KV_DEVERR_BAD_PAGE);
            return -1;
        }
        return (static_cast<int64_t>(pg) << p.page_shift) | (t & ((1 << p.page_shift) - 1));
    }
}

template <bool kSparse>
__global__ void __maxnreg__(152) mla_decode_kernel(const DecodeParams p) {
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
    const int start = s * p.tokens_per_split;
    const int end = min(start + p.tokens_per_split, L);
    const int n_tiles = end > start ? (end - start + kTile - 1) / kTile : 0;

    float* red = reinterpret_cast<float*>(smem + SM_RED);
    float* mrow = reinterpret_cast<float*>(smem + SM_MROW);
    float* alpha = reinterpret_cast<float*>(smem + SM_ALPHA);
    float* qscale = reinterpret_cast<float*>(smem + SM_QSCALE);
    int* limit = reinterpret_cast<int*>(smem + SM_LIMIT);
    float* lsum = reinterpret_cast<float*>(smem + SM_LSUM);
    int64_t* rowoff = reinterpret_cast<int64_t*>(smem + SM_ROWOFF);
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
        flags[0] = 0;
        flags[1] = 0;
        mbar_fence_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(sbase + SM_FLAGS + 8, kTmemCols);
        tmem_relinquish();
    }

    // ---- Q rows -> fp16 (per-row power-of-two scale keeps them inside fp16 range exactly)
    const int rows_total = p.q_len * p.num_heads;
    for (int n = warp; n < kNQ; n += kThreads / 32) {
        const int r = g * kNQ + n;
        const bool real = r < rows_total;
        const int qi = real ? r / p.num_heads : 0;
        const int h = real ? r % p.num_heads : 0;
        uint4 u0 = make_uint4(0, 0, 0, 0), u1 = u0;
        if (real) {
            const __nv_bfloat16* qp = p.q + b * p.q_sb + qi * p.q_sq + h * p.q_sh + 16 * lane;
            u0 = *reinterpret_cast<const uint4*>(qp);
            u1 = *reinterpret_cast<const uint4*>(qp + 8);
        }
        const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        float x[16];
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            x[2 * j] = __uint_as_float(w[j] << 16);
            x[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
            amax = fmaxf(amax, fmaxf(fabsf(x[2 * j]), fabsf(x[2 * j + 1])));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        const int e = (amax > 0.0f && amax <= 3.0e38f) ? ilogbf(amax) - 14 : 0;
        const float mul = ldexpf(1.0f, -e);
        uint32_t hw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) hw[j] = pack_half2(x[2 * j] * mul, x[2 * j + 1] * mul);
        const int db = lane >> 2, j0 = (lane & 3) * 2;
        uint8_t* qrow = smem + SM_Q + db * (kNQ * 128) + n * 128;
        *reinterpret_cast<uint4*>(qrow + (((j0 + 0) ^ (n & 7)) << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(qrow + (((j0 + 1) ^ (n & 7)) << 4)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        if (lane == 0) {
            qscale[n] = real ? p.scale_log2 * ldexpf(1.0f, e) : 0.0f;
            limit[n] = real ? (kSparse ? L : L - (p.q_len - 1 - qi)) : -1;
            rowoff[n] = real ? b * p.o_sb + qi * p.o_sq + h * p.o_sh : -1;
            mrow[n] = -INFINITY;
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + SM_FLAGS + 8);

    if (warp >= kMmaWarp + 1) {
        // ================================================================ producers
        const int pw = warp - (kMmaWarp + 1);
        const int hh = pw >> 2;                  // which d-block of each 128-d chunk
        const int tl = 32 * (pw & 3) + lane;     // token within the tile
        uint8_t* kv = smem + SM_KV;
        for (int i = 0; i < n_tiles; ++i) {
            const int t = start + i * kTile + tl;
            const int64_t row = token_row<kSparse>(p, b, t, end, hh == 0);
            uint4 cl[4], ch[4];
            uint32_t sc[4];
            if (row >= 0) {
                const uint8_t* src = p.pool + row * kRowBytes;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int db = 2 * c + hh;
                    cl[c] = ldg_nc_v4(src + 32 * db);
                    ch[c] = ldg_nc_v4(src + 32 * db + 16);
                    sc[c] = ldg_nc_u32(src + 256 + 4 * db);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    cl[c] = make_uint4(0, 0, 0, 0);
                    ch[c] = cl[c];
                    sc[c] = 0;
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                mbar_wait(bar(B_KV_EMPTY + c), (i & 1) ^ 1, abort_flag, p.err);
                const int db = 2 * c + hh;
                const uint32_t s01 = e4m3x2_to_f16x2(static_cast<uint16_t>(sc[c] & 0xFFFFu));
                const uint32_t s23 = e4m3x2_to_f16x2(static_cast<uint16_t>(sc[c] >> 16));
                const uint32_t S[4] = {__byte_perm(s01, 0, 0x1010), __byte_perm(s01, 0, 0x3232),
                                       __byte_perm(s23, 0, 0x1010), __byte_perm(s23, 0, 0x3232)};
                const uint32_t cw[8] = {cl[c].x, cl[c].y, cl[c].z, cl[c].w,
                                        ch[c].x, ch[c].y, ch[c].z, ch[c].w};
                uint8_t* dst = kv + db * (kTile * 128) + tl * 128;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    uint32_t hv[4];
                    e2m1x8_to_f16x2x4(cw[k], hv);
#pragma unroll
                    for (int j = 0; j < 4; ++j) hv[j] = hmul2_u32(hv[j], S[k >> 1]);
                    *reinterpret_cast<uint4*>(dst + ((k ^ (tl & 7)) << 4)) =
                        make_uint4(hv[0], hv[1], hv[2], hv[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_KV_FULL + c));
            }
        }
    } else if (warp == kMmaWarp) {
        // ================================================================ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_f16_f32(128, kNQ, false, false);
            constexpr uint32_t idesc_pv = idesc_f16_f32(128, kNQ, true, true);
            const uint32_t q_addr = sbase + SM_Q, kv_addr = sbase + SM_KV, p_addr = sbase + SM_P;
            const uint32_t tS = tmem + kTmemS, tO = tmem + kTmemO;
            for (int i = 0; i < n_tiles; ++i) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    mbar_wait(bar(B_KV_FULL + c), i & 1, abort_flag, p.err);
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const int db = 2 * c + (ks >> 2);
                        const uint32_t koff = (ks & 3) * 32;
                        const uint64_t ad = smem_desc_sw128(kv_addr + db * (kTile * 128) + koff, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(q_addr + db * (kNQ * 128) + koff, 16, 1024);
                        tc_mma_f16(tS, ad, bd, idesc_qk, (c | ks) != 0);
                    }
                }
                tc_commit(bar(B_S_FULL));
                mbar_wait(bar(B_P_FULL), i & 1, abort_flag, p.err);
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t ad = smem_desc_sw128(kv_addr + 2 * c * (kTile * 128) + ks * 2048,
                                                            kTile * 128, 1024);
                        const uint64_t bd = smem_desc_sw128(p_addr + ks * 2048, kTile * 128, 1024);
                        tc_mma_f16(tO + 64 * c, ad, bd, idesc_pv, (i > 0 || ks > 0) ? 1u : 0u);
                    }
                    tc_commit(bar(B_KV_EMPTY + c));
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
        const int w = warp;
        const int tl = 32 * w + lane;
        const uint32_t lane_base = static_cast<uint32_t>(32 * w) << 16;
        const uint32_t tS = tmem + kTmemS + lane_base, tO = tmem + kTmemO + lane_base;
        float l0 = 0.0f, l1 = 0.0f;  // row sums of rows 2*lane, 2*lane+1 over this warp's tokens
        float2* coef = reinterpret_cast<float2*>(smem + SM_COEF);
        const bool row_limits = p.q_len > 1;  // causal MTP rows see different token counts
        for (int i = 0; i < n_tiles; ++i) {
            const int t = start + i * kTile + tl;
            const bool valid = token_row<kSparse>(p, b, t, end, false) >= 0;
            mbar_wait(bar(B_S_FULL), i & 1, abort_flag, p.err);
            tc_fence_after();
            // ---- pass 1: row maxima of this tile (raw scores; the row scale is > 0)
            float v[64];
            {
                uint32_t sr[64];
                tmem_ld32(tS, sr);
                tmem_ld32(tS + 32, sr + 32);
                tmem_wait_ld();
#pragma unroll
                for (int n = 0; n < 64; ++n) {
                    const bool ok = valid && (!row_limits || t < limit[n]);
                    v[n] = ok ? __uint_as_float(sr[n]) : -INFINITY;
                }
            }
            float m0, m1;
            reduce_scatter64<true>(v, lane, m0, m1);
            red[w * 64 + 2 * lane] = m0 * qscale[2 * lane];
            red[w * 64 + 2 * lane + 1] = m1 * qscale[2 * lane + 1];
            named_bar_sync(1, kSoftmaxWarps * 32);
            if (tl < 64) {
                const float tm = fmaxf(fmaxf(red[tl], red[64 + tl]), fmaxf(red[128 + tl], red[192 + tl]));
                const float mo = mrow[tl];
                float a = 1.0f, mn = mo;
                if (tm > mo + kRescaleLog2) {
                    a = (mo == -INFINITY) ? 0.0f : ex2_approx(mo - tm);
                    mn = tm;
                    mrow[tl] = tm;
                    flags[0] = i + 1;
                }
                alpha[tl] = a;
                coef[tl] = make_float2(qscale[tl], mn == -INFINITY ? 0.0f : -mn);
            }
            named_bar_sync(1, kSoftmaxWarps * 32);
            const bool rescale = (i > 0) && (flags[0] == i + 1);
            if (i > 0) {  // PV(i-1) must be done before O is rescaled or P overwritten
                mbar_wait(bar(B_PV_DONE), (i - 1) & 1, abort_flag, p.err);
                tc_fence_after();
            }
            if (rescale) {
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t ob[32];
                    tmem_ld32(tO + 32 * c, ob);
                    tmem_wait_ld();
                    const int n0 = (c & 1) * 32;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        ob[j] = __float_as_uint(__uint_as_float(ob[j]) * alpha[n0 + j]);
                    tmem_st32(tO + 32 * c, ob);
                }
                tmem_wait_st();
            }
            l0 *= alpha[2 * lane];
            l1 *= alpha[2 * lane + 1];
            // ---- pass 2: probabilities p = 2^(s * qscale - m), written as fp16 for PV
            {
                uint32_t sr[64];
                tmem_ld32(tS, sr);
                tmem_ld32(tS + 32, sr + 32);
                tmem_wait_ld();
#pragma unroll
                for (int n = 0; n < 64; n += 2) {
                    const float4 cf = *reinterpret_cast<const float4*>(coef + n);
                    const bool ok0 = valid && (!row_limits || t < limit[n]);
                    const bool ok1 = valid && (!row_limits || t < limit[n + 1]);
                    v[n] = ok0 ? ex2_approx(fmaf(__uint_as_float(sr[n]), cf.x, cf.y)) : 0.0f;
                    v[n + 1] = ok1 ? ex2_approx(fmaf(__uint_as_float(sr[n + 1]), cf.z, cf.w)) : 0.0f;
                }
            }
            uint8_t* prow = smem + SM_P + (tl >> 3) * 1024 + (tl & 7) * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                *reinterpret_cast<uint4*>(prow + ((j ^ (tl & 7)) << 4)) =
                    make_uint4(pack_half2(v[8 * j], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                               pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_P_FULL));
            float s0, s1;
            reduce_scatter64<false>(v, lane, s0, s1);
            l0 += s0;
            l1 += s1;
        }
        if (n_tiles > 0) {
            mbar_wait(bar(B_PV_DONE), (n_tiles - 1) & 1, abort_flag, p.err);
            tc_fence_after();
        }
        // ---- epilogue: row sums, then O (thread = d within each 128-d chunk)
        named_bar_sync(1, kSoftmaxWarps * 32);
        red[w * 64 + 2 * lane] = l0;
        red[w * 64 + 2 * lane + 1] = l1;
        named_bar_sync(1, kSoftmaxWarps * 32);
        if (tl < 64) lsum[tl] = red[tl] + red[64 + tl] + red[128 + tl] + red[192 + tl];
        named_bar_sync(1, kSoftmaxWarps * 32);
        const int rows_here = min(kNQ, rows_total - g * kNQ);
        if (p.splits == 1) {
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t ob[32];
                if (n_tiles > 0) {
                    tmem_ld32(tO + 32 * c, ob);
                    tmem_wait_ld();
                }
                const int d = 128 * (c >> 1) + tl;
                const int n0 = (c & 1) * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int n = n0 + j;
                    if (n < rows_here) {
                        const float l = lsum[n];
                        const float o = (n_tiles > 0 && l > 0.0f) ? __uint_as_float(ob[j]) * (p.bmm2_scale / l) : 0.0f;
                        p.out[rowoff[n] + d] = __float2bfloat16_rn(o);
                    }
                }
            }
        } else {
            const int64_t unit = (static_cast<int64_t>(s) * p.batch + b) * p.groups + g;
            float* po = p.part_o + unit * (kNQ * kLatent);
            if (n_tiles > 0) {
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t ob[32];
                    tmem_ld32(tO + 32 * c, ob);
                    tmem_wait_ld();
                    const int d = 128 * (c >> 1) + tl;
                    const int n0 = (c & 1) * 32;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int n = n0 + j;
                        if (n < rows_here) po[n * kLatent + d] = __uint_as_float(ob[j]);
                    }
                }
            }
            if (tl < 64) {
                float* ml = p.part_ml + unit * (kNQ * 2) + 2 * tl;
                ml[0] = n_tiles > 0 ? mrow[tl] : -INFINITY;
                ml[1] = n_tiles > 0 ? lsum[tl] : 0.0f;
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

// Merge split partials: out = sum_s w_s O_s / sum_s w_s l_s * bmm2_scale,
// w_s = 2^(m_s - max m).  One CTA per query group, one thread per latent dim.
__global__ void __launch_bounds__(512)
combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits,
               int batch, int groups, int q_len, int num_heads, float bmm2_scale,
               __nv_bfloat16* __restrict__ out, int64_t o_sb, int64_t o_sq, int64_t o_sh) {
    __shared__ float wts[kNQ][kMaxSplits];
    const int g = blockIdx.x % groups, b = blockIdx.x / groups;
    const int rows_total = q_len * num_heads;
    const int rows_here = min(kNQ, rows_total - g * kNQ);
    const int tid = threadIdx.x;
    if (tid < rows_here) {
        float M = -INFINITY;
        for (int s = 0; s < splits; ++s) {
            const float* ml = part_ml + (((static_cast<int64_t>(s) * batch + b) * groups + g) * kNQ + tid) * 2;
            if (ml[1] > 0.0f) M = fmaxf(M, ml[0]);
        }
        float Ls = 0.0f;
        for (int s = 0; s < splits; ++s) {
            const float* ml = part_ml + (((static_cast<int64_t>(s) * batch + b) * groups + g) * kNQ + tid) * 2;
            const float wgt = ml[1] > 0.0f ? exp2f(ml[0] - M) : 0.0f;
            wts[tid][s] = wgt;
            Ls += wgt * ml[1];
        }
        const float inv = Ls > 0.0f ? bmm2_scale / Ls : 0.0f;
        for (int s = 0; s < splits; ++s) wts[tid][s] *= inv;
    }
    __syncthreads();
    const int d = tid;
    for (int n = 0; n < rows_here; ++n) {
        float acc = 0.0f;
        for (int s = 0; s < splits; ++s) {
            const float wgt = wts[n][s];
            if (wgt != 0.0f)
                acc += wgt * part_o[(((static_cast<int64_t>(s) * batch + b) * groups + g) * kNQ + n) * kLatent + d];
        }
        const int r = g * kNQ + n;
        const int qi = r / num_heads, h = r % num_heads;
        out[b * o_sb + qi * o_sq + h * o_sh + d] = __float2bfloat16_rn(acc);
    }
}

struct Plan {
    int groups, splits, tokens_per_split;
    size_t ws_bytes;
};

Plan make_plan(int batch, int q_len, int num_heads, int max_seq_len, int sparse_topk) {
    Plan pl{};
    pl.groups = (q_len * num_heads + kNQ - 1) / kNQ;
    const int ctx = sparse_topk > 0 ? sparse_topk : max_seq_len;
    const int tiles = ctx > 0 ? (ctx + kTile - 1) / kTile : 1;
    const int units = batch * pl.groups;
    const int sms = device_sm_count();
    int want = units >= sms ? 1 : sms / units;
    want = want < 1 ? 1 : (want > kMaxSplits ? kMaxSplits : want);
    want = want > tiles ? tiles : want;
    const int tiles_per_split = (tiles + want - 1) / want;
    pl.tokens_per_split = tiles_per_split * kTile;
    pl.splits = (tiles + tiles_per_split - 1) / tiles_per_split;
    if (pl.splits < 1) pl.splits = 1;
    pl.ws_bytes = pl.splits > 1
                      ? static_cast<size_t>(pl.splits) * units * kNQ * (kLatent + 2) * sizeof(float)
                      : 0;
    return pl;
}

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
}  // namespace nvfp4kv

extern "C" int nvfp4kv_mla_decode_workspace_size(int batch, int q_len, int num_heads,
                                                 int max_seq_len, int sparse_topk, size_t* bytes) {
    using namespace nvfp4kv;
    if (!bytes) return fail(NVFP4KV_EINVAL, "workspace_size: null output");
    if (batch < 0 || q_len < 1 || num_heads < 1 || max_seq_len < 0 || sparse_topk < 0)
        return fail(NVFP4KV_EINVAL, "workspace_size: bad shape");
    *bytes = batch == 0 ? 0 : make_plan(batch, q_len, num_heads, max_seq_len, sparse_topk).ws_bytes;
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
    if (reinterpret_cast<uintptr_t>(out) % 2)
        return fail(NVFP4KV_EINVAL, "mla_decode: out must be 2-byte aligned");
    const Plan pl = make_plan(batch, q_len, num_heads, max_seq_len, sparse_topk);
    if (pl.splits > 1) {
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
    prm.tokens_per_split = pl.tokens_per_split;
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
        mla_decode_kernel<true><<<grid, kThreads, kSmemBytes, st>>>(prm);
    } else {
        if ((rc = ensure_smem_attr<false>()) != NVFP4KV_OK) return rc;
        mla_decode_kernel<false><<<grid, kThreads, kSmemBytes, st>>>(prm);
    }
    if ((rc = check_launch("nvfp4kv_mla_decode")) != NVFP4KV_OK) return rc;
    if (pl.splits > 1) {
        combine_kernel<<<batch * pl.groups, 512, 0, st>>>(prm.part_o, prm.part_ml, pl.splits, batch,
                                                          pl.groups, q_len, num_heads, bmm2_scale,
                                                          prm.out, out_stride_b, out_stride_q, out_stride_h);
        if ((rc = check_launch("nvfp4kv_mla_decode combine")) != NVFP4KV_OK) return rc;
    }
    return NVFP4KV_OK;
}
