// Fused NVFP4 paged gather + MLA decode attention for sm_100a, with Q.K^T on the block-scaled
// fp4 tensor-core path (tcgen05.mma kind::mxf4nvf4).
//
// The 288-byte pool rows already are NVFP4: 512 e2m1 codes plus one e4m3 scale per 16
// latent dims.  So the tile of 128 rows goes into shared memory unchanged (TMA, 128-byte
// swizzled) and is the A operand of the QK product, with its scales as the A scale factors.
// Q is written as a sum of four NVFP4 terms (each term codes the residual of the previous
// ones with its own per-16 scales, after a per-row power-of-two prescale); four terms leave a
// relative error of about 5e-5 in q, below bf16's own rounding.  The terms sit on the MMA's N
// side in two passes of N = 128 (terms 1|2, then 3|4 accumulated on top), so S^T needs only
// 128 TMEM columns: column n holds term-1+3 of query row n, column 64+n term-2+4.
//
// PV stays exact: V (= the same latent rows) is dequantised to fp16 (code x scale is exact in
// fp16) in 16-token chunks and multiplied with fp16 probabilities, latent dims on M:
//   O^T[d, n] += V^T[d, t] P^T[t, n]      M = 128 dims (4 blocks), N = 64 query rows, K = 16.
//
// Work unit (one CTA): query group (b, g) of up to 64 rows (MTP token i, head h) x token split.
// Warps: 0-7 softmax (warp w: TMEM sub-partition w & 3 = tokens of the tile, query rows
// 32 (w >> 2) .. +32), 8-11 producers, 12 MMA issue, 13 loads.  Per 128-token tile i:
//   loads    3-slot ring of tiles: codes [2 x 128 rows x 128 B] swizzled + scales [128 x 32 B].
//            Dense (paged): TMA boxes straight from the pages; pages missing or beyond the
//            context load as out-of-range boxes (zeros).  Sparse (top-k rows): TMA row gathers
//            (tile::gather4, four rows per instruction) into the same slot layout, so everything
//            downstream is shared with the dense path; masked rows never reach the output
//            (probability 0, V written as zeros).
//   producers  V chunks of 16 tokens -> fp16 [8 d-atoms x 16 tokens x 128 B] (2 buffers).
//   MMA      QK(i): 16 fp4 MMAs M128 N128 K64 -> S^T; PV(i-1): 8 chunks x 4 fp16 MMAs.
//   softmax  S^T row t -> x = s * log2(e) * bmm1_scale, masked; the running max of each query
//            row is raised only when some x exceeds it by more than 8 (a CTA vote), and then
//            O^T is rescaled; p = 2^(x - m) in fp16 -> P^T row t (swizzled), row sums kept
//            per thread and reduced once at the end.
// Splits write partial O and (max, sum) per row; the combine kernel of the caller merges
// them.  Every wait is bounded (common.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "abi_common.h"
#include "common.cuh"
#include "decode_shared.h"

namespace nvfp4kv {
namespace {

constexpr int kTile = kDecTile;                   // 128 tokens: QK M
constexpr int kNQ = kDecRows;                     // 64 query rows: PV N
constexpr int kChunk = 16;                        // tokens per V chunk = PV K
constexpr int kChunks = kTile / kChunk;           // 8
// Four warpgroups.  Registers are moved between them at run time (setmaxnreg): the block is
// launched with 128 per thread; softmax takes 168, producers keep 96, the control group 80.
constexpr int kSoftmaxWarps = 8;                  // warpgroups 0-1: 2 per TMEM sub-partition, 32 rows each
constexpr int kProducerWarp0 = 8;                 // warpgroup 2: V chunks and the pool scale factors
constexpr int kProducerWarps = 4;
constexpr int kMmaWarp = 12;                      // warpgroup 3: MMA issue,
constexpr int kTmaWarp = 13;                      //   every TMA / bulk load, and two spare warps
constexpr int kLoadBar = 2;                       // named barrier of the control warpgroup's shared loads
constexpr int kRefillBar = 3;                     // named barrier of the sparse refill warps (13-15)
constexpr int kThreads = 16 * 32;                 // 512
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr uint32_t kRegsSoftmax = 168, kRegsProducer = 96, kRegsCtl = 80;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsProducer + 128 * kRegsCtl == kThreads * 128,
              "the register split uses exactly what the block is launched with");
constexpr float kRescaleLog2 = 8.0f;

// Shared memory map (offsets from a 1024-byte aligned base) of a ring of S raw tiles and V
// V-chunk buffers.  Two shapes are built: S = 3, V = 2 (tiles loaded two ahead; long contexts)
// and S = 2, V = 4 (the third tile's 36 KB hold two more V chunks, so four chunks are in flight
// between the producers and the tensor core; splits of at most two tiles, where a third slot
// would never be loaded).
constexpr int kCodeBytes = kTile * 256;               // 2 atom columns x [128 rows x 128 B]
constexpr int kScaleBytes = kTile * 32;               // [128 rows x 32 B]
constexpr int kSlotBytes = kCodeBytes + kScaleBytes;  // 36864
constexpr int kVtBytes = 8 * kChunk * 128;            // one V chunk: [8 d-atoms x 16 tokens x 128 B] fp16
constexpr int SM_STAGE = 0;
constexpr int kMaxIdx = 768;                          // staged page ids / top-k rows of the split
constexpr int kIdxTiles = kMaxIdx / kTile;            // sparse: a window of 6 tiles' rows, refilled ahead
template <int S, int V>
struct DecCfg {
    static constexpr int kSlots = S;                                 // tile ring depth
    static constexpr int kVBufs = V;                                 // V chunk buffers
    static constexpr int SM_QB = SM_STAGE + S * kSlotBytes;          // Q terms: 2 passes x 2 atom columns x [128 x 128 B]
    static constexpr int SM_VT = SM_QB + 2 * kCodeBytes;             // V x [8 d-atoms x 16 tokens x 128 B] fp16
    static constexpr int SM_PT = SM_VT + V * kVtBytes;               // [128 tokens x 128 B] fp16 P^T
    static constexpr int SM_M = SM_PT + kTile * 128;                 // 64 f32: running row max (log2 units)
    static constexpr int SM_ALPHA = SM_M + 256;                      // 64 f32: rescale factors / epilogue 1/l
    static constexpr int SM_QS = SM_ALPHA + 256;                     // 64 f32: log2e * bmm1_scale * 2^e_row
    static constexpr int SM_LIM = SM_QS + 256;                       // 64 i32: visible positions < lim
    static constexpr int SM_LSUM = SM_LIM + 256;                     // 64 f32: row sums
    static constexpr int SM_RED = SM_LSUM + 256;                     // 4 sub-partitions x 64 f32
    static constexpr int SM_ROWOFF = SM_RED + 4 * 64 * 4;            // 64 i64: output row offsets
    static constexpr int SM_FLAGS = SM_ROWOFF + 64 * 8;              // [0] TMEM base, [1] abort
    static constexpr int SM_TMASK = SM_FLAGS + 16;                   // S x 4 words: tile rows that are valid
    static constexpr int SM_BARS = SM_TMASK + S * 16;
    static constexpr int B_FULL = 0;                    // [S] raw tile landed (TMA bytes / cp.async arrivals)
    static constexpr int B_FREE = B_FULL + S;           // [S] producers finished reading the slot
    static constexpr int B_QKD = B_FREE + S;            // [S] QK finished reading the slot
    static constexpr int B_SFA_FULL = B_QKD + S;        // [2] pool scales of a tile written to TMEM
    static constexpr int B_S_FULL = B_SFA_FULL + 2;     // S^T complete in TMEM
    static constexpr int B_S_FREE = B_S_FULL + 1;       // softmax has S^T in registers
    static constexpr int B_P_FULL = B_S_FREE + 1;       // P^T complete in shared memory
    static constexpr int B_PV_DONE = B_P_FULL + 1;      // PV of a tile complete (O^T stable, P^T free)
    static constexpr int B_V_FULL = B_PV_DONE + 1;      // [V] V chunk written
    static constexpr int B_V_EMPTY = B_V_FULL + V;      // [V] PV finished reading the V chunk
    static constexpr int B_Q = B_V_EMPTY + V;           // prepared Q landed (set-up)
    static constexpr int B_DRAIN = B_Q + 1;             // every MMA of the CTA complete (before TMEM is freed)
    static constexpr int B_SFB = B_DRAIN + 1;           // Q-term scales (B scale factors) in TMEM
    static constexpr int kNumBars = B_SFB + 1;
    static constexpr int SM_IDX = SM_BARS + ((kNumBars * 8 + 15) / 16) * 16;
    static constexpr int SM_END = SM_IDX + kMaxIdx * 4;
    static constexpr int kSmemBytes = SM_END + 1024;                 // slack to align the base
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static_assert(SM_VT >= kNQ * kLatent * 4, "epilogue staging fits below the V buffers");
};
static_assert(kQImageBytes == 2 * kCodeBytes + 2 * 4096 + 256, "prepared-Q image layout");

// Tensor memory columns (all 128 lanes).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTS = 0;      // S^T: 128 columns
constexpr uint32_t kTO = 128;    // O^T: 4 d-blocks x 64 rows
constexpr uint32_t kTSFA = 384;  // 2 slots x 32 columns: pool scales of a tile
constexpr uint32_t kTSFB = 448;  // 2 passes x 32 columns: Q-term scales

struct Fp4Params {
    const uint8_t* pool;           // sparse: rows are bulk-copied from here
    int64_t pool_rows;
    const int32_t* tables;
    int64_t tables_stride;
    const int32_t* seq_lens;
    int batch, q_len, num_heads, groups, splits;
    int page_shift, box_rows;
    int64_t num_pages;
    int max_seq_len, tiles_total;   // tiles of the planned context, spread over the splits
    float bmm2_scale;
    __nv_bfloat16* out;
    int64_t o_sb, o_sq, o_sh;
    float* part_o;
    float* part_ml;
    const uint8_t* qimg;
    float* lse;                    // optional [batch][q_len][heads] (single-split plans)
    int32_t* err;
    const float* rope_logits;      // rope scores [units][64][rope_ld] (rope side-pool only)
    int64_t rope_ld;
};

struct QPrepParams {
    const __nv_bfloat16* q;
    int64_t q_sb, q_sq, q_sh;
    int q_len, num_heads, groups;
    float scale_log2;
    uint8_t* qimg;
    float* rope_q;   // [units][64][64] fp32: q's rope part times the row's 2^-e_n (null: no rope)
};

// Q of one query group (64 rows) -> four NVFP4 terms, written as the fused kernel's shared
// memory image: term tt goes to pass tt>>1, B-operand row 64 (tt&1) + n (K-major, 128-byte
// swizzle); its per-16 e4m3 scales to [pass][row][32]; qs[n] = log2e * bmm1_scale * 2^e_n.
// Each row is first scaled by 2^-e_n (exact) so its largest |q| lies in [2^10, 2^11) and the
// first term's scales stay within e4m3; each later term codes the residual of the earlier
// ones.  One warp per row, one lane per 16-dim block: q_prep_row quantises row n of the
// group from its 16 bf16 values per lane (u0, u1; zeros for rows past the group).
__device__ __forceinline__ void q_prep_row(const QPrepParams& p, int unit, int n, bool real, int lane,
                                           uint4 u0, uint4 u1, uint32_t rope_w) {
    const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    float x[16];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        x[2 * j] = __uint_as_float(w8[j] << 16);
        x[2 * j + 1] = __uint_as_float(w8[j] & 0xFFFF0000u);
        amax = fmaxf(amax, fmaxf(fabsf(x[2 * j]), fabsf(x[2 * j + 1])));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
    // e = floor(log2 amax) - 10 from the exponent bits (a subnormal or zero row keeps e = 0 and
    // its terms quantise to zero, as the reference data never has such rows in practice)
    const int eb = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu);
    int e = (eb > 0 && eb < 255) ? eb - 127 - 10 : 0;
    e = max(-100, min(100, e));
    const float mul = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);   // 2^-e, exact
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] *= mul;
    if (p.rope_q)   // rope dims 512 + 2 lane, +1, on the same power-of-two scale as the terms
        reinterpret_cast<float2*>(p.rope_q + (static_cast<size_t>(unit) * kNQ + n) * 64)[lane] =
            make_float2(__uint_as_float(rope_w << 16) * mul, __uint_as_float(rope_w & 0xFFFF0000u) * mul);
    uint8_t* img = p.qimg + static_cast<size_t>(unit) * kQImageBytes;
    const int chunk = (lane & 15) >> 1;
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
        // block amax as a tree (the chain of each term is the kernel's latency); the scale and
        // its reciprocal need not be exact: they only place the codes, which the next terms
        // correct, and the decode uses the stored e4m3 scale itself
        float a8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) a8[j] = fmaxf(fabsf(x[2 * j]), fabsf(x[2 * j + 1]));
#pragma unroll
        for (int j = 0; j < 4; ++j) a8[j] = fmaxf(a8[j], a8[j + 4]);
        const float am = fmaxf(fmaxf(a8[0], a8[2]), fmaxf(a8[1], a8[3]));
        const uint8_t sb = am > 0.0f ? f32_to_e4m3(am * (1.0f / 6.0f)) : static_cast<uint8_t>(0);
        const float sf = e4m3_to_f32(sb);
        const float inv = sf > 0.0f ? rcp_approx(sf) : 0.0f;
        uint32_t wlo = 0, whi = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t byte = f32x2_to_e2m1x2(x[2 * j] * inv, x[2 * j + 1] * inv);
            if (j < 4) wlo |= byte << (8 * j);
            else whi |= byte << (8 * (j - 4));
            const uint32_t dqw = e2m1x2_to_f16x2(byte);
            x[2 * j] -= __half2float(__ushort_as_half(static_cast<unsigned short>(dqw & 0xFFFFu))) * sf;
            x[2 * j + 1] -= __half2float(__ushort_as_half(static_cast<unsigned short>(dqw >> 16))) * sf;
        }
        const int ps = tt >> 1, R = 64 * (tt & 1) + n;
        uint8_t* dst = img + ps * (2 * 16384) + (lane >> 4) * 16384 + (R >> 3) * 1024 + (R & 7) * 128 +
                       ((chunk ^ (R & 7)) << 4) + 8 * (lane & 1);
        *reinterpret_cast<uint2*>(dst) = make_uint2(wlo, whi);
        img[2 * kCodeBytes + ps * 4096 + R * 32 + lane] = sb;
    }
    if (lane == 0)
        reinterpret_cast<float*>(img + 2 * kCodeBytes + 2 * 4096)[n] = real ? p.scale_log2 * ldexpf(1.0f, e) : 0.0f;
}

// grid = groups x 8 blocks of 8 rows (one warp per row).
__global__ void __launch_bounds__(256) q_prep_kernel(const QPrepParams p) {
    griddep_launch_dependents();   // the attention kernel may start its set-up meanwhile
    const int unit = blockIdx.x >> 3;
    const int b = unit / p.groups, g = unit % p.groups;
    const int lane = threadIdx.x & 31;
    const int n = ((blockIdx.x & 7) << 3) | (threadIdx.x >> 5);
    const int rows_here = min(kNQ, p.q_len * p.num_heads - g * kNQ);
    const bool real = n < rows_here;
    uint4 u0 = make_uint4(0, 0, 0, 0), u1 = make_uint4(0, 0, 0, 0);
    uint32_t rope_w = 0;
    if (real) {
        const int r = g * kNQ + n, qi = r / p.num_heads, h = r % p.num_heads;
        const __nv_bfloat16* row = p.q + b * p.q_sb + qi * p.q_sq + h * p.q_sh;
        u0 = ldg_nc_v4(row + 16 * lane);
        u1 = ldg_nc_v4(row + 16 * lane + 8);
        if (p.rope_q) rope_w = __ldg(reinterpret_cast<const uint32_t*>(row + kLatent) + lane);
    }
    q_prep_row(p, unit, n, real, lane, u0, u1, rope_w);
}

// Rope scores of the rope side-pool: for query group `unit` (64 rows) and token position pos
// of its entry, logits[unit][n][pos] = (q_rope[n] 2^-e_n) . k_rope[row(pos)] in fp32, in the
// units of the attention kernel's raw scores (the Q terms carry the same 2^-e_n), 0 where the
// position is masked.  One block per (unit, 128-token tile); thread = token x 32 rows.
struct RopeParams {
    const uint16_t* rope_pool;
    int64_t pool_rows, num_pages;
    const int32_t* tables;
    int64_t tables_stride;
    const int32_t* seq_lens;
    int groups, page_shift, max_seq_len, tiles_total;
    const float* rope_q;
    float* logits;
    int64_t ld;                        // tiles_total * 128
};

template <bool kSparse>
__global__ void __launch_bounds__(256) rope_logits_kernel(const RopeParams p) {
    __shared__ float4 qs[kNQ * 16];    // [64 rows][64 dims]
    const int unit = blockIdx.x / p.tiles_total, tile = blockIdx.x % p.tiles_total;
    const int b = unit / p.groups;
    const float4* qsrc = reinterpret_cast<const float4*>(p.rope_q + static_cast<size_t>(unit) * kNQ * 64);
    for (int k = threadIdx.x; k < kNQ * 16; k += blockDim.x) qs[k] = qsrc[k];
    const int t = threadIdx.x & (kTile - 1), half = threadIdx.x >> 7;
    const int pos = tile * kTile + t;
    int L = __ldg(p.seq_lens + b);
    L = L < 0 ? 0 : (L > p.max_seq_len ? p.max_seq_len : L);
    int64_t row = -1;
    if (pos < L) {
        if constexpr (kSparse) {
            const int idx = __ldg(p.tables + b * p.tables_stride + pos);
            if (idx >= 0 && idx < p.pool_rows) row = idx;
        } else {
            const int pg = __ldg(p.tables + b * p.tables_stride + (pos >> p.page_shift));
            if (pg >= 0 && pg < p.num_pages)
                row = (static_cast<int64_t>(pg) << p.page_shift) | (pos & ((1 << p.page_shift) - 1));
        }
    }
    float k[64];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 w = row >= 0 ? ldg_nc_v4(p.rope_pool + row * 64 + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            k[8 * c + 2 * h] = __uint_as_float(ws[h] << 16);
            k[8 * c + 2 * h + 1] = __uint_as_float(ws[h] & 0xFFFF0000u);
        }
    }
    __syncthreads();
    float* out = p.logits + (static_cast<int64_t>(unit) * kNQ + 32 * half) * p.ld + pos;
#pragma unroll 2
    for (int j = 0; j < 32; ++j) {
        const float4* qr = qs + (32 * half + j) * 16;
        float acc = 0.0f;
#pragma unroll
        for (int d4 = 0; d4 < 16; ++d4) {
            const float4 qv = qr[d4];
            acc = fmaf(qv.x, k[4 * d4], acc);
            acc = fmaf(qv.y, k[4 * d4 + 1], acc);
            acc = fmaf(qv.z, k[4 * d4 + 2], acc);
            acc = fmaf(qv.w, k[4 * d4 + 3], acc);
        }
        out[static_cast<int64_t>(j) * p.ld] = acc;
    }
}

__device__ __forceinline__ int page_id(const Fp4Params& p, const int* sidx, bool staged, int idx_base,
                                       int b, int pos) {
    const int pi = pos >> p.page_shift;
    return staged ? sidx[pi - idx_base] : __ldg(p.tables + b * p.tables_stride + pi);
}

// TMA loads of tile `tile_start` into ring slot `slot`.  Every box is issued (a missing page
// or a box past the context is addressed out of range and reads as zeros), so the slot always
// receives kSlotBytes.
// Rows [lo, hi) of a tile -> bits of a 128-bit row mask.
__device__ __forceinline__ void mask_rows(uint32_t (&m)[4], int lo, int hi) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const int a = max(lo, 32 * w), e = min(hi, 32 * w + 32);
        if (a < e) m[w] |= (e - a == 32 ? 0xFFFFFFFFu : ((1u << (e - a)) - 1u)) << (a - 32 * w);
    }
}

// TMA loads of tile `tile_start` into ring slot `slot`.  Every box is issued (a missing page
// or a box past the context is addressed out of range and reads as zeros), so the slot always
// receives kSlotBytes.  The tile's valid rows (in range, on a valid page) go to `mask` first,
// published to the slot's waiters by the barrier arrival.
__device__ __forceinline__ void load_tile(const Fp4Params& p, const void* tm_codes, const void* tm_scales,
                                          uint32_t sbase, uint32_t bar_full, const int* sidx, bool staged,
                                          int idx_base, int b, int tile_start, int end, int slot,
                                          uint32_t* mask) {
    const int box = p.box_rows;
    int y[kTile / 16];
    uint32_t m[4] = {0u, 0u, 0u, 0u};
#pragma unroll 1
    for (int r0 = 0, k = 0; r0 < kTile; r0 += box, ++k) {
        const int pos = tile_start + r0;
        y[k] = -box;
        if (pos < end) {
            const int pg = page_id(p, sidx, staged, idx_base, b, pos);
            if (pg >= 0 && pg < p.num_pages) {
                y[k] = (pg << p.page_shift) | (pos & ((1 << p.page_shift) - 1));
                mask_rows(m, r0, min(r0 + box, end - tile_start));
            } else {
                set_error(p.err, NVFP4KV_DEVERR_BAD_PAGE);
            }
        }
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) mask[w] = m[w];
    mbar_arrive_expect_tx(bar_full, kSlotBytes);
    const uint32_t codes = sbase + SM_STAGE + slot * kSlotBytes;
    const uint32_t scales = codes + kCodeBytes;
#pragma unroll 1
    for (int r0 = 0, k = 0; r0 < kTile; r0 += box, ++k) {
        tma_load_2d(codes + r0 * 128, tm_codes, 0, y[k], bar_full);
        tma_load_2d(codes + 16384 + r0 * 128, tm_codes, 128, y[k], bar_full);
        tma_load_2d(scales + r0 * 32, tm_scales, 256, y[k], bar_full);
    }
}

// Pool row of token position `pos` (< end), or -1 when the token is masked.  Dense: the page
// table entry must name a page of the pool.  Sparse: the table holds pool rows, -1 padded;
// with `report`, entries < -1 or >= pool_rows set NVFP4KV_DEVERR_BAD_INDEX.
template <bool kSparse>
__device__ __forceinline__ int64_t token_row(const Fp4Params& p, const int* sidx, bool staged, int idx_base,
                                             int b, int pos, bool report) {
    if constexpr (kSparse) {
        // sparse rows are staged as a window of kIdxTiles tiles (tile j at j % kIdxTiles)
        const int idx = staged ? sidx[(pos - idx_base) % kMaxIdx] : __ldg(p.tables + b * p.tables_stride + pos);
        if (idx < 0 || idx >= p.pool_rows) {
            if (report && idx != -1) set_error(p.err, NVFP4KV_DEVERR_BAD_INDEX);
            return -1;
        }
        return idx;
    } else {
        const int pg = page_id(p, sidx, staged, idx_base, b, pos);
        if (pg < 0 || pg >= p.num_pages) return -1;
        return (static_cast<int64_t>(pg) << p.page_shift) | (pos & ((1 << p.page_shift) - 1));
    }
}

// Sparse: the rows of tile `tile_start` into the ring slot at `slot_base` by TMA row gathers
// (tile::gather4: four arbitrary pool rows per instruction, the box one row high), issued by a
// group of NW warps of the control warpgroup together: the issue of a gather4 serialises over
// the lanes of a warp (measured, 148 CTAs x 16 tiles of 128 random rows: 3.6 us per tile from
// one warp, 2.4 us from two, 1.9 us from four), so warp wq of the group takes mask words
// wq, wq + NW, ... (word k: rows 32k .. 32k + 31), eight lanes of four rows per word.  Four
// rows are three gathers: the two 128-byte halves of their codes (written 128-byte swizzled,
// the layout the dense path's tile boxes produce) and their 32 scale bytes.  A masked row (-1
// padding, an out-of-range entry, a position past `end`) is fetched from pool row 0: its bit
// stays clear in the slot's valid-row mask, the softmax gives it probability 0 and the
// producers write its V as zeros, so nothing of that row reaches the output.  Named barrier
// `bar_id` (the group's NW x 32 threads) orders every mask word before the arming arrive
// (warp 0 of the group) and that before any copy of the phase.
template <int NW>
__device__ __forceinline__ void load_rows_gather4_grp(const Fp4Params& p, const void* tm_codes, const void* tm_scales,
                                                      uint32_t slot_base, uint32_t bar_full, uint32_t* slot_mask,
                                                      const int* sidx, int idx_base, int b, int tile_start, int end,
                                                      int wq, int lane, int bar_id) {
    const int k = lane >> 3;                 // which of this warp's words
    const int w = wq + NW * k;               // the mask word, rows 32w .. 32w + 31
    const bool act = w < 4;
    const int r0 = 32 * w + 4 * (lane & 7);
    int rows[4];
    uint32_t live = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int pos = tile_start + r0 + j;
        const int64_t row = act && pos < end ? token_row<true>(p, sidx, true, idx_base, b, pos, true) : -1;
        live |= static_cast<uint32_t>(row >= 0) << j;
        rows[j] = row >= 0 ? static_cast<int>(row) : 0;
    }
    uint32_t bits[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) bits[j] = __ballot_sync(0xFFFFFFFFu, (live >> j) & 1u);
    if (act && (lane & 7) == 0) {   // row 32w + 4m + j is bit 4m + j of word w
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int m = 0; m < 8; ++m) word |= ((bits[j] >> (8 * k + m)) & 1u) << (4 * m + j);
        slot_mask[w] = word;
    }
    named_bar_sync(bar_id, NW * 32);   // every mask word written before the arming arrive
    if (wq == 0 && lane == 0) mbar_arrive_expect_tx(bar_full, kSlotBytes);
    named_bar_sync(bar_id, NW * 32);   // armed before any copy of the phase issues
    if (act) {
        tma_gather4(slot_base + r0 * 128, tm_codes, 0, rows, bar_full);
        tma_gather4(slot_base + 16384 + r0 * 128, tm_codes, 128, rows, bar_full);
        tma_gather4(slot_base + kCodeBytes + r0 * 32, tm_scales, 256, rows, bar_full);
    }
}

// The prepared Q image of (sequence b, query group g) -> shared memory: Q-term codes, their
// scale image (in the P^T buffer until the set-up moves it to TMEM) and the per-row constants.
// It is the output of the Q preparation kernel this one may overlap (all else this kernel reads
// was complete before that kernel started), hence the grid dependency wait.
template <int kQB, int kPT, int kQS>
__device__ __forceinline__ void load_q_image(const Fp4Params& p, uint32_t sbase, uint32_t bar_q, int b, int g) {
    griddep_wait();
    const uint8_t* img = p.qimg + static_cast<size_t>(b * p.groups + g) * kQImageBytes;
    mbar_arrive_expect_tx(bar_q, static_cast<uint32_t>(kQImageBytes));
    bulk_copy_g2s(sbase + kQB, img, 2 * kCodeBytes, bar_q);
    bulk_copy_g2s(sbase + kPT, img + 2 * kCodeBytes, 2 * 4096, bar_q);
    bulk_copy_g2s(sbase + kQS, img + 2 * kCodeBytes + 2 * 4096, 256, bar_q);
}

// Pool scales of the tile in `slot` -> TMEM scale-factor columns `col` of this warp's
// sub-partition: column 4kk+q of lane r holds the 4 scales (dims 64kk..64kk+63) of token
// 32q + r.  Every sub-partition needs a full copy.
__device__ __forceinline__ void scales_to_tmem(const uint8_t* scales, uint32_t taddr, int lane) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {   // columns 16 half .. +16: dims 256 half .. +256
        uint32_t rr[16];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 w = reinterpret_cast<const uint4*>(scales + (32 * q4 + lane) * 32)[half];
            rr[0 + q4] = w.x;
            rr[4 + q4] = w.y;
            rr[8 + q4] = w.z;
            rr[12 + q4] = w.w;
        }
        tmem_st16(taddr + 16 * half, rr);
    }
    tmem_wait_st();
}

// scales_to_tmem four columns at a time (same layout), for call sites where registers are
// scarce: column 4kk+q of lane r holds word kk of token 32q + r's 32 scale bytes.
__device__ __forceinline__ void scales_to_tmem_narrow(const uint8_t* scales, uint32_t taddr, int lane) {
#pragma unroll 1
    for (int kk = 0; kk < 8; ++kk) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(scales + lane * 32 + 4 * kk);
        tmem_st4(taddr + 4 * kk, w[0], w[32 * 8], w[64 * 8], w[96 * 8]);
    }
    tmem_wait_st();
}

// Max (kSum = false) or sum over the 32 lanes of 32 values per lane; lane L returns the
// result for value index L.  `v` is left unchanged: the first exchange step writes into a
// 16-value scratch, which later steps halve in place.
template <bool kSum>
__device__ __forceinline__ float warp_reduce_scatter32(const float (&v)[32], int lane) {
    float w[16];
    {
        const bool upper = (lane & 16) != 0;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float send = upper ? v[j] : v[j + 16];
            const float keep = upper ? v[j + 16] : v[j];
            const float recv = __shfl_xor_sync(0xFFFFFFFFu, send, 16);
            w[j] = kSum ? keep + recv : fmaxf(keep, recv);
        }
    }
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < off; ++j) {
            const float send = upper ? w[j] : w[j + off];
            const float keep = upper ? w[j + off] : w[j];
            const float recv = __shfl_xor_sync(0xFFFFFFFFu, send, off);
            w[j] = kSum ? keep + recv : fmaxf(keep, recv);
        }
    }
    return w[0];
}

// Max over the 32 lanes of 16 values per lane; lane L returns the result for value L & 15.
__device__ __forceinline__ float warp_max_scatter16(const float (&v)[16], int lane) {
    float w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = fmaxf(v[j], __shfl_xor_sync(0xFFFFFFFFu, v[j], 16));
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < off; ++j) {
            const float send = upper ? w[j] : w[j + off];
            const float keep = upper ? w[j + off] : w[j];
            w[j] = fmaxf(keep, __shfl_xor_sync(0xFFFFFFFFu, send, off));
        }
    }
    return w[0];
}

// p = 2^(s qs - m) for the 32 rows of this thread (0 where not visible), packed as fp16 pairs;
// row sums accumulate in l.
__device__ __forceinline__ void probs32(const float (&sraw)[32], const float* qs_h, const float* M_h,
                                        const int* lim_h, bool tok_ok, bool per_row_lim, int pos,
                                        float (&l)[32], uint32_t (&pk)[16]) {
#pragma unroll
    for (int n4 = 0; n4 < 8; ++n4) {
        const float4 q4 = reinterpret_cast<const float4*>(qs_h)[n4];
        const float4 m4 = reinterpret_cast<const float4*>(M_h)[n4];
        const int4 l4 = reinterpret_cast<const int4*>(lim_h)[n4];
        const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
        const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
        const int lv[4] = {l4.x, l4.y, l4.z, l4.w};
        float pv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const bool vis = tok_ok && (!per_row_lim || pos < lv[k]);
            pv[k] = vis ? ex2_approx(fmaf(sraw[4 * n4 + k], qv[k], -mv[k])) : 0.0f;
            l[4 * n4 + k] += pv[k];
        }
        pk[2 * n4] = pack_half2(pv[0], pv[1]);
        pk[2 * n4 + 1] = pack_half2(pv[2], pv[3]);
    }
}

// kSparse: the table holds pool rows (top-k, -1 padded) instead of page ids; the tensor maps
// have one-row boxes for the row gathers.
template <bool kSparse, int kRing, int kVBuf, bool kRope>
__global__ void __launch_bounds__(kThreads, 1)
decode_fp4_kernel(const __grid_constant__ Fp4Params p, const __grid_constant__ CUtensorMap tm_codes,
                  const __grid_constant__ CUtensorMap tm_scales) {
    using C = DecCfg<kRing, kVBuf>;
    constexpr int kSlots = C::kSlots, kVBufs = C::kVBufs;
    constexpr int SM_QB = C::SM_QB, SM_VT = C::SM_VT, SM_PT = C::SM_PT, SM_M = C::SM_M, SM_ALPHA = C::SM_ALPHA;
    constexpr int SM_QS = C::SM_QS, SM_LIM = C::SM_LIM, SM_LSUM = C::SM_LSUM, SM_RED = C::SM_RED;
    constexpr int SM_ROWOFF = C::SM_ROWOFF, SM_FLAGS = C::SM_FLAGS, SM_TMASK = C::SM_TMASK, SM_BARS = C::SM_BARS;
    constexpr int SM_IDX = C::SM_IDX;
    // Sparse: the control warpgroup writes tile 1's pool scales into TMEM (the slot's first
    // use), each warp its sub-partition's copy (warps 12-15 are sub-partitions 0-3), as the
    // tile lands; on the softmax side that write sat between P(0) and QK(1).  Tile 0's (set-up)
    // and every later pool-scale write is the softmax warps'; the MMA warp writing tile 0's
    // copy delayed QK(0) by 0.6 us.
    constexpr bool kSfaByCtl = kSparse;
    constexpr int B_FULL = C::B_FULL, B_FREE = C::B_FREE, B_QKD = C::B_QKD, B_SFA_FULL = C::B_SFA_FULL;
    constexpr int B_S_FULL = C::B_S_FULL, B_S_FREE = C::B_S_FREE, B_P_FULL = C::B_P_FULL, B_PV_DONE = C::B_PV_DONE;
    constexpr int B_V_FULL = C::B_V_FULL, B_V_EMPTY = C::B_V_EMPTY, B_Q = C::B_Q, B_DRAIN = C::B_DRAIN;
    constexpr int B_SFB = C::B_SFB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int s = blockIdx.x % p.splits;
    const int bg = blockIdx.x / p.splits;
    const int g = bg % p.groups;
    const int b = bg / p.groups;

    int L = __ldg(p.seq_lens + b);
    if (L > p.max_seq_len) {
        if (threadIdx.x == 0) set_error(p.err, NVFP4KV_DEVERR_SEQ_LEN);
        L = p.max_seq_len;
    }
    if (L < 0) L = 0;
    // split s covers tiles [s T / splits, (s + 1) T / splits) of the planned context
    const int start = static_cast<int>((static_cast<int64_t>(s) * p.tiles_total) / p.splits) * kTile;
    const int end = min(static_cast<int>((static_cast<int64_t>(s + 1) * p.tiles_total) / p.splits) * kTile, L);
    const int n_tiles = end > start ? (end - start + kTile - 1) / kTile : 0;
    const int rows_here = min(kNQ, p.q_len * p.num_heads - g * kNQ);

    float* Mrow = reinterpret_cast<float*>(smem + SM_M);
    float* alpha = reinterpret_cast<float*>(smem + SM_ALPHA);
    float* qs = reinterpret_cast<float*>(smem + SM_QS);
    int* lim = reinterpret_cast<int*>(smem + SM_LIM);
    float* lsum = reinterpret_cast<float*>(smem + SM_LSUM);
    float* red = reinterpret_cast<float*>(smem + SM_RED);
    int64_t* rowoff = reinterpret_cast<int64_t*>(smem + SM_ROWOFF);
    int* sidx = reinterpret_cast<int*>(smem + SM_IDX);
    uint32_t* tmask = reinterpret_cast<uint32_t*>(smem + SM_TMASK);   // [slot][4]: valid rows
    volatile int* flags = reinterpret_cast<volatile int*>(smem + SM_FLAGS);
    volatile int* abort_flag = flags + 1;
    auto bar = [&](int i) -> uint32_t { return sbase + SM_BARS + 8 * i; };

    if (threadIdx.x == 0) {
        for (int k = 0; k < kSlots; ++k) {
            mbar_init(bar(B_FULL + k), 1);
            mbar_init(bar(B_FREE + k), kProducerWarps);
            mbar_init(bar(B_QKD + k), 1);
        }
        for (int k = 0; k < 2; ++k) mbar_init(bar(B_SFA_FULL + k), 4);
        for (int k = 0; k < kVBufs; ++k) {
            mbar_init(bar(B_V_FULL + k), kProducerWarps);
            mbar_init(bar(B_V_EMPTY + k), 1);
        }
        mbar_init(bar(B_S_FULL), 1);
        mbar_init(bar(B_S_FREE), kSoftmaxWarps);
        mbar_init(bar(B_P_FULL), kSoftmaxWarps);
        mbar_init(bar(B_PV_DONE), 1);
        mbar_init(bar(B_Q), 1);
        mbar_init(bar(B_SFB), kSoftmaxWarps);
        mbar_init(bar(B_DRAIN), 1);
        flags[1] = 0;
        mbar_fence_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(sbase + SM_FLAGS, kTmemCols);
        tmem_relinquish();
    }
    // page ids (dense) / pool rows (sparse) of this split
    const int idx_base = kSparse ? start : start >> p.page_shift;
    const int idx_count = end <= start ? 0 : kSparse ? end - start : ((end - 1) >> p.page_shift) - idx_base + 1;
    // dense: the split's page ids when they fit; sparse: always, as a window of the first
    // kIdxTiles tiles' rows that the load warp refills ahead of its copies
    const bool staged = kSparse || idx_count <= kMaxIdx;
    if (staged)
        for (int k = threadIdx.x; k < min(idx_count, kMaxIdx); k += kThreads)
            sidx[k] = __ldg(p.tables + b * p.tables_stride + idx_base + k);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = static_cast<uint32_t>(flags[0]);
    auto sfa_by_ctl = [&](int j) {   // tile j < 2 (first ring pass): ring slot j, TMEM scale slot j
        mbar_wait(bar(B_FULL + j), 0, abort_flag, p.err);
        scales_to_tmem_narrow(smem + SM_STAGE + j * kSlotBytes + kCodeBytes,
                              tmem + kTSFA + 32 * j + (static_cast<uint32_t>(32 * (warp & 3)) << 16), lane);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_SFA_FULL + j));
    };
    griddep_launch_dependents();   // the split combine may be scheduled; it waits for this grid

    if (warp >= kMmaWarp) {
    warpgroup_reg_dealloc<kRegsCtl>();
    if constexpr (kSparse) {
        // the first ring tiles: rows gathered by all four warps of the group
        if (lane == 0) {
            tma_prefetch_desc(&tm_codes);
            tma_prefetch_desc(&tm_scales);
        }
        for (int j = 0; j < kSlots && j < n_tiles; ++j)
            load_rows_gather4_grp<4>(p, &tm_codes, &tm_scales, sbase + SM_STAGE + j * kSlotBytes, bar(B_FULL + j),
                                     tmask + 4 * j, sidx, idx_base, b, start + j * kTile, end, warp - kMmaWarp,
                                     lane, kLoadBar);
        // the MMA warp writes its copy after QK(0) is issued
        if (kSfaByCtl && warp != kMmaWarp && n_tiles > 1) sfa_by_ctl(1);
        if (warp != kMmaWarp) {
            // ======================================================== sparse refills
            // tile j -> slot j % kSlots once QK(j - kSlots) and the producers are done with it,
            // gathered by the load warp and the two spare warps together
            const int wq = warp - kTmaWarp;
            int issued = n_tiles < kSlots ? n_tiles : kSlots;   // tile j completes phase j / kSlots of its slot
            // Splits longer than the index window: after tile t is issued, the load warp loads
            // the rows of tile t + kSlots into registers (window slot (t + kSlots) % kIdxTiles,
            // whose tile t + kSlots - kIdxTiles was issued long before) and stores them before
            // the next issue, so no copy waits on a table load.
            static_assert(2 * kSlots <= kIdxTiles, "index window covers the refill distance");
            const bool refill = idx_count > kMaxIdx;
            int pend[4] = {-1, -1, -1, -1};
            int pend_tile = -1;
#pragma unroll 1
            for (int i = 0; i + kSlots < n_tiles; ++i) {
                const int slot = i % kSlots;
                const uint32_t sph = (i / kSlots) & 1;
                const bool f = mbar_wait(bar(B_FREE + slot), sph, abort_flag, p.err);
                const bool d = mbar_wait(bar(B_QKD + slot), sph, abort_flag, p.err);
                // after an abort nothing more is issued (the drain below waits for what was);
                // the three warps decide together, so none is left at a named barrier
                if (named_bar_red_or(kRefillBar, 96, !(f && d) || *abort_flag)) break;
                if (wq == 0 && pend_tile >= 0) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) sidx[(pend_tile % kIdxTiles) * kTile + 32 * k + lane] = pend[k];
                }
                fence_proxy_async_smem();
                named_bar_sync(kRefillBar, 96);   // the refreshed row ids visible to the group
                const int t = i + kSlots;
                load_rows_gather4_grp<3>(p, &tm_codes, &tm_scales, sbase + SM_STAGE + slot * kSlotBytes,
                                         bar(B_FULL + slot), tmask + 4 * slot, sidx, idx_base, b, start + t * kTile,
                                         end, wq, lane, kRefillBar);
                issued = t + 1;
                pend_tile = -1;
                if (wq == 0 && refill && t + kSlots >= kIdxTiles && t + kSlots < n_tiles) {
                    pend_tile = t + kSlots;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int pos = start + pend_tile * kTile + 32 * k + lane;
                        pend[k] = pos < end ? __ldg(p.tables + b * p.tables_stride + pos) : -1;
                    }
                }
            }
            if (wq == 0)
                for (int j = issued > kSlots ? issued - kSlots : 0; j < issued; ++j)
                    mbar_drain_wait(bar(B_FULL + j % kSlots), (j / kSlots) & 1);
        }
    }
    if (warp == kTmaWarp) {
        // ============================================================ TMA / bulk loads
        // The Q image (the output of the Q preparation kernel this one may overlap) is copied
        // first for dense (measured: the dense step lost 0.2 us the other way round); for
        // sparse a softmax thread copies it while the row gathers issue.
        if (lane == 0) {
            tma_prefetch_desc(&tm_codes);
            tma_prefetch_desc(&tm_scales);
        }
        if constexpr (kSparse) {
            // the row gathers are issued above
        } else if (lane == 0) {
            load_q_image<SM_QB, SM_PT, SM_QS>(p, sbase, bar(B_Q), b, g);
            int issued = 0;   // tiles loaded; tile j completes phase j / kSlots of slot j % kSlots
            for (int j = 0; j < kSlots && j < n_tiles; ++j) {
                load_tile(p, &tm_codes, &tm_scales, sbase, bar(B_FULL + j), sidx, staged, idx_base, b,
                          start + j * kTile, end, j, tmask + 4 * j);
                issued = j + 1;
            }
#pragma unroll 1
            for (int i = 0; i + kSlots < n_tiles; ++i) {
                const int slot = i % kSlots;
                const uint32_t sph = (i / kSlots) & 1;
                const bool f = mbar_wait(bar(B_FREE + slot), sph, abort_flag, p.err);
                const bool d = mbar_wait(bar(B_QKD + slot), sph, abort_flag, p.err);
                // after an abort nothing more is issued: a slot is re-armed only once its last
                // transfer was consumed (the drain below waits for what is in flight)
                if (!f || !d || *abort_flag) break;
                fence_proxy_async_smem();
                load_tile(p, &tm_codes, &tm_scales, sbase, bar(B_FULL + slot), sidx, staged, idx_base, b,
                          start + (i + kSlots) * kTile, end, slot, tmask + 4 * slot);
                issued = i + kSlots + 1;
            }
            for (int j = issued > kSlots ? issued - kSlots : 0; j < issued; ++j)
                mbar_drain_wait(bar(B_FULL + j % kSlots), (j / kSlots) & 1);
        }
        // the Q image copy lands before the CTA can exit
        if (lane == 0) mbar_drain_wait(bar(B_Q), 0);
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ============================================================ MMA issue
        constexpr uint32_t idq = idesc_fp4_f32(kTile, 128);
        constexpr uint32_t idp = idesc_f16_f32(128, kNQ, true, true);
        const uint64_t dq0 = smem_desc_sw128(sbase + SM_QB, 16, 1024);
        const uint64_t dpt = smem_desc_sw128(sbase + SM_PT, 16, 1024);
        mbar_wait(bar(B_Q), 0, abort_flag, p.err);   // Q-term codes in shared memory
        mbar_wait(bar(B_SFB), 0, abort_flag, p.err); // and their scales in TMEM (both passes)
#pragma unroll 1
        for (int i = 0; i <= n_tiles; ++i) {
            if (i < n_tiles) {
                const int slot = i % kSlots, fb = i & 1;
                if (kSfaByCtl && i == 1) sfa_by_ctl(1);
                mbar_wait(bar(B_FULL + slot), (i / kSlots) & 1, abort_flag, p.err);
                mbar_wait(bar(B_SFA_FULL + fb), (i >> 1) & 1, abort_flag, p.err);
                if (i > 0) mbar_wait(bar(B_S_FREE), (i - 1) & 1, abort_flag, p.err);
                tc_fence_after();
                const uint64_t da0 = smem_desc_sw128(sbase + SM_STAGE + slot * kSlotBytes, 16, 1024);
                const uint32_t sfa = tmem + kTSFA + 32 * fb, sfb = tmem + kTSFB;
                if (elect_one()) {
#pragma unroll
                    for (int ps = 0; ps < 2; ++ps)
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                            tc_mma_fp4(tmem + kTS, da0 + off, dq0 + ((ps * 32768) >> 4) + off, idq,
                                       (ps | kk) != 0, sfa + 4 * kk, sfb + 32 * ps + 4 * kk);
                        }
                    tc_commit(bar(B_S_FULL));
                    tc_commit(bar(B_QKD + slot));
                }
                __syncwarp();
            }
            if (i > 0) {
                const int t = i - 1;
                mbar_wait(bar(B_P_FULL), t & 1, abort_flag, p.err);
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < kChunks; ++c) {
                    const int u = kChunks * t + c, vb = u % kVBufs;
                    mbar_wait(bar(B_V_FULL + vb), (u / kVBufs) & 1, abort_flag, p.err);
                    tc_fence_after();
                    const uint64_t dv = smem_desc_sw128(sbase + SM_VT + vb * kVtBytes, 2048, 1024);
                    const uint64_t dp = dpt + ((c * kChunk * 128) >> 4);
                    if (elect_one()) {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            tc_mma_f16(tmem + kTO + 64 * j, dv + ((j * 4096) >> 4), dp, idp, (t | c) != 0);
                        tc_commit(bar(B_V_EMPTY + vb));
                        if (c == kChunks - 1) tc_commit(bar(B_PV_DONE));
                    }
                    __syncwarp();
                }
            }
        }
        // every MMA of this CTA completes before its TMEM is freed, on the abort path too
        if (elect_one()) tc_commit(bar(B_DRAIN));
        __syncwarp();
        mbar_drain_wait(bar(B_DRAIN), 0);
    }
    } else if (warp >= kProducerWarp0) {
        warpgroup_reg_dealloc<kRegsProducer>();
        // ============================================================ producers: V chunks
        // lane -> token tq = lane & 15 of the chunk; 16-byte code chunks (32 dims) sc0 =
        // 4 pw + (lane >> 4) and sc0 + 2.
        const int pw = warp - kProducerWarp0;
#pragma unroll 1
        for (int i = 0; i < n_tiles; ++i) {
            const int slot = i % kSlots;
            mbar_wait(bar(B_FULL + slot), (i / kSlots) & 1, abort_flag, p.err);
            const uint8_t* codes = smem + SM_STAGE + slot * kSlotBytes;
            const uint8_t* scales = codes + kCodeBytes;
#pragma unroll 1
            for (int c = 0; c < kChunks; ++c) {
                const int u = kChunks * i + c, vb = u % kVBufs;
                const int tq = lane & 15;
                const int tok = c * kChunk + tq;
                const int sc0 = 4 * pw + (lane >> 4);
                // dequantise both 32-dim pieces into registers first; the destination buffer
                // is awaited only for the stores
                uint32_t hv[2][16];
#pragma unroll
                for (int it = 0; it < 2; ++it) {
                    const int sc = sc0 + 2 * it;
                    const uint4 cw = *reinterpret_cast<const uint4*>(
                        codes + (sc >> 3) * 16384 + (tok >> 3) * 1024 + (tok & 7) * 128 + (((sc & 7) ^ (tok & 7)) << 4));
                    const uint32_t s2 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(scales + tok * 32 + 2 * sc));
                    const uint32_t slo = (s2 & 0xFFFFu) * 0x10001u, shi = (s2 >> 16) * 0x10001u;
                    const uint32_t cws[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        uint32_t t4[4];
                        e2m1x8_to_f16x2x4(cws[w], t4);
                        const uint32_t sv = w < 2 ? slo : shi;
#pragma unroll
                        for (int k = 0; k < 4; ++k) hv[it][4 * w + k] = hmul2_u32(t4[k], sv);
                    }
                }
                // a masked row (padding, a bad entry, a missing page, past the context) may hold
                // anything, even NaN scales: its V is written as zeros (its probability is 0)
                if (!((tmask[4 * slot + (tok >> 5)] >> (tok & 31)) & 1u)) {
#pragma unroll
                    for (int it = 0; it < 2; ++it)
#pragma unroll
                        for (int k = 0; k < 16; ++k) hv[it][k] = 0u;
                }
                if (u >= kVBufs) mbar_wait(bar(B_V_EMPTY + vb), ((u / kVBufs) - 1) & 1, abort_flag, p.err);
                uint8_t* vt = smem + SM_VT + vb * kVtBytes + tq * 128;
#pragma unroll
                for (int it = 0; it < 2; ++it) {
                    const int sc = sc0 + 2 * it;
                    // dims 32sc + 8j .. +8 -> d-atom sc>>1, 16-byte chunk 4(sc&1) + j
                    uint8_t* row = vt + (sc >> 1) * 2048;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4*>(row + (((4 * (sc & 1) + j) ^ (tq & 7)) << 4)) =
                            make_uint4(hv[it][4 * j], hv[it][4 * j + 1], hv[it][4 * j + 2], hv[it][4 * j + 3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_V_FULL + vb));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_FREE + slot));
        }
    } else {
        warpgroup_reg_alloc<kRegsSoftmax>();
        // ============================================================ softmax
        // warp w: TMEM sub-partition sp = w & 3 (token t = 32 sp + lane), query rows 32 hh .. +32
        const int sp = warp & 3, hh = warp >> 2;
        const int t = 32 * sp + lane;
        const uint32_t lane_base = static_cast<uint32_t>(32 * sp) << 16;
        const float* qs_h = qs + 32 * hh;
        const int* lim_h = lim + 32 * hh;
        const float* M_h = Mrow + 32 * hh;
        const float* alpha_h = alpha + 32 * hh;
        const bool per_row_lim = p.q_len > 1;   // q_len 1: every row sees the whole context

        // ---- set-up: per-row constants, Q-term scales (B scale factors) and tile 0's pool
        // scales (A scale factors) into TMEM; every sub-partition gets a full copy
        if (kSparse && threadIdx.x == 0) load_q_image<SM_QB, SM_PT, SM_QS>(p, sbase, bar(B_Q), b, g);
        mbar_wait(bar(B_Q), 0, abort_flag, p.err);
        if (threadIdx.x < kNQ) {
            const int n = threadIdx.x;
            const bool real = n < rows_here;
            const int r = g * kNQ + n;
            const int qi = real ? r / p.num_heads : 0, h = real ? r % p.num_heads : 0;
            lim[n] = real ? L - (p.q_len - 1 - qi) : -1;
            rowoff[n] = real ? b * p.o_sb + qi * p.o_sq + h * p.o_sh : 0;
            Mrow[n] = -INFINITY;
        }
        {
            const uint8_t* sfb_img = smem + SM_PT;   // [2 passes][128 rows][32 scale bytes]
            uint32_t rr[32];
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
                    rr[4 * kk + q4] = *reinterpret_cast<const uint32_t*>(sfb_img + hh * 4096 +
                                                                         (32 * q4 + lane) * 32 + 4 * kk);
            tmem_st32(tmem + kTSFB + 32 * hh + lane_base, rr);
            tmem_wait_st();
            // every softmax warp writes a part (pass hh, its sub-partition): the MMA waits for all
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_SFB));
        }
        if (hh == 0 && n_tiles > 0) {
            mbar_wait(bar(B_FULL + 0), 0, abort_flag, p.err);
            scales_to_tmem(smem + SM_STAGE + kCodeBytes, tmem + kTSFA + lane_base, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_SFA_FULL + 0));
        }
        named_bar_sync(1, kSoftmaxThreads);   // per-row constants visible; the SFB image is read

        float l[32];
#pragma unroll
        for (int n = 0; n < 32; ++n) l[n] = 0.0f;
#pragma unroll 1
        for (int i = 0; i < n_tiles; ++i) {
            mbar_wait(bar(B_S_FULL), i & 1, abort_flag, p.err);
            tc_fence_after();
            // pool scales of tile i+1 -> its TMEM slot (QK(i-1), the slot's last reader, is
            // complete: S_FULL(i) tracks every earlier MMA).  In a long split the ring loads
            // tiles two ahead, so tile i+1 has landed and its scales go now: QK(i+1) runs while
            // P(i) is computed.  Short sparse splits (one or two tiles, the two-slot ring) start
            // with both tiles' row gathers in flight: there they go after P(i), which must not
            // wait for tile i+1 to land.
            const bool next_tile = hh == 0 && i + 1 < n_tiles && !(kSfaByCtl && i == 0);
            const bool early = next_tile && !(kSparse && kSlots == 2);
            if (early) {
                mbar_wait(bar(B_FULL + (i + 1) % kSlots), ((i + 1) / kSlots) & 1, abort_flag, p.err);
                scales_to_tmem(smem + SM_STAGE + ((i + 1) % kSlots) * kSlotBytes + kCodeBytes,
                               tmem + kTSFA + 32 * ((i + 1) & 1) + lane_base, lane);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_SFA_FULL + ((i + 1) & 1)));
            }

            // Scores of this thread's token for its 32 query rows (S^T stays allocated until
            // the vote below: a rescale reads it again).
            float sv[32];
            auto load_scores = [&]() {
                uint32_t a[32], c2[32];
                tmem_ld32(tmem + kTS + 32 * hh + lane_base, a);
                tmem_ld32(tmem + kTS + 64 + 32 * hh + lane_base, c2);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) sv[j] = __uint_as_float(a[j]) + __uint_as_float(c2[j]);
                if constexpr (kRope) {   // + the rope scores of this token for the 32 rows
                    const float* rl = p.rope_logits + (static_cast<int64_t>(bg) * kNQ + 32 * hh) * p.rope_ld +
                                      start + i * kTile + t;
#pragma unroll
                    for (int j = 0; j < 32; ++j) sv[j] += __ldg(rl + j * p.rope_ld);
                }
            };
            load_scores();
            const int pos = start + i * kTile + t;
            // valid row of the tile: the load warp publishes the mask with the slot's barrier
            // (complete long before S^T of the tile exists, and not re-armed before P(i))
            mbar_wait(bar(B_FULL + i % kSlots), (i / kSlots) & 1, abort_flag, p.err);
            const bool tok_ok = (tmask[4 * (i % kSlots) + (t >> 5)] >> (t & 31)) & 1u;
            // Probabilities against the running row maxima, computed speculatively in place:
            // p = 2^(s qs - m).  They stand unless some visible score exceeds its row's max by
            // more than 2^8 (a vote over the CTA); then the maxima move and p is recomputed.
            // Sparse tile 0: the maxima are -inf, so the update below always runs; it skips this
            // pass and the vote and works on the raw scores still in sv (a tile with no visible
            // score leaves the maxima at -inf and every probability at 0).  In a sparse split
            // of two tiles that is half the softmax work; dense keeps one code path (its
            // registers are at the limit).
            const bool first = kSparse && i == 0;
            bool grow = false;
            if (!first) {
#pragma unroll
                for (int n4 = 0; n4 < 8; ++n4) {
                    const float4 q4 = reinterpret_cast<const float4*>(qs_h)[n4];
                    const float4 m4 = reinterpret_cast<const float4*>(M_h)[n4];
                    const int4 l4 = reinterpret_cast<const int4*>(lim_h)[n4];
                    const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
                    const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
                    const int lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const bool vis = tok_ok && (!per_row_lim || pos < lv[k]);
                        const float x = fmaf(sv[4 * n4 + k], qv[k], -mv[k]);
                        grow |= vis && x > kRescaleLog2;
                        sv[4 * n4 + k] = vis ? ex2_approx(x) : 0.0f;
                    }
                }
            }
            const bool any = first || named_bar_red_or(1, kSoftmaxThreads, grow);
            uint32_t pk[16];
            if (!any) {
                // common case: P is ready before PV(i-1) completes
#pragma unroll
                for (int n = 0; n < 32; ++n) l[n] += sv[n];
#pragma unroll
                for (int k = 0; k < 16; ++k) pk[k] = pack_half2(sv[2 * k], sv[2 * k + 1]);
            } else {
                // new row max = max(old, tile max); alpha = 2^(old - new)
                if (!first) load_scores();
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {   // 16 rows at a time keeps the register count down
                    float xv[16];
#pragma unroll
                    for (int n4 = 0; n4 < 4; ++n4) {
                        const float4 q4 = reinterpret_cast<const float4*>(qs_h + 16 * hf)[n4];
                        const int4 l4 = reinterpret_cast<const int4*>(lim_h + 16 * hf)[n4];
                        const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
                        const int lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const bool vis = tok_ok && (!per_row_lim || pos < lv[k]);
                            xv[4 * n4 + k] = vis ? sv[16 * hf + 4 * n4 + k] * qv[k] : -INFINITY;
                        }
                    }
                    const float mx = warp_max_scatter16(xv, lane);
                    if (lane < 16) red[sp * 64 + 32 * hh + 16 * hf + lane] = mx;
                }
                named_bar_sync(1, kSoftmaxThreads);
                if (threadIdx.x < 64) {
                    const int n = threadIdx.x;
                    const float mo = Mrow[n];
                    const float tmx = fmaxf(fmaxf(red[n], red[64 + n]), fmaxf(red[128 + n], red[192 + n]));
                    const float mn = fmaxf(mo, tmx);
                    alpha[n] = (mn == -INFINITY) ? 1.0f : ex2_approx(mo - mn);
                    Mrow[n] = mn;
                }
                named_bar_sync(1, kSoftmaxThreads);
#pragma unroll
                for (int n4 = 0; n4 < 8; ++n4) {
                    const float4 a4 = reinterpret_cast<const float4*>(alpha_h)[n4];
                    l[4 * n4] *= a4.x;
                    l[4 * n4 + 1] *= a4.y;
                    l[4 * n4 + 2] *= a4.z;
                    l[4 * n4 + 3] *= a4.w;
                }
            }
            // S^T is no longer needed (QK(i+1) may overwrite it)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_S_FREE));
            if (i > 0) {
                // P^T is single-buffered and O^T must be stable: wait for PV(i-1).  QK(i+1) is
                // queued on the tensor core ahead of PV(i), so the work below stays hidden.
                mbar_wait(bar(B_PV_DONE), (i - 1) & 1, abort_flag, p.err);
                tc_fence_after();
                if (any) {
#pragma unroll 1
                    for (int cc = 0; cc < 8; ++cc) {   // 16 columns at a time
                        const int jh = 16 * (cc & 1);
                        const uint32_t col = tmem + kTO + 64 * (cc >> 1) + 32 * hh + jh + lane_base;
                        uint32_t o[16];
                        tmem_ld16(col, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha_h[jh + j]);
                        tmem_st16(col, o);
                    }
                    tmem_wait_st();
                }
            }
            if (any) probs32(sv, qs_h, M_h, lim_h, tok_ok, per_row_lim, pos, l, pk);
            // P^T row t, 16-byte chunks 4hh .. 4hh+3 (rows 32hh .. 32hh+31), 128-byte swizzled
            uint8_t* prow = smem + SM_PT + t * 128;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                *reinterpret_cast<uint4*>(prow + (((4 * hh + k) ^ (t & 7)) << 4)) =
                    make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_P_FULL));
            if (next_tile && !early) {
                mbar_wait(bar(B_FULL + (i + 1) % kSlots), ((i + 1) / kSlots) & 1, abort_flag, p.err);
                scales_to_tmem_narrow(smem + SM_STAGE + ((i + 1) % kSlots) * kSlotBytes + kCodeBytes,
                               tmem + kTSFA + 32 * ((i + 1) & 1) + lane_base, lane);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_SFA_FULL + ((i + 1) & 1)));
            }
        }

        // ---- epilogue
        if (n_tiles > 0) {
            mbar_wait(bar(B_PV_DONE), (n_tiles - 1) & 1, abort_flag, p.err);
            tc_fence_after();
        }
        red[sp * 64 + 32 * hh + lane] = warp_reduce_scatter32<true>(l, lane);
        named_bar_sync(1, kSoftmaxThreads);
        const bool final_out = p.splits == 1;
        if (threadIdx.x < 64) {
            const int n = threadIdx.x;
            const float ls = red[n] + red[64 + n] + red[128 + n] + red[192 + n];
            lsum[n] = ls;
            alpha[n] = (n_tiles > 0 && ls > 0.0f) ? p.bmm2_scale / ls : 0.0f;
            // log-sum-exp of the row's scores: sum_t 2^(x_t) = 2^m l, x in log2 units
            if (final_out && p.lse && n < rows_here)
                p.lse[static_cast<int64_t>(b) * p.q_len * p.num_heads + g * kNQ + n] =
                    (n_tiles > 0 && ls > 0.0f) ? 0.69314718055994531f * (Mrow[n] + log2f(ls)) : -INFINITY;
        }
        named_bar_sync(1, kSoftmaxThreads);
        if (final_out) {
            // O^T -> row-major bf16 staging at offset 0 (the ring and Q regions are idle
            // now), then one bulk copy per output row (the output has caller strides):
            // warp (sp, hh) moves rows 32hh .. +32 of dims 128 jb + 32 sp + lane.
#pragma unroll 1
            for (int jb = 0; jb < 4; ++jb) {
                uint32_t o[32];
                if (n_tiles > 0) {
                    tmem_ld32(tmem + kTO + 64 * jb + 32 * hh + lane_base, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int k = 0; k < 32; ++k) o[k] = 0u;
                }
                const int d = 128 * jb + t;
                __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem);
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    const int n = 32 * hh + k;
                    stg[n * kLatent + d] = __float2bfloat16_rn(__uint_as_float(o[k]) * alpha[n]);
                }
            }
            fence_proxy_async_smem();
            named_bar_sync(1, kSoftmaxThreads);
            const int n = threadIdx.x;
            if (n < rows_here) {
                bulk_copy_s2g(p.out + rowoff[n], sbase + n * kLatent * 2, kLatent * 2);
                bulk_commit_group();
                bulk_wait_group_read0();
            }
        } else {
            // split partial: unnormalised O rows straight from TMEM to global memory (for one
            // row k a warp writes 32 consecutive floats), then (max, sum) per row.  A split
            // that saw no token writes no O values: its sums are 0 and the combine skips it.
            const int64_t unit = (static_cast<int64_t>(s) * p.batch + b) * p.groups + g;
            float* po = p.part_o + unit * kNQ * kLatent;
            if (n_tiles > 0) {
#pragma unroll 1
                for (int jb = 0; jb < 4; ++jb) {
                    uint32_t o[32];
                    tmem_ld32(tmem + kTO + 64 * jb + 32 * hh + lane_base, o);
                    tmem_wait_ld();
                    const int d = 128 * jb + t;
#pragma unroll
                    for (int k = 0; k < 32; ++k)
                        if (32 * hh + k < rows_here) __stcg(po + (32 * hh + k) * kLatent + d, __uint_as_float(o[k]));
                }
            }
            const int n = threadIdx.x;
            if (n < kNQ) {
                const bool live = n < rows_here && n_tiles > 0;
                __stcg(reinterpret_cast<float2*>(p.part_ml + (unit * kNQ + n) * 2),
                       live ? make_float2(Mrow[n], lsum[n]) : make_float2(-INFINITY, 0.0f));
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

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// L2 promotion: dense boxes are whole pages, so 256-byte fills cost nothing; sparse boxes are
// single random 288-byte rows, where 256-byte fills read about 512 bytes per row from DRAM
// (measured: 16.0 MB for 9.4 MB of rows), so those maps promote nothing.
int make_pool_map(CUtensorMap* m, const uint8_t* pool, int64_t pool_rows, uint32_t box_x, uint32_t box_y,
                  CUtensorMapSwizzle swz, CUtensorMapL2promotion promo) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(NVFP4KV_ECUDA, "mla_decode: cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kRowBytes), static_cast<cuuint64_t>(pool_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kRowBytes)};
    const cuuint32_t box[2] = {box_x, box_y};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(pool), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, promo,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NVFP4KV_ECUDA, "mla_decode: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return NVFP4KV_OK;
}

template <bool kSparse, int kRing, int kVBuf, bool kRope>
int ensure_fp4_smem_attr() {
    static int done[64] = {0};
    constexpr int bytes = DecCfg<kRing, kVBuf>::kSmemBytes;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaGetDevice failed");
    if (dev >= 0 && dev < 64 && done[dev]) return NVFP4KV_OK;
    const cudaError_t e = cudaFuncSetAttribute(decode_fp4_kernel<kSparse, kRing, kVBuf, kRope>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess)
        return fail(NVFP4KV_ECUDA, "cudaFuncSetAttribute(max dynamic smem %d): %s", bytes, cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) done[dev] = 1;
    return NVFP4KV_OK;
}

// The attention launch for one kernel shape (a programmatic dependent of the Q preparation:
// its set-up overlaps that kernel's tail).
template <bool kSparse, int kRing, int kVBuf, bool kRope>
int launch_attention(const Fp4Params& p, const CUtensorMap& tm_codes, const CUtensorMap& tm_scales, dim3 grid,
                     cudaStream_t st) {
    int rc;
    if ((rc = ensure_fp4_smem_attr<kSparse, kRing, kVBuf, kRope>()) != NVFP4KV_OK) return rc;
    const cudaError_t le = launch_dependent(decode_fp4_kernel<kSparse, kRing, kVBuf, kRope>, grid, dim3(kThreads),
                                            DecCfg<kRing, kVBuf>::kSmemBytes, st, p, tm_codes, tm_scales);
    if (le != cudaSuccess)
        return fail(NVFP4KV_ECUDA, "nvfp4kv_mla_decode: attention launch failed: %s", cudaGetErrorString(le));
    return check_launch(kSparse ? "nvfp4kv_mla_decode (fp4 sparse)" : "nvfp4kv_mla_decode (fp4 dense)");
}

// Ring shape of a call: splits of at most two tiles never load a third ring slot, so its
// space goes to two more V-chunk buffers.
bool short_ring(const DecodePlan& pl) {
    const int longest = (pl.tiles_total + pl.splits - 1) / pl.splits;
    return longest <= 2;
}

}  // namespace

int launch_decode_fp4(const DecodeArgs& a, const DecodePlan& pl, cudaStream_t st) {
    const bool sparse = a.sparse_topk > 0;
    if (!sparse && a.page_size < 16)
        return fail(NVFP4KV_EINVAL, "mla_decode: page_size must be >= 16 (got %d)", a.page_size);
    if (!a.qimg || reinterpret_cast<uintptr_t>(a.qimg) % 16)
        return fail(NVFP4KV_EWORKSPACE, "mla_decode: no 16-byte aligned workspace for the prepared Q");
    if (a.pool_rows > 0x7FFFFFFFll)
        return fail(NVFP4KV_EINVAL, "mla_decode: pool_rows %lld beyond 2^31 - 1", static_cast<long long>(a.pool_rows));
    // dense: boxes of up to a page of rows; sparse: one-row boxes for the row gathers
    const int box_rows = sparse ? 1 : (a.page_size < kTile ? a.page_size : kTile);
    CUtensorMap tm_codes{}, tm_scales{};
    int rc;
    const CUtensorMapL2promotion promo = sparse ? CU_TENSOR_MAP_L2_PROMOTION_NONE : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
    if ((rc = make_pool_map(&tm_codes, a.pool, a.pool_rows, 128, box_rows, CU_TENSOR_MAP_SWIZZLE_128B, promo)) !=
        NVFP4KV_OK)
        return rc;
    if ((rc = make_pool_map(&tm_scales, a.pool, a.pool_rows, 32, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE, promo)) !=
        NVFP4KV_OK)
        return rc;
    QPrepParams qp{};
    qp.q = static_cast<const __nv_bfloat16*>(a.q);
    qp.q_sb = a.q_sb; qp.q_sq = a.q_sq; qp.q_sh = a.q_sh;
    qp.q_len = a.q_len; qp.num_heads = a.num_heads; qp.groups = pl.groups;
    qp.scale_log2 = a.bmm1_scale * 1.4426950408889634f;
    qp.qimg = a.qimg;
    qp.rope_q = a.rope_q;
    q_prep_kernel<<<a.batch * pl.groups * 8, 256, 0, st>>>(qp);
    if ((rc = check_launch("nvfp4kv_mla_decode (Q preparation)")) != NVFP4KV_OK) return rc;
    if (a.rope_pool) {   // rope scores, after the Q preparation and before the attention
        RopeParams rp{};
        rp.rope_pool = a.rope_pool;
        rp.pool_rows = a.pool_rows;
        rp.num_pages = sparse ? 0 : a.pool_rows / a.page_size;
        rp.tables = a.tables; rp.tables_stride = a.tables_stride; rp.seq_lens = a.seq_lens;
        rp.groups = pl.groups; rp.page_shift = sparse ? 0 : a.page_shift;
        rp.max_seq_len = sparse ? a.sparse_topk : a.max_seq_len;
        rp.tiles_total = pl.tiles_total;
        rp.rope_q = a.rope_q; rp.logits = a.rope_logits;
        rp.ld = static_cast<int64_t>(pl.tiles_total) * kTile;
        const dim3 rg(static_cast<unsigned>(static_cast<int64_t>(a.batch) * pl.groups * pl.tiles_total));
        if (sparse) rope_logits_kernel<true><<<rg, 256, 0, st>>>(rp);
        else rope_logits_kernel<false><<<rg, 256, 0, st>>>(rp);
        if ((rc = check_launch("nvfp4kv_mla_decode_rope (rope scores)")) != NVFP4KV_OK) return rc;
    }
    Fp4Params p{};
    p.pool = a.pool; p.pool_rows = a.pool_rows;
    p.tables = a.tables; p.tables_stride = a.tables_stride;
    p.seq_lens = a.seq_lens;
    p.batch = a.batch; p.q_len = a.q_len; p.num_heads = a.num_heads;
    p.groups = pl.groups; p.splits = pl.splits;
    p.page_shift = sparse ? 0 : a.page_shift; p.box_rows = box_rows;
    p.num_pages = sparse ? 0 : a.pool_rows / a.page_size;
    p.max_seq_len = sparse ? a.sparse_topk : a.max_seq_len;   // seq_lens beyond it are clamped
    p.tiles_total = pl.tiles_total;
    p.bmm2_scale = a.bmm2_scale;
    p.out = static_cast<__nv_bfloat16*>(a.out);
    p.o_sb = a.o_sb; p.o_sq = a.o_sq; p.o_sh = a.o_sh;
    p.part_o = a.part_o; p.part_ml = a.part_ml;
    p.qimg = a.qimg;
    p.lse = a.lse;
    p.err = a.err;
    p.rope_logits = a.rope_logits;
    p.rope_ld = static_cast<int64_t>(pl.tiles_total) * kTile;
    const dim3 grid(static_cast<unsigned>(a.batch * pl.groups * pl.splits));
    cudaEvent_t ev0, ev1;
    take_kernel_events(&ev0, &ev1);
    if (ev0 && cudaEventRecord(ev0, st) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaEventRecord failed");
    const bool shrt = short_ring(pl);
    if (a.rope_pool) {
        rc = sparse ? (shrt ? launch_attention<true, 2, 4, true>(p, tm_codes, tm_scales, grid, st)
                            : launch_attention<true, 3, 2, true>(p, tm_codes, tm_scales, grid, st))
                    : (shrt ? launch_attention<false, 2, 4, true>(p, tm_codes, tm_scales, grid, st)
                            : launch_attention<false, 3, 2, true>(p, tm_codes, tm_scales, grid, st));
    } else {
        rc = sparse ? (shrt ? launch_attention<true, 2, 4, false>(p, tm_codes, tm_scales, grid, st)
                            : launch_attention<true, 3, 2, false>(p, tm_codes, tm_scales, grid, st))
                    : (shrt ? launch_attention<false, 2, 4, false>(p, tm_codes, tm_scales, grid, st)
                            : launch_attention<false, 3, 2, false>(p, tm_codes, tm_scales, grid, st));
    }
    if (rc != NVFP4KV_OK) return rc;
    if (ev1 && cudaEventRecord(ev1, st) != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaEventRecord failed");
    return NVFP4KV_OK;
}

}  // namespace nvfp4kv
