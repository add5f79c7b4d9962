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
//   index_score_kernel  one block per (query, run of its 128-position tiles), one wave over the
//                       SMs: whole pages of key rows bulk-copied into a ring, each tile of 128
//                       keys the NVFP4 A operand of tcgen05 block-scaled fp4 MMAs (its e4m3
//                       scales as the A scale factors) against q written as four NVFP4 terms
//                       (after an exact power-of-two scale per head, folded into the head's
//                       weight), fp32 accumulators in TMEM, then the ReLU-weighted head sum per
//                       position from the accumulators.
//   index_topk_kernel   one thread-block cluster of 8 CTAs per query, each CTA an eighth of
//                       the positions: an 8-pass 4-bit radix select of the k-th largest score
//                       (digit counts exchanged through distributed shared memory), then the
//                       selected positions written in ascending order (ties at the threshold
//                       go to the lowest positions), mapped to pool rows.
#include <algorithm>

#include "abi_common.h"
#include "common.cuh"

namespace nvfp4kv {
namespace {

constexpr int kITile = 128;                         // positions per score block
constexpr int kIHeads = 64;                         // indexer heads
constexpr int kIDim = NVFP4KV_INDEX_DIM;            // 128
constexpr int kIRow = NVFP4KV_INDEX_ROW_BYTES;      // 72

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
    int runs;                     // blocks per entry
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

// ------------------------------------------------------------------ scores (tcgen05)
// A 72-byte key row already is NVFP4 (64 code bytes, one e4m3 scale per 16 dims), so a tile of
// 128 keys is the A operand of tcgen05.mma kind::mxf4nvf4.block_scale.block16 with its scales
// as the A scale factors, and q is written as four NVFP4 terms on the N side, as the attention
// kernel does for its queries: column h of the accumulator holds terms 1 + 3 of head h, column
// 64 + h terms 2 + 4 (two passes of N = 128).  Each head is first scaled by 2^-e_h (exact, so
// that its largest |q| lies in [2^10, 2^11)); 2^e_h goes into the head's weight, since
// max(c x, 0) = c max(x, 0) for c > 0.
//
// Every stage works on tiles of 128 keys, and each hand-off between stages costs about a memory
// latency, so the stages run as several copies over interleaved tiles: warps 0, 2 and 3 load
// (tile j from loader j mod 3: page runs of the pool bulk-copied into a ring of raw tiles, the run's
// page ids staged in shared memory a window at a time, so no copy waits on a table load);
// warp 1 issues the MMAs; warps 4-7 rewrite each raw tile into the 128-byte swizzled operand
// layout and its scales into TMEM (warp w: sub-partition w & 3), three operand buffers; warps
// 8-19, three sets of four, read a finished tile's 128 accumulator columns (thread = key
// position) and write the ReLU-weighted head sum, set e taking the tiles j = e mod 3 in
// accumulator e.  Warps 4-7 quantise q at the start.  Warp 2 also owns the TMEM allocation.
// Every wait is bounded (common.cuh).
//
// Every slot of every ring is waited on by one warp (or one set of warps) only, in phase order:
// a parity wait cannot tell phase u - 1 from phase u + 1, so a second consumer of a slot that
// reached its wait one phase early would pass at once.  Hence the ring depths: the 9 key
// stages split over 3 loaders (stage s always loader s mod 3), 3 operand buffers and 3
// accumulators each served by the one converter set, the one MMA warp and epilogue set e.
constexpr int kSStages = 9;                                  // raw key tiles in flight
constexpr int kSDepth = 3;                                   // operand buffers, accumulators, epilogue sets
constexpr int kSLoaders = 3;                                 // warps 0, 2, 3
static_assert(kSStages % kSLoaders == 0, "a stage is always refilled by the same loader");
constexpr int kKeyTileBytes = kITile * kIRow;                // 9216
constexpr int kSThreads = 640;                               // 20 warps
constexpr int kSMmaWarp = 1, kSAllocWarp = 2, kSConvWarp0 = 4, kSEpiWarp0 = 8;
constexpr int kSPrepBar = 1;                                 // named barrier of warps 4-19
constexpr int kSLoadBar = 2;                                 // named barrier of the loaders
constexpr int kPgWin = 512;                                  // page ids a loader stages at a time
// Registers moved between warpgroups at run time (setmaxnreg).  The block is launched with
// kSLaunchRegs a thread (ptxas's figure for 640 threads, one block per SM).
constexpr uint32_t kSLaunchRegs = 96;
constexpr uint32_t kSRegsCtl = 80, kSRegsConv = 72, kSRegsEpi = 96;
static_assert(128 * (kSRegsCtl + kSRegsConv + kSDepth * kSRegsEpi) <= kSThreads * kSLaunchRegs,
              "register split within the launch");
constexpr int SS_QB = 0;                                     // Q terms: 2 passes x [128 rows x 128 B], 64 B used
constexpr int SS_A = SS_QB + 2 * 16384;                      // kSDepth x key codes [128 rows x 128 B], 64 B used
constexpr int SS_STG = SS_A + kSDepth * 16384;               // kSStages x [128 rows x 72 B] as copied
constexpr int SS_QSF = SS_STG + kSStages * kKeyTileBytes;    // [2 passes][128 rows][8] Q-term scales
constexpr int SS_WQ = SS_QSF + 2 * 128 * 8;                  // 64 f32: w[h] 2^e_h
constexpr int SS_PG = SS_WQ + 256;                           // kSLoaders x kPgWin i32: each loader's page ids
constexpr int SS_LAST = SS_PG + kSLoaders * kPgWin * 4;      // kSLoaders i32: each loader's last tile
constexpr int SS_FLAGS = SS_LAST + 16;                       // [0] TMEM base, [1] abort
constexpr int SS_BARS = SS_FLAGS + 16;
constexpr int SB_FULL = 0;                                   // [stages] raw tile landed
constexpr int SB_FREE = SB_FULL + kSStages;                  // [stages] converters done with it
constexpr int SB_AFULL = SB_FREE + kSStages;                 // [depth] operand tile + its scales ready
constexpr int SB_AFREE = SB_AFULL + kSDepth;                 // [depth] MMAs done reading them
constexpr int SB_DFULL = SB_AFREE + kSDepth;                 // [depth] accumulator complete
constexpr int SB_DFREE = SB_DFULL + kSDepth;                 // [depth] accumulator read
constexpr int SB_DRAIN = SB_DFREE + kSDepth;                 // every MMA complete (before TMEM is freed)
constexpr int SB_QREADY = SB_DRAIN + 1;                      // Q-term scales in TMEM (every sub-partition)
constexpr int kSBars = SB_QREADY + 1;
constexpr int kScoreSmem = SS_BARS + kSBars * 8 + 1024;      // slack to align the base
static_assert(kScoreSmem <= 232448, "shared memory budget");
constexpr uint32_t kSTD = 0;        // kSDepth x 128 columns: accumulators
constexpr uint32_t kSTSFA = 384;    // kSDepth x 8 columns: key scales (column 4 kk + q: word kk of row 32 q + lane)
constexpr uint32_t kSTSFB = 416;    // 16 columns: Q-term scales (8 pass + 4 kk + q)
constexpr uint32_t kSTCols = 512;
static_assert(kIDim == 2 * 64 && kIRow == kIDim / 2 + kIDim / 16, "a key row: two K-chunks of 64 codes, then their scales");

// Packed pairs of fp32 (sm_100 f32x2 arithmetic: one instruction for two lanes of work).
__device__ __forceinline__ uint64_t pack_f32x2(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, uint32_t& lo, uint32_t& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// Four floats from shared memory, issued where written (not hoisted out of a loop).
__device__ __forceinline__ float4 lds_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// q of entry b -> four NVFP4 terms in the B-operand image (term tt: pass tt >> 1, row
// 64 (tt & 1) + h, K-major, 128-byte swizzle), their scales [pass][row][8], and w[h] 2^e_h.
// The four converter warps (wi = 0..3), eight lanes per head (lane j: dims 16 j .. 16 j + 15),
// four heads per warp and round.
__device__ __forceinline__ void index_q_prep(const ScoreParams& p, int b, uint8_t* smem, int wi, int lane) {
    const int j = lane & 7;
#pragma unroll 1
    for (int it = 0; it < 4; ++it) {
        const int h = 16 * it + 4 * wi + (lane >> 3);
        const __nv_bfloat16* src = p.q + b * p.q_sb + h * p.q_sh + 16 * j;
        const uint4 u0 = ldg_nc_v4(src), u1 = ldg_nc_v4(src + 8);
        const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        float x[16];
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            x[2 * k] = __uint_as_float(w8[k] << 16);
            x[2 * k + 1] = __uint_as_float(w8[k] & 0xFFFF0000u);
            amax = fmaxf(amax, fmaxf(fabsf(x[2 * k]), fabsf(x[2 * k + 1])));
        }
#pragma unroll
        for (int off = 4; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
        const int eb = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu);
        int e = (eb > 0 && eb < 255) ? eb - 127 - 10 : 0;
        e = max(-100, min(100, e));
        const float mul = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);   // 2^-e, exact
#pragma unroll
        for (int k = 0; k < 16; ++k) x[k] *= mul;
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
            float am = 0.0f;
#pragma unroll
            for (int k = 0; k < 16; ++k) am = fmaxf(am, fabsf(x[k]));
            const uint8_t sb = am > 0.0f ? f32_to_e4m3(am * (1.0f / 6.0f)) : static_cast<uint8_t>(0);
            const float sf = e4m3_to_f32(sb);
            const float inv = sf > 0.0f ? rcp_approx(sf) : 0.0f;
            uint32_t wlo = 0, whi = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t byte = f32x2_to_e2m1x2(x[2 * k] * inv, x[2 * k + 1] * inv);
                if (k < 4) wlo |= byte << (8 * k);
                else whi |= byte << (8 * (k - 4));
                const uint32_t dq = e2m1x2_to_f16x2(byte);
                x[2 * k] -= __half2float(__ushort_as_half(static_cast<unsigned short>(dq & 0xFFFFu))) * sf;
                x[2 * k + 1] -= __half2float(__ushort_as_half(static_cast<unsigned short>(dq >> 16))) * sf;
            }
            const int ps = tt >> 1, R = 64 * (tt & 1) + h, c = j >> 1;
            *reinterpret_cast<uint2*>(smem + SS_QB + ps * 16384 + (R >> 3) * 1024 + (R & 7) * 128 +
                                      ((c ^ (R & 7)) << 4) + 8 * (j & 1)) = make_uint2(wlo, whi);
            smem[SS_QSF + (ps * 128 + R) * 8 + j] = sb;
        }
        if (j == 0)
            reinterpret_cast<float*>(smem + SS_WQ)[h] = __ldg(p.w + b * p.w_sb + h) * ldexpf(1.0f, e);
    }
}

// Block = (entry b, run r of its tiles): the tiles of visible positions are cut into p.runs
// equal runs, so a batch of B entries fills about B x runs SMs in one wave.
__global__ void __launch_bounds__(kSThreads, 1) index_score_kernel(const ScoreParams p, int32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const int b = blockIdx.x / p.runs, run = blockIdx.x % p.runs;
    const int L = clamp_len(p.seq_lens, b, p.max_seq_len, err);
    const int tiles_b = (L + kITile - 1) / kITile;
    const int per = (tiles_b + p.runs - 1) / p.runs;
    const int t0 = run * per, t1 = min(t0 + per, tiles_b);
    if (t0 >= t1) return;                            // the whole block: nothing visible here
    const int n = t1 - t0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* flags = reinterpret_cast<volatile int*>(smem + SS_FLAGS);
    volatile int* abort_flag = flags + 1;
    auto bar = [&](int i) -> uint32_t { return sbase + SS_BARS + 8 * i; };
    if (tid == 0) {
        for (int s = 0; s < kSStages; ++s) {
            mbar_init(bar(SB_FULL + s), 1);
            mbar_init(bar(SB_FREE + s), 4);
        }
        for (int a = 0; a < kSDepth; ++a) {
            mbar_init(bar(SB_AFULL + a), 4);
            mbar_init(bar(SB_AFREE + a), 1);
            mbar_init(bar(SB_DFULL + a), 1);
            mbar_init(bar(SB_DFREE + a), 4);
        }
        mbar_init(bar(SB_DRAIN), 1);
        mbar_init(bar(SB_QREADY), 4);
        flags[1] = 0;
        mbar_fence_init();
    }
    if (warp == kSAllocWarp) {
        tmem_alloc(sbase + SS_FLAGS, kSTCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = static_cast<uint32_t>(flags[0]);

    // each role's code follows its own register budget change (setmaxnreg), so the compiler
    // allocates every role within its budget
    if (warp < kSConvWarp0) {
    warpgroup_reg_dealloc<kSRegsCtl>();
    if (warp != kSMmaWarp) {
        // ============================================================ loads
        // loader li takes tiles j = li mod kSLoaders.  A tile is 128 / page runs of one page each
        // (pages of <= 128 positions) or 128 rows of one page; runs of pages that are missing
        // or lie wholly past the visible end are not copied (their positions score -inf or are
        // not written).  A bulk copy that overwrites a stage the converters only read needs no
        // proxy fence: their reads are ordered before it by the stage's barrier.
        const int li = warp == 0 ? 0 : warp - 1;
        const int run_rows = p.page_shift >= 7 ? kITile : (1 << p.page_shift);
        const int runs_per_tile = kITile / run_rows;
        const uint32_t run_bytes = static_cast<uint32_t>(run_rows * kIRow);
        int* pgw = reinterpret_cast<int*>(smem + SS_PG) + li * kPgWin;   // pages wbase .. wbase + kPgWin - 1
        const int last_page = (min(t1 * kITile, L) - 1) >> p.page_shift;
        int wbase = -2 * kPgWin;
        int last = -1;                               // the last tile this loader issued
#pragma unroll 1
        for (int j = li; j < n; j += kSLoaders) {
            const int s = j % kSStages;
            if (j >= kSStages) {
                const bool ok = mbar_wait(bar(SB_FREE + s), ((j / kSStages) - 1) & 1, abort_flag, err);
                if (!ok || *abort_flag) break;
            }
            const int pos0 = (t0 + j) * kITile;
            const int pfirst = pos0 >> p.page_shift, plast = (min(pos0 + kITile, L) - 1) >> p.page_shift;
            if (pfirst < wbase || plast >= wbase + kPgWin) {   // the tile's pages: one window (<= 64 pages)
                __syncwarp();
                wbase = pfirst;
                const int cnt = min(kPgWin, last_page - wbase + 1);
                for (int k = lane; k < cnt; k += 32) pgw[k] = __ldg(p.tables + b * p.tables_stride + wbase + k);
                __syncwarp();
            }
            // runs r = lane, lane + 32 (at most 64 a tile): page id, or -1 (not copied)
            int pg[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = lane + 32 * h, pos = pos0 + r * run_rows;
                pg[h] = -1;
                if (r < runs_per_tile && pos < L) {
                    const int v = pgw[(pos >> p.page_shift) - wbase];
                    pg[h] = (v < 0 || v >= p.num_pages) ? -1 : v;
                }
            }
            const uint32_t nrun = __popc(__ballot_sync(0xFFFFFFFFu, pg[0] >= 0)) +
                                  __popc(__ballot_sync(0xFFFFFFFFu, pg[1] >= 0));
            if (lane == 0) mbar_arrive_expect_tx(bar(SB_FULL + s), nrun * run_bytes);
            __syncwarp();
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (pg[h] >= 0) {
                    const int r = lane + 32 * h, pos = pos0 + r * run_rows;
                    const int64_t row = (static_cast<int64_t>(pg[h]) << p.page_shift) | (pos & ((1 << p.page_shift) - 1));
                    bulk_copy_g2s(sbase + SS_STG + s * kKeyTileBytes + r * run_bytes, p.pool + row * kIRow, run_bytes,
                                  bar(SB_FULL + s));
                }
            last = j;
        }
        // Copies in flight land before the CTA can exit.  Only a stage's last issued tile can
        // still be in flight (a stage is re-armed after its tile was consumed), and only its
        // phase is certain not to have been passed by a later tile of another loader, so once
        // every loader has stopped, lane s of loader 0 waits for stage s's last tile.
        if (lane == 0) reinterpret_cast<volatile int*>(smem + SS_LAST)[li] = last;
        named_bar_sync(kSLoadBar, kSLoaders * 32);
        if (li == 0 && lane < kSStages) {
            int t = -1;
#pragma unroll 1
            for (int l = 0; l < kSLoaders; ++l) {   // loader l's last tile on stage `lane`
                const int lj = reinterpret_cast<volatile int*>(smem + SS_LAST)[l];
#pragma unroll 1
                for (int j = lj; j >= 0 && j > lj - kSLoaders * kSStages; j -= kSLoaders)
                    if (j % kSStages == lane) {
                        t = max(t, j);
                        break;
                    }
            }
            if (t >= 0) mbar_drain_wait(bar(SB_FULL + lane), (t / kSStages) & 1);
        }
        __syncwarp();
    } else if (warp == kSMmaWarp) {
        // ============================================================ MMA issue
        constexpr uint32_t idq = idesc_fp4_f32(kITile, 128);
        const uint64_t dq = smem_desc_sw128(sbase + SS_QB, 16, 1024);
        const uint64_t da = smem_desc_sw128(sbase + SS_A, 16, 1024);
        // the Q-term scales in TMEM, written by the converter warps before their first tile
        const bool qready = mbar_wait(bar(SB_QREADY), 0, abort_flag, err);
        tc_fence_after();
#pragma unroll 1
        for (int j = 0; qready && j < n; ++j) {
            const int a = j % kSDepth, u = j / kSDepth;
            if (!mbar_wait(bar(SB_AFULL + a), u & 1, abort_flag, err)) break;
            if (u > 0 && !mbar_wait(bar(SB_DFREE + a), (u - 1) & 1, abort_flag, err)) break;
            tc_fence_after();
            if (elect_one()) {
#pragma unroll
                for (int ps = 0; ps < 2; ++ps)
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk)
                        tc_mma_fp4(tmem + kSTD + 128 * a, da + ((a * 16384 + kk * 32) >> 4),
                                   dq + ((ps * 16384 + kk * 32) >> 4), idq, (ps | kk) != 0,
                                   tmem + kSTSFA + 8 * a + 4 * kk, tmem + kSTSFB + 8 * ps + 4 * kk);
                tc_commit(bar(SB_AFREE + a));
                tc_commit(bar(SB_DFULL + a));
            }
            __syncwarp();
        }
        // every MMA of this CTA completes before its TMEM is freed, on the abort path too
        if (elect_one()) tc_commit(bar(SB_DRAIN));
        __syncwarp();
        mbar_drain_wait(bar(SB_DRAIN), 0);
    }
    } else if (warp < kSEpiWarp0) {
        warpgroup_reg_dealloc<kSRegsConv>();
        index_q_prep(p, b, smem, warp - kSConvWarp0, lane);
        fence_proxy_async_smem();                    // the Q terms are read by the tensor core
        named_bar_sync(kSPrepBar, (kSThreads / 32 - kSConvWarp0) * 32);
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        // ============================================================ operand tiles
        {   // Q-term scales into this sub-partition: column 8 ps + 4 kk + q = word kk of row 32 q + lane
            uint32_t v[16];
#pragma unroll
            for (int ps = 0; ps < 2; ++ps)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint2 w = *reinterpret_cast<const uint2*>(smem + SS_QSF + (ps * 128 + 32 * q + lane) * 8);
                    v[8 * ps + q] = w.x;
                    v[8 * ps + 4 + q] = w.y;
                }
            tmem_st16(tmem + lane_base + kSTSFB, v);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(SB_QREADY));
        }
        const int m = tid - kSConvWarp0 * 32;        // key row of the tile this thread rewrites
#pragma unroll 1
        for (int j = 0; j < n; ++j) {
            const int s = j % kSStages, a = j % kSDepth, u = j / kSDepth;
            if (!mbar_wait(bar(SB_FULL + s), (j / kSStages) & 1, abort_flag, err)) break;
            if (u > 0 && !mbar_wait(bar(SB_AFREE + a), (u - 1) & 1, abort_flag, err)) break;
            const uint8_t* stg = smem + SS_STG + s * kKeyTileBytes;
            const uint2* src = reinterpret_cast<const uint2*>(stg + m * kIRow);
            uint2 c[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) c[k] = src[k];
            uint8_t* arow = smem + SS_A + a * 16384 + (m >> 3) * 1024 + (m & 7) * 128;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
                *reinterpret_cast<uint4*>(arow + ((ch ^ (m & 7)) << 4)) =
                    make_uint4(c[2 * ch].x, c[2 * ch].y, c[2 * ch + 1].x, c[2 * ch + 1].y);
            // key scales of rows lane, 32 + lane, 64 + lane, 96 + lane into this sub-partition
            uint32_t sv[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint2 w = *reinterpret_cast<const uint2*>(stg + (32 * q + lane) * kIRow + 64);
                sv[q] = w.x;
                sv[4 + q] = w.y;
            }
            tmem_st4(tmem + lane_base + kSTSFA + 8 * a, sv[0], sv[1], sv[2], sv[3]);
            tmem_st4(tmem + lane_base + kSTSFA + 8 * a + 4, sv[4], sv[5], sv[6], sv[7]);
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(SB_FREE + s));
                mbar_arrive(bar(SB_AFULL + a));
            }
        }
    } else {
        warpgroup_reg_alloc<kSRegsEpi>();
        named_bar_sync(kSPrepBar, (kSThreads / 32 - kSConvWarp0) * 32);
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        // ============================================================ weighted head sums
        const uint32_t wq = sbase + SS_WQ;          // read every tile (kept in registers, they spill)
        float* out = p.scores + static_cast<int64_t>(b) * p.tiles * kITile;
        const int a = (warp - kSEpiWarp0) >> 2;      // this set's accumulator: tiles j = a mod kSDepth
        const int my = 32 * (warp & 3) + lane;
        // the table entry of this thread's position in tile jj (-1 past the visible end),
        // loaded a tile of this set ahead and tested only where it is used, so the load's
        // latency is hidden behind a whole tile
        auto page_of = [&](int jj) -> int {
            const int pos = (t0 + jj) * kITile + my;
            return (jj < n && pos < L) ? __ldg(p.tables + b * p.tables_stride + (pos >> p.page_shift)) : -1;
        };
        int pg_cur = page_of(a);
#pragma unroll 1
        for (int j = a; j < n; j += kSDepth) {
            const int pg_next = page_of(j + kSDepth);
            if (!mbar_wait(bar(SB_DFULL + a), (j / kSDepth) & 1, abort_flag, err)) break;
            tc_fence_after();
            // heads 16 r .. 16 r + 15 in round r: columns 16 r + h (terms 1 + 3) and 64 + 16 r + h
            // (terms 2 + 4); round r + 1's loads are issued before round r is summed
            const uint32_t dcol = tmem + lane_base + kSTD + 128 * a;
            uint64_t acc2[2] = {0ull, 0ull};   // two f32x2 accumulators
            uint32_t lo0[16], hi0[16], lo1[16], hi1[16];
            auto sum16 = [&](const uint32_t (&lo)[16], const uint32_t (&hi)[16], int r) {
#pragma unroll
                for (int h4 = 0; h4 < 4; ++h4) {
                    const float4 w4 = lds_f32x4(wq + 64 * r + 16 * h4);
#pragma unroll
                    for (int hp = 0; hp < 2; ++hp) {
                        const int h = 4 * h4 + 2 * hp;
                        uint64_t s2 = add_f32x2(pack_f32x2(lo[h], lo[h + 1]), pack_f32x2(hi[h], hi[h + 1]));
                        uint32_t s0, s1;
                        unpack_f32x2(s2, s0, s1);
                        s2 = pack_f32x2(__float_as_uint(fmaxf(__uint_as_float(s0), 0.0f)),
                                        __float_as_uint(fmaxf(__uint_as_float(s1), 0.0f)));
                        const uint64_t w2 = hp ? pack_f32x2(__float_as_uint(w4.z), __float_as_uint(w4.w))
                                               : pack_f32x2(__float_as_uint(w4.x), __float_as_uint(w4.y));
                        acc2[hp] = fma_f32x2(w2, s2, acc2[hp]);
                    }
                }
            };
            tmem_ld16(dcol, lo0);
            tmem_ld16(dcol + 64, hi0);
#pragma unroll 1
            for (int rp = 0; rp < 4; rp += 2) {
                tmem_wait_ld();
                tmem_ld16(dcol + 16 * (rp + 1), lo1);
                tmem_ld16(dcol + 64 + 16 * (rp + 1), hi1);
                sum16(lo0, hi0, rp);
                tmem_wait_ld();
                if (rp == 0) {
                    tmem_ld16(dcol + 32, lo0);
                    tmem_ld16(dcol + 96, hi0);
                }
                sum16(lo1, hi1, rp + 1);
            }
            uint32_t a0, a1, a2, a3;
            unpack_f32x2(acc2[0], a0, a1);
            unpack_f32x2(acc2[1], a2, a3);
            const float tot = (__uint_as_float(a0) + __uint_as_float(a2)) + (__uint_as_float(a1) + __uint_as_float(a3));
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(SB_DFREE + a));
            const int pos = (t0 + j) * kITile + my;
            if (pos < L) out[pos] = (pg_cur >= 0 && pg_cur < p.num_pages) ? tot : -INFINITY;
            pg_cur = pg_next;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kSAllocWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kSTCols);
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
    if (page_size < 2 || (page_size & (page_size - 1)) || page_size > 4096 || pool_rows % page_size)
        return fail(NVFP4KV_EINVAL, "index_topk: page_size must be a power of two in [2, 4096] dividing pool_rows");
    if (reinterpret_cast<uintptr_t>(q) % 16 || q_stride_b % 8 || q_stride_h % 8 ||
        reinterpret_cast<uintptr_t>(index_pool) % 16)
        return fail(NVFP4KV_EINVAL, "index_topk: q must be 16-byte aligned with strides multiples of 8, "
                                    "the index pool 16-byte aligned");
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
        // one wave: B entries x runs blocks on the SMs (one block per SM), at least one tile a run
        static int sm_count[64] = {0};
        int sms = dev >= 0 && dev < 64 ? sm_count[dev] : 0;
        if (sms <= 0) {
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
                return fail(NVFP4KV_ECUDA, "index_topk: SM count unavailable");
            if (dev >= 0 && dev < 64) sm_count[dev] = sms;
        }
        sp.runs = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, sms / batch)));
        index_score_kernel<<<static_cast<unsigned>(static_cast<int64_t>(batch) * sp.runs), kSThreads, kScoreSmem,
                             st>>>(sp, err_flag);
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
