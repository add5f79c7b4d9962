// Pool-row readers: the 656-byte fp8_ds_mla gather (byte-identical to the reference's
// _gather_kernel) and a bf16 dequantiser.  Both are HBM-bound; one warp handles one row,
// each lane one 16-element scale block (8 code bytes + 1 scale byte).
#include <atomic>

#include "abi_common.h"
#include "common.cuh"

namespace nvfp4kv {
namespace {

// e2m1 magnitude (3 bits) -> fp32 value {0, .5, 1, 1.5, 2, 3, 4, 6}, built from bits.
__device__ __forceinline__ float e2m1_mag(uint32_t mag) {
    const uint32_t e = mag >> 1, m = mag & 1u;
    const uint32_t bits = e == 0 ? (m ? 0x3F000000u : 0u) : (((126u + e) << 23) | (m << 22));
    return __uint_as_float(bits);
}

// Signed code value as the reference decodes it (glm53_nvfp4_runtime.py:101-104): the
// negative branch is Triton's unary minus, `0 - x`, so code 0x8 gives +0.0.
__device__ __forceinline__ float e2m1_value(uint32_t code) {
    const float mag = e2m1_mag(code & 7u);
    return (code & 8u) ? __fsub_rn(0.0f, mag) : mag;
}

// The 16 code values e2m1_value(c) in shared memory, filled by the block's first 16 threads
// (every thread of the block calls this before any of them returns).  Looking a code up costs a
// shared-memory load instead of the ~10 integer operations of building its value from bits,
// which bound these kernels by the ALU pipe.
__device__ __forceinline__ void fill_code_table(float* table) {
    if (threadIdx.x < 16) table[threadIdx.x] = e2m1_value(threadIdx.x);
    __syncthreads();
}

// Decode one lane's block: 8 code bytes (16 elements) times the block scale, in fp32; the
// product of the exact table value and the scale, as the reference computes it.
__device__ __forceinline__ void decode_block(uint2 codes, uint8_t scale_byte, const float* table,
                                             float (&v)[16]) {
    const float s = e4m3_to_f32(scale_byte);
    const uint32_t w[2] = {codes.x, codes.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
        v[2 * i] = __fmul_rn(table[byte & 15u], s);
        v[2 * i + 1] = __fmul_rn(table[byte >> 4], s);
    }
}

// a / b with the PTX instruction div.full.f32, which is what GPU Triton emits for an fp32 `/`
// (checked on the B200 against the reference's own compiled `amax / 448.0` and `1.0 / gscale`,
// every one of 500,882 quotients equal).  Used only in the Triton-division mode.
__device__ __forceinline__ float div_full(float a, float b) {
    float d;
    asm("div.full.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// runtime:87-122.  One warp: the 656-byte row at `dst` re-encodes pool row clamp(src, 0, R-1).
// kTritonDiv = false divides exactly (IEEE: the reference run on the CPU); true divides as the
// reference compiled by Triton for the GPU does (div.full.f32), byte for byte.
// `rope` (may be null): a rope side-pool of 64 bf16 per row (128 B), whose row src fills the
// 656-byte row's rope bytes [528, 656); null writes them as zeros, as the reference does.
template <bool kTritonDiv>
__device__ __forceinline__ void gather_row_ds656(const uint8_t* __restrict__ pool, int64_t R, int64_t src,
                                                 const float* table, uint8_t* __restrict__ dst, int lane,
                                                 const uint32_t* __restrict__ rope = nullptr) {
    src = src < 0 ? 0 : (src > R - 1 ? R - 1 : src);          // :98
    const uint8_t* row = pool + src * kRowBytes;
    const uint2 codes = ldg_nc_v2(row + 8 * lane);
    const uint8_t sb = row[256 + lane];
    float v[16];
    decode_block(codes, sb, table, v);                          // :99-108
    float amax = 0.0f;                                          // :109-112 (max includes 0.0)
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fmaxf(fabsf(v[2 * i]), fabsf(v[2 * i + 1])));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));  // 8 lanes = 128 elements
    const float gscale = fmaxf(kTritonDiv ? div_full(amax, 448.0f) : __fdiv_rn(amax, 448.0f), 1e-12f);  // :113
    const float inv = kTritonDiv ? div_full(1.0f, gscale) : __fdiv_rn(1.0f, gscale);                    // :115-116
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        // two values per conversion (round to nearest even, saturating; .x -> low byte)
        const uint32_t lo = __nv_cvt_float2_to_fp8x2(
            make_float2(__fmul_rn(v[4 * j], inv), __fmul_rn(v[4 * j + 1], inv)), __NV_SATFINITE, __NV_E4M3);
        const uint32_t hi = __nv_cvt_float2_to_fp8x2(
            make_float2(__fmul_rn(v[4 * j + 2], inv), __fmul_rn(v[4 * j + 3], inv)), __NV_SATFINITE, __NV_E4M3);
        o[j] = (lo & 0xFFFFu) | (hi << 16);
    }
    *reinterpret_cast<uint4*>(dst + 16 * lane) = make_uint4(o[0], o[1], o[2], o[3]);  // :117-120
    if ((lane & 7) == 0) *reinterpret_cast<float*>(dst + 512 + 4 * (lane >> 3)) = gscale;  // :114
    *reinterpret_cast<uint32_t*>(dst + 528 + 4 * lane) = rope ? __ldg(rope + src * 32 + lane) : 0u;  // :121-122
}

// Row r of `out` re-encodes pool row clamp(idx[r], 0, R-1).
template <bool kTritonDiv>
__global__ void __launch_bounds__(256)
gather_ds656_kernel(const uint8_t* __restrict__ pool, int64_t R, const int32_t* __restrict__ idx,
                    int64_t S, uint8_t* __restrict__ out, const uint32_t* __restrict__ rope) {
    __shared__ float table[16];
    fill_code_table(table);
    const int lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= S) return;
    gather_row_ds656<kTritonDiv>(pool, R, idx[r], table, out + r * kDsBytes, lane, rope);
}

// ------------------------------------------------------------------ sync-free dedup
// The distinct values of the block tables, ascending, as torch.unique sorts them
// (runtime:177-182): a mark per possible value (key 0 = -1, key r + 1 = pool row r), an
// exclusive scan of the marks giving each value its position, the inverse tables read off
// the scan, and the gather driven by the device-side count.  Fixed grids: no host sync.
constexpr int kScanBlock = 1024;
constexpr int kScanPerThread = 4;
constexpr int kScanTile = kScanBlock * kScanPerThread;   // marks per scan block

__device__ __forceinline__ int64_t dedup_key(int32_t e, int64_t R, int32_t* err) {
    if (e == -1) return 0;
    if (e < 0 || e >= R) {   // counted as -1; the reference would keep it as its own value
        set_error(err, NVFP4KV_DEVERR_BAD_INDEX);
        return 0;
    }
    return static_cast<int64_t>(e) + 1;
}

// Key 0 (every -1 entry, typically ~10 % of a step's table) is recorded once per block
// through a shared flag: stores to one word serialise in L2.
__global__ void __launch_bounds__(256)
dedup_mark_kernel(const int32_t* __restrict__ entries, int64_t n, int64_t R, int32_t* __restrict__ marks,
                  int32_t* __restrict__ err) {
    __shared__ int any_minus_one;
    if (threadIdx.x == 0) any_minus_one = 0;
    __syncthreads();
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j < n) {
        const int64_t key = dedup_key(entries[j], R, err);
        if (key == 0) any_minus_one = 1;
        else marks[key] = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0 && any_minus_one) marks[0] = 1;
}

// Block-wide exclusive scan of one value per thread; returns this thread's prefix and sets
// `total` (every thread) to the block's sum.
__device__ __forceinline__ int32_t block_exclusive_scan(int32_t v, int32_t& total) {
    __shared__ int32_t warp_sums[kScanBlock / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int32_t w = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        warp_sums[lane] = w;   // inclusive over warps
    }
    __syncthreads();
    total = warp_sums[kScanBlock / 32 - 1];
    const int32_t before = warp == 0 ? 0 : warp_sums[warp - 1];
    __syncthreads();           // warp_sums is reused by the next call
    return before + x - v;
}

__global__ void __launch_bounds__(kScanBlock)
dedup_block_sums_kernel(const int32_t* __restrict__ marks, int64_t M, int32_t* __restrict__ bsum) {
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + kScanPerThread * threadIdx.x;
    int32_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanPerThread; ++k)
        if (base + k < M) s += marks[base + k];
    int32_t total;
    block_exclusive_scan(s, total);
    if (threadIdx.x == 0) bsum[blockIdx.x] = total;
}

// One block: exclusive scan of the nb block sums in place, in chunks of kScanBlock with a
// running carry; the grand total is the number of distinct entries.
__global__ void __launch_bounds__(kScanBlock)
dedup_scan_sums_kernel(int32_t* __restrict__ bsum, int64_t nb, int32_t* __restrict__ n_unique) {
    int32_t carry = 0;
    for (int64_t c = 0; c < nb; c += kScanBlock) {
        const int64_t i = c + threadIdx.x;
        const int32_t v = i < nb ? bsum[i] : 0;
        int32_t total;
        const int32_t ex = block_exclusive_scan(v, total);
        if (i < nb) bsum[i] = carry + ex;
        carry += total;
    }
    if (threadIdx.x == 0) *n_unique = carry;
}

// Marks -> positions (in place), and the ascending list of distinct values.
__global__ void __launch_bounds__(kScanBlock)
dedup_offsets_kernel(int32_t* __restrict__ marks, int64_t M, const int32_t* __restrict__ bsum,
                     int32_t* __restrict__ uniq) {
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + kScanPerThread * threadIdx.x;
    int32_t m[kScanPerThread];
    int32_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanPerThread; ++k) {
        m[k] = base + k < M ? marks[base + k] : 0;
        s += m[k];
    }
    int32_t total;
    int32_t pos = bsum[blockIdx.x] + block_exclusive_scan(s, total);
#pragma unroll
    for (int k = 0; k < kScanPerThread; ++k) {
        if (base + k < M) {
            marks[base + k] = pos;
            if (m[k]) uniq[pos] = static_cast<int32_t>(base + k - 1);   // key 0 -> -1
        }
        pos += m[k];
    }
}

__global__ void __launch_bounds__(256)
dedup_tables_kernel(const int32_t* __restrict__ entries, int64_t n, int64_t R, const int32_t* __restrict__ pos,
                    int32_t* __restrict__ tables) {
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j < n) tables[j] = pos[dedup_key(entries[j], R, nullptr)];
}

// Warp u (grid-stride) writes scratch row u: the gathered row of distinct value u for
// u < n_unique, zeros up to the next multiple of 64 rows, within `cap` rows.
template <bool kTritonDiv>
__global__ void __launch_bounds__(256)
dedup_gather_kernel(const uint8_t* __restrict__ pool, int64_t R, const int32_t* __restrict__ uniq,
                    const int32_t* __restrict__ n_unique, uint8_t* __restrict__ scratch, int64_t cap,
                    int32_t* __restrict__ err) {
    __shared__ float table[16];
    fill_code_table(table);
    const int lane = threadIdx.x & 31;
    const int64_t nu = *n_unique;
    const int64_t padded = (nu + 63) / 64 * 64;
    const int64_t end = padded < cap ? padded : cap;
    if (blockIdx.x == 0 && threadIdx.x == 0 && nu > cap) set_error(err, NVFP4KV_DEVERR_CAPACITY);
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t u = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); u < end;
         u += warps) {
        uint8_t* dst = scratch + u * kDsBytes;
        if (u < nu) {
            gather_row_ds656<kTritonDiv>(pool, R, uniq[u], table, dst, lane);
        } else {
            reinterpret_cast<uint4*>(dst)[lane] = make_uint4(0u, 0u, 0u, 0u);   // 512 B
            if (lane < 9) reinterpret_cast<uint4*>(dst + 512)[lane] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
}

struct DedupLayout {
    int64_t M, nb, uniq_len, ints;   // marks [M], block sums [nb], uniq [uniq_len]
};
DedupLayout dedup_layout(int64_t pool_rows, int64_t n) {
    DedupLayout l{};
    l.M = pool_rows + 1;
    l.nb = (l.M + kScanTile - 1) / kScanTile;
    l.uniq_len = n < l.M ? n : l.M;
    l.ints = l.M + l.nb + l.uniq_len;
    return l;
}

template <int IDT>
__global__ void __launch_bounds__(256)
dequant_bf16_kernel(const uint8_t* __restrict__ pool, int64_t R, const void* __restrict__ rows,
                    int64_t n, __nv_bfloat16* __restrict__ out, int32_t* __restrict__ err) {
    __shared__ float table[16];
    fill_code_table(table);
    const int lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= n) return;
    int64_t src;
    if constexpr (IDT == NVFP4KV_INDEX_I64) src = static_cast<const int64_t*>(rows)[r];
    else src = static_cast<const int32_t*>(rows)[r];
    uint32_t packed[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (src >= 0 && src < R) {
        const uint8_t* row = pool + src * kRowBytes;
        float v[16];
        decode_block(ldg_nc_v2(row + 8 * lane), row[256 + lane], table, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);  // exact
            packed[i] = *reinterpret_cast<uint32_t*>(&h);
        }
    } else if (lane == 0 && src != -1) {
        set_error(err, NVFP4KV_DEVERR_BAD_INDEX);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + r * kLatent + 16 * lane);
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
}

// Division mode of the 656-byte row encoders (nvfp4kv_set_gather_division), process-wide.
std::atomic<int> g_gather_division{NVFP4KV_DIV_IEEE};

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_set_gather_division(int mode) {
    using namespace nvfp4kv;
    if (mode != NVFP4KV_DIV_IEEE && mode != NVFP4KV_DIV_TRITON)
        return fail(NVFP4KV_EINVAL, "set_gather_division: mode must be NVFP4KV_DIV_IEEE or NVFP4KV_DIV_TRITON (got %d)",
                    mode);
    g_gather_division.store(mode);
    return NVFP4KV_OK;
}

extern "C" int nvfp4kv_get_gather_division(void) { return nvfp4kv::g_gather_division.load(); }

namespace nvfp4kv {
namespace {

int gather_ds656_impl(const char* name, const uint8_t* pool, const void* rope, int64_t pool_rows,
                      const int32_t* idx, int64_t num_rows, uint8_t* out, nvfp4kv_stream_t stream) {
    if (num_rows < 0) return fail(NVFP4KV_EINVAL, "%s: num_rows < 0", name);
    if (num_rows == 0) return NVFP4KV_OK;
    if (!pool || !idx || !out) return fail(NVFP4KV_EINVAL, "%s: null pointer", name);
    if (pool_rows <= 0) return fail(NVFP4KV_EINVAL, "%s: empty pool", name);
    if (reinterpret_cast<uintptr_t>(pool) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
        reinterpret_cast<uintptr_t>(rope) % 16)
        return fail(NVFP4KV_EINVAL, "%s: pool, rope pool and out must be 16-byte aligned", name);
    const int warps = 8;
    const dim3 grid(static_cast<unsigned>((num_rows + warps - 1) / warps));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint32_t* r = static_cast<const uint32_t*>(rope);
    if (g_gather_division.load() == NVFP4KV_DIV_TRITON)
        gather_ds656_kernel<true><<<grid, warps * 32, 0, st>>>(pool, pool_rows, idx, num_rows, out, r);
    else
        gather_ds656_kernel<false><<<grid, warps * 32, 0, st>>>(pool, pool_rows, idx, num_rows, out, r);
    return check_launch(name);
}

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_gather_ds656(const uint8_t* pool, int64_t pool_rows, const int32_t* idx,
                                    int64_t num_rows, uint8_t* out, nvfp4kv_stream_t stream) {
    return nvfp4kv::gather_ds656_impl("nvfp4kv_gather_ds656", pool, nullptr, pool_rows, idx, num_rows, out, stream);
}

extern "C" int nvfp4kv_gather_ds656_rope(const uint8_t* pool, const void* rope_pool, int64_t pool_rows,
                                         const int32_t* idx, int64_t num_rows, uint8_t* out,
                                         nvfp4kv_stream_t stream) {
    if (!rope_pool && num_rows > 0)
        return nvfp4kv::fail(NVFP4KV_EINVAL, "nvfp4kv_gather_ds656_rope: null rope pool");
    return nvfp4kv::gather_ds656_impl("nvfp4kv_gather_ds656_rope", pool, rope_pool, pool_rows, idx, num_rows, out,
                                      stream);
}

extern "C" int nvfp4kv_dequant_bf16(const uint8_t* pool, int64_t pool_rows, const void* rows,
                                    int rows_dtype, int64_t num_rows, void* out,
                                    int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (num_rows < 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_dequant_bf16: num_rows < 0");
    if (num_rows == 0) return NVFP4KV_OK;
    if (!pool || !rows || !out) return fail(NVFP4KV_EINVAL, "nvfp4kv_dequant_bf16: null pointer");
    if (reinterpret_cast<uintptr_t>(pool) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_dequant_bf16: pool and out must be 16-byte aligned");
    const int warps = 8;
    const dim3 grid(static_cast<unsigned>((num_rows + warps - 1) / warps));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    auto* o = static_cast<__nv_bfloat16*>(out);
    if (rows_dtype == NVFP4KV_INDEX_I64)
        dequant_bf16_kernel<NVFP4KV_INDEX_I64><<<grid, warps * 32, 0, st>>>(pool, pool_rows, rows, num_rows, o, err_flag);
    else if (rows_dtype == NVFP4KV_INDEX_I32)
        dequant_bf16_kernel<NVFP4KV_INDEX_I32><<<grid, warps * 32, 0, st>>>(pool, pool_rows, rows, num_rows, o, err_flag);
    else
        return fail(NVFP4KV_EINVAL, "nvfp4kv_dequant_bf16: rows dtype must be int64 or int32");
    return check_launch("nvfp4kv_dequant_bf16");
}

extern "C" int nvfp4kv_dedup_workspace_ints(int64_t pool_rows, int64_t num_entries, int64_t* ints) {
    using namespace nvfp4kv;
    if (!ints) return fail(NVFP4KV_EINVAL, "nvfp4kv_dedup_workspace_ints: null output");
    if (pool_rows <= 0 || num_entries < 0 || pool_rows >= (int64_t(1) << 31) - 1)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_dedup_workspace_ints: bad pool_rows / num_entries");
    *ints = dedup_layout(pool_rows, num_entries).ints;
    return NVFP4KV_OK;
}

extern "C" int nvfp4kv_dedup_gather_ds656(const uint8_t* pool, int64_t pool_rows, const int32_t* entries,
                                          int64_t num_entries, int32_t* workspace, int64_t workspace_ints,
                                          int32_t* tables, uint8_t* scratch, int64_t scratch_rows,
                                          int32_t* n_unique, int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (num_entries < 0 || scratch_rows < 0)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_dedup_gather_ds656: negative size");
    if (!pool || !workspace || !n_unique || (num_entries > 0 && (!entries || !tables)) ||
        (scratch_rows > 0 && !scratch))
        return fail(NVFP4KV_EINVAL, "nvfp4kv_dedup_gather_ds656: null pointer");
    if (pool_rows <= 0 || pool_rows >= (int64_t(1) << 31) - 1)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_dedup_gather_ds656: bad pool_rows");
    if (reinterpret_cast<uintptr_t>(pool) % 16 || reinterpret_cast<uintptr_t>(scratch) % 16)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_dedup_gather_ds656: pool and scratch must be 16-byte aligned");
    const DedupLayout l = dedup_layout(pool_rows, num_entries);
    if (workspace_ints < l.ints)
        return fail(NVFP4KV_EWORKSPACE, "nvfp4kv_dedup_gather_ds656: workspace %lld ints < %lld",
                    (long long)workspace_ints, (long long)l.ints);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int32_t* marks = workspace;
    int32_t* bsum = workspace + l.M;
    int32_t* uniq = bsum + l.nb;
    cudaError_t e = cudaMemsetAsync(marks, 0, static_cast<size_t>(l.M) * sizeof(int32_t), st);
    if (e != cudaSuccess) return fail(NVFP4KV_ECUDA, "nvfp4kv_dedup_gather_ds656: memset: %s", cudaGetErrorString(e));
    int rc;
    const unsigned eb = static_cast<unsigned>((num_entries + 255) / 256);
    if (num_entries > 0) {
        dedup_mark_kernel<<<eb, 256, 0, st>>>(entries, num_entries, pool_rows, marks, err_flag);
        if ((rc = check_launch("nvfp4kv_dedup_gather_ds656 (mark)")) != NVFP4KV_OK) return rc;
    }
    dedup_block_sums_kernel<<<static_cast<unsigned>(l.nb), kScanBlock, 0, st>>>(marks, l.M, bsum);
    if ((rc = check_launch("nvfp4kv_dedup_gather_ds656 (block sums)")) != NVFP4KV_OK) return rc;
    dedup_scan_sums_kernel<<<1, kScanBlock, 0, st>>>(bsum, l.nb, n_unique);
    if ((rc = check_launch("nvfp4kv_dedup_gather_ds656 (scan)")) != NVFP4KV_OK) return rc;
    dedup_offsets_kernel<<<static_cast<unsigned>(l.nb), kScanBlock, 0, st>>>(marks, l.M, bsum, uniq);
    if ((rc = check_launch("nvfp4kv_dedup_gather_ds656 (positions)")) != NVFP4KV_OK) return rc;
    if (num_entries > 0) {
        dedup_tables_kernel<<<eb, 256, 0, st>>>(entries, num_entries, pool_rows, marks, tables);
        if ((rc = check_launch("nvfp4kv_dedup_gather_ds656 (tables)")) != NVFP4KV_OK) return rc;
    }
    if (scratch_rows > 0) {
        const int64_t want = (scratch_rows + 7) / 8;   // 8 warps a block, one row each per pass
        const unsigned grid = static_cast<unsigned>(want < 148 * 16 ? want : 148 * 16);
        if (g_gather_division.load() == NVFP4KV_DIV_TRITON)
            dedup_gather_kernel<true><<<grid, 256, 0, st>>>(pool, pool_rows, uniq, n_unique, scratch, scratch_rows,
                                                            err_flag);
        else
            dedup_gather_kernel<false><<<grid, 256, 0, st>>>(pool, pool_rows, uniq, n_unique, scratch, scratch_rows,
                                                             err_flag);
        if ((rc = check_launch("nvfp4kv_dedup_gather_ds656 (gather)")) != NVFP4KV_OK) return rc;
    }
    return NVFP4KV_OK;
}
