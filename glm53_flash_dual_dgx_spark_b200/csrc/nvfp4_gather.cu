// Pool-row readers: the 656-byte fp8_ds_mla gather (byte-identical to the reference's
// _gather_kernel) and a bf16 dequantiser.  Both are HBM-bound; one warp handles one row,
// each lane one 16-element scale block (8 code bytes + 1 scale byte).
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

// Decode one lane's block: 8 code bytes (16 elements) times the block scale, in fp32.
__device__ __forceinline__ void decode_block(uint2 codes, uint8_t scale_byte, float (&v)[16]) {
    const float s = e4m3_to_f32(scale_byte);
    const uint32_t w[2] = {codes.x, codes.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
        v[2 * i] = __fmul_rn(e2m1_value(byte & 15u), s);
        v[2 * i + 1] = __fmul_rn(e2m1_value(byte >> 4), s);
    }
}

// runtime:87-122.  Row r of `out` re-encodes pool row clamp(idx[r], 0, R-1).
__global__ void __launch_bounds__(256)
gather_ds656_kernel(const uint8_t* __restrict__ pool, int64_t R, const int32_t* __restrict__ idx,
                    int64_t S, uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= S) return;
    int64_t src = idx[r];
    src = src < 0 ? 0 : (src > R - 1 ? R - 1 : src);          // :98
    const uint8_t* row = pool + src * kRowBytes;
    const uint2 codes = ldg_nc_v2(row + 8 * lane);
    const uint8_t sb = row[256 + lane];
    float v[16];
    decode_block(codes, sb, v);                                 // :99-108
    float amax = 0.0f;                                          // :109-112 (max includes 0.0)
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fmaxf(fabsf(v[2 * i]), fabsf(v[2 * i + 1])));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));  // 8 lanes = 128 elements
    const float gscale = fmaxf(__fdiv_rn(amax, 448.0f), 1e-12f);  // :113
    const float inv = __fdiv_rn(1.0f, gscale);                     // :115-116
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t w = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            w |= static_cast<uint32_t>(f32_to_e4m3(__fmul_rn(v[4 * j + k], inv))) << (8 * k);
        o[j] = w;
    }
    uint8_t* dst = out + r * kDsBytes;
    *reinterpret_cast<uint4*>(dst + 16 * lane) = make_uint4(o[0], o[1], o[2], o[3]);  // :117-120
    if ((lane & 7) == 0) *reinterpret_cast<float*>(dst + 512 + 4 * (lane >> 3)) = gscale;  // :114
    *reinterpret_cast<uint32_t*>(dst + 528 + 4 * lane) = 0u;                           // :121-122
}

template <int IDT>
__global__ void __launch_bounds__(256)
dequant_bf16_kernel(const uint8_t* __restrict__ pool, int64_t R, const void* __restrict__ rows,
                    int64_t n, __nv_bfloat16* __restrict__ out, int32_t* __restrict__ err) {
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
        decode_block(ldg_nc_v2(row + 8 * lane), row[256 + lane], v);
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

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_gather_ds656(const uint8_t* pool, int64_t pool_rows, const int32_t* idx,
                                    int64_t num_rows, uint8_t* out, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (num_rows < 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_gather_ds656: num_rows < 0");
    if (num_rows == 0) return NVFP4KV_OK;
    if (!pool || !idx || !out) return fail(NVFP4KV_EINVAL, "nvfp4kv_gather_ds656: null pointer");
    if (pool_rows <= 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_gather_ds656: empty pool");
    if (reinterpret_cast<uintptr_t>(pool) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_gather_ds656: pool and out must be 16-byte aligned");
    const int warps = 8;
    const dim3 grid(static_cast<unsigned>((num_rows + warps - 1) / warps));
    gather_ds656_kernel<<<grid, warps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        pool, pool_rows, idx, num_rows, out);
    return check_launch("nvfp4kv_gather_ds656");
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
