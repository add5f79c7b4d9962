// Quantize-on-append: bf16/fp16 MLA latent rows -> 288-byte NVFP4 pool rows.
//
// Restates _quant_kernel (reference nvfp4-kv/glm53_nvfp4_runtime.py:37-65) for sm_100a:
// one warp per token, two fully coalesced 16-byte loads per lane (elements [8l, 8l+8) and
// [256+8l, 256+8l+8)) issued together with the slot load, the block amax completed with one
// shuffle (a 16-element block spans two neighbouring lanes), and coalesced 4-byte code
// stores / 1-byte scale stores.
//
// Bit-exactness.  The reference computes v = x / s in fp32 and walks the ladder
// `|v| < 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5` (ties go up; NaN fails every `<`).  Here the
// division is replaced by the exact comparison |x| < t*s: t*s has at most 7 significant
// bits and so is exact in fp32, and a bf16/fp16 x can never lie within half an fp32 ulp of
// t*s without being equal to it, so fl(x/s) < t  <=>  |x| < t*s.  s == 0 makes every
// threshold 0 and every code 7, like x/0 = +-inf and 0/0 = NaN in the reference; the sign
// nibble is (x < 0), which equals (x/s < 0) for every s >= 0 and a bf16/fp16 x.
//
// Fast path.  The ladder is round-to-nearest onto the e2m1 grid {0, 0.5, 1, 1.5, 2, 3, 4, 6}
// with ties rounded up (each threshold is the midpoint of two neighbours) and everything
// from 5 up mapped to 6.  So the code of x is the hardware conversion
// cvt.rn.satfinite.e2m1x2.f32 of v = x * r, where r = RN(RN(1/s) * (1 + 2^-18)):
// v / (x/s) lies in (1, 1 + 2^-17), which moves an exact tie x = t*s strictly above t (so
// it rounds up, not to even), while a bf16/fp16 x != t*s is at least 2^-11 (relative) away
// from t*s (t*s has at most 7 significant bits and is itself a bf16/fp16 value), so it stays
// on its side.  v is formed as fma(x, r, +0.0) so that x = -0.0 gives +0.0 (code 0, as in
// the reference), while a negative x that rounds to zero keeps its sign (code 8).  A block
// whose scale byte is 0 (x/0) or whose elements include a NaN takes the exact compare
// ladder below instead, for its whole warp.
#include "abi_common.h"
#include "common.cuh"

namespace nvfp4kv {
namespace {

template <int DT>
__device__ __forceinline__ float to_f32(uint16_t v) {
    if constexpr (DT == NVFP4KV_DTYPE_BF16) return __uint_as_float(static_cast<uint32_t>(v) << 16);
    else return __half2float(__ushort_as_half(v));
}

// 8 consecutive 16-bit elements, as raw words (converted after every load is in flight).
template <bool VEC>
__device__ __forceinline__ uint4 load8_raw(const uint16_t* p) {
    if constexpr (VEC) {
        return ldg_nc_v4(p);              // streamed once: no L1 allocation
    } else {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = static_cast<uint32_t>(p[2 * j]) | (static_cast<uint32_t>(p[2 * j + 1]) << 16);
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
}

template <int DT>
__device__ __forceinline__ void unpack8(uint4 u, float (&x)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x[2 * j] = to_f32<DT>(static_cast<uint16_t>(w[j] & 0xFFFFu));
        x[2 * j + 1] = to_f32<DT>(static_cast<uint16_t>(w[j] >> 16));
    }
}

// Code of one element given the block's 7 exact thresholds t_k * s (see file comment): the
// number of thresholds with !(|x| < t_k s), found by a three-level search over the sorted
// thresholds (3 compares instead of 7; a NaN fails every `<` and lands on 7 as before).
__device__ __forceinline__ uint32_t nvfp4_code(float x, const float (&th)[7]) {
    const float a = fabsf(x);
    const bool b2 = !(a < th[3]);                      // >= 1.75 s: codes 4..7
    const bool b1 = !(a < (b2 ? th[5] : th[1]));       // >= 3.5 s / 0.75 s
    const float t0 = b2 ? (b1 ? th[6] : th[4]) : (b1 ? th[2] : th[0]);
    const bool b0 = !(a < t0);
    const uint32_t c = (b2 ? 4u : 0u) | (b1 ? 2u : 0u) | (b0 ? 1u : 0u);
    return c | (x < 0.0f ? 8u : 0u);
}

// Quantise 8 consecutive elements of one block half: returns the 4 packed code bytes and
// the block's e4m3 scale byte.  `amax_half` is this lane's |x| max; the block max needs
// the partner lane (lane ^ 1).
__device__ __forceinline__ uint32_t quant_half(const float (&x)[8], uint8_t& scale_byte) {
    float m = fabsf(x[0]);
#pragma unroll
    for (int j = 1; j < 8; ++j) m = fmaxf(m, fabsf(x[j]));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    const float sc = fmaxf(__fdiv_rn(m, 6.0f), 1e-8f);     // runtime:47
    scale_byte = f32_to_e4m3(sc);
    const float s = e4m3_to_f32(scale_byte);
    const float tmul[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
    float th[7];
#pragma unroll
    for (int k = 0; k < 7; ++k) th[k] = __fmul_rn(tmul[k], s);
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = nvfp4_code(x[2 * j], th);
        const uint32_t hi = nvfp4_code(x[2 * j + 1], th);
        packed |= (lo | (hi << 4)) << (8 * j);
    }
    return packed;
}

__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}
__device__ __forceinline__ float abs_max_nan8(const float (&x)[8]) {
    float m = fabsf(x[0]);
#pragma unroll
    for (int j = 1; j < 8; ++j) m = max_nan(m, fabsf(x[j]));
    return m;
}

// Fast-path codes of 8 consecutive elements: cvt.rn.satfinite.e2m1x2 of fma(x, r, +0.0)
// (see the file comment), packed with element 0 in the low nibble of byte 0.
__device__ __forceinline__ uint32_t e2m1x8_scaled(const float (&x)[8], float r) {
    uint32_t packed;
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        ".reg .f32 v0, v1, v2, v3, v4, v5, v6, v7;\n\t"
        "fma.rn.f32 v0, %1, %9, 0f00000000;\n\t"
        "fma.rn.f32 v1, %2, %9, 0f00000000;\n\t"
        "fma.rn.f32 v2, %3, %9, 0f00000000;\n\t"
        "fma.rn.f32 v3, %4, %9, 0f00000000;\n\t"
        "fma.rn.f32 v4, %5, %9, 0f00000000;\n\t"
        "fma.rn.f32 v5, %6, %9, 0f00000000;\n\t"
        "fma.rn.f32 v6, %7, %9, 0f00000000;\n\t"
        "fma.rn.f32 v7, %8, %9, 0f00000000;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b0, v1, v0;\n\t"   // first source -> high nibble
        "cvt.rn.satfinite.e2m1x2.f32 b1, v3, v2;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b2, v5, v4;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b3, v7, v6;\n\t"
        "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
        : "=r"(packed)
        : "f"(x[0]), "f"(x[1]), "f"(x[2]), "f"(x[3]), "f"(x[4]), "f"(x[5]), "f"(x[6]), "f"(x[7]), "f"(r));
    return packed;
}

// At most 32 registers a thread, so that 8 blocks (64 warps, 64 tokens in flight) fit on an
// SM: the latency of the row loads is covered by occupancy (two or four tokens per warp, at
// fewer warps an SM, measured slower).
template <int DT, int SLOT_DT, bool VEC>
__global__ void __launch_bounds__(256, 8)
append_kernel(const uint16_t* __restrict__ src, int64_t T, int64_t stride,
              uint8_t* __restrict__ pool, int64_t pool_rows, const void* __restrict__ slot,
              int32_t* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    // the row and its slot are loaded together (token t's row exists whatever its slot says;
    // a skipped token's row is simply not stored), so a warp waits one memory latency, not two
    const uint16_t* row = src + t * stride;
    const uint4 ua = load8_raw<VEC>(row + 8 * lane);
    const uint4 ub = load8_raw<VEC>(row + 256 + 8 * lane);
    int64_t sl;
    if constexpr (SLOT_DT == NVFP4KV_INDEX_I64) sl = __ldg(static_cast<const long long*>(slot) + t);
    else sl = __ldg(static_cast<const int32_t*>(slot) + t);
    if (sl < 0) return;                                        // runtime:42-43
    if (sl >= pool_rows) {
        if (lane == 0) set_error(err, NVFP4KV_DEVERR_BAD_SLOT);
        return;
    }
    float xa[8], xb[8];
    unpack8<DT>(ua, xa);
    unpack8<DT>(ub, xb);
    uint8_t* dst = pool + sl * kRowBytes;
    // block amax, NaN-propagating: a NaN anywhere in the block sends the warp to the ladder
    float ma = abs_max_nan8(xa), mb = abs_max_nan8(xb);
    ma = max_nan(ma, __shfl_xor_sync(0xFFFFFFFFu, ma, 1));
    mb = max_nan(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, 1));
    // the two lanes of a pair share blocks l/2 (half a) and 16 + l/2 (half b): the even lane
    // computes the first one's scale, the odd lane the second one's
    const bool odd = lane & 1;
    const float m = odd ? mb : ma;
    const uint8_t sbyte = f32_to_e4m3(fmaxf(__fdiv_rn(m, 6.0f), 1e-8f));   // runtime:47-48
    const float s = e4m3_to_f32(sbyte);                                   // runtime:49
    // r > 0 only on the fast path (s > 0 and no NaN); 1 + 2^-18 is exact in fp32
    const float r = (s > 0.0f && m == m) ? __fmul_rn(__frcp_rn(s), 1.0000038146972656f) : 0.0f;
    if (__all_sync(0xFFFFFFFFu, r > 0.0f)) {
        const float r_other = __shfl_xor_sync(0xFFFFFFFFu, r, 1);
        dst[256 + 16 * odd + (lane >> 1)] = sbyte;             // block l/2 or 16 + l/2
        *reinterpret_cast<uint32_t*>(dst + 4 * lane) = e2m1x8_scaled(xa, odd ? r_other : r);
        *reinterpret_cast<uint32_t*>(dst + 128 + 4 * lane) = e2m1x8_scaled(xb, odd ? r : r_other);
    } else {
        uint8_t sa, sb;
        const uint32_t ca = quant_half(xa, sa);
        const uint32_t cb = quant_half(xb, sb);
        *reinterpret_cast<uint32_t*>(dst + 4 * lane) = ca;         // bytes [4l, 4l+4)
        *reinterpret_cast<uint32_t*>(dst + 128 + 4 * lane) = cb;   // bytes [128+4l, ...)
        dst[256 + 16 * odd + (lane >> 1)] = odd ? sb : sa;          // NaN-ignoring amax here
    }
}

template <int DT, int SLOT_DT>
void launch_append(const void* kv_c, int64_t T, int64_t stride, uint8_t* pool, int64_t rows,
                   const void* slot, int32_t* err, cudaStream_t st, bool vec) {
    const int warps = 8;
    const dim3 grid(static_cast<unsigned>((T + warps - 1) / warps));
    const uint16_t* src = static_cast<const uint16_t*>(kv_c);
    if (vec)
        append_kernel<DT, SLOT_DT, true><<<grid, warps * 32, 0, st>>>(src, T, stride, pool, rows, slot, err);
    else
        append_kernel<DT, SLOT_DT, false><<<grid, warps * 32, 0, st>>>(src, T, stride, pool, rows, slot, err);
}

// Indexer keys: a 128-d key per token quantised by the same rule as the latent rows (per-16
// scale e4m3(max(amax / 6, 1e-8)), codes by the `<` ladder with ties up), into a 72-byte row:
// bytes [0, 64) codes (byte i = code[2i] | code[2i+1] << 4), bytes [64, 72) the 8 block
// scales.  A half-warp per token, a lane per 8 elements (a block spans two lanes); the exact
// compare ladder throughout.  Lanes of a token past T compute on zeros and store nothing (the
// block's partner shuffle needs every lane).
template <int SLOT_DT, bool VEC>
__global__ void __launch_bounds__(256)
index_append_kernel(const uint16_t* __restrict__ k, int64_t T, int64_t stride, uint8_t* __restrict__ pool,
                    int64_t rows, const void* __restrict__ slot_mapping, int32_t* __restrict__ err) {
    const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
    const int l = threadIdx.x & 15;
    const bool live = t < T;
    int64_t slot = -1;
    float x[8];
    if (live) {
        slot = SLOT_DT == NVFP4KV_INDEX_I64 ? static_cast<const int64_t*>(slot_mapping)[t]
                                            : static_cast<const int32_t*>(slot_mapping)[t];
        unpack8<NVFP4KV_DTYPE_BF16>(load8_raw<VEC>(k + t * stride + 8 * l), x);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = 0.0f;
    }
    uint8_t sb;
    const uint32_t codes = quant_half(x, sb);
    if (!live || slot < 0) return;
    if (slot >= rows) {
        if (l == 0) set_error(err, NVFP4KV_DEVERR_BAD_SLOT);
        return;
    }
    uint8_t* row = pool + slot * NVFP4KV_INDEX_ROW_BYTES;
    *reinterpret_cast<uint32_t*>(row + 4 * l) = codes;
    if ((l & 1) == 0) row[64 + (l >> 1)] = sb;
}

template <int SLOT_DT>
void launch_index_append(const uint16_t* k, int64_t T, int64_t stride, uint8_t* pool, int64_t rows,
                         const void* slot, int32_t* err, bool vec, cudaStream_t st) {
    const dim3 grid(static_cast<unsigned>((T * 16 + 255) / 256));
    if (vec) index_append_kernel<SLOT_DT, true><<<grid, 256, 0, st>>>(k, T, stride, pool, rows, slot, err);
    else index_append_kernel<SLOT_DT, false><<<grid, 256, 0, st>>>(k, T, stride, pool, rows, slot, err);
}

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_index_append(const void* k, int64_t num_tokens, int64_t src_stride, uint8_t* index_pool,
                                    int64_t pool_rows, const void* slot_mapping, int slot_dtype,
                                    int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (num_tokens < 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_index_append: num_tokens < 0");
    if (num_tokens == 0) return NVFP4KV_OK;
    if (!k || !index_pool || !slot_mapping) return fail(NVFP4KV_EINVAL, "nvfp4kv_index_append: null pointer");
    if (src_stride < NVFP4KV_INDEX_DIM)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_index_append: src_stride %lld < 128", (long long)src_stride);
    if (pool_rows <= 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_index_append: empty index pool");
    if (reinterpret_cast<uintptr_t>(index_pool) % 8 || reinterpret_cast<uintptr_t>(k) % 2)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_index_append: index pool must be 8-byte and k 2-byte aligned");
    if (slot_dtype != NVFP4KV_INDEX_I64 && slot_dtype != NVFP4KV_INDEX_I32)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_index_append: slot dtype must be int64 or int32");
    const bool vec = reinterpret_cast<uintptr_t>(k) % 16 == 0 && src_stride % 8 == 0;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint16_t* src = static_cast<const uint16_t*>(k);
    if (slot_dtype == NVFP4KV_INDEX_I64)
        launch_index_append<NVFP4KV_INDEX_I64>(src, num_tokens, src_stride, index_pool, pool_rows, slot_mapping,
                                               err_flag, vec, st);
    else
        launch_index_append<NVFP4KV_INDEX_I32>(src, num_tokens, src_stride, index_pool, pool_rows, slot_mapping,
                                               err_flag, vec, st);
    return check_launch("nvfp4kv_index_append");
}

extern "C" int nvfp4kv_append(const void* kv_c, int kv_dtype, int64_t num_tokens, int64_t src_stride,
                              uint8_t* pool, int64_t pool_rows, const void* slot_mapping,
                              int slot_dtype, int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (num_tokens < 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_append: num_tokens < 0");
    if (num_tokens == 0) return NVFP4KV_OK;                     // runtime:73-74
    if (!kv_c || !pool || !slot_mapping) return fail(NVFP4KV_EINVAL, "nvfp4kv_append: null pointer");
    if (src_stride < NVFP4KV_LATENT)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_append: src_stride %lld < 512", (long long)src_stride);
    if (pool_rows <= 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_append: empty pool");
    if (reinterpret_cast<uintptr_t>(pool) % 16 != 0)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_append: pool must be 16-byte aligned");
    if (kv_dtype != NVFP4KV_DTYPE_BF16 && kv_dtype != NVFP4KV_DTYPE_F16)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_append: kv_dtype must be bf16 or fp16");
    if (slot_dtype != NVFP4KV_INDEX_I64 && slot_dtype != NVFP4KV_INDEX_I32)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_append: slot dtype must be int64 or int32");
    const bool vec = (reinterpret_cast<uintptr_t>(kv_c) % 16 == 0) && (src_stride % 8 == 0);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (kv_dtype == NVFP4KV_DTYPE_BF16) {
        if (slot_dtype == NVFP4KV_INDEX_I64)
            launch_append<NVFP4KV_DTYPE_BF16, NVFP4KV_INDEX_I64>(kv_c, num_tokens, src_stride, pool, pool_rows, slot_mapping, err_flag, st, vec);
        else
            launch_append<NVFP4KV_DTYPE_BF16, NVFP4KV_INDEX_I32>(kv_c, num_tokens, src_stride, pool, pool_rows, slot_mapping, err_flag, st, vec);
    } else {
        if (slot_dtype == NVFP4KV_INDEX_I64)
            launch_append<NVFP4KV_DTYPE_F16, NVFP4KV_INDEX_I64>(kv_c, num_tokens, src_stride, pool, pool_rows, slot_mapping, err_flag, st, vec);
        else
            launch_append<NVFP4KV_DTYPE_F16, NVFP4KV_INDEX_I32>(kv_c, num_tokens, src_stride, pool, pool_rows, slot_mapping, err_flag, st, vec);
    }
    return check_launch("nvfp4kv_append");
}
