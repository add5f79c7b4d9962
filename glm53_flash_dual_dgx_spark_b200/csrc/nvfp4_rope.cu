// Rope side-pool writer.  The reference's model is NoPE: its write seam drops k_pe
// (nvfp4-kv/patch_nvfp4_kv.py:70) and its 656-byte rows carry zero rope bytes
// (nvfp4-kv/glm53_nvfp4_runtime.py:121-122).  For MLA models whose keys do carry a 64-d rope
// part, this library keeps it next to the 288-byte pool, in a pool of its own: 64 bf16 per
// token slot (128-byte rows), addressed by the same slots.  The 288-byte layout is unchanged.
//
// The copy is HBM-bound (128 B read + 128 B written + the slot per token): eight lanes move
// one token's row as 16-byte pieces, four tokens per warp.
#include "abi_common.h"
#include "common.cuh"

namespace nvfp4kv {
namespace {

template <int SLOT_DT, bool kVec>
__global__ void __launch_bounds__(256)
rope_append_kernel(const uint16_t* __restrict__ k_pe, int64_t T, int64_t stride, uint16_t* __restrict__ rope,
                   int64_t rows, const void* __restrict__ slot_mapping, int32_t* __restrict__ err) {
    const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t t = g >> 3;            // token
    const int piece = static_cast<int>(g & 7);   // 16-byte piece of its row (8 bf16)
    if (t >= T) return;
    const int64_t slot = SLOT_DT == NVFP4KV_INDEX_I64 ? static_cast<const int64_t*>(slot_mapping)[t]
                                                      : static_cast<const int32_t*>(slot_mapping)[t];
    if (slot < 0) return;                // padding slots are skipped, as by the append
    if (slot >= rows) {
        if (piece == 0) set_error(err, NVFP4KV_DEVERR_BAD_SLOT);
        return;
    }
    const uint16_t* src = k_pe + t * stride + 8 * piece;
    uint16_t* dst = rope + slot * NVFP4KV_ROPE + 8 * piece;
    if constexpr (kVec) {
        *reinterpret_cast<uint4*>(dst) = ldg_nc_v4(src);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) dst[k] = src[k];
    }
}

template <int SLOT_DT>
void launch_rope_append(const uint16_t* k_pe, int64_t T, int64_t stride, uint16_t* rope, int64_t rows,
                        const void* slot, int32_t* err, bool vec, cudaStream_t st) {
    const int64_t threads = T * 8;
    const dim3 grid(static_cast<unsigned>((threads + 255) / 256));
    if (vec)
        rope_append_kernel<SLOT_DT, true><<<grid, 256, 0, st>>>(k_pe, T, stride, rope, rows, slot, err);
    else
        rope_append_kernel<SLOT_DT, false><<<grid, 256, 0, st>>>(k_pe, T, stride, rope, rows, slot, err);
}

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_append_rope(const void* k_pe, int64_t num_tokens, int64_t src_stride, void* rope_pool,
                                   int64_t pool_rows, const void* slot_mapping, int slot_dtype,
                                   int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (num_tokens < 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_append_rope: num_tokens < 0");
    if (num_tokens == 0) return NVFP4KV_OK;
    if (!k_pe || !rope_pool || !slot_mapping) return fail(NVFP4KV_EINVAL, "nvfp4kv_append_rope: null pointer");
    if (src_stride < NVFP4KV_ROPE)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_append_rope: src_stride %lld < 64", (long long)src_stride);
    if (pool_rows <= 0) return fail(NVFP4KV_EINVAL, "nvfp4kv_append_rope: empty rope pool");
    if (reinterpret_cast<uintptr_t>(rope_pool) % 16 || reinterpret_cast<uintptr_t>(k_pe) % 2)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_append_rope: rope pool must be 16-byte and k_pe 2-byte aligned");
    if (slot_dtype != NVFP4KV_INDEX_I64 && slot_dtype != NVFP4KV_INDEX_I32)
        return fail(NVFP4KV_EINVAL, "nvfp4kv_append_rope: slot dtype must be int64 or int32");
    const bool vec = reinterpret_cast<uintptr_t>(k_pe) % 16 == 0 && src_stride % 8 == 0;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint16_t* src = static_cast<const uint16_t*>(k_pe);
    uint16_t* dst = static_cast<uint16_t*>(rope_pool);
    if (slot_dtype == NVFP4KV_INDEX_I64)
        launch_rope_append<NVFP4KV_INDEX_I64>(src, num_tokens, src_stride, dst, pool_rows, slot_mapping, err_flag,
                                              vec, st);
    else
        launch_rope_append<NVFP4KV_INDEX_I32>(src, num_tokens, src_stride, dst, pool_rows, slot_mapping, err_flag,
                                              vec, st);
    return check_launch("nvfp4kv_append_rope");
}
