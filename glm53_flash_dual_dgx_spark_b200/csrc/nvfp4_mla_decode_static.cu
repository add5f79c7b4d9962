// nvfp4kv_mla_decode_static: the fused NVFP4 MLA decode with its workspace (split-K partials,
// prepared Q) kept in a fixed file-scope device array instead of a caller-provided one.
//
// Some callers cannot allocate device memory on the decode path: a host binding with no
// caching allocator of its own (a cgo / JNI / ctypes caller) would have to cudaMalloc per
// call, which synchronises the whole device and can fail with out-of-memory in the middle of
// a serving step; and an engine that has handed all free HBM to the KV pool after profiling
// has no headroom left for a per-call workspace.  This entry point needs neither: the
// workspace (split partials, prepared Q) lives in `g_decode_scratch`, which the CUDA module
// reserves once when it is loaded on a device.
//
// Limits:
//   - at most kStaticScratchBytes (32 MiB) of workspace; nvfp4kv_mla_decode_workspace_size()
//     of the shape must not exceed it (larger shapes are rejected with NVFP4KV_EWORKSPACE).
//     On a 148-SM device the split planner keeps splits * (batch * head groups) <= 148, so
//     the split partials never pass 148 * 64 rows * 514 floats = 19.5 MB; the prepared Q adds
//     72.25 KB per 64-row query group, which stays within the scratch up to 453 groups
//     (e.g. batch 453 at 64 heads and q_len 1);
//   - one scratch array per device: two calls whose kernels overlap on the same device (on
//     different streams, or from different host threads) race on it.  Calls must be ordered
//     on one stream or otherwise serialised;
//   - nothing in the scratch needs to start at zero: every split CTA writes its (max, sum)
//     pair for all 64 rows of its unit, and writes its O rows whenever its sum can be
//     non-zero, before the combine kernel reads them; the Q preparation kernel writes every
//     byte of the prepared-Q images before the attention kernel reads them;
//   - the first call on each device looks up the array's address (cudaGetSymbolAddress,
//     with that device current) and keeps it for the life of the process.  Make that first
//     call before any stream capture begins.  A cudaDeviceReset (or any re-creation of the
//     device's primary context) reloads the module and may move the array, so the library
//     must not be used on a device after it has been reset.
#include <cuda_runtime.h>

#include <mutex>

#include "abi_common.h"
#include "decode_shared.h"

namespace nvfp4kv {
namespace {

constexpr size_t kStaticScratchBytes = NVFP4KV_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Address of g_decode_scratch on the current device, looked up once per device.
int scratch_address(void** addr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(NVFP4KV_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(NVFP4KV_EINVAL, "mla_decode_static: device ordinal %d beyond %d", dev, kMaxDevices);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess || !p)
            return fail(NVFP4KV_ECUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
                        cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *addr = g_scratch_addr[dev];
    return NVFP4KV_OK;
}

}  // namespace
}  // namespace nvfp4kv

extern "C" int nvfp4kv_mla_decode_static(const void* q, int64_t q_stride_b, int64_t q_stride_q,
                                         int64_t q_stride_h, const uint8_t* pool, int64_t pool_rows,
                                         const int32_t* tables, int64_t tables_stride,
                                         const int32_t* seq_lens, int batch, int q_len, int num_heads,
                                         int head_dim_qk, int kv_lora_rank, int sparse_topk,
                                         int page_size, int max_seq_len, float bmm1_scale,
                                         float bmm2_scale, void* out, int64_t out_stride_b,
                                         int64_t out_stride_q, int64_t out_stride_h,
                                         int32_t* err_flag, nvfp4kv_stream_t stream) {
    using namespace nvfp4kv;
    if (batch < 0) return fail(NVFP4KV_EINVAL, "mla_decode_static: batch < 0");
    if (batch == 0) return NVFP4KV_OK;
    // the argument errors of nvfp4kv_mla_decode come first, then the capacity
    int rc = check_decode_args(q, q_stride_b, q_stride_q, q_stride_h, pool, pool_rows, tables, seq_lens, batch,
                               q_len, num_heads, head_dim_qk, kv_lora_rank, sparse_topk, page_size, max_seq_len,
                               out, out_stride_b, out_stride_q, out_stride_h, nullptr);
    if (rc != NVFP4KV_OK) return rc;
    size_t need = 0;
    rc = nvfp4kv_mla_decode_workspace_size(batch, q_len, num_heads, max_seq_len, sparse_topk, &need);
    if (rc != NVFP4KV_OK) return rc;
    if (need > kStaticScratchBytes)
        return fail(NVFP4KV_EWORKSPACE,
                    "mla_decode_static: shape needs %zu bytes of workspace, the static scratch "
                    "holds %zu; use nvfp4kv_mla_decode with a caller workspace",
                    need, kStaticScratchBytes);
    void* scratch = nullptr;
    if ((rc = scratch_address(&scratch)) != NVFP4KV_OK) return rc;
    return nvfp4kv_mla_decode(q, q_stride_b, q_stride_q, q_stride_h, pool, pool_rows, tables,
                              tables_stride, seq_lens, batch, q_len, num_heads, head_dim_qk,
                              kv_lora_rank, sparse_topk, page_size, max_seq_len, bmm1_scale,
                              bmm2_scale, out, out_stride_b, out_stride_q, out_stride_h, scratch,
                              kStaticScratchBytes, err_flag, stream);
}
