// Pieces shared by the fused-decode kernels: the split plan, the validated call arguments
// and the launchers each kernel file provides.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace nvfp4kv {

constexpr int kDecTile = 128;       // tokens per tile
constexpr int kDecRows = 64;        // query rows per CTA (one "group")
constexpr int kDecMaxSplits = 64;   // split-K partitions per group

// Bytes of one query group's prepared Q: the four NVFP4 terms as the fused
// kernel's shared-memory image (64 KB), their scales (8 KB) and 64 per-row score factors.
constexpr size_t kQImageBytes = 65536 + 8192 + 256;

struct DecodePlan {
    int groups, splits, tiles_total;   // split s: tiles [s T / splits, (s+1) T / splits)
    size_t part_bytes;   // splits * batch * groups * 64 * (512 + 2) floats when splits > 1, else 0
    size_t qimg_bytes;   // batch * groups * kQImageBytes
    size_t ws_bytes;     // part_bytes + qimg_bytes
};
DecodePlan make_decode_plan(int batch, int q_len, int num_heads, int max_seq_len, int sparse_topk);

// Arguments of nvfp4kv_mla_decode after validation.
struct DecodeArgs {
    const void* q;
    int64_t q_sb, q_sq, q_sh;
    const uint8_t* pool;
    int64_t pool_rows;
    const int32_t* tables;
    int64_t tables_stride;
    const int32_t* seq_lens;
    int batch, q_len, num_heads;
    int sparse_topk, page_size, page_shift, max_seq_len;
    float bmm1_scale, bmm2_scale;
    void* out;
    int64_t o_sb, o_sq, o_sh;
    float* part_o;    // [splits][batch][groups][64][512] when splits > 1
    float* part_ml;   // [splits][batch][groups][64][2]
    uint8_t* qimg;    // [batch][groups][kQImageBytes]
    float* lse;       // optional [batch][q_len][heads]: natural-log sum of exp(bmm1_scale q.k)
    int32_t* err;
    // rope side-pool (all null without one): 64 bf16 per pool row; the prepared rope part of q
    // ([batch][groups][64][64] fp32, scaled like the Q terms) and the rope scores
    // ([batch][groups][64][tiles_total * 128] fp32) the attention kernel adds to its scores
    const uint16_t* rope_pool;
    float* rope_q;
    float* rope_logits;
};

// Workspace bytes the rope side of a decode adds to DecodePlan::ws_bytes (placed after it).
inline size_t rope_q_bytes(const DecodePlan& pl, int batch) {
    return static_cast<size_t>(batch) * pl.groups * kDecRows * 64 * sizeof(float);
}
inline size_t rope_logit_bytes(const DecodePlan& pl, int batch) {
    return static_cast<size_t>(batch) * pl.groups * kDecRows * pl.tiles_total * kDecTile * sizeof(float);
}

// Launch `kernel` as a programmatic dependent of the kernel before it on `st`: it may start
// while that kernel still runs, and reads that kernel's output only after griddepcontrol.wait.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Argument checks of nvfp4kv_mla_decode that need no workspace (pointers, alignment, shape,
// page geometry); `page_shift` receives log2(page_size) in dense mode.  No device call.
int check_decode_args(const void* q, int64_t q_stride_b, int64_t q_stride_q, int64_t q_stride_h,
                      const uint8_t* pool, int64_t pool_rows, const int32_t* tables, const int32_t* seq_lens,
                      int batch, int q_len, int num_heads, int head_dim_qk, int kv_lora_rank, int sparse_topk,
                      int page_size, int max_seq_len, const void* out, int64_t out_stride_b,
                      int64_t out_stride_q, int64_t out_stride_h, int* page_shift);

// Q preparation + the fused decode kernel (QK^T on the block-scaled fp4 tensor-core path),
// paged (sparse_topk == 0) or top-k rows (sparse_topk > 0).
int launch_decode_fp4(const DecodeArgs& a, const DecodePlan& pl, cudaStream_t st);

}  // namespace nvfp4kv
