// Internal launcher declarations (C++), wrapped by the C ABI in capi.cu.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ms {

cudaError_t launch_quantize_rows(const void* x, int64_t ldx, int64_t M, int K, void* xq, float* sx,
                                 cudaStream_t stream);
// Per-row amax of fp16 rows, and row quantisation with a given amax (exact scales
// of K-sharded rows after an all-reduce max).
cudaError_t launch_row_amax(const void* x, int64_t ldx, int64_t M, int K, float* amax, cudaStream_t stream);
cudaError_t launch_quantize_rows_amax(const void* x, int64_t ldx, int64_t M, int K, const float* amax, void* xq,
                                      float* sx, cudaStream_t stream);
cudaError_t launch_rmsnorm(const void* x, const void* residual, const void* weight, int64_t M, int H, float eps,
                           void* residual_out, void* y, void* yq, float* sy, cudaStream_t stream);
cudaError_t launch_silu_mul(const void* gu, int64_t M, int I, void* out, void* aq, float* sa, cudaStream_t stream);

cudaError_t launch_store_kv_fp8(const void* k, const void* v, int64_t T, int kv_heads, int head_dim,
                                const int64_t* slots, void* k_cache, void* v_cache, float* k_scale, float* v_scale,
                                cudaStream_t stream);
cudaError_t launch_qkv_post(const void* qkv, int64_t T, int q_heads, int kv_heads, int head_dim, const void* q_norm_w,
                            const void* k_norm_w, float eps, const int64_t* positions, const void* cos_tab,
                            const void* sin_tab, const int64_t* slots, void* q_out, void* k_out, void* v_out,
                            void* k_cache, void* v_cache, float* k_scale, float* v_scale, cudaStream_t stream);

int decode_num_splits(int B, int Hkv, int max_blocks, int block_size, int num_sms);
size_t decode_workspace_bytes(int B, int Hq, int splits);
size_t decode_noalloc_scratch_bytes();
cudaError_t decode_noalloc_scratch(void** ptr);
cudaError_t launch_decode_attention(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                                    const float* v_scale, const int32_t* seqlens, const int32_t* block_tables,
                                    void* out, int B, int Hq, int Hkv, int head_dim, int block_size, int max_blocks,
                                    float softmax_scale, int splits, void* workspace, cudaStream_t stream);

cudaError_t launch_prefill_attention(bool paged, const void* q, const void* k16, const void* v16,
                                     const void* k_cache, const void* v_cache, const float* k_scale,
                                     const float* v_scale, const int32_t* block_tables, const int32_t* cu_q,
                                     const int32_t* kv_lens, void* out, int num_seqs, int total_q, int Hq, int Hkv,
                                     int head_dim, int block_size, int max_blocks, float softmax_scale,
                                     cudaStream_t stream);

// One rank's communication buffer for the fused tensor-parallel op: byte offsets
// (peers write [recv, ctrl); outq/outs/outh are the normalised rows this rank's
// next op reads).
struct TpLayout {
  int64_t partial, recv, grq, grs, grh, ctrl, outq, outs, outh, total;
};
TpLayout tp_layout(int world, int64_t H, int64_t max_rows);
cudaError_t launch_tp_buffer_init(void* base, int world, int64_t H, int64_t max_rows, cudaStream_t stream);
cudaError_t launch_tp_allreduce_rmsnorm_fp8(void* const* bases, int rank, int world, int64_t H, int64_t max_rows,
                                            void* residual, const void* weight, int M, float eps, int want_h,
                                            int pushed, int num_sms, cudaStream_t stream);

size_t argmax_workspace_bytes(int64_t M);
cudaError_t launch_argmax_rows(const void* x, int64_t M, int V, int64_t ldx, int64_t* idx, float* vmax,
                               void* workspace, cudaStream_t stream);

// out[6]: token-tile width BN (0: CUDA-core kernel), CTAs, K parts per tile
// (split-K, else 0), 256 x 256 tiles (0/1), whole tiles (0/1), K chunks per stage.
void gemm_plan(int M, int N, int K, int num_sms, int* out);
size_t gemm_workspace_bytes(int M, int N, int K, int num_sms);
struct TpRows;
// rp (optional): push each output row to its owner's receive slot (row-parallel
// GEMM of tensor parallelism, see tp_rows.cuh) instead of writing y. tail (with
// rp): in, a request to do the tensor-parallel row work (reduce + residual +
// RMSNorm + FP8 + gather, the fields of *rp) in the GEMM's own tail; out, whether
// it will (otherwise the caller launches the separate op with pushed rows).
// f16: fp16 operands x [M, K/2] and w [N, K/2] (K in bytes, a multiple of 16), no
// scales (sx, sw null), no row-parallel push: y = fp16(x . w^T), fp32 accumulation.
cudaError_t launch_fp8_gemm(const void* xq, const float* sx, const void* wq, const float* sw, const void* bias,
                            void* y, int M, int N, int K, void* workspace, size_t workspace_bytes, int num_sms,
                            cudaStream_t stream, const TpRows* rp = nullptr, bool* tail = nullptr, bool f16 = false);

}  // namespace ms
