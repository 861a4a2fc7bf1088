// extern "C" entry points declared in include/microserve_b200.h: argument
// validation, error codes and the per-device facts (SM count) the launchers need.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <string>

#include "../../include/microserve_b200.h"
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tp_rows.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MS_OK;
  if (e == cudaErrorInvalidValue) return fail(MS_ERR_UNSUPPORTED, "%s: unsupported shape or argument", what);
  return fail(MS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

int ms_version(void) { return 100; }

const char* ms_last_error(void) { return g_err.c_str(); }

int64_t ms_launch_count(void) { return ms::g_host_launches.load(std::memory_order_relaxed); }

int ms_set_pdl(int enable) { return ms::g_pdl_enabled.exchange(enable ? 1 : 0); }

int ms_set_pair_tiles(int enable) { return ms::g_pair_tiles_enabled.exchange(enable ? 1 : 0); }

int ms_get_device_status(int* status, void* stream) {
  if (status == nullptr) return fail(MS_ERR_INVALID, "ms_get_device_status: status is NULL");
  int host = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&host, ms::g_device_status, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                            S(stream));
  if (e == cudaSuccess)
    e = cudaMemcpyToSymbolAsync(ms::g_device_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, S(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(S(stream));
  *status = host;
  return check_cuda(e, "ms_get_device_status");
}

int ms_quantize_rows_fp8(const void* x, int64_t ldx, int64_t M, int64_t K, void* xq, float* sx, void* stream) {
  if (M < 0 || K < 0 || ldx < K) return fail(MS_ERR_INVALID, "ms_quantize_rows_fp8: bad sizes M=%lld K=%lld ldx=%lld",
                                              (long long)M, (long long)K, (long long)ldx);
  if (M > 0 && K > 0 && (!x || !xq || !sx)) return fail(MS_ERR_INVALID, "ms_quantize_rows_fp8: null pointer");
  if (K > (1 << 20)) return fail(MS_ERR_UNSUPPORTED, "ms_quantize_rows_fp8: K too large");
  return check_cuda(ms::launch_quantize_rows(x, ldx, M, (int)K, xq, sx, S(stream)), "ms_quantize_rows_fp8");
}

size_t ms_fp8_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return ms::gemm_workspace_bytes((int)M, (int)N, (int)K, num_sms());
}

int ms_fp8_gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int* plan) {
  if (M <= 0 || N <= 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || sms <= 0 || !plan)
    return fail(MS_ERR_INVALID, "ms_fp8_gemm_plan: bad arguments");
  ms::gemm_plan((int)M, (int)N, (int)K, sms, plan);
  return MS_OK;
}

int ms_fp8_gemm(const void* xq, const float* sx, const void* wq, const float* sw, const void* bias, void* y,
                int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(MS_ERR_INVALID, "ms_fp8_gemm: bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                (long long)K);
  if (M == 0 || N == 0) return MS_OK;
  if (!xq || !sx || !wq || !sw || !y) return fail(MS_ERR_INVALID, "ms_fp8_gemm: null pointer");
  const size_t need = ms::gemm_workspace_bytes((int)M, (int)N, (int)K, num_sms());
  if (workspace_bytes < need || (need > 0 && workspace == nullptr))
    return fail(MS_ERR_WORKSPACE, "ms_fp8_gemm: workspace %zu < %zu bytes", workspace_bytes, need);
  return check_cuda(ms::launch_fp8_gemm(xq, sx, wq, sw, bias, y, (int)M, (int)N, (int)K, workspace,
                                        workspace_bytes, num_sms(), S(stream)),
                    "ms_fp8_gemm");
}

size_t ms_f16_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || K > INT32_MAX / 2) return 0;
  return ms::gemm_workspace_bytes((int)M, (int)N, (int)(2 * K), num_sms());
}

int ms_f16_gemm(const void* x, const void* w, void* y, int64_t M, int64_t N, int64_t K, void* workspace,
                size_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX / 2)
    return fail(MS_ERR_INVALID, "ms_f16_gemm: bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                (long long)K);
  if (M == 0 || N == 0) return MS_OK;
  if (!x || !w || !y) return fail(MS_ERR_INVALID, "ms_f16_gemm: null pointer");
  if (K % 8 != 0) return fail(MS_ERR_UNSUPPORTED, "ms_f16_gemm: K=%lld is not a multiple of 8", (long long)K);
  if (((uintptr_t)x & 15) != 0 || ((uintptr_t)w & 15) != 0)
    return fail(MS_ERR_INVALID, "ms_f16_gemm: x and w must be 16-byte aligned");
  const size_t need = ms::gemm_workspace_bytes((int)M, (int)N, (int)(2 * K), num_sms());
  if (workspace_bytes < need || (need > 0 && workspace == nullptr))
    return fail(MS_ERR_WORKSPACE, "ms_f16_gemm: workspace %zu < %zu bytes", workspace_bytes, need);
  return check_cuda(ms::launch_fp8_gemm(x, nullptr, w, nullptr, nullptr, y, (int)M, (int)N, (int)(2 * K), workspace,
                                        workspace_bytes, num_sms(), S(stream), nullptr, nullptr, true),
                    "ms_f16_gemm");
}

int ms_rmsnorm(const void* x, const void* residual, const void* weight, int64_t M, int64_t H, float eps,
               void* residual_out, void* y, void* yq, float* sy, void* stream) {
  if (M < 0 || H <= 0) return fail(MS_ERR_INVALID, "ms_rmsnorm: bad sizes");
  if (M == 0) return MS_OK;
  if (!x || !weight) return fail(MS_ERR_INVALID, "ms_rmsnorm: null pointer");
  if (residual && !residual_out) return fail(MS_ERR_INVALID, "ms_rmsnorm: residual without residual_out");
  if ((yq == nullptr) != (sy == nullptr)) return fail(MS_ERR_INVALID, "ms_rmsnorm: yq and sy go together");
  if (H % 16 != 0) return fail(MS_ERR_UNSUPPORTED, "ms_rmsnorm: H=%lld is not a multiple of 16", (long long)H);
  if (H > 32768) return fail(MS_ERR_UNSUPPORTED, "ms_rmsnorm: H=%lld > 32768", (long long)H);
  return check_cuda(ms::launch_rmsnorm(x, residual, weight, M, (int)H, eps, residual_out, y, yq, sy, S(stream)),
                    "ms_rmsnorm");
}

int ms_silu_mul(const void* gu, int64_t M, int64_t I, void* out, void* aq, float* sa, void* stream) {
  if (M < 0 || I <= 0) return fail(MS_ERR_INVALID, "ms_silu_mul: bad sizes");
  if (M == 0) return MS_OK;
  if (!gu) return fail(MS_ERR_INVALID, "ms_silu_mul: null pointer");
  if ((aq == nullptr) != (sa == nullptr)) return fail(MS_ERR_INVALID, "ms_silu_mul: aq and sa go together");
  if (I % 16 != 0) return fail(MS_ERR_UNSUPPORTED, "ms_silu_mul: I=%lld is not a multiple of 16", (long long)I);
  if (I > 32768) return fail(MS_ERR_UNSUPPORTED, "ms_silu_mul: I=%lld > 32768", (long long)I);
  return check_cuda(ms::launch_silu_mul(gu, M, (int)I, out, aq, sa, S(stream)), "ms_silu_mul");
}

int ms_store_kv_fp8(const void* k, const void* v, int64_t T, int kv_heads, int head_dim, const int64_t* slots,
                    void* k_cache, void* v_cache, float* k_scale, float* v_scale, void* stream) {
  if (T < 0 || kv_heads <= 0) return fail(MS_ERR_INVALID, "ms_store_kv_fp8: bad sizes");
  if (T == 0) return MS_OK;
  if (head_dim != 128) return fail(MS_ERR_UNSUPPORTED, "ms_store_kv_fp8: head_dim %d != 128", head_dim);
  if (!k || !v || !slots || !k_cache || !v_cache || !k_scale || !v_scale)
    return fail(MS_ERR_INVALID, "ms_store_kv_fp8: null pointer");
  return check_cuda(ms::launch_store_kv_fp8(k, v, T, kv_heads, head_dim, slots, k_cache, v_cache, k_scale, v_scale,
                                            S(stream)),
                    "ms_store_kv_fp8");
}

int ms_qkv_post(const void* qkv, int64_t T, int q_heads, int kv_heads, int head_dim, const void* q_norm_w,
                const void* k_norm_w, float eps, const int64_t* positions, const void* cos_tab, const void* sin_tab,
                const int64_t* slots, void* q_out, void* k_out, void* v_out, void* k_cache, void* v_cache,
                float* k_scale, float* v_scale, void* stream) {
  if (T < 0 || q_heads <= 0 || kv_heads <= 0) return fail(MS_ERR_INVALID, "ms_qkv_post: bad sizes");
  if (T == 0) return MS_OK;
  if (head_dim != 128) return fail(MS_ERR_UNSUPPORTED, "ms_qkv_post: head_dim %d != 128", head_dim);
  if (!qkv || !positions || !cos_tab || !sin_tab || !q_out) return fail(MS_ERR_INVALID, "ms_qkv_post: null pointer");
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
    return fail(MS_ERR_INVALID, "ms_qkv_post: q_norm_w and k_norm_w go together");
  if (slots && (!k_cache || !v_cache || !k_scale || !v_scale))
    return fail(MS_ERR_INVALID, "ms_qkv_post: slots without a cache");
  return check_cuda(ms::launch_qkv_post(qkv, T, q_heads, kv_heads, head_dim, q_norm_w, k_norm_w, eps, positions,
                                        cos_tab, sin_tab, slots, q_out, k_out, v_out, k_cache, v_cache, k_scale,
                                        v_scale, S(stream)),
                    "ms_qkv_post");
}

size_t ms_paged_decode_workspace_size(int B, int Hq, int Hkv, int max_blocks, int block_size) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || max_blocks <= 0 || block_size <= 0) return 0;
  const int splits = ms::decode_num_splits(B, Hkv, max_blocks, block_size, num_sms());
  return ms::decode_workspace_bytes(B, Hq, splits);
}

int ms_paged_decode_fp8(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                        const float* v_scale, const int32_t* seqlens, const int32_t* block_tables, void* out, int B,
                        int Hq, int Hkv, int head_dim, int block_size, int max_blocks, float softmax_scale,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || block_size <= 0 || max_blocks <= 0)
    return fail(MS_ERR_INVALID, "ms_paged_decode_fp8: bad sizes");
  if (B == 0) return MS_OK;
  if (!q || !k_cache || !v_cache || !k_scale || !v_scale || !seqlens || !block_tables || !out)
    return fail(MS_ERR_INVALID, "ms_paged_decode_fp8: null pointer");
  if (head_dim != 128 || Hq % Hkv != 0 || Hq / Hkv > 8 || block_size % 16 != 0)
    return fail(MS_ERR_UNSUPPORTED, "ms_paged_decode_fp8: head_dim=%d Hq=%d Hkv=%d block_size=%d unsupported",
                head_dim, Hq, Hkv, block_size);
  const int splits = ms::decode_num_splits(B, Hkv, max_blocks, block_size, num_sms());
  const size_t need = ms::decode_workspace_bytes(B, Hq, splits);
  if (workspace_bytes < need || (need > 0 && workspace == nullptr))
    return fail(MS_ERR_WORKSPACE, "ms_paged_decode_fp8: workspace %zu < %zu bytes", workspace_bytes, need);
  return check_cuda(ms::launch_decode_attention(q, k_cache, v_cache, k_scale, v_scale, seqlens, block_tables, out, B,
                                                Hq, Hkv, head_dim, block_size, max_blocks, softmax_scale, splits,
                                                workspace, S(stream)),
                    "ms_paged_decode_fp8");
}

int ms_paged_decode_fp8_noalloc(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                                const float* v_scale, const int32_t* seqlens, const int32_t* block_tables, void* out,
                                int B, int Hq, int Hkv, int head_dim, int block_size, int max_blocks,
                                float softmax_scale, void* stream) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || block_size <= 0 || max_blocks <= 0)
    return fail(MS_ERR_INVALID, "ms_paged_decode_fp8_noalloc: bad sizes");
  if (B == 0) return MS_OK;
  if (!q || !k_cache || !v_cache || !k_scale || !v_scale || !seqlens || !block_tables || !out)
    return fail(MS_ERR_INVALID, "ms_paged_decode_fp8_noalloc: null pointer");
  if (head_dim != 128 || Hq % Hkv != 0 || Hq / Hkv > 8 || block_size % 16 != 0)
    return fail(MS_ERR_UNSUPPORTED, "ms_paged_decode_fp8_noalloc: head_dim=%d Hq=%d Hkv=%d block_size=%d unsupported",
                head_dim, Hq, Hkv, block_size);
  const int splits = ms::decode_num_splits(B, Hkv, max_blocks, block_size, num_sms());
  const size_t need = ms::decode_workspace_bytes(B, Hq, splits);
  const size_t have = ms::decode_noalloc_scratch_bytes();
  if (need > have)
    return fail(MS_ERR_UNSUPPORTED,
                "ms_paged_decode_fp8_noalloc: this batch needs %zu bytes of scratch but the built-in buffer holds "
                "%zu bytes; use ms_paged_decode_fp8 with a caller-provided workspace",
                need, have);
  void* ws = nullptr;
  if (need > 0) {
    const cudaError_t e = ms::decode_noalloc_scratch(&ws);
    if (e != cudaSuccess) return check_cuda(e, "ms_paged_decode_fp8_noalloc: scratch address");
  }
  return check_cuda(ms::launch_decode_attention(q, k_cache, v_cache, k_scale, v_scale, seqlens, block_tables, out, B,
                                                Hq, Hkv, head_dim, block_size, max_blocks, softmax_scale, splits, ws,
                                                S(stream)),
                    "ms_paged_decode_fp8_noalloc");
}

int ms_paged_prefill_fp8(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                         const float* v_scale, const int32_t* block_tables, const int32_t* cu_q,
                         const int32_t* kv_lens, void* out, int num_seqs, int64_t total_q, int Hq, int Hkv,
                         int head_dim, int block_size, int max_blocks, float softmax_scale, void* stream) {
  if (num_seqs < 0 || total_q < 0 || Hq <= 0 || Hkv <= 0 || block_size <= 0 || max_blocks <= 0 ||
      total_q > INT32_MAX)
    return fail(MS_ERR_INVALID, "ms_paged_prefill_fp8: bad sizes");
  if (num_seqs == 0 || total_q == 0) return MS_OK;
  if (!q || !k_cache || !v_cache || !k_scale || !v_scale || !block_tables || !cu_q || !kv_lens || !out)
    return fail(MS_ERR_INVALID, "ms_paged_prefill_fp8: null pointer");
  if (head_dim != 128 || Hq % Hkv != 0 || 64 % (Hq / Hkv) != 0 || block_size % 64 != 0)
    return fail(MS_ERR_UNSUPPORTED, "ms_paged_prefill_fp8: head_dim=%d Hq=%d Hkv=%d block_size=%d unsupported",
                head_dim, Hq, Hkv, block_size);
  return check_cuda(ms::launch_prefill_attention(true, q, nullptr, nullptr, k_cache, v_cache, k_scale, v_scale,
                                                 block_tables, cu_q, kv_lens, out, num_seqs, (int)total_q, Hq, Hkv,
                                                 head_dim, block_size, max_blocks, softmax_scale, S(stream)),
                    "ms_paged_prefill_fp8");
}

int ms_varlen_prefill(const void* q, const void* k, const void* v, const int32_t* cu, void* out, int num_seqs,
                      int64_t total, int Hq, int Hkv, int head_dim, float softmax_scale, void* stream) {
  if (num_seqs < 0 || total < 0 || Hq <= 0 || Hkv <= 0 || total > INT32_MAX)
    return fail(MS_ERR_INVALID, "ms_varlen_prefill: bad sizes");
  if (num_seqs == 0 || total == 0) return MS_OK;
  if (!q || !k || !v || !cu || !out) return fail(MS_ERR_INVALID, "ms_varlen_prefill: null pointer");
  if (head_dim != 128 || Hq % Hkv != 0 || 64 % (Hq / Hkv) != 0)
    return fail(MS_ERR_UNSUPPORTED, "ms_varlen_prefill: head_dim=%d Hq=%d Hkv=%d unsupported", head_dim, Hq, Hkv);
  return check_cuda(ms::launch_prefill_attention(false, q, k, v, nullptr, nullptr, nullptr, nullptr, nullptr, cu,
                                                 nullptr, out, num_seqs, (int)total, Hq, Hkv, head_dim, 256, 1,
                                                 softmax_scale, S(stream)),
                    "ms_varlen_prefill");
}

size_t ms_argmax_workspace_size(int64_t M) { return M > 0 ? ms::argmax_workspace_bytes(M) : 0; }

int ms_argmax_rows(const void* x, int64_t M, int64_t V, int64_t ldx, int64_t* idx, float* vmax, void* workspace,
                   size_t workspace_bytes, void* stream) {
  if (M < 0 || V <= 0 || V > INT32_MAX || ldx < V || M > 16384)
    return fail(MS_ERR_INVALID, "ms_argmax_rows: bad sizes M=%lld V=%lld ldx=%lld", (long long)M, (long long)V,
                (long long)ldx);
  if (M == 0) return MS_OK;
  if (!x || !idx || !workspace) return fail(MS_ERR_INVALID, "ms_argmax_rows: null pointer");
  if (workspace_bytes < ms::argmax_workspace_bytes(M))
    return fail(MS_ERR_WORKSPACE, "ms_argmax_rows: workspace %zu < %zu bytes", workspace_bytes,
                ms::argmax_workspace_bytes(M));
  return check_cuda(ms::launch_argmax_rows(x, M, (int)V, ldx, idx, vmax, workspace, S(stream)), "ms_argmax_rows");
}

// --------------------------------------------------------------------------- tensor parallel
int ms_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return fail(MS_ERR_INVALID, "ms_ipc_handle: null pointer");
  // the allocation that holds ptr (driver entry point: the library does not link libcuda)
  typedef CUresult (*RangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<RangeFn>(f);
  });
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn == nullptr || range_fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS)
    return fail(MS_ERR_CUDA, "ms_ipc_handle: cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, (void*)base);
  if (e != cudaSuccess) return check_cuda(e, "ms_ipc_handle");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)((CUdeviceptr)ptr - base);
  return MS_OK;
}

int ms_ipc_open(const void* handle, int64_t offset, void** base_out, void** ptr_out) {
  if (!handle || !base_out || !ptr_out || offset < 0) return fail(MS_ERR_INVALID, "ms_ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return check_cuda(e, "ms_ipc_open");
  *base_out = base;
  *ptr_out = (char*)base + offset;
  return MS_OK;
}

int ms_ipc_close(void* base) {
  if (!base) return fail(MS_ERR_INVALID, "ms_ipc_close: null pointer");
  return check_cuda(cudaIpcCloseMemHandle(base), "ms_ipc_close");
}

int ms_tp_layout(int world, int64_t hidden, int64_t max_rows, int64_t* offsets) {
  if (world < 1 || world > 8 || hidden <= 0 || max_rows <= 0 || !offsets)
    return fail(MS_ERR_INVALID, "ms_tp_layout: bad arguments");
  const ms::TpLayout l = ms::tp_layout(world, hidden, max_rows);
  const int64_t o[5] = {l.partial, l.outq, l.outs, l.outh, l.total};
  memcpy(offsets, o, sizeof(o));
  return MS_OK;
}

int ms_tp_buffer_init(void* base, int world, int64_t hidden, int64_t max_rows, void* stream) {
  if (!base || world < 1 || world > 8 || hidden <= 0 || max_rows <= 0)
    return fail(MS_ERR_INVALID, "ms_tp_buffer_init: bad arguments");
  if (((uintptr_t)base & 255) != 0) return fail(MS_ERR_INVALID, "ms_tp_buffer_init: base not 256-byte aligned");
  return check_cuda(ms::launch_tp_buffer_init(base, world, hidden, max_rows, S(stream)), "ms_tp_buffer_init");
}

int ms_tp_allreduce_rmsnorm_fp8(void* const* bases, int rank, int world, int64_t hidden, int64_t max_rows,
                                void* residual, const void* weight, int64_t M, float eps, int want_fp16, int pushed,
                                void* stream) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world || M < 0 || max_rows <= 0 || M > max_rows ||
      max_rows > INT32_MAX || hidden <= 0)
    return fail(MS_ERR_INVALID, "ms_tp_allreduce_rmsnorm_fp8: bad sizes rank=%d world=%d M=%lld max_rows=%lld", rank,
                world, (long long)M, (long long)max_rows);
  if (hidden % 16 != 0 || hidden > 16384)
    return fail(MS_ERR_UNSUPPORTED, "ms_tp_allreduce_rmsnorm_fp8: hidden=%lld (needs a multiple of 16, <= 16384)",
                (long long)hidden);
  if (M == 0) return MS_OK;
  if (!bases || !residual || !weight) return fail(MS_ERR_INVALID, "ms_tp_allreduce_rmsnorm_fp8: null pointer");
  for (int p = 0; p < world; ++p)
    if (!bases[p] || ((uintptr_t)bases[p] & 255) != 0)
      return fail(MS_ERR_INVALID, "ms_tp_allreduce_rmsnorm_fp8: buffer of rank %d null or not 256-byte aligned", p);
  if (((uintptr_t)residual & 15) != 0 || ((uintptr_t)weight & 15) != 0)
    return fail(MS_ERR_INVALID, "ms_tp_allreduce_rmsnorm_fp8: residual/weight not 16-byte aligned");
  return check_cuda(ms::launch_tp_allreduce_rmsnorm_fp8(bases, rank, world, hidden, max_rows, residual, weight,
                                                        (int)M, eps, want_fp16, pushed, num_sms(), S(stream)),
                    "ms_tp_allreduce_rmsnorm_fp8");
}

int ms_fp8_gemm_rowpar(const void* xq, const float* sx, const void* wq, const float* sw, int64_t M, int64_t N,
                       int64_t K, void* workspace, size_t workspace_bytes, void* const* bases, int rank, int world,
                       int64_t max_rows, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || M > max_rows || max_rows > INT32_MAX || N > 16384 || K > INT32_MAX ||
      world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(MS_ERR_INVALID, "ms_fp8_gemm_rowpar: bad sizes M=%lld N=%lld K=%lld rank=%d world=%d", (long long)M,
                (long long)N, (long long)K, rank, world);
  if (M == 0) return MS_OK;
  if (N % 16 != 0 || K % 16 != 0)
    return fail(MS_ERR_UNSUPPORTED, "ms_fp8_gemm_rowpar: N and K must be multiples of 16");
  if (!xq || !sx || !wq || !sw || !bases) return fail(MS_ERR_INVALID, "ms_fp8_gemm_rowpar: null pointer");
  for (int p = 0; p < world; ++p)
    if (!bases[p] || ((uintptr_t)bases[p] & 255) != 0)
      return fail(MS_ERR_INVALID, "ms_fp8_gemm_rowpar: buffer of rank %d null or not 256-byte aligned", p);
  const size_t need = ms::gemm_workspace_bytes((int)M, (int)N, (int)K, num_sms());
  if (workspace_bytes < need || (need > 0 && workspace == nullptr))
    return fail(MS_ERR_WORKSPACE, "ms_fp8_gemm_rowpar: workspace %zu < %zu bytes", workspace_bytes, need);
  const ms::TpRows rp = ms::tp_rows_args(bases, rank, world, N, max_rows, (int)M);
  return check_cuda(ms::launch_fp8_gemm(xq, sx, wq, sw, nullptr, nullptr, (int)M, (int)N, (int)K, workspace,
                                        workspace_bytes, num_sms(), S(stream), &rp),
                    "ms_fp8_gemm_rowpar");
}

int ms_fp8_gemm_rowpar_ar_rmsnorm(const void* xq, const float* sx, const void* wq, const float* sw, int64_t M,
                                  int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* const* bases,
                                  int rank, int world, int64_t max_rows, void* residual, const void* weight,
                                  float eps, int want_fp16, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || M > max_rows || max_rows > INT32_MAX || N > 16384 || K > INT32_MAX ||
      world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(MS_ERR_INVALID, "ms_fp8_gemm_rowpar_ar_rmsnorm: bad sizes M=%lld N=%lld K=%lld rank=%d world=%d",
                (long long)M, (long long)N, (long long)K, rank, world);
  if (M == 0) return MS_OK;
  if (N % 16 != 0 || K % 16 != 0)
    return fail(MS_ERR_UNSUPPORTED, "ms_fp8_gemm_rowpar_ar_rmsnorm: N and K must be multiples of 16");
  if (!xq || !sx || !wq || !sw || !bases || !residual || !weight)
    return fail(MS_ERR_INVALID, "ms_fp8_gemm_rowpar_ar_rmsnorm: null pointer");
  for (int p = 0; p < world; ++p)
    if (!bases[p] || ((uintptr_t)bases[p] & 255) != 0)
      return fail(MS_ERR_INVALID, "ms_fp8_gemm_rowpar_ar_rmsnorm: buffer of rank %d null or not 256-byte aligned",
                  p);
  if (((uintptr_t)residual & 15) != 0 || ((uintptr_t)weight & 15) != 0)
    return fail(MS_ERR_INVALID, "ms_fp8_gemm_rowpar_ar_rmsnorm: residual/weight not 16-byte aligned");
  const size_t need = ms::gemm_workspace_bytes((int)M, (int)N, (int)K, num_sms());
  if (workspace_bytes < need || (need > 0 && workspace == nullptr))
    return fail(MS_ERR_WORKSPACE, "ms_fp8_gemm_rowpar_ar_rmsnorm: workspace %zu < %zu bytes", workspace_bytes,
                need);
  ms::TpRows rp = ms::tp_rows_args(bases, rank, world, N, max_rows, (int)M);
  rp.residual = static_cast<__half*>(residual);
  rp.weight = static_cast<const __half*>(weight);
  rp.eps = eps;
  rp.want_h = want_fp16 ? 1 : 0;
  rp.pushed = 1;
  bool tail = true;
  const int rc = check_cuda(ms::launch_fp8_gemm(xq, sx, wq, sw, nullptr, nullptr, (int)M, (int)N, (int)K, workspace,
                                                workspace_bytes, num_sms(), S(stream), &rp, &tail),
                            "ms_fp8_gemm_rowpar_ar_rmsnorm");
  if (rc != MS_OK || tail) return rc;
  // the row work did not fit the GEMM's tail (many rows per CTA, or a very wide row):
  // the separate op on the pushed rows
  return check_cuda(ms::launch_tp_allreduce_rmsnorm_fp8(bases, rank, world, N, max_rows, residual, weight, (int)M,
                                                        eps, want_fp16, 1, num_sms(), S(stream)),
                    "ms_fp8_gemm_rowpar_ar_rmsnorm");
}

int ms_set_wait_limit(uint64_t ns) {
  if (ns == 0) return fail(MS_ERR_INVALID, "ms_set_wait_limit: limit must be > 0");
  const unsigned long long v = ns;
  return check_cuda(cudaMemcpyToSymbol(ms::g_wait_limit_ns, &v, sizeof(v)), "ms_set_wait_limit");
}

int ms_row_amax(const void* x, int64_t ldx, int64_t M, int64_t K, float* amax, void* stream) {
  if (M < 0 || K <= 0 || ldx < K || K > (1 << 20)) return fail(MS_ERR_INVALID, "ms_row_amax: bad sizes");
  if (M == 0) return MS_OK;
  if (!x || !amax) return fail(MS_ERR_INVALID, "ms_row_amax: null pointer");
  return check_cuda(ms::launch_row_amax(x, ldx, M, (int)K, amax, S(stream)), "ms_row_amax");
}

int ms_quantize_rows_fp8_amax(const void* x, int64_t ldx, int64_t M, int64_t K, const float* amax, void* xq,
                              float* sx, void* stream) {
  if (M < 0 || K <= 0 || ldx < K || K > (1 << 20)) return fail(MS_ERR_INVALID, "ms_quantize_rows_fp8_amax: bad sizes");
  if (M == 0) return MS_OK;
  if (!x || !amax || !xq || !sx) return fail(MS_ERR_INVALID, "ms_quantize_rows_fp8_amax: null pointer");
  return check_cuda(ms::launch_quantize_rows_amax(x, ldx, M, (int)K, amax, xq, sx, S(stream)),
                    "ms_quantize_rows_fp8_amax");
}

}  // extern "C"
