// FP8 KV-cache writes.
//
//  * store_kv_fp8: the reference's `store_fp8_kvcache`
//    (microserve/layers/fp8_kv_cache.py:11-61): per (token, kv head) an fp32
//    scale = max(amax over head_dim, 1e-8) / 448 and e4m3 codes of x / scale,
//    scattered to `slot` of a [num_blocks, block_size, kv_heads, head_dim]
//    cache. Bit-exact target.
//  * qkv_post: the attention prologue of Qwen3Attention.forward
//    (microserve/models/qwen3.py:44-53) fused into one pass over the QKV GEMM
//    output: per-head q/k RMSNorm (torch path of layers/layernorm.py:55-57,82-83),
//    neox RoPE with fp16 cos/sin tables (layers/rotary_embedding.py:24-31,
//    every product and sum rounded to fp16 as torch does), then the FP8 store
//    of k and v. One warp per (token, head); lane l owns elements 4l..4l+3 so
//    the rotate-half partner (d +- 64) sits in lane l^16.
#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kHeadDim = 128;

struct alignas(8) H4 {
  __half2 a, b;
};

__device__ __forceinline__ void quant_store_head(const float (&v)[4], int64_t slot, int kv_heads, int head,
                                                 uint8_t* __restrict__ cache, float* __restrict__ scale_cache) {
  const int lane = threadIdx.x & 31;
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float s = fp8_scale_from_amax(amax);
  uint16_t lo = f32x2_to_e4m3x2(v[0] / s, v[1] / s);
  uint16_t hi = f32x2_to_e4m3x2(v[2] / s, v[3] / s);
  const int64_t row = slot * kv_heads + head;
  reinterpret_cast<uint32_t*>(cache + row * kHeadDim)[lane] = (uint32_t)lo | ((uint32_t)hi << 16);
  if (lane == 0) scale_cache[row] = s;
}

__global__ void __launch_bounds__(256) store_kv_fp8_kernel(const __half* __restrict__ k, const __half* __restrict__ v,
                                                           int64_t T, int kv_heads, const int64_t* __restrict__ slots,
                                                           uint8_t* __restrict__ k_cache,
                                                           uint8_t* __restrict__ v_cache, float* __restrict__ k_scale,
                                                           float* __restrict__ v_scale) {
  pdl_wait();
  pdl_trigger();
  const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (item >= T * kv_heads) return;
  const int64_t t = item / kv_heads;
  const int h = (int)(item % kv_heads);
  const int lane = threadIdx.x & 31;
  const int64_t slot = slots[t];
  if (slot < 0) return;
  H4 kk = reinterpret_cast<const H4*>(k + item * kHeadDim)[lane];
  H4 vv = reinterpret_cast<const H4*>(v + item * kHeadDim)[lane];
  float kf[4], vf[4];
  float2 t0 = __half22float2(kk.a), t1 = __half22float2(kk.b);
  kf[0] = t0.x; kf[1] = t0.y; kf[2] = t1.x; kf[3] = t1.y;
  t0 = __half22float2(vv.a); t1 = __half22float2(vv.b);
  vf[0] = t0.x; vf[1] = t0.y; vf[2] = t1.x; vf[3] = t1.y;
  quant_store_head(kf, slot, kv_heads, h, k_cache, k_scale);
  quant_store_head(vf, slot, kv_heads, h, v_cache, v_scale);
}

struct QkvPostArgs {
  const __half* qkv;  // [T, (Hq + 2 Hkv) * D]
  int64_t T;
  int q_heads, kv_heads;
  const __half* q_norm_w;  // [D] or null (no q/k norm)
  const __half* k_norm_w;
  float eps;
  const int64_t* positions;  // [T]
  const __half* cos_tab;     // [max_pos, D/2]
  const __half* sin_tab;
  const int64_t* slots;  // [T] or null (no cache write)
  __half* q_out;         // [T, Hq, D]
  __half* k_out;         // [T, Hkv, D] or null
  __half* v_out;         // [T, Hkv, D] or null
  uint8_t* k_cache;
  uint8_t* v_cache;
  float* k_scale;
  float* v_scale;
};

__device__ __forceinline__ void head_rmsnorm(float (&x)[4], const __half* __restrict__ w, float eps) {
  const int lane = threadIdx.x & 31;
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)kHeadDim + eps);
  H4 wv = reinterpret_cast<const H4*>(w)[lane];
  __half2 n0 = __floats2half2_rn(x[0] * inv, x[1] * inv);
  __half2 n1 = __floats2half2_rn(x[2] * inv, x[3] * inv);
  n0 = __hmul2(n0, wv.a);
  n1 = __hmul2(n1, wv.b);
  float2 a = __half22float2(n0), b = __half22float2(n1);
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}

// x holds fp16-exact values; returns fp16(fp16(x*cos) + fp16(rot*sin)).
__device__ __forceinline__ void head_rope(float (&x)[4], const __half* __restrict__ cos_row,
                                          const __half* __restrict__ sin_row) {
  const int lane = threadIdx.x & 31;
  float p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, x[i], 16);
  const int f = (lane & 15) * 4;
  H4 c = *reinterpret_cast<const H4*>(cos_row + f);
  H4 s = *reinterpret_cast<const H4*>(sin_row + f);
  __half cs[4] = {__low2half(c.a), __high2half(c.a), __low2half(c.b), __high2half(c.b)};
  __half sn[4] = {__low2half(s.a), __high2half(s.a), __low2half(s.b), __high2half(s.b)};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half xi = __float2half_rn(x[i]);
    __half rot = __float2half_rn(lane < 16 ? -p[i] : p[i]);
    // __hmul_rn: each product rounded to fp16 on its own (no fma contraction), as torch does
    __half r = __hadd(__hmul_rn(xi, cs[i]), __hmul_rn(rot, sn[i]));
    x[i] = __half2float(r);
  }
}

__global__ void __launch_bounds__(256) qkv_post_kernel(QkvPostArgs a) {
  pdl_wait();
  pdl_trigger();
  const int heads = a.q_heads + 2 * a.kv_heads;
  const int hd = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (hd >= heads) return;
  const int64_t t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const __half* src = a.qkv + t * (int64_t)heads * kHeadDim + (int64_t)hd * kHeadDim;
  H4 xv = reinterpret_cast<const H4*>(src)[lane];
  float x[4];
  {
    float2 t0 = __half22float2(xv.a), t1 = __half22float2(xv.b);
    x[0] = t0.x; x[1] = t0.y; x[2] = t1.x; x[3] = t1.y;
  }
  const bool is_q = hd < a.q_heads;
  const bool is_k = !is_q && hd < a.q_heads + a.kv_heads;
  if (is_q || is_k) {
    if (a.q_norm_w != nullptr) head_rmsnorm(x, is_q ? a.q_norm_w : a.k_norm_w, a.eps);
    const int64_t pos = a.positions[t];
    head_rope(x, a.cos_tab + pos * (kHeadDim / 2), a.sin_tab + pos * (kHeadDim / 2));
  }
  H4 o;
  o.a = __floats2half2_rn(x[0], x[1]);
  o.b = __floats2half2_rn(x[2], x[3]);
  if (is_q) {
    reinterpret_cast<H4*>(a.q_out + (t * a.q_heads + hd) * kHeadDim)[lane] = o;
    return;
  }
  const int kvh = is_k ? hd - a.q_heads : hd - a.q_heads - a.kv_heads;
  __half* dst16 = is_k ? a.k_out : a.v_out;
  if (dst16 != nullptr) reinterpret_cast<H4*>(dst16 + (t * a.kv_heads + kvh) * kHeadDim)[lane] = o;
  if (a.slots == nullptr) return;
  const int64_t slot = a.slots[t];
  if (slot < 0) return;
  quant_store_head(x, slot, a.kv_heads, kvh, is_k ? a.k_cache : a.v_cache, is_k ? a.k_scale : a.v_scale);
}

}  // namespace

cudaError_t launch_store_kv_fp8(const void* k, const void* v, int64_t T, int kv_heads, int head_dim,
                                const int64_t* slots, void* k_cache, void* v_cache, float* k_scale, float* v_scale,
                                cudaStream_t stream) {
  if (head_dim != kHeadDim) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  const int64_t items = T * kv_heads;
  return launch_kernel(store_kv_fp8_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0, stream, (const __half*)k,
                       (const __half*)v, T, kv_heads, slots, (uint8_t*)k_cache, (uint8_t*)v_cache, k_scale, v_scale);
}

cudaError_t launch_qkv_post(const void* qkv, int64_t T, int q_heads, int kv_heads, int head_dim, const void* q_norm_w,
                            const void* k_norm_w, float eps, const int64_t* positions, const void* cos_tab,
                            const void* sin_tab, const int64_t* slots, void* q_out, void* k_out, void* v_out,
                            void* k_cache, void* v_cache, float* k_scale, float* v_scale, cudaStream_t stream) {
  if (head_dim != kHeadDim) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  QkvPostArgs a;
  a.qkv = (const __half*)qkv;
  a.T = T;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.q_norm_w = (const __half*)q_norm_w;
  a.k_norm_w = (const __half*)k_norm_w;
  a.eps = eps;
  a.positions = positions;
  a.cos_tab = (const __half*)cos_tab;
  a.sin_tab = (const __half*)sin_tab;
  a.slots = slots;
  a.q_out = (__half*)q_out;
  a.k_out = (__half*)k_out;
  a.v_out = (__half*)v_out;
  a.k_cache = (uint8_t*)k_cache;
  a.v_cache = (uint8_t*)v_cache;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  const int heads = q_heads + 2 * kv_heads;
  dim3 grid((unsigned)T, (unsigned)((heads + 7) / 8));
  return launch_kernel(qkv_post_kernel, grid, dim3(256), 0, stream, a);
}

}  // namespace ms
