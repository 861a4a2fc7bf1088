// Row-wise kernels of the FP8 decoder layer: per-row FP8 quantisation,
// (residual +) RMSNorm with an optional FP8 epilogue, SiLU*mul with an
// optional FP8 epilogue. They are short and latency-bound: a row belongs to a
// group of 1-8 warps that copies the row into shared memory with cp.async up
// front (every byte in flight at once), so the amax needed by the FP8 scale is
// known before any byte is written; outputs are written as 8- or 16-byte
// vectors.
//
// Reference semantics followed (microserve, file:line):
//   quantize rows      layers/fp8_linear.py:14-23   (and the offline weight quant :51-54)
//   residual RMSNorm   layers/layernorm.py:22-42    (residual rounded to fp16 before the norm)
//   plain RMSNorm      layers/layernorm.py:7-19
//   SiLU*mul           layers/activation.py:5-8     (silu in fp32 -> fp16, then fp16 multiply)
#include "common.cuh"
#include "kernels.h"
#include "rowops.cuh"

namespace ms {
namespace {

constexpr int kRowThreads = 512;

// x: [M, K] fp16 with row stride ldx (elements), any K and alignment (scalar
// loads and stores; irregular layer widths). Writes xq [M, K] e4m3 and sx [M].
__global__ void __launch_bounds__(kRowThreads) quantize_rows_scalar_kernel(const __half* __restrict__ x,
                                                                          int64_t ldx, int K,
                                                                          uint8_t* __restrict__ xq,
                                                                          float* __restrict__ sx) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* row = reinterpret_cast<__half*>(smem_raw);
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;
  const __half* xr = x + m * ldx;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const __half a = xr[k];
    amax = fmaxf(amax, fabsf(__half2float(a)));
    row[k] = a;
  }
  amax = block_reduce<true>(amax, red);
  const float scale = fp8_scale_from_amax(amax);
  for (int k = threadIdx.x; k < K; k += blockDim.x)
    xq[m * (int64_t)K + k] = f32_to_e4m3(__half2float(row[k]) / scale);
  if (threadIdx.x == 0) sx[m] = scale;
}

// ---------------------------------------------------------------------------
// Row-group kernels: W warps per row (T = 32 W threads), one row per CTA
// (blockDim = T). Each thread loads its own 16-byte vectors (v = t, t + T, ...,
// at most kRowVec of them) into registers, all loads issued before any is used,
// and keeps them there: no shared-memory staging, so a CTA fits beside a GEMM
// CTA (~195 KB of shared memory) and, launched early under programmatic
// dependent launch, starts the moment that GEMM ends. A row's reductions are
// warp shuffles plus, for W > 1, one named barrier (one 512-thread CTA per row
// spent about a microsecond in each block-wide reduction). FP8 codes use
// div_by_rcp: the IEEE quotient x / scale in five flops.
// ---------------------------------------------------------------------------
// Reduction over the T threads of the CTA's row (red: a distinct shared array
// of kMaxRowWarps floats per reduction, so none is reused).
template <int W, bool kMax>
__device__ __forceinline__ float group_reduce(float v, float* red, int t) {
  v = kMax ? warp_max(v) : warp_sum(v);
  if constexpr (W == 1) {
    return v;
  } else {
    if ((t & 31) == 0) red[t >> 5] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < W; ++i) r = kMax ? fmaxf(r, red[i]) : r + red[i];
    return r;
  }
}

// Per-row FP8 quantisation (16-byte aligned rows, K % 16 == 0, K / 8 <= kRowVec * T).
// amax_in: row amax given (exact scales of a K-sharded row); amax_out: write the
// row amax and nothing else.
template <int W>
__global__ void __launch_bounds__(32 * W) quantize_rows_group_kernel(const __half* __restrict__ x, int64_t ldx, int K,
                                                                    uint8_t* __restrict__ xq, float* __restrict__ sx,
                                                                    const float* __restrict__ amax_in,
                                                                    float* __restrict__ amax_out) {
  __shared__ float red_max[kMaxRowWarps];
  constexpr int T = 32 * W;
  const int t = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;
  const int nv = K / 8;
  const __half* xr = x + m * ldx;
  H8 a[kRowVec];
#pragma unroll
  for (int i = 0; i < kRowVec; ++i)
    if (t + i * T < nv) a[i] = ld_h8(xr + (t + i * T) * 8);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kRowVec; ++i)
    if (t + i * T < nv) amax = amax8(a[i], amax);
  amax = group_reduce<W, true>(amax, red_max, t);
  if (amax_out != nullptr) {
    if (t == 0) amax_out[m] = amax;
    return;
  }
  if (amax_in != nullptr) amax = amax_in[m];
  const float scale = fp8_scale_from_amax(amax), rcp = 1.0f / scale;
  uint8_t* dst = xq + m * (int64_t)K;
#pragma unroll
  for (int i = 0; i < kRowVec; ++i)
    if (t + i * T < nv) *reinterpret_cast<uint2*>(dst + (size_t)(t + i * T) * 8) = encode8(a[i], scale, rcp);
  if (t == 0) sx[m] = scale;
}

// (residual +) RMSNorm with optional fp16 / FP8 outputs: r' = fp16(x + r)
// (written to residual_out) when a residual is given, y = fp16(fp16(v *
// rsqrt(mean(v^2) + eps)) * w) for v = r' (or x), FP8 row quantisation of y.
template <int W>
__global__ void __launch_bounds__(32 * W) rmsnorm_group_kernel(const __half* __restrict__ x,
                                                              const __half* __restrict__ residual,
                                                              const __half* __restrict__ weight, int H, float eps,
                                                              __half* __restrict__ residual_out,
                                                              __half* __restrict__ y, uint8_t* __restrict__ yq,
                                                              float* __restrict__ sy) {
  __shared__ float red_ss[kMaxRowWarps];
  __shared__ float red_max[kMaxRowWarps];
  constexpr int T = 32 * W;
  const int t = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;
  const int nv = H / 8;
  const int64_t base = m * (int64_t)H;
  H8 a[kRowVec], w[kRowVec];
#pragma unroll
  for (int i = 0; i < kRowVec; ++i) {
    if (t + i * T < nv) {
      a[i] = ld_h8(x + base + (t + i * T) * 8);
      w[i] = ld_h8(weight + (t + i * T) * 8);
    }
  }
  if (residual != nullptr) {
    H8 r[kRowVec];
#pragma unroll
    for (int i = 0; i < kRowVec; ++i)
      if (t + i * T < nv) r[i] = ld_h8(residual + base + (t + i * T) * 8);
#pragma unroll
    for (int i = 0; i < kRowVec; ++i) {
      if (t + i * T < nv) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fa = __half22float2(a[i].h[j]);
          const float2 fr = __half22float2(r[i].h[j]);
          a[i].h[j] = __floats2half2_rn(fa.x + fr.x, fa.y + fr.y);
        }
        st_h8(residual_out + base + (t + i * T) * 8, a[i]);
      }
    }
  }
  float ss = 0.f;  // the canonical sum of squares (rowops.cuh), shared with the TP op
#pragma unroll
  for (int i = 0; i < kRowVec; ++i)
    if (t + i * T < nv) ss = sumsq8(a[i], ss);
  ss = group_reduce<W, false>(ss, red_ss, t);
  const float inv = rsqrtf(ss / (float)H + eps);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kRowVec; ++i) {
    if (t + i * T < nv) {
      a[i] = norm8(a[i], w[i], inv);
      amax = amax8(a[i], amax);
      if (y != nullptr) st_h8(y + base + (t + i * T) * 8, a[i]);
    }
  }
  if (yq == nullptr) return;
  amax = group_reduce<W, true>(amax, red_max, t);
  const float scale = fp8_scale_from_amax(amax), rcp = 1.0f / scale;
#pragma unroll
  for (int i = 0; i < kRowVec; ++i)
    if (t + i * T < nv) *reinterpret_cast<uint2*>(yq + base + (size_t)(t + i * T) * 8) = encode8(a[i], scale, rcp);
  if (t == 0) sy[m] = scale;
}

// gu: [M, 2I] fp16 (gate | up). a = fp16(fp16(silu(g)) * u), optional fp16 and FP8 outputs.
template <int W>
__global__ void __launch_bounds__(32 * W) silu_mul_group_kernel(const __half* __restrict__ gu, int I,
                                                               __half* __restrict__ out, uint8_t* __restrict__ aq,
                                                               float* __restrict__ sa) {
  __shared__ float red_max[kMaxRowWarps];
  constexpr int T = 32 * W;
  const int t = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;
  const int nv = I / 8;
  const __half* g = gu + m * (int64_t)(2 * I);
  H8 a[kRowVec], b[kRowVec];
#pragma unroll
  for (int i = 0; i < kRowVec; ++i) {
    if (t + i * T < nv) {
      a[i] = ld_h8(g + (t + i * T) * 8);
      b[i] = ld_h8(g + I + (t + i * T) * 8);
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kRowVec; ++i) {
    if (t + i * T < nv) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __half22float2(a[i].h[j]);
        const __half2 sg = __floats2half2_rn(fa.x / (1.0f + expf(-fa.x)), fa.y / (1.0f + expf(-fa.y)));
        a[i].h[j] = __hmul2(sg, b[i].h[j]);
      }
      amax = amax8(a[i], amax);
      if (out != nullptr) st_h8(out + m * (int64_t)I + (t + i * T) * 8, a[i]);
    }
  }
  if (aq == nullptr) return;
  amax = group_reduce<W, true>(amax, red_max, t);
  const float scale = fp8_scale_from_amax(amax), rcp = 1.0f / scale;
  uint8_t* dst = aq + m * (int64_t)I;
#pragma unroll
  for (int i = 0; i < kRowVec; ++i)
    if (t + i * T < nv) *reinterpret_cast<uint2*>(dst + (size_t)(t + i * T) * 8) = encode8(a[i], scale, rcp);
  if (t == 0) sa[m] = scale;
}

// Opt a kernel in to the largest dynamic shared memory these launchers request
// (200 KB), once per kernel (a function-local static at each call site); the
// default 48 KB limit also counts the static reduction buffer.
#define ALLOW_BIG_SMEM(kernel)                                                                        \
  do {                                                                                                \
    static const cudaError_t set_once =                                                               \
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);       \
    (void)set_once;                                                                                   \
  } while (0)

inline int row_threads(int K) {
  int t = (K + 7) / 8;
  t = (t + 31) / 32 * 32;
  return t < kRowThreads ? (t < 32 ? 32 : t) : kRowThreads;
}

#define MS_ROW_SWITCH(w, CALL) \
  switch (w) {                 \
    case 1: return CALL(1);    \
    case 2: return CALL(2);    \
    case 4: return CALL(4);    \
    case 8: return CALL(8);    \
    case 16: return CALL(16);  \
    default: return cudaErrorInvalidValue; \
  }

}  // namespace

cudaError_t launch_quantize_rows(const void* x, int64_t ldx, int64_t M, int K, void* xq, float* sx,
                                 cudaStream_t stream) {
  if (M == 0 || K == 0) return cudaSuccess;
  const size_t smem = (size_t)K * 2;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  const bool vec = (K % 16 == 0) && (ldx % 8 == 0) && (((uintptr_t)x & 15) == 0) && (((uintptr_t)xq & 15) == 0);
  if (vec && row_warps(K / 8) > 0) {
#define MS_CALL(W)                                                                                      \
  launch_kernel(quantize_rows_group_kernel<W>, dim3((unsigned)M), dim3(32 * W), 0, stream, (const __half*)x, \
                ldx, K, (uint8_t*)xq, sx, (const float*)nullptr, (float*)nullptr)
    MS_ROW_SWITCH(row_warps(K / 8), MS_CALL)
#undef MS_CALL
  } else {
    ALLOW_BIG_SMEM(quantize_rows_scalar_kernel);
    return launch_kernel(quantize_rows_scalar_kernel, dim3((unsigned)M), dim3(row_threads(K)), smem, stream,
                         (const __half*)x, ldx, K, (uint8_t*)xq, sx);
  }
}

static bool rows_vectorised(const void* x, int64_t ldx, int K) {
  return (K % 16 == 0) && (ldx % 8 == 0) && (((uintptr_t)x & 15) == 0) && row_warps(K / 8) > 0;
}

cudaError_t launch_row_amax(const void* x, int64_t ldx, int64_t M, int K, float* amax, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (!rows_vectorised(x, ldx, K)) return cudaErrorInvalidValue;
#define MS_CALL(W)                                                                                      \
  launch_kernel(quantize_rows_group_kernel<W>, dim3((unsigned)M), dim3(32 * W), 0, stream, (const __half*)x, \
                ldx, K, (uint8_t*)nullptr, (float*)nullptr, (const float*)nullptr, amax)
  MS_ROW_SWITCH(row_warps(K / 8), MS_CALL)
#undef MS_CALL
}

cudaError_t launch_quantize_rows_amax(const void* x, int64_t ldx, int64_t M, int K, const float* amax, void* xq,
                                      float* sx, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (!rows_vectorised(x, ldx, K) || ((uintptr_t)xq & 15) != 0) return cudaErrorInvalidValue;
#define MS_CALL(W)                                                                                      \
  launch_kernel(quantize_rows_group_kernel<W>, dim3((unsigned)M), dim3(32 * W), 0, stream, (const __half*)x, \
                ldx, K, (uint8_t*)xq, sx, amax, (float*)nullptr)
  MS_ROW_SWITCH(row_warps(K / 8), MS_CALL)
#undef MS_CALL
}

cudaError_t launch_rmsnorm(const void* x, const void* residual, const void* weight, int64_t M, int H, float eps,
                           void* residual_out, void* y, void* yq, float* sy, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (H % 16 != 0 || row_warps(H / 8) == 0) return cudaErrorInvalidValue;
#define MS_CALL(W)                                                                                          \
  launch_kernel(rmsnorm_group_kernel<W>, dim3((unsigned)M), dim3(32 * W), 0, stream, (const __half*)x,       \
                (const __half*)residual, (const __half*)weight, H, eps, (__half*)residual_out, (__half*)y,   \
                (uint8_t*)yq, sy)
  MS_ROW_SWITCH(row_warps(H / 8), MS_CALL)
#undef MS_CALL
}

cudaError_t launch_silu_mul(const void* gu, int64_t M, int I, void* out, void* aq, float* sa, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (I % 16 != 0 || row_warps(I / 8) == 0) return cudaErrorInvalidValue;
#define MS_CALL(W)                                                                                               \
  launch_kernel(silu_mul_group_kernel<W>, dim3((unsigned)M), dim3(32 * W), 0, stream, (const __half*)gu, I,       \
                (__half*)out, (uint8_t*)aq, sa)
  MS_ROW_SWITCH(row_warps(I / 8), MS_CALL)
#undef MS_CALL
}

}  // namespace ms
