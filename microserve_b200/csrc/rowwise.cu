// Row-wise kernels of the FP8 decoder layer: per-row FP8 quantisation,
// (residual +) RMSNorm with an optional FP8 epilogue, SiLU*mul with an
// optional FP8 epilogue. All are HBM-bound; each CTA owns one row and copies
// all of its inputs into shared memory with cp.async up front (every byte of
// the row in flight at once: these kernels are short and latency-bound), so the
// amax needed by the FP8 scale is known before any byte is written; outputs are
// written as 16-byte vectors.
//
// Reference semantics followed (microserve, file:line):
//   quantize rows      layers/fp8_linear.py:14-23   (and the offline weight quant :51-54)
//   residual RMSNorm   layers/layernorm.py:22-42    (residual rounded to fp16 before the norm)
//   plain RMSNorm      layers/layernorm.py:7-19
//   SiLU*mul           layers/activation.py:5-8     (silu in fp32 -> fp16, then fp16 multiply)
#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kRowThreads = 512;

// Copy n16 16-byte chunks global -> shared with cp.async (L2 only), spread over
// the block; completes with cp_async_wait_all().
__device__ __forceinline__ void stage_row(void* dst_smem, const void* src, int n16) {
  const uint32_t d = smem_u32(dst_smem);
  const char* sp = static_cast<const char*>(src);
  for (int v = threadIdx.x; v < n16; v += blockDim.x)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d + 16u * v), "l"(sp + (size_t)16 * v)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();
}

struct alignas(16) H8 {
  __half2 h[4];
};

__device__ __forceinline__ void store_fp8_row(const __half* __restrict__ src_smem, int K, float scale,
                                              uint8_t* __restrict__ dst) {
  // dst row of K bytes, K % 16 == 0: each thread writes 16 bytes at a time.
  for (int v = threadIdx.x; v < K / 16; v += blockDim.x) {
    const H8* s = reinterpret_cast<const H8*>(src_smem + v * 16);
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      H8 x = s[j];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        float2 a = __half22float2(x.h[2 * p]);
        float2 b = __half22float2(x.h[2 * p + 1]);
        uint16_t lo = f32x2_to_e4m3x2(a.x / scale, a.y / scale);
        uint16_t hi = f32x2_to_e4m3x2(b.x / scale, b.y / scale);
        w[2 * j + p] = (uint32_t)lo | ((uint32_t)hi << 16);
      }
    }
    *reinterpret_cast<uint4*>(dst + (size_t)v * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// x: [M, K] fp16 with row stride ldx (elements). Writes xq [M, K] e4m3 and sx [M].
// kVec: K % 16 == 0 and 16-byte aligned rows (16-byte vectors); else scalar
// loads and stores (irregular layer widths).
template <bool kVec>
__global__ void __launch_bounds__(kRowThreads) quantize_rows_kernel(const __half* __restrict__ x, int64_t ldx,
                                                                   int K, uint8_t* __restrict__ xq,
                                                                   float* __restrict__ sx) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* row = reinterpret_cast<__half*>(smem_raw);
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;
  const __half* xr = x + m * ldx;
  float amax = 0.f;
  if (kVec) {
    stage_row(row, xr, K / 8);
    cp_async_wait_all();
    for (int v = threadIdx.x; v < K / 8; v += blockDim.x) {
      H8 a = *reinterpret_cast<const H8*>(row + v * 8);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(a.h[j]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const __half a = xr[k];
      amax = fmaxf(amax, fabsf(__half2float(a)));
      row[k] = a;
    }
  }
  amax = block_reduce<true>(amax, red);
  const float scale = fp8_scale_from_amax(amax);
  if (kVec) {
    store_fp8_row(row, K, scale, xq + m * (int64_t)K);
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x)
      xq[m * (int64_t)K + k] = f32_to_e4m3(__half2float(row[k]) / scale);
  }
  if (threadIdx.x == 0) sx[m] = scale;
}

// (residual +) RMSNorm. If residual != nullptr: r' = fp16(x + r) is written to
// residual_out and normalised; else x is normalised. y = fp16(fp16(v * rsqrt(mean(v^2) + eps)) * w).
// Optional outputs: y (fp16), yq/sy (FP8 row quantisation of y).
__global__ void __launch_bounds__(kRowThreads) rmsnorm_kernel(const __half* __restrict__ x,
                                                             const __half* __restrict__ residual,
                                                             const __half* __restrict__ weight, int H, float eps,
                                                             __half* __restrict__ residual_out,
                                                             __half* __restrict__ y, uint8_t* __restrict__ yq,
                                                             float* __restrict__ sy) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* row = reinterpret_cast<__half*>(smem_raw);
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;
  const int64_t base = m * (int64_t)H;
  __half* rres = row + H;     // residual row
  __half* wrow = row + 2 * H;  // weight
  stage_row(row, x + base, H / 8);
  if (residual != nullptr) stage_row(rres, residual + base, H / 8);
  stage_row(wrow, weight, H / 8);
  cp_async_wait_all();
  float ss = 0.f;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    H8 a = *reinterpret_cast<const H8*>(row + v * 8);
    if (residual != nullptr) {
      H8 r = *reinterpret_cast<const H8*>(rres + v * 8);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 fa = __half22float2(a.h[j]);
        float2 fr = __half22float2(r.h[j]);
        a.h[j] = __floats2half2_rn(fa.x + fr.x, fa.y + fr.y);
      }
      *reinterpret_cast<H8*>(residual_out + base + v * 8) = a;
      *reinterpret_cast<H8*>(row + v * 8) = a;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(a.h[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  ss = block_reduce<false>(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
  float amax = 0.f;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    H8 a = *reinterpret_cast<const H8*>(row + v * 8);
    H8 w = *reinterpret_cast<const H8*>(wrow + v * 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(a.h[j]);
      __half2 n = __floats2half2_rn(f.x * inv, f.y * inv);
      a.h[j] = __hmul2(n, w.h[j]);
      float2 o = __half22float2(a.h[j]);
      amax = fmaxf(amax, fmaxf(fabsf(o.x), fabsf(o.y)));
    }
    if (y != nullptr) *reinterpret_cast<H8*>(y + base + v * 8) = a;
    *reinterpret_cast<H8*>(row + v * 8) = a;
  }
  if (yq == nullptr) return;
  amax = block_reduce<true>(amax, red);
  const float scale = fp8_scale_from_amax(amax);
  store_fp8_row(row, H, scale, yq + base);
  if (threadIdx.x == 0) sy[m] = scale;
}

// gu: [M, 2I] fp16 (gate | up). a = fp16(fp16(silu(g)) * u).
__global__ void __launch_bounds__(kRowThreads) silu_mul_kernel(const __half* __restrict__ gu, int I,
                                                              __half* __restrict__ out, uint8_t* __restrict__ aq,
                                                              float* __restrict__ sa) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* row = reinterpret_cast<__half*>(smem_raw);
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;
  __half* urow = row + I;
  stage_row(row, gu + m * (int64_t)(2 * I), I / 4);  // gate and up halves are contiguous
  cp_async_wait_all();
  float amax = 0.f;
  for (int v = threadIdx.x; v < I / 8; v += blockDim.x) {
    H8 a = *reinterpret_cast<const H8*>(row + v * 8);
    H8 b = *reinterpret_cast<const H8*>(urow + v * 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 fa = __half22float2(a.h[j]);
      __half2 s = __floats2half2_rn(fa.x / (1.0f + expf(-fa.x)), fa.y / (1.0f + expf(-fa.y)));
      a.h[j] = __hmul2(s, b.h[j]);
      float2 o = __half22float2(a.h[j]);
      amax = fmaxf(amax, fmaxf(fabsf(o.x), fabsf(o.y)));
    }
    if (out != nullptr) *reinterpret_cast<H8*>(out + m * (int64_t)I + v * 8) = a;
    *reinterpret_cast<H8*>(row + v * 8) = a;
  }
  if (aq == nullptr) return;
  amax = block_reduce<true>(amax, red);
  const float scale = fp8_scale_from_amax(amax);
  store_fp8_row(row, I, scale, aq + m * (int64_t)I);
  if (threadIdx.x == 0) sa[m] = scale;
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

}  // namespace

cudaError_t launch_quantize_rows(const void* x, int64_t ldx, int64_t M, int K, void* xq, float* sx,
                                 cudaStream_t stream) {
  if (M == 0 || K == 0) return cudaSuccess;
  const size_t smem = (size_t)K * 2;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  const bool vec = (K % 16 == 0) && (ldx % 8 == 0) && (((uintptr_t)x & 15) == 0) && (((uintptr_t)xq & 15) == 0);
  if (vec) {
    ALLOW_BIG_SMEM(quantize_rows_kernel<true>);
    return launch_kernel(quantize_rows_kernel<true>, dim3((unsigned)M), dim3(row_threads(K)), smem, stream,
                         (const __half*)x, ldx, K, (uint8_t*)xq, sx);
  } else {
    ALLOW_BIG_SMEM(quantize_rows_kernel<false>);
    return launch_kernel(quantize_rows_kernel<false>, dim3((unsigned)M), dim3(row_threads(K)), smem, stream,
                         (const __half*)x, ldx, K, (uint8_t*)xq, sx);
  }
}

cudaError_t launch_rmsnorm(const void* x, const void* residual, const void* weight, int64_t M, int H, float eps,
                           void* residual_out, void* y, void* yq, float* sy, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (H % 16 != 0 || H * 6 > 200 * 1024) return cudaErrorInvalidValue;
  size_t smem = (size_t)H * 6;  // x, residual, weight
  ALLOW_BIG_SMEM(rmsnorm_kernel);
  return launch_kernel(rmsnorm_kernel, dim3((unsigned)M), dim3(row_threads(H)), smem, stream, (const __half*)x,
                       (const __half*)residual, (const __half*)weight, H, eps, (__half*)residual_out, (__half*)y,
                       (uint8_t*)yq, sy);
}

cudaError_t launch_silu_mul(const void* gu, int64_t M, int I, void* out, void* aq, float* sa, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (I % 16 != 0 || I * 4 > 200 * 1024) return cudaErrorInvalidValue;
  size_t smem = (size_t)I * 4;  // gate, up
  ALLOW_BIG_SMEM(silu_mul_kernel);
  return launch_kernel(silu_mul_kernel, dim3((unsigned)M), dim3(row_threads(I)), smem, stream, (const __half*)gu, I,
                       (__half*)out, (uint8_t*)aq, sa);
}

}  // namespace ms
