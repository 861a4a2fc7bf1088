// Greedy token selection: the row-wise argmax of the logits, the greedy branch
// of the reference's `_sample` (microserve/engine/model_runner.py:33-34,
// `torch.argmax(logits.float())`): the first index of the maximum, NaN counting
// as larger than every number (torch's rule), -0.0 equal to +0.0.
//
// One pass over the logits: (kChunks x M) CTAs each reduce a slice of a row to
// a 64-bit key (order-preserving bits of the value, then the complement of the
// index, so the largest key is the largest value at the smallest index); the
// last CTA of a row (per-row arrival counter in the workspace) reduces the
// kChunks keys and writes the index and the value (the value lets a
// vocab-parallel caller merge ranks). Counters return to zero for the next call.
#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kChunks = 8;
constexpr int kThreads = 256;
// Per-row arrival counters sit at the start of the workspace with a fixed
// capacity, so calls with different row counts can share one workspace: the
// keys of one call never overlap the counters of another.
constexpr int64_t kMaxRows = 16384;
constexpr size_t kCounterBytes = kMaxRows * sizeof(int);

__device__ __forceinline__ uint64_t make_key(float f, uint32_t idx) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;  // -0.0 ties with +0.0
  uint32_t k;
  if (f != f) {
    k = 0xFFFFFFFFu;  // NaN above everything
  } else {
    k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  return ((uint64_t)k << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}

__device__ __forceinline__ float key_value(uint64_t key) {
  const uint32_t k = (uint32_t)(key >> 32);
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

template <bool kVec>
__global__ void __launch_bounds__(kThreads) argmax_rows_kernel(const __half* __restrict__ x, int64_t ldx, int V,
                                                              int64_t* __restrict__ idx_out,
                                                              float* __restrict__ max_out,
                                                              uint64_t* __restrict__ keys, int* __restrict__ counters) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint64_t red[kThreads / 32];
  __shared__ bool last;
  const int chunk = blockIdx.x;
  const int64_t row = blockIdx.y;
  const __half* xr = x + row * ldx;
  const int per = ((V + kChunks - 1) / kChunks + 7) & ~7;  // chunk length, a multiple of 8
  const int lo = min(V, chunk * per), hi = min(V, lo + per);
  uint64_t best = 0;
  if (kVec) {
    for (int v = lo / 8 + threadIdx.x; v < hi / 8; v += kThreads) {
      const uint4 w = *reinterpret_cast<const uint4*>(xr + (int64_t)v * 8);
      const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        const uint64_t a = make_key(f.x, (uint32_t)(v * 8 + 2 * j));
        const uint64_t b = make_key(f.y, (uint32_t)(v * 8 + 2 * j + 1));
        best = a > best ? a : best;
        best = b > best ? b : best;
      }
    }
  } else {
    for (int i = lo + threadIdx.x; i < hi; i += kThreads) {
      const uint64_t a = make_key(__half2float(xr[i]), (uint32_t)i);
      best = a > best ? a : best;
    }
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint64_t v = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0;
    v = warp_max_u64(v);
    if (threadIdx.x == 0) {
      keys[row * kChunks + chunk] = v;
      __threadfence();
      last = atomicAdd(&counters[row], 1) == kChunks - 1;
    }
  }
  __syncthreads();
  if (!last) return;
  if (threadIdx.x == 0) {
    __threadfence();
    uint64_t m = 0;
    for (int c = 0; c < kChunks; ++c) {
      const uint64_t k = *reinterpret_cast<volatile const uint64_t*>(&keys[row * kChunks + c]);
      m = k > m ? k : m;
    }
    idx_out[row] = (int64_t)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFu));
    if (max_out != nullptr) max_out[row] = key_value(m);
    counters[row] = 0;
  }
}

}  // namespace

size_t argmax_workspace_bytes(int64_t M) { return kCounterBytes + (size_t)M * kChunks * sizeof(uint64_t); }

cudaError_t launch_argmax_rows(const void* x, int64_t M, int V, int64_t ldx, int64_t* idx, float* vmax,
                               void* workspace, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (M > kMaxRows) return cudaErrorInvalidValue;
  int* counters = static_cast<int*>(workspace);
  uint64_t* keys = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + kCounterBytes);
  const bool vec = V % 8 == 0 && ldx % 8 == 0 && ((uintptr_t)x & 15) == 0;
  const dim3 grid(kChunks, (unsigned)M);
  return vec ? launch_kernel(argmax_rows_kernel<true>, grid, dim3(kThreads), 0, stream, (const __half*)x, ldx, V, idx,
                             vmax, keys, counters)
             : launch_kernel(argmax_rows_kernel<false>, grid, dim3(kThreads), 0, stream, (const __half*)x, ldx, V,
                             idx, vmax, keys, counters);
}

}  // namespace ms
