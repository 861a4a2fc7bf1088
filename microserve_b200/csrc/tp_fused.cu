// Tensor-parallel all-reduce fused with the residual add, RMSNorm and FP8 row
// quantisation that follow every row-parallel linear of the decoder layer
// (o_proj -> post_attention_layernorm, down_proj -> next input_layernorm), over
// NVLink peer memory (CUDA IPC mappings; plain loads and stores, no multicast).
//
// Reference semantics (microserve, file:line): RowParallelLinear sums its partial
// outputs over the group (layers/linear.py:70-77, dist.all_reduce of the fp16
// output), then the decoder layer's fused add + RMSNorm (layers/layernorm.py:22-42,
// residual rounded to fp16 before the norm) and the next FP8DynamicLinear's
// activation quantisation (layers/fp8_linear.py:14-23).
//
// Work split: rank r owns rows [r*R, (r+1)*R), R = ceil(M / world). For each owned
// row one CTA reads that row of every rank's partial output (peer memory), sums
// the parts in rank order in fp32 and rounds to fp16 (the all-reduce result), adds
// the local residual row (fp16), normalises, quantises to e4m3 and writes the
// codes and the scale into every rank's gather buffer (optionally the fp16 row
// too). The residual stream is therefore only kept current for owned rows on each
// rank, which is all that the next op reads.
//
// Synchronisation, per call, with a per-rank epoch e (device counter):
//  * ready: block 0 stores e into flags[peer][rank] of every rank (release,
//    system scope): "my partial output is complete" (the GEMM that wrote it
//    precedes this kernel in the stream). Every block waits until flags[p] >= e
//    for all p in its own flag array before reading peer partials.
//  * done: after its stores every block arrives on a local counter; the last
//    one stores e into flags[peer][world + rank] of every rank and waits for all
//    of its own done flags, then advances the epoch. The kernel therefore ends
//    only when every rank's rows are in this rank's gather buffer.
// All waits are bounded (kWaitLimitNs); a timeout records kStatusPeerTimeout.
#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kMaxWorld = 8;
constexpr int kThreads = 512;
constexpr int kMaxVec = 4;  // 16-byte vectors per thread: H <= 4 * 8 * 512 = 16384

struct TpArgs {
  const __half* partial[kMaxWorld];  // every rank's partial output [M, H]
  uint8_t* gather_q[kMaxWorld];      // every rank's FP8 gather buffer [M, H]
  float* gather_s[kMaxWorld];        // every rank's row scales [M]
  __half* gather_h[kMaxWorld];       // optional: every rank's fp16 gather buffer [M, H]
  int* flags[kMaxWorld];             // every rank's flags [2 * world]
  int* ctrl;                         // this rank: [0] epoch, [1] block arrivals
  __half* residual;                  // this rank [M, H] (owned rows read and updated)
  const __half* weight;              // [H]
  int rank, world, M, H, row0, rows;
  float eps;
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until flags[first + q] >= e for q < world (one thread).
__device__ __forceinline__ bool wait_flags(const int* flags, int first, int world, int e) {
  const uint64_t t0 = global_ns();
  for (int q = 0; q < world; ++q) {
    uint32_t spins = 0;
    while (ld_acquire_sys(flags + first + q) < e) {
      if ((++spins & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
        set_device_status(kStatusPeerTimeout);
        return false;
      }
    }
  }
  return true;
}

struct alignas(16) H8 {
  __half2 h[4];
};

__device__ __forceinline__ void row_work(const TpArgs& a, int64_t m, float* red);

__global__ void __launch_bounds__(kThreads) tp_allreduce_rmsnorm_fp8_kernel(TpArgs a) {
  __shared__ float red[32];
  __shared__ int s_e, s_last;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    const int e = a.ctrl[0] + 1;
    s_e = e;
    if (blockIdx.x == 0)
      for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + a.rank, e);  // ready
    wait_flags(a.flags[a.rank], 0, a.world, e);
  }
  __syncthreads();
  const int e = s_e;
  if (blockIdx.x < a.rows) row_work(a, a.row0 + blockIdx.x, red);
  // done: the last block publishes this rank's rows and waits for everyone's. One
  // system-scope fence per block, after the block barrier, orders every thread's
  // peer stores before the arrival (the fence is cumulative); a fence in every
  // thread would serialise thousands of system-scope fences.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(a.ctrl + 1, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (threadIdx.x == 0 && s_last) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + a.world + a.rank, e);
    wait_flags(a.flags[a.rank], a.world, a.world, e);
    a.ctrl[1] = 0;
    a.ctrl[0] = e;
  }
}

// One owned row (all threads of the block).
__device__ __forceinline__ void row_work(const TpArgs& a, int64_t m, float* red) {
  const int nv = a.H / 8;
  const int64_t base = m * (int64_t)a.H;

  // all-reduce of the row: fp32 sum of the ranks' parts in rank order, rounded to fp16
  float v[kMaxVec][8];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nv) {
      // every rank's vector in flight before any add (one round trip over NVLink);
      // L1 bypassed: the same addresses were read one op earlier with other contents
      uint4 u[kMaxWorld];
#pragma unroll
      for (int p = 0; p < kMaxWorld; ++p)
        if (p < a.world) u[p] = __ldcg(reinterpret_cast<const uint4*>(a.partial[p] + base) + c);
#pragma unroll
      for (int p = 0; p < kMaxWorld; ++p) {
        if (p < a.world) {
          H8 x;
          memcpy(&x, &u[p], sizeof(x));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(x.h[j]);
            v[i][2 * j] += f.x;
            v[i][2 * j + 1] += f.y;
          }
        }
      }
    }
  }
  // + residual (fp16 rounding of the all-reduce result, then of the sum), sum of squares
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nv) {
      H8 r = *reinterpret_cast<const H8*>(a.residual + base + 8 * c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fr = __half22float2(r.h[j]);
        const float x0 = __half2float(__float2half_rn(v[i][2 * j]));
        const float x1 = __half2float(__float2half_rn(v[i][2 * j + 1]));
        r.h[j] = __floats2half2_rn(x0 + fr.x, x1 + fr.y);
        const float2 f = __half22float2(r.h[j]);
        v[i][2 * j] = f.x;
        v[i][2 * j + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
      *reinterpret_cast<H8*>(a.residual + base + 8 * c) = r;
    }
  }
  ss = block_reduce<false>(ss, red);
  const float inv = rsqrtf(ss / (float)a.H + a.eps);
  // y = fp16(fp16(r * inv) * w); amax of y
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nv) {
      const H8 w = *reinterpret_cast<const H8*>(a.weight + 8 * c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 n = __floats2half2_rn(v[i][2 * j] * inv, v[i][2 * j + 1] * inv);
        const float2 y = __half22float2(__hmul2(n, w.h[j]));
        v[i][2 * j] = y.x;
        v[i][2 * j + 1] = y.y;
        amax = fmaxf(amax, fmaxf(fabsf(y.x), fabsf(y.y)));
      }
    }
  }
  amax = block_reduce<true>(amax, red);
  const float scale = fp8_scale_from_amax(amax);
  // codes (and optionally the fp16 row) into every rank's gather buffers
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nv) {
      uint32_t code[2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
        code[j] = (uint32_t)f32x2_to_e4m3x2(v[i][4 * j] / scale, v[i][4 * j + 1] / scale) |
                  ((uint32_t)f32x2_to_e4m3x2(v[i][4 * j + 2] / scale, v[i][4 * j + 3] / scale) << 16);
      H8 yh;
#pragma unroll
      for (int j = 0; j < 4; ++j) yh.h[j] = __floats2half2_rn(v[i][2 * j], v[i][2 * j + 1]);
      for (int p = 0; p < a.world; ++p) {
        *reinterpret_cast<uint2*>(a.gather_q[p] + base + 8 * c) = make_uint2(code[0], code[1]);
        if (a.gather_h[p] != nullptr) *reinterpret_cast<H8*>(a.gather_h[p] + base + 8 * c) = yh;
      }
    }
  }
  if (threadIdx.x == 0)
    for (int p = 0; p < a.world; ++p) a.gather_s[p][m] = scale;
}

}  // namespace

cudaError_t launch_tp_allreduce_rmsnorm_fp8(const void* const* partial, void* const* gather_q,
                                            float* const* gather_s, void* const* gather_h, int* const* flags,
                                            int* ctrl, void* residual, const void* weight, int rank, int world,
                                            int M, int H, float eps, cudaStream_t stream) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || H % 8 != 0 || H > kMaxVec * 8 * kThreads)
    return cudaErrorInvalidValue;
  TpArgs a = {};
  for (int p = 0; p < world; ++p) {
    a.partial[p] = static_cast<const __half*>(partial[p]);
    a.gather_q[p] = static_cast<uint8_t*>(gather_q[p]);
    a.gather_s[p] = gather_s[p];
    a.gather_h[p] = gather_h != nullptr ? static_cast<__half*>(gather_h[p]) : nullptr;
    a.flags[p] = flags[p];
  }
  a.ctrl = ctrl;
  a.residual = static_cast<__half*>(residual);
  a.weight = static_cast<const __half*>(weight);
  a.rank = rank;
  a.world = world;
  a.M = M;
  a.H = H;
  a.eps = eps;
  const int R = (M + world - 1) / world;
  a.row0 = rank * R;
  a.rows = M - a.row0 < R ? (M - a.row0 > 0 ? M - a.row0 : 0) : R;
  // A rank that owns no rows still takes part in both barriers with one block.
  const int blocks = a.rows > 0 ? a.rows : 1;
  return launch_kernel(tp_allreduce_rmsnorm_fp8_kernel, dim3(blocks), dim3(kThreads), 0, stream, a);
}

}  // namespace ms
