// Shared device helpers for the microserve-b200 kernels (sm_100a only).
//
// Numerics contract: every FP8 encode in this library is
//   scale = max(amax, 1e-8f) * fl32(1/448)
//   q     = e4m3(clamp(x / scale, -448, 448)) (IEEE divide, round-to-nearest-even, satfinite)
// The reference writes `max(amax, 1e-8) / 448.0` (microserve/layers/fp8_linear.py:20-21,
// :52; microserve/layers/fp8_kv_cache.py:34-37), but both of its executions of that
// expression - the Triton kernels and torch on CUDA (a tensor divided by a scalar) -
// multiply by the fp32 reciprocal, which differs from an IEEE divide by one ulp for about
// half of the inputs; the golden outputs of the reference's own GPU kernels
// (tests/golden/reference_gpu.pt) pin this. The library is compiled without
// --use_fast_math so that `x / scale` is div.rn.f32.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#define MS_FP8_MAX 448.0f

namespace ms {

// ---------------------------------------------------------------------------
// Device status word: kernels that wait on barriers never spin forever; on a
// timeout they record a code here and return. The host reads it with
// ms_get_device_status().
// ---------------------------------------------------------------------------
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusMbarTimeout = 1,
  kStatusPeerTimeout = 2,
};

extern __device__ int g_device_status;

// Host-side count of kernel launches issued by the library (for launch
// accounting in benchmarks; a CUDA-graph replay re-runs captured launches
// without counting them again).
extern std::atomic<long long> g_host_launches;
#define MS_COUNT_LAUNCH() (::ms::g_host_launches.fetch_add(1, std::memory_order_relaxed))

__device__ __forceinline__ void set_device_status(int code) {
  atomicCAS(&g_device_status, 0, code);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Every kernel of the library is launched
// with programmatic stream serialization allowed, so it may start while the
// preceding kernel in the stream is still running. Contract for each kernel:
//  * pdl_wait() before its first access to memory that earlier work in the
//    stream writes or reads (inputs, outputs, workspaces); only immutable data
//    (weights, tensor maps) and on-chip state may be touched before it;
//  * pdl_trigger() once the CTA no longer blocks the next kernel from starting
//    its own prologue. The next kernel starts when every CTA has triggered or
//    exited, so all CTAs of this grid are resident by then.
// Without the launch attribute both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: whether launches carry the programmatic-serialization attribute.
extern std::atomic<int> g_pdl_enabled;
extern std::atomic<int> g_pair_tiles_enabled;  // FP8/fp16 GEMM: SM-pair schedules allowed

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl_enabled.load(std::memory_order_relaxed) ? 1 : 0;
  MS_COUNT_LAUNCH();
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// FP8 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fp8_scale_from_amax(float amax) {
  return fmaxf(amax, 1e-8f) * (1.0f / MS_FP8_MAX);
}

// Encode two fp32 values (already divided by the scale) into two e4m3 bytes,
// clamped to +-448 first (the clamp is a no-op for finite values under
// satfinite, kept for NaN-free parity with the reference's explicit clamp).
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  a = fminf(fmaxf(a, -MS_FP8_MAX), MS_FP8_MAX);
  b = fminf(fmaxf(b, -MS_FP8_MAX), MS_FP8_MAX);
  __nv_fp8x2_storage_t r = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  return (uint16_t)r;
}

// x / s rounded to nearest (the IEEE quotient) from r = RN(1/s), in five
// flops instead of a full-precision divide: q0 = RN(x r) is within ~1.5 ulp of
// x/s; one correction q1 = RN(q0 + r RN(x - s q0)) brings it within half an ulp
// plus a negligible term, i.e. faithful; a second correction from the faithful
// q1 is correctly rounded by Markstein's theorem (with r within half an ulp of
// 1/s the remainder x - s q1 is exact under FMA and RN(q1 + r (x - s q1)) =
// RN(x/s)). Needs no underflow in the remainder: holds for the FP8 encoders
// here (fp16 x, s >= 1e-8 / 448, |x/s| <= 448). Zeros are returned as they are:
// the corrections would turn -0 into +0 (-0 + +0 = +0), and -0 / s is -0.
__device__ __forceinline__ float div_by_rcp(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float q1 = __fmaf_rn(__fmaf_rn(-q0, s, x), r, q0);
  const float q2 = __fmaf_rn(__fmaf_rn(-q1, s, x), r, q1);
  return x == 0.f ? x : q2;
}

__device__ __forceinline__ uint8_t f32_to_e4m3(float a) {
  a = fminf(fmaxf(a, -MS_FP8_MAX), MS_FP8_MAX);
  return (uint8_t)__nv_cvt_float_to_fp8(a, __NV_SATFINITE, __NV_E4M3);
}

// Two e4m3 bytes (low byte = first element) -> half2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)v, __NV_E4M3);
  return __half2float(__half(h));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// ---------------------------------------------------------------------------
// Warp / block reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reduction; `smem` must hold >= 32 floats. All threads get the result.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = kMax ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? smem[lane] : (kMax ? 0.f : 0.f);
  if (wid == 0) {
    r = kMax ? warp_max(r) : warp_sum(r);
    if (lane == 0) smem[0] = r;
  }
  __syncthreads();
  return smem[0];
}

// ---------------------------------------------------------------------------
// mbarrier helpers (bounded waits)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Nanoseconds of the GPU's global timer.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any in-kernel wait, per device (ms_set_wait_limit). Legitimate
// waits last microseconds to milliseconds; the limit only ends a wait whose
// event can no longer come (a peer that died or never joined). Default 4 s.
constexpr uint64_t kDefaultWaitLimitNs = 4000000000ull;
extern __device__ unsigned long long g_wait_limit_ns;

__device__ __forceinline__ uint64_t wait_limit_ns() {
  return *static_cast<volatile unsigned long long*>(&g_wait_limit_ns);
}

// Wait until the barrier's phase `phase` completed. try_wait already suspends
// the thread in hardware until the phase completes (or a short time limit
// passes), so the loop adds no sleep of its own: a __nanosleep here delays the
// wake-up by its own granularity. Gives up after wait_limit_ns(), records
// kStatusMbarTimeout and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = global_ns(), limit = wait_limit_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((i & 255u) == 0 && global_ns() - t0 > limit) break;
  }
  set_device_status(kStatusMbarTimeout);
  return false;
}

}  // namespace ms
