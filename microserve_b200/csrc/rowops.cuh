// Row helpers shared by the single-GPU row kernels (rowwise.cu) and the
// tensor-parallel op (tp_fused.cu). The RMSNorm sum of squares is defined here
// ONCE, with every rounding explicit, so that the two kernels that normalise a
// decoder row produce the same bits for the same fp16 row:
//
//   canonical row layout: W warps (T = 32 W threads, W = row_warps(H / 8));
//   thread t owns the 16-byte vectors v = t, t + T, ..., t + (kRowVec - 1) T;
//   ss_t = sum over its vectors in order, over the vector's four element pairs
//          in order, of RN(x0 * x0 + RN(x1 * x1))   (one FMA, one add per pair)
//   ss   = red[0] + red[1] + ... + red[W-1], red[w] = the butterfly warp sum
//          (xor 16, 8, 4, 2, 1) of warp w's ss_t.
#pragma once

#include "common.cuh"

namespace ms {

constexpr int kMaxRowWarps = 16;
constexpr int kRowVec = 8;  // 16-byte vectors per thread at most

struct alignas(16) H8 {
  __half2 h[4];
};

__device__ __forceinline__ H8 ld_h8(const __half* p) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  H8 h;
  memcpy(&h, &u, sizeof(h));
  return h;
}
__device__ __forceinline__ void st_h8(__half* p, const H8& h) {
  uint4 u;
  memcpy(&u, &h, sizeof(u));
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ H8 as_h8(const uint4& u) {
  H8 h;
  memcpy(&h, &u, sizeof(h));
  return h;
}
__device__ __forceinline__ uint4 as_u4(const H8& h) {
  uint4 u;
  memcpy(&u, &h, sizeof(u));
  return u;
}

// Eight fp16 values -> eight e4m3 codes (x / s rounded as the IEEE quotient, r = 1/s).
__device__ __forceinline__ uint2 encode8(const H8& a, float s, float r) {
  uint32_t w[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const float2 f0 = __half22float2(a.h[2 * p]);
    const float2 f1 = __half22float2(a.h[2 * p + 1]);
    const uint16_t lo = f32x2_to_e4m3x2(div_by_rcp(f0.x, s, r), div_by_rcp(f0.y, s, r));
    const uint16_t hi = f32x2_to_e4m3x2(div_by_rcp(f1.x, s, r), div_by_rcp(f1.y, s, r));
    w[p] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
  return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ float amax8(const H8& a, float amax) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(a.h[j]);
    amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return amax;
}

// The canonical per-vector step of the sum of squares (see the file comment).
__device__ __forceinline__ float sumsq8(const H8& a, float ss) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(a.h[j]);
    ss = __fadd_rn(ss, __fmaf_rn(f.x, f.x, __fmul_rn(f.y, f.y)));
  }
  return ss;
}

// y = fp16(fp16(v * inv) * w), elementwise (the reference's RMSNorm rounding points).
__device__ __forceinline__ H8 norm8(const H8& a, const H8& w, float inv) {
  H8 y;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(a.h[j]);
    const __half2 n = __floats2half2_rn(f.x * inv, f.y * inv);
    y.h[j] = __hmul2(n, w.h[j]);
  }
  return y;
}

// Warps per row so that a thread holds at most kRowVec 16-byte vectors (a power
// of two, <= kMaxRowWarps); 0 if the row is too long.
__host__ __device__ inline int row_warps(int nv) {
  int w = 1;
  while (w * 32 * kRowVec < nv && w < kMaxRowWarps) w <<= 1;
  return w * 32 * kRowVec >= nv ? w : 0;
}

}  // namespace ms
