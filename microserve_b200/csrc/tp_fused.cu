// Tensor-parallel all-reduce fused with the residual add, RMSNorm and FP8 row
// quantisation that follow every row-parallel linear of the decoder layer
// (o_proj -> post_attention_layernorm, down_proj -> next input_layernorm), over
// NVLink peer memory (CUDA IPC mappings; plain loads and stores, no multicast).
//
// Reference semantics (microserve, file:line): RowParallelLinear sums its partial
// outputs over the group (layers/linear.py:70-77, dist.all_reduce of the fp16
// output), then the decoder layer's fused add + RMSNorm (layers/layernorm.py:22-42,
// residual rounded to fp16 before the norm) and the next FP8DynamicLinear's
// activation quantisation (layers/fp8_linear.py:14-23). The sum is taken in fp32
// in rank order and rounded to fp16 once.
//
// Work split: with R = ceil(M / world), rank r owns rows [r R, (r + 1) R). Row
// index j (0 <= j < R) is handled by the same CTA on every rank (CTA j mod grid,
// grid <= SM count); for each of its j it does, pushes first, waits last:
//   1. push   rows p R + j (p != r) of its partial output into rank p's receive
//             slot [b][r][j] (b = epoch parity), 16-byte peer stores;
//   2. reduce its own row r R + j: the world parts in rank order (its own part
//             straight from the partial buffer), + residual, RMSNorm with the
//             canonical sum of squares of rowops.cuh (the same bits as
//             ms_rmsnorm), FP8 codes and scale;
//   3. gather the codes / scale (and the fp16 row for the final norm) into every
//             rank's gather buffer;
//   4. wait   until the rows p R + j of every other owner have landed here.
//
// Readiness travels with the data, not with flags: every buffer a peer writes
// holds the pattern 0xFF..FF ("not yet written") until the write lands, and
// no value a writer stores has that pattern (fp16 0xFFFF and e4m3 0xFF are
// NaN encodings; writers turn them into the positive NaN; scales are finite).
// A reader polls each 16-byte vector until none of its elements is the
// pattern. So there is no ready/done flag and no system-scope fence between
// data and flag on the critical path. Buffers return to the pattern by:
//   * receive slots: cleared by their owner right after it read them; there
//     are two sets by epoch parity, so a slot read in call e is written again
//     in call e + 2 - after its writer finished call e + 1, which needed rows
//     this rank produced after this rank finished call e (and its clears);
//   * gather rows (one fixed buffer, so the next GEMM's tensor map stays
//     valid): each CTA clears the rows it is about to wait for BEFORE it pushes
//     its partial rows (one CTA-level system fence between the two); the owner
//     of such a row writes it only after it received that push.
// The epoch (ctrl[0]) is advanced by the last CTA of the grid. Every wait is
// bounded (ms_set_wait_limit); a wait that runs out records kStatusPeerTimeout,
// the CTA skips its remaining work and the epoch is NOT advanced: the group's
// buffers are then inconsistent and the caller must tear the group down.
#include "common.cuh"
#include "kernels.h"
#include "rowops.cuh"

namespace ms {

namespace {

constexpr int kMaxWorld = 8;
constexpr int kTpThreads = 512;
constexpr uint32_t kPattern = 0xFFFFFFFFu;

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

struct TpArgs {
  __half* recv[kMaxWorld];  // every rank's receive slots [2][world][Rc][H]
  uint8_t* gq[kMaxWorld];   // every rank's gather codes [max_rows][H]
  float* gs[kMaxWorld];     // every rank's gather scales [max_rows]
  __half* gh[kMaxWorld];    // every rank's gather fp16 rows [max_rows][H] (want_h)
  const __half* partial;    // this rank's row-parallel output [M][H]
  __half* residual;         // this rank's residual [M][H] (owned rows read and updated)
  const __half* weight;     // [H]
  int* ctrl;                // this rank: [0] epoch, [1] CTA arrivals, [2] failed
  int64_t recv_half;        // elements of one parity set (world * Rc * H)
  int64_t recv_src;         // elements of one source's slots (Rc * H)
  int rank, world, M, H, R, W;
  int want_h;
  float eps;
};

__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_volatile_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_v4(void* p, const uint4& v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_volatile_v2(void* p, const uint2& v) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void st_volatile_u32(void* p, uint32_t v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// "Not yet written" tests, per element.
__device__ __forceinline__ bool pending16(const uint4& v) {
  return (__vcmpeq2(v.x, kPattern) | __vcmpeq2(v.y, kPattern) | __vcmpeq2(v.z, kPattern) |
          __vcmpeq2(v.w, kPattern)) != 0u;
}
__device__ __forceinline__ bool pending8(const uint4& v) {
  return (__vcmpeq4(v.x, kPattern) | __vcmpeq4(v.y, kPattern) | __vcmpeq4(v.z, kPattern) |
          __vcmpeq4(v.w, kPattern)) != 0u;
}
// Writers never store the pattern: fp16 0xFFFF (a NaN) becomes 0x7FFF, e4m3
// 0xFF (a NaN) becomes 0x7F.
__device__ __forceinline__ uint32_t unpattern16(uint32_t w) { return w & ~(__vcmpeq2(w, kPattern) & 0x80008000u); }
__device__ __forceinline__ uint32_t unpattern8(uint32_t w) { return w & ~(__vcmpeq4(w, kPattern) & 0x80808080u); }
__device__ __forceinline__ uint4 unpattern16(uint4 v) {
  return make_uint4(unpattern16(v.x), unpattern16(v.y), unpattern16(v.z), unpattern16(v.w));
}

// Re-reads *p until `v` has no pending element; false after `limit` ns.
template <bool kCodes>
__device__ __noinline__ bool poll_v4(const void* p, uint4& v, uint64_t limit) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    v = ld_volatile_v4(p);
    if (!(kCodes ? pending8(v) : pending16(v))) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > limit) return false;
  }
}

// One owned row: sum the parts in rank order, + residual, RMSNorm, FP8 codes,
// gathered into every rank's buffers. Returns false if a peer's part did not
// arrive within the wait limit (CTA-uniform).
template <int NVT>
__device__ __forceinline__ bool reduce_row(const TpArgs& a, int j, int b, uint64_t limit, H8* srow, float* red_ss,
                                           float* red_max) {
  const int t = threadIdx.x, T = blockDim.x;
  const int H = a.H, nv = H / 8;
  const int64_t Hl = H;
  const int m0 = a.rank * a.R + j;
  __half* recv_me = a.recv[a.rank] + (int64_t)b * a.recv_half;
  bool fail = false;
  H8 rn[NVT];
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int c = t + i * T;
    if (c >= nv) continue;
    uint4 x[kMaxWorld];
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p) {
      if (p >= a.world) continue;
      x[p] = p == a.rank ? __ldcg(reinterpret_cast<const uint4*>(a.partial + m0 * Hl) + c)
                         : ld_volatile_v4(recv_me + p * a.recv_src + j * Hl + 8 * c);
    }
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p)
      if (p < a.world && p != a.rank && !fail && pending16(x[p]))
        fail = !poll_v4<false>(recv_me + p * a.recv_src + j * Hl + 8 * c, x[p], limit);
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p) {
      if (p >= a.world) continue;
      const H8 h = as_h8(x[p]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h.h[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    // the slots are read: back to "not yet written" for the call after next
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p)
      if (p < a.world && p != a.rank)
        *reinterpret_cast<uint4*>(recv_me + p * a.recv_src + j * Hl + 8 * c) =
            make_uint4(kPattern, kPattern, kPattern, kPattern);
    H8 r = ld_h8(a.residual + m0 * Hl + 8 * c);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 fr = __half22float2(r.h[k]);
      const float x0 = __half2float(__float2half_rn(acc[2 * k]));
      const float x1 = __half2float(__float2half_rn(acc[2 * k + 1]));
      r.h[k] = __floats2half2_rn(x0 + fr.x, x1 + fr.y);
    }
    if (!fail) st_h8(a.residual + m0 * Hl + 8 * c, r);
    rn[i] = r;
    srow[c] = r;
  }
  if (__syncthreads_or(fail)) return false;

  // canonical sum of squares (rowops.cuh): W warps over the staged row
  float ss = 0.f;
  const int TW = 32 * a.W;
  if (t < TW)
    for (int i = 0; i < kRowVec; ++i)
      if (t + i * TW < nv) ss = sumsq8(srow[t + i * TW], ss);
  ss = warp_sum(ss);
  if ((t & 31) == 0 && (t >> 5) < a.W) red_ss[t >> 5] = ss;
  __syncthreads();
  float tot = red_ss[0];
  for (int w = 1; w < a.W; ++w) tot = tot + red_ss[w];
  const float inv = rsqrtf(tot / (float)H + a.eps);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int c = t + i * T;
    if (c >= nv) continue;
    rn[i] = norm8(rn[i], ld_h8(a.weight + 8 * c), inv);
    amax = amax8(rn[i], amax);
  }
  amax = block_reduce<true>(amax, red_max);  // ends with a barrier: srow and red_ss are free again
  const float scale = fp8_scale_from_amax(amax), rcp = 1.0f / scale;
  // gather: codes (and the fp16 row) into every rank's buffers
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int c = t + i * T;
    if (c >= nv) continue;
    uint2 q = encode8(rn[i], scale, rcp);
    q = make_uint2(unpattern8(q.x), unpattern8(q.y));
    const uint4 yh = unpattern16(as_u4(rn[i]));
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p) {
      if (p >= a.world) continue;
      if (p == a.rank) {
        *reinterpret_cast<uint2*>(a.gq[p] + m0 * Hl + 8 * c) = q;
        if (a.want_h) *reinterpret_cast<uint4*>(a.gh[p] + m0 * Hl + 8 * c) = yh;
      } else {
        st_volatile_v2(a.gq[p] + m0 * Hl + 8 * c, q);
        if (a.want_h) st_volatile_v4(a.gh[p] + m0 * Hl + 8 * c, yh);
      }
    }
  }
  if (t == 0)
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) a.gs[p][m0] = scale;
      else st_volatile_u32(a.gs[p] + m0, __float_as_uint(scale));
    }
  return true;
}

// NVT: 16-byte vectors of an fp16 row per thread (ceil(H / 8 / blockDim)). The grid
// has at most one CTA per SM, so every CTA of every rank is resident at once; CTA c
// handles the row indices j = c, c + gridDim, ... < R and issues all of its pushes
// before its first wait.
template <int NVT>
__global__ void __launch_bounds__(kTpThreads) tp_rowpar_norm_kernel(TpArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];  // the owned row after the residual add, [H] fp16
  H8* srow = reinterpret_cast<H8*>(smem_raw);
  __shared__ float red_ss[kMaxRowWarps];
  __shared__ float red_max[32];
  const int t = threadIdx.x, T = blockDim.x;
  const int H = a.H, nv = H / 8, ncv = H / 16;
  const int64_t Hl = H;
  pdl_wait();
  const int e = *reinterpret_cast<volatile int*>(a.ctrl);
  const int b = e & 1;
  const uint64_t limit = wait_limit_ns();
  uint8_t* gq_me = a.gq[a.rank];
  __half* gh_me = a.want_h ? a.gh[a.rank] : nullptr;

  // 0. clear the gather rows this CTA waits for (rows p R + j of the other owners) ...
  for (int j = blockIdx.x; j < a.R; j += gridDim.x)
    for (int p = 0; p < a.world; ++p) {
      const int m = p * a.R + j;
      if (p == a.rank || m >= a.M) continue;
      for (int c = t; c < ncv; c += T)
        *reinterpret_cast<uint4*>(gq_me + m * Hl + 16 * c) = make_uint4(kPattern, kPattern, kPattern, kPattern);
      if (gh_me != nullptr)
        for (int c = t; c < nv; c += T)
          *reinterpret_cast<uint4*>(gh_me + m * Hl + 8 * c) = make_uint4(kPattern, kPattern, kPattern, kPattern);
      if (t == 0) *reinterpret_cast<uint32_t*>(a.gs[a.rank] + m) = kPattern;
    }
  // ... performed system-wide before any owner can answer the pushes below
  __syncthreads();
  if (t == 0) asm volatile("fence.acq_rel.sys;" ::: "memory");
  __syncthreads();
  pdl_trigger();

  // 1. push the rows owned by other ranks into their receive slots
  for (int j = blockIdx.x; j < a.R; j += gridDim.x) {
#pragma unroll
    for (int i = 0; i < NVT; ++i) {
      const int c = t + i * T;
      if (c >= nv) continue;
      uint4 x[kMaxWorld];
#pragma unroll
      for (int p = 0; p < kMaxWorld; ++p) {
        const int m = p * a.R + j;
        if (p < a.world && p != a.rank && m < a.M)
          x[p] = __ldcg(reinterpret_cast<const uint4*>(a.partial + m * Hl) + c);
      }
#pragma unroll
      for (int p = 0; p < kMaxWorld; ++p) {
        const int m = p * a.R + j;
        if (p < a.world && p != a.rank && m < a.M)
          st_volatile_v4(a.recv[p] + (int64_t)b * a.recv_half + a.rank * a.recv_src + j * Hl + 8 * c,
                         unpattern16(x[p]));
      }
    }
  }

  // 2-3. reduce, normalise and gather the owned rows
  bool fail = false;
  for (int j = blockIdx.x; j < a.R && !fail; j += gridDim.x)
    if (a.rank * a.R + j < a.M) fail = !reduce_row<NVT>(a, j, b, limit, srow, red_ss, red_max);

  // 4. wait for the rows the other owners write into this rank's gather buffers
  for (int j = blockIdx.x; j < a.R && !fail; j += gridDim.x) {
    for (int p = 0; p < a.world && !fail; ++p) {
      const int m = p * a.R + j;
      if (p == a.rank || m >= a.M) continue;
      for (int c = t; c < ncv && !fail; c += T) {
        const uint8_t* src = gq_me + m * Hl + 16 * c;
        uint4 v = ld_volatile_v4(src);
        if (pending8(v)) fail = !poll_v4<true>(src, v, limit);
      }
      if (gh_me != nullptr)
        for (int c = t; c < nv && !fail; c += T) {
          const __half* src = gh_me + m * Hl + 8 * c;
          uint4 v = ld_volatile_v4(src);
          if (pending16(v)) fail = !poll_v4<false>(src, v, limit);
        }
      if (t == 0 && !fail) {
        const float* sp = a.gs[a.rank] + m;
        const uint64_t t0 = global_ns();
        for (uint32_t i = 1; ld_volatile_u32(sp) == kPattern; ++i)
          if ((i & 63u) == 0 && global_ns() - t0 > limit) {
            fail = true;
            break;
          }
      }
    }
  }
  fail = __syncthreads_or(fail) != 0;

  // 5. the last CTA advances the epoch (not after a timeout)
  if (t == 0) {
    if (fail) {
      set_device_status(kStatusPeerTimeout);
      atomicOr(a.ctrl + 2, 1);
    }
    __threadfence();
    if (atomicAdd(a.ctrl + 1, 1) == (int)gridDim.x - 1) {
      a.ctrl[1] = 0;
      if (atomicAdd(a.ctrl + 2, 0) == 0) a.ctrl[0] = e + 1;
    }
  }
}

}  // namespace

TpLayout tp_layout(int world, int64_t H, int64_t max_rows) {
  TpLayout l;
  const int64_t rc = (max_rows + world - 1) / world;
  int64_t off = 0;
  l.partial = off;
  off = align256(off + max_rows * H * 2);
  l.recv = off;
  off = align256(off + 2 * (int64_t)world * rc * H * 2);
  l.gq = off;
  off = align256(off + max_rows * H);
  l.gs = off;
  off = align256(off + max_rows * 4);
  l.gh = off;
  off = align256(off + max_rows * H * 2);
  l.ctrl = off;
  off = align256(off + 256);
  l.total = off;
  return l;
}

cudaError_t launch_tp_buffer_init(void* base, int world, int64_t H, int64_t max_rows, cudaStream_t stream) {
  const TpLayout l = tp_layout(world, H, max_rows);
  cudaError_t e = cudaMemsetAsync(base, 0xFF, (size_t)l.ctrl, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(static_cast<char*>(base) + l.ctrl, 0, (size_t)(l.total - l.ctrl), stream);
  return e;
}

cudaError_t launch_tp_allreduce_rmsnorm_fp8(void* const* bases, int rank, int world, int64_t H, int64_t max_rows,
                                            void* residual, const void* weight, int M, float eps, int want_h,
                                            int num_sms, cudaStream_t stream) {
  if (num_sms < 1 || world < 1 || world > kMaxWorld || rank < 0 || rank >= world || H % 16 != 0 || H > 16384 || M > max_rows)
    return cudaErrorInvalidValue;
  if (M <= 0) return cudaSuccess;
  const TpLayout l = tp_layout(world, H, max_rows);
  const int64_t rc = (max_rows + world - 1) / world;
  TpArgs a = {};
  for (int p = 0; p < world; ++p) {
    char* base = static_cast<char*>(bases[p]);
    a.recv[p] = reinterpret_cast<__half*>(base + l.recv);
    a.gq[p] = reinterpret_cast<uint8_t*>(base + l.gq);
    a.gs[p] = reinterpret_cast<float*>(base + l.gs);
    a.gh[p] = reinterpret_cast<__half*>(base + l.gh);
  }
  char* me = static_cast<char*>(bases[rank]);
  a.partial = reinterpret_cast<const __half*>(me + l.partial);
  a.residual = static_cast<__half*>(residual);
  a.weight = static_cast<const __half*>(weight);
  a.ctrl = reinterpret_cast<int*>(me + l.ctrl);
  a.recv_src = rc * H;
  a.recv_half = (int64_t)world * rc * H;
  a.rank = rank;
  a.world = world;
  a.M = M;
  a.H = (int)H;
  a.R = (M + world - 1) / world;
  a.W = row_warps((int)(H / 8));
  a.want_h = want_h ? 1 : 0;
  a.eps = eps;
  const int nv = (int)(H / 8);
  int T = (nv + 31) / 32 * 32;
  if (T > kTpThreads) T = kTpThreads;
  const int nvt = (nv + T - 1) / T;
  const size_t smem = (size_t)H * 2;
  // at most one CTA per SM (a 512-thread CTA fits any SM beside the kernels that
  // precede it): every CTA of every rank is then resident at once, whatever the
  // order in which the hardware dispatches them
  const dim3 grid(a.R < num_sms ? a.R : num_sms);
  switch (nvt) {
    case 1: return launch_kernel(tp_rowpar_norm_kernel<1>, grid, dim3(T), smem, stream, a);
    case 2: return launch_kernel(tp_rowpar_norm_kernel<2>, grid, dim3(T), smem, stream, a);
    case 3: return launch_kernel(tp_rowpar_norm_kernel<3>, grid, dim3(T), smem, stream, a);
    case 4: return launch_kernel(tp_rowpar_norm_kernel<4>, grid, dim3(T), smem, stream, a);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ms
