// Row work of the fused tensor-parallel all-reduce + residual add + RMSNorm + FP8
// quantisation, shared by the standalone op (tp_fused.cu) and the row-parallel
// GEMM that pushes its output tiles itself (fp8_gemm.cu, row-parallel mode).
//
// Reference semantics (microserve, file:line): RowParallelLinear sums its partial
// outputs over the group (layers/linear.py:70-77, dist.all_reduce of the fp16
// output), then the decoder layer's fused add + RMSNorm (layers/layernorm.py:22-42,
// residual rounded to fp16 before the norm) and the next FP8DynamicLinear's
// activation quantisation (layers/fp8_linear.py:14-23). The sum is taken in fp32
// in rank order and rounded to fp16 once.
//
// With R = ceil(M / world), rank r owns rows [r R, (r + 1) R). Row index j
// (0 <= j < R) is handled by the same CTA on every rank; per call and j:
//   push     rows p R + j (p != r) of the rank's partial output go to rank p's
//            receive slot [b][r][j] (b = epoch parity) - done by the GEMM's
//            epilogue when it pushes its tiles itself;
//   reduce   the owned row r R + j: the world parts in rank order, + residual,
//            RMSNorm with the canonical sum of squares of rowops.cuh (the same
//            bits as ms_rmsnorm), FP8 codes and scale, written to this rank's
//            output and to every other rank's gather slot [b] of that row;
//   collect  rows p R + j of the other owners: wait for their gather slots,
//            copy them to this rank's output, reset the slots.
//
// Readiness travels with the data: every slot a peer writes holds the pattern
// 0xFF..FF ("not yet written") until the write lands, and no value a writer
// stores has that pattern (fp16 0xFFFF and e4m3 0xFF are NaN encodings and are
// stored as the positive NaN; scales are finite). A reader polls each 16-byte
// vector until none of its elements is the pattern and resets the slot after
// reading it. Slots come in two sets by epoch parity: a slot read in call e is
// written again in call e + 2, by a writer that has finished call e + 1, which
// needed rows that this rank produced after it finished call e (and its
// resets) - so no flag and no memory fence is needed anywhere. The consumer of
// the normalised rows (the next GEMM) reads the fixed output area, so its
// tensor map never changes.
#pragma once

#include "common.cuh"
#include "rowops.cuh"

namespace ms {

constexpr int kTpMaxWorld = 8;
constexpr uint32_t kTpPattern = 0xFFFFFFFFu;

struct TpRows {
  __half* recv[kTpMaxWorld];   // every rank's partial receive slots [2][world][Rc][H]
  uint8_t* grq[kTpMaxWorld];   // every rank's gather slots, codes [2][max_rows][H]
  float* grs[kTpMaxWorld];     // every rank's gather slots, scales [2][max_rows]
  __half* grh[kTpMaxWorld];    // every rank's gather slots, fp16 rows [2][max_rows][H]
  uint8_t* outq;               // this rank's output codes [max_rows][H]
  float* outs;                 // this rank's output scales [max_rows]
  __half* outh;                // this rank's output fp16 rows [max_rows][H]
  const __half* partial;       // this rank's row-parallel output [M][H] (not pushed)
  __half* residual;            // this rank's residual [M][H] (owned rows read and updated)
  const __half* weight;        // [H]
  int* ctrl;                   // this rank: [0] epoch, [1] CTA arrivals, [2] failed
  int64_t recv_half, recv_src; // elements of one parity set / of one source's slots
  int64_t g_half;              // rows of one gather parity set (max_rows)
  int rank, world, M, H, R, W;
  int want_h;                  // write fp16 rows (the final norm) instead of FP8 codes
  int pushed;                  // the partial rows are already in the receive slots (own one too)
  float eps;
};

__device__ __forceinline__ uint4 tp_ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint32_t tp_ld_volatile_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void tp_st_volatile_v4(void* p, const uint4& v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void tp_st_volatile_v2(void* p, const uint2& v) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void tp_st_volatile_u32(void* p, uint32_t v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 tp_pattern4() { return make_uint4(kTpPattern, kTpPattern, kTpPattern, kTpPattern); }

// "Not yet written" tests, per element.
__device__ __forceinline__ bool tp_pending16(const uint4& v) {
  return (__vcmpeq2(v.x, kTpPattern) | __vcmpeq2(v.y, kTpPattern) | __vcmpeq2(v.z, kTpPattern) |
          __vcmpeq2(v.w, kTpPattern)) != 0u;
}
__device__ __forceinline__ bool tp_pending8(const uint4& v) {
  return (__vcmpeq4(v.x, kTpPattern) | __vcmpeq4(v.y, kTpPattern) | __vcmpeq4(v.z, kTpPattern) |
          __vcmpeq4(v.w, kTpPattern)) != 0u;
}
// Writers never store the pattern: fp16 0xFFFF becomes 0x7FFF, e4m3 0xFF becomes 0x7F.
__device__ __forceinline__ uint32_t tp_unpattern16(uint32_t w) {
  return w & ~(__vcmpeq2(w, kTpPattern) & 0x80008000u);
}
__device__ __forceinline__ uint32_t tp_unpattern8(uint32_t w) { return w & ~(__vcmpeq4(w, kTpPattern) & 0x80808080u); }
__device__ __forceinline__ uint4 tp_unpattern16(uint4 v) {
  return make_uint4(tp_unpattern16(v.x), tp_unpattern16(v.y), tp_unpattern16(v.z), tp_unpattern16(v.w));
}

// Re-reads *p until no element is pending and returns the vector; after `limit` ns it
// returns the last read, still pending. (Returned by value: a vector passed by
// reference would live in local memory, and storing each load's result there would
// serialise the loads that should be in flight together.)
template <bool kCodes>
__device__ __noinline__ uint4 tp_poll_v4(const void* p, uint64_t limit) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    const uint4 v = tp_ld_volatile_v4(p);
    if (!(kCodes ? tp_pending8(v) : tp_pending16(v))) return v;
    if ((i & 63u) == 0 && global_ns() - t0 > limit) return v;
  }
}

// The compile-time bound on the ranks that the row work is instantiated for.
__host__ __device__ constexpr int tp_world_bound(int world) { return world <= 2 ? 2 : world <= 4 ? 4 : 8; }

// Host: the arguments for one call (pointers from every rank's buffer base, sizes);
// residual, weight, eps, want_h and pushed are left for the caller.
TpRows tp_rows_args(void* const* bases, int rank, int world, int64_t H, int64_t max_rows, int M);

// Receive slot of source rank `src` for owner-row j, parity b, on rank `owner`.
__device__ __forceinline__ __half* tp_slot(const TpRows& a, int owner, int b, int src, int j) {
  return a.recv[owner] + (int64_t)b * a.recv_half + src * a.recv_src + (int64_t)j * a.H;
}

// push: rows p R + j (p != rank) of the partial output into their owners' slots.
__device__ __forceinline__ void tp_push_rows(const TpRows& a, int j, int b) {
  const int T = blockDim.x, nv = a.H / 8;
  for (int c = threadIdx.x; c < nv; c += T) {
    uint4 x[kTpMaxWorld];
#pragma unroll
    for (int p = 0; p < kTpMaxWorld; ++p) {
      const int m = p * a.R + j;
      if (p < a.world && p != a.rank && m < a.M)
        x[p] = __ldcg(reinterpret_cast<const uint4*>(a.partial + (int64_t)m * a.H) + c);
    }
#pragma unroll
    for (int p = 0; p < kTpMaxWorld; ++p) {
      const int m = p * a.R + j;
      if (p < a.world && p != a.rank && m < a.M)
        tp_st_volatile_v4(tp_slot(a, p, b, a.rank, j) + 8 * c, tp_unpattern16(x[p]));
    }
  }
}

// Vectors a thread keeps in flight at once in reduce and collect: the row's
// vectors are taken in groups of kI (NVT per thread in all, WB parts or peers
// each), and every load of a group is issued before the first one is used, so a
// group costs one memory round trip instead of one per vector (at most 16
// vectors, 64 registers).
template <int NVT, int WB>
struct TpGroup {
  static constexpr int kI = (16 / WB) < NVT ? (16 / WB) : NVT;
};

// reduce: the owned row rank R + j (all threads of the CTA; srow: the row, [H] fp16
// in shared memory; red_ss >= kMaxRowWarps floats, red_max >= 32 floats). WB >=
// world. Returns false if a part did not arrive within the wait limit
// (CTA-uniform).
template <int NVT, int WB>
__device__ __forceinline__ bool tp_reduce_row(const TpRows& a, int j, int b, uint64_t limit, H8* srow,
                                              float* red_ss, float* red_max) {
  constexpr int kI = TpGroup<NVT, WB>::kI;
  const int t = threadIdx.x, T = blockDim.x;
  const int H = a.H, nv = H / 8;
  const int64_t m0 = (int64_t)a.rank * a.R + j;
  bool fail = false;
  H8 rn[NVT];
#pragma unroll
  for (int g = 0; g < NVT; g += kI) {
    uint4 x[kI][WB];
    H8 r[kI];
#pragma unroll
    for (int i = 0; i < kI; ++i) {  // the group's loads: every part and the residual
      const int c = t + (g + i) * T;
      if (g + i >= NVT || c >= nv) continue;
#pragma unroll
      for (int p = 0; p < WB; ++p) {
        if (p >= a.world) continue;
        x[i][p] = (p == a.rank && !a.pushed) ? __ldcg(reinterpret_cast<const uint4*>(a.partial + m0 * H) + c)
                                             : tp_ld_volatile_v4(tp_slot(a, a.rank, b, p, j) + 8 * c);
      }
      r[i] = ld_h8(a.residual + m0 * H + 8 * c);
    }
#pragma unroll
    for (int i = 0; i < kI; ++i) {  // parts not yet written: wait for them
      const int c = t + (g + i) * T;
      if (g + i >= NVT || c >= nv) continue;
#pragma unroll
      for (int p = 0; p < WB; ++p)
        if (p < a.world && (p != a.rank || a.pushed) && !fail && tp_pending16(x[i][p])) {
          x[i][p] = tp_poll_v4<false>(tp_slot(a, a.rank, b, p, j) + 8 * c, limit);
          fail = tp_pending16(x[i][p]);
        }
    }
#pragma unroll
    for (int i = 0; i < kI; ++i) {
      const int c = t + (g + i) * T;
      if (g + i >= NVT || c >= nv) continue;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
      for (int p = 0; p < WB; ++p) {  // rank order
        if (p >= a.world) continue;
        const H8 h = as_h8(x[i][p]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(h.h[k]);
          acc[2 * k] += f.x;
          acc[2 * k + 1] += f.y;
        }
      }
      // the slots are read: back to "not yet written" for the call after next
#pragma unroll
      for (int p = 0; p < WB; ++p)
        if (p < a.world && (p != a.rank || a.pushed))
          *reinterpret_cast<uint4*>(tp_slot(a, a.rank, b, p, j) + 8 * c) = tp_pattern4();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 fr = __half22float2(r[i].h[k]);
        const float x0 = __half2float(__float2half_rn(acc[2 * k]));
        const float x1 = __half2float(__float2half_rn(acc[2 * k + 1]));
        r[i].h[k] = __floats2half2_rn(x0 + fr.x, x1 + fr.y);
      }
      if (!fail) st_h8(a.residual + m0 * H + 8 * c, r[i]);
      rn[g + i] = r[i];
      srow[c] = r[i];
    }
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
  const int64_t gslot = (int64_t)b * a.g_half + m0;  // the row in a gather parity set
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int c = t + i * T;
    if (c >= nv) continue;
    if (a.want_h) {
      const uint4 yh = tp_unpattern16(as_u4(rn[i]));
      *reinterpret_cast<uint4*>(a.outh + m0 * H + 8 * c) = yh;
#pragma unroll
      for (int p = 0; p < WB; ++p)
        if (p < a.world && p != a.rank) tp_st_volatile_v4(a.grh[p] + gslot * H + 8 * c, yh);
    } else {
      uint2 q = encode8(rn[i], scale, rcp);
      q = make_uint2(tp_unpattern8(q.x), tp_unpattern8(q.y));
      *reinterpret_cast<uint2*>(a.outq + m0 * H + 8 * c) = q;
#pragma unroll
      for (int p = 0; p < WB; ++p)
        if (p < a.world && p != a.rank) tp_st_volatile_v2(a.grq[p] + gslot * H + 8 * c, q);
    }
  }
  if (t == 0 && !a.want_h) {
    a.outs[m0] = scale;
    for (int p = 0; p < a.world; ++p)
      if (p != a.rank) tp_st_volatile_u32(a.grs[p] + gslot, __float_as_uint(scale));
  }
  return true;
}

// collect: rows p R + j of the other owners, from this rank's gather slots into its
// output (the slots are reset after reading): every peer's vectors of a group are
// loaded at once, and thread p waits for peer p's scale. WB >= world. Returns
// false on a timeout.
template <int NVT, int WB>
__device__ __forceinline__ bool tp_collect_rows(const TpRows& a, int j, int b, uint64_t limit) {
  constexpr int kI = TpGroup<NVT, WB>::kI;
  const int t = threadIdx.x, T = blockDim.x;
  const int64_t H = a.H;
  const int me = a.rank;
  const int nvec = a.want_h ? (int)(H / 8) : (int)(H / 16);  // 16-byte vectors of a gathered row
  const size_t vbytes = a.want_h ? (size_t)H * 2 : (size_t)H;
  unsigned char* const slots = a.want_h ? reinterpret_cast<unsigned char*>(a.grh[me]) : a.grq[me];
  unsigned char* const out = a.want_h ? reinterpret_cast<unsigned char*>(a.outh) : a.outq;
  bool fail = false;
#pragma unroll
  for (int g = 0; g < NVT; g += kI) {
    uint4 v[kI][WB];
#pragma unroll
    for (int i = 0; i < kI; ++i) {
      const int c = t + (g + i) * T;
      if (g + i >= NVT || c >= nvec) continue;
#pragma unroll
      for (int p = 0; p < WB; ++p) {
        const int64_t m = (int64_t)p * a.R + j;
        if (p >= a.world || p == me || m >= a.M) continue;
        v[i][p] = tp_ld_volatile_v4(slots + ((int64_t)b * a.g_half + m) * vbytes + 16 * c);
      }
    }
#pragma unroll
    for (int i = 0; i < kI; ++i) {
      const int c = t + (g + i) * T;
      if (g + i >= NVT || c >= nvec) continue;
#pragma unroll
      for (int p = 0; p < WB; ++p) {
        const int64_t m = (int64_t)p * a.R + j;
        if (p >= a.world || p == me || m >= a.M || fail) continue;
        unsigned char* src = slots + ((int64_t)b * a.g_half + m) * vbytes + 16 * c;
        if (a.want_h ? tp_pending16(v[i][p]) : tp_pending8(v[i][p])) {
          v[i][p] = a.want_h ? tp_poll_v4<false>(src, limit) : tp_poll_v4<true>(src, limit);
          fail = a.want_h ? tp_pending16(v[i][p]) : tp_pending8(v[i][p]);
        }
      }
    }
    if (fail) return false;
#pragma unroll
    for (int i = 0; i < kI; ++i) {
      const int c = t + (g + i) * T;
      if (g + i >= NVT || c >= nvec) continue;
#pragma unroll
      for (int p = 0; p < WB; ++p) {
        const int64_t m = (int64_t)p * a.R + j;
        if (p >= a.world || p == me || m >= a.M) continue;
        *reinterpret_cast<uint4*>(out + m * vbytes + 16 * c) = v[i][p];
        *reinterpret_cast<uint4*>(slots + ((int64_t)b * a.g_half + m) * vbytes + 16 * c) = tp_pattern4();
      }
    }
  }
  if (!a.want_h && t < a.world && t != me) {  // thread p: peer p's scale
    const int64_t m = (int64_t)t * a.R + j;
    if (m < a.M) {
      float* sp = a.grs[me] + (int64_t)b * a.g_half + m;
      const uint64_t t0 = global_ns();
      uint32_t v;
      for (uint32_t i = 1; (v = tp_ld_volatile_u32(sp)) == kTpPattern; ++i)
        if ((i & 63u) == 0 && global_ns() - t0 > limit) return false;
      a.outs[m] = __uint_as_float(v);
      *reinterpret_cast<uint32_t*>(sp) = kTpPattern;
    }
  }
  return true;
}

// End of a call, one thread per CTA after the CTA's last wait: the last CTA of
// the grid advances the epoch, unless a wait of this call ran out.
__device__ __forceinline__ void tp_finish_call(const TpRows& a, bool fail, int e) {
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

}  // namespace ms
