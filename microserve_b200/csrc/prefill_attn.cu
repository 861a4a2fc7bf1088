// Causal prefill attention, varlen over several sequences in one launch.
//
//  * kPaged = true : chunked prefill over the paged FP8 KV cache, the
//    reference's `_fp8_chunk_prefill_attention`
//    (microserve/layers/fp8_chunk_prefill_attention.py:8-67): K/V tiles are
//    dequantised as fp16(x_fp8 * scale) (the reference's rounding, :296-297),
//    scores = q . k^T in fp32 * softmax_scale, causal against
//    prefix_len + query index, P rounded to fp16 for P . V. The reference
//    handles one sequence per launch; here every sequence of the batch is
//    handled in one launch (prefix_len_s = kv_len_s - q_len_s).
//  * kPaged = false: first-chunk prefill over the fresh (unquantised) fp16
//    k and v, the FP8 PREFILL branch of the reference's Attention.forward
//    (microserve/layers/attention.py:49-55, flash_attn_varlen_func, causal).
//
// Design: one CTA per (64 query rows, kv head). The 64 rows are
// (token, q head) pairs of the G = Hq/Hkv heads sharing the kv head, so a K/V
// tile is staged once for all of them. K/V tiles of 64 keys are staged in
// shared memory as fp16 in a 16-byte-chunk XOR swizzle; products run on
// mma.m16n8k16 fed by ldmatrix (FlashAttention-2 register layout), online
// softmax in the exp2 domain with fp32 statistics.
#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kD = 128;
constexpr int kRows = 64;   // query rows per CTA
constexpr int kKeys = 64;   // keys per tile
constexpr float kLog2e = 1.4426950408889634f;

struct PrefillArgs {
  const __half* q;  // [T, Hq, D]
  const __half* k16;  // fresh mode: [T, Hkv, D]
  const __half* v16;
  const uint8_t* k_cache;  // paged mode: [NB, BS, Hkv, D]
  const uint8_t* v_cache;
  const float* k_scale;
  const float* v_scale;
  const int32_t* block_tables;  // [S, max_blocks]
  const int32_t* cu_q;          // [S + 1]
  const int32_t* kv_lens;       // [S] keys per sequence (paged); null in fresh mode
  __half* out;                  // [T, Hq, D]
  int num_seqs, Hq, Hkv, block_size, max_blocks;
  float scale_log2;
};

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t x) {
  __half2 h;
  memcpy(&h, &x, 4);
  return __half22float2(h);
}

template <bool kPaged>
__global__ void __launch_bounds__(128) prefill_kernel(PrefillArgs a) {
  __shared__ __align__(128) unsigned char sQ[kRows * 256];
  __shared__ __align__(128) unsigned char sK[kKeys * 256];
  __shared__ __align__(128) unsigned char sV[kKeys * 256];
  pdl_wait();
  pdl_trigger();

  const int kvh = blockIdx.y;
  const int G = a.Hq / a.Hkv;
  const int tpc = kRows / G;  // query tokens per CTA
  // Locate (sequence, block) of this CTA.
  int bx = blockIdx.x, seq = -1;
  for (int s = 0; s < a.num_seqs; ++s) {
    const int ql = a.cu_q[s + 1] - a.cu_q[s];
    const int nb = (ql + tpc - 1) / tpc;
    if (bx < nb) {
      seq = s;
      break;
    }
    bx -= nb;
  }
  if (seq < 0) return;
  const int q_start = a.cu_q[seq];
  const int q_len = a.cu_q[seq + 1] - q_start;
  const int kv_len = kPaged ? a.kv_lens[seq] : q_len;
  const int prefix = kv_len - q_len;
  const int tok0 = bx * tpc;  // first query index (within the sequence) of this CTA
  const int ntok = min(tpc, q_len - tok0);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;

  // ---- stage Q: row r = (token r / G, head r % G) --------------------------------
  for (int i = tid; i < kRows * 16; i += 128) {
    const int r = i >> 4, ch = i & 15;
    const int t = r / G, h = r % G;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < ntok) {
      const __half* src = a.q + ((int64_t)(q_start + tok0 + t) * a.Hq + kvh * G + h) * kD + ch * 8;
      v = *reinterpret_cast<const uint4*>(src);
    }
    *reinterpret_cast<uint4*>(sQ + swz(r, ch)) = v;
  }
  __syncthreads();

  // Q fragments for this warp's 16 rows: 8 k-steps of 16 d.
  uint32_t qa[8][4];
  {
    const int r = warp * 16 + (lane & 15);
    const uint32_t base = smem_u32(sQ);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int ch = 2 * s + (lane >> 4);
      ldsm_x4(base + swz(r, ch), qa[s][0], qa[s][1], qa[s][2], qa[s][3]);
    }
  }

  // Rows this thread owns in the accumulator layout: r0 = 16w + g, r1 = r0 + 8.
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  const int t0 = r0 / G, t1 = r1 / G;
  const int lim0 = (t0 < ntok) ? prefix + tok0 + t0 : -1;  // last visible key position
  const int lim1 = (t1 < ntok) ? prefix + tok0 + t1 : -1;

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  const int last_key = min(kv_len - 1, prefix + tok0 + ntok - 1);
  const int n_tiles = last_key / kKeys + 1;
  const int32_t* bt = kPaged ? a.block_tables + (int64_t)seq * a.max_blocks : nullptr;

  for (int kt = 0; kt < n_tiles; ++kt) {
    const int kbase = kt * kKeys;
    __syncthreads();  // previous tile fully consumed
    // ---- stage K and V tile as fp16 ------------------------------------------------
    if (kPaged) {
      const int page = kbase / a.block_size;
      const int64_t slot0 = (int64_t)bt[page] * a.block_size + (kbase - page * a.block_size);
      // 64 keys x 8 chunks of 16 fp8 bytes, per cache
      for (int i = tid; i < kKeys * 8; i += 128) {
        const int key = i >> 3, ch = i & 7;  // fp8 chunk -> fp16 chunks 2ch, 2ch+1
        uint4 kq = make_uint4(0, 0, 0, 0), vq = make_uint4(0, 0, 0, 0);
        float ks = 0.f, vs = 0.f;
        if (kbase + key < kv_len) {
          const int64_t row = (slot0 + key) * a.Hkv + kvh;
          kq = *reinterpret_cast<const uint4*>(a.k_cache + row * kD + ch * 16);
          vq = *reinterpret_cast<const uint4*>(a.v_cache + row * kD + ch * 16);
          ks = a.k_scale[row];
          vs = a.v_scale[row];
        }
        const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w};
        const uint32_t vw[4] = {vq.x, vq.y, vq.z, vq.w};
        uint32_t ko[8], vo[8];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float2 kf = h2_to_f2(e4m3x2_to_f16x2((uint16_t)(hh ? (kw[w] >> 16) : (kw[w] & 0xffff))));
            const float2 vf = h2_to_f2(e4m3x2_to_f16x2((uint16_t)(hh ? (vw[w] >> 16) : (vw[w] & 0xffff))));
            ko[2 * w + hh] = pack_h2(kf.x * ks, kf.y * ks);
            vo[2 * w + hh] = pack_h2(vf.x * vs, vf.y * vs);
          }
        }
        *reinterpret_cast<uint4*>(sK + swz(key, 2 * ch)) = make_uint4(ko[0], ko[1], ko[2], ko[3]);
        *reinterpret_cast<uint4*>(sK + swz(key, 2 * ch + 1)) = make_uint4(ko[4], ko[5], ko[6], ko[7]);
        *reinterpret_cast<uint4*>(sV + swz(key, 2 * ch)) = make_uint4(vo[0], vo[1], vo[2], vo[3]);
        *reinterpret_cast<uint4*>(sV + swz(key, 2 * ch + 1)) = make_uint4(vo[4], vo[5], vo[6], vo[7]);
      }
    } else {
      for (int i = tid; i < kKeys * 16; i += 128) {
        const int key = i >> 4, ch = i & 15;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (kbase + key < kv_len) {
          const int64_t row = (int64_t)(q_start + kbase + key) * a.Hkv + kvh;
          kv = *reinterpret_cast<const uint4*>(a.k16 + row * kD + ch * 8);
          vv = *reinterpret_cast<const uint4*>(a.v16 + row * kD + ch * 8);
        }
        *reinterpret_cast<uint4*>(sK + swz(key, ch)) = kv;
        *reinterpret_cast<uint4*>(sV + swz(key, ch)) = vv;
      }
    }
    __syncthreads();
    // skip the products when none of this warp's rows sees any key of the tile
    if (__all_sync(0xffffffffu, lim0 < kbase && lim1 < kbase)) continue;

    // ---- S = Q K^T : 16 rows x 64 keys -----------------------------------------------
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const uint32_t kb = smem_u32(sK);
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // key groups of 8
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {  // pairs of k-steps (32 d)
        uint32_t b0, b1, b2, b3;
        const int key = j * 8 + (lane & 7);
        const int ch = 4 * sp + (lane >> 3);
        ldsm_x4(kb + swz(key, ch), b0, b1, b2, b3);
        mma16816(s[j], qa[2 * sp], b0, b1);
        mma16816(s[j], qa[2 * sp + 1], b2, b3);
      }
    }
    // ---- mask, online softmax -----------------------------------------------------
    float tmax0 = -INFINITY, tmax1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k0 = kbase + j * 8 + 2 * c;
      s[j][0] = (k0 <= lim0) ? s[j][0] * a.scale_log2 : -INFINITY;
      s[j][1] = (k0 + 1 <= lim0) ? s[j][1] * a.scale_log2 : -INFINITY;
      s[j][2] = (k0 <= lim1) ? s[j][2] * a.scale_log2 : -INFINITY;
      s[j][3] = (k0 + 1 <= lim1) ? s[j][3] * a.scale_log2 : -INFINITY;
      tmax0 = fmaxf(tmax0, fmaxf(s[j][0], s[j][1]));
      tmax1 = fmaxf(tmax1, fmaxf(s[j][2], s[j][3]));
    }
    tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, 1));
    tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, 2));
    tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, 1));
    tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, 2));
    const float mn0 = fmaxf(m0, tmax0), mn1 = fmaxf(m1, tmax1);
    const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;  // rows with nothing visible yet
    const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
    const float al0 = ex2(m0 - mu0), al1 = ex2(m1 - mu1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = ex2(s[j][0] - mu0), p1 = ex2(s[j][1] - mu0);
      const float p2 = ex2(s[j][2] - mu1), p3 = ex2(s[j][3] - mu1);
      ps0 += p0 + p1;
      ps1 += p2 + p3;
      // accumulator tiles (2kk, 2kk+1) -> A operand of k-step kk
      const int kk = j >> 1, hi = j & 1;
      pa[kk][hi ? 2 : 0] = pack_h2(p0, p1);
      pa[kk][hi ? 3 : 1] = pack_h2(p2, p3);
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= al0; o[i][1] *= al0;
      o[i][2] *= al1; o[i][3] *= al1;
    }
    // ---- O += P V : 16 rows x 128 d -------------------------------------------------
    const uint32_t vb = smem_u32(sV);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
#pragma unroll
      for (int np = 0; np < 8; ++np) {  // pairs of 8-wide d tiles
        uint32_t b0, b1, b2, b3;
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = 2 * np + (lane >> 4);
        ldsm_x4_t(vb + swz(key, ch), b0, b1, b2, b3);
        mma16816(o[2 * np], pa[kk], b0, b1);
        mma16816(o[2 * np + 1], pa[kk], b2, b3);
      }
    }
  }

  // ---- normalise and store ------------------------------------------------------------
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  if (t0 < ntok) {
    __half* dst = a.out + ((int64_t)(q_start + tok0 + t0) * a.Hq + kvh * G + r0 % G) * kD;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      *reinterpret_cast<uint32_t*>(dst + 8 * i + 2 * c) = pack_h2(o[i][0] * inv0, o[i][1] * inv0);
  }
  if (t1 < ntok) {
    __half* dst = a.out + ((int64_t)(q_start + tok0 + t1) * a.Hq + kvh * G + r1 % G) * kD;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      *reinterpret_cast<uint32_t*>(dst + 8 * i + 2 * c) = pack_h2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

}  // namespace

cudaError_t launch_prefill_attention(bool paged, const void* q, const void* k16, const void* v16,
                                     const void* k_cache, const void* v_cache, const float* k_scale,
                                     const float* v_scale, const int32_t* block_tables, const int32_t* cu_q,
                                     const int32_t* kv_lens, void* out, int num_seqs, int total_q, int Hq, int Hkv,
                                     int head_dim, int block_size, int max_blocks, float softmax_scale,
                                     cudaStream_t stream) {
  if (head_dim != kD || Hq % Hkv != 0) return cudaErrorInvalidValue;
  const int G = Hq / Hkv;
  if (kRows % G != 0 || (paged && block_size % kKeys != 0)) return cudaErrorInvalidValue;
  if (total_q == 0 || num_seqs == 0) return cudaSuccess;
  const int tpc = kRows / G;
  // upper bound on CTAs over all sequences: sum ceil(len/tpc) <= total/tpc + num_seqs
  const int blocks = total_q / tpc + num_seqs;
  PrefillArgs a;
  a.q = (const __half*)q;
  a.k16 = (const __half*)k16;
  a.v16 = (const __half*)v16;
  a.k_cache = (const uint8_t*)k_cache;
  a.v_cache = (const uint8_t*)v_cache;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.block_tables = block_tables;
  a.cu_q = cu_q;
  a.kv_lens = kv_lens;
  a.out = (__half*)out;
  a.num_seqs = num_seqs;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.block_size = block_size;
  a.max_blocks = max_blocks;
  a.scale_log2 = softmax_scale * kLog2e;
  dim3 grid(blocks, Hkv);
  return paged ? launch_kernel(prefill_kernel<true>, grid, dim3(128), 0, stream, a)
               : launch_kernel(prefill_kernel<false>, grid, dim3(128), 0, stream, a);
}

}  // namespace ms
