// Paged FP8-KV decode attention (one query token per sequence), the
// reference's `_fp8_decode_flashAttention` (microserve/layers/fp8_decode_attention.py:8-59):
//   o[b, hq] = softmax_t(q[b,hq] . (k_fp8[t] * k_scale[t]) * sm_scale) . (v_fp8[t] * v_scale[t])
// over t < cache_seqlens[b], pages looked up in block_tables[b]. Rows with
// cache_seqlens == 0 produce 0.
//
// B200 design:
//  * One CTA per (split, kv head, sequence); the G = Hq/Hkv query heads that
//    share a kv head are processed together so every K/V byte is read once
//    (the reference re-reads K/V once per query head).
//  * Each warp streams its 16-token tiles of K, V and their scales through a
//    private ring of kStages shared-memory stages with cp.async (16-byte
//    copies, L2 only), so kStages tiles per warp are in flight without holding
//    registers; the 16-byte chunks of a row are XOR-swizzled so that both
//    fragment read patterns below are bank-conflict free. Fragments are
//    widened e4m3 -> f16 in registers (exact), and both products run on the
//    tensor cores with mma.m16n8k16 (f16 in, f32 accumulate):
//        S^T[tok, head] = K[tok, d] . Q^T[d, head]      (M = 16 tokens, N = 8 heads)
//        O^T[d, head]  += V^T[d, tok] . P'^T[tok, head] (M = 16 of d, N = 8 heads)
//    The head_dim axis of each product is permuted so that every thread's
//    fragment comes from contiguous bytes it loaded itself; Q and O use the
//    same permutation, so results are unchanged. The per-token k scale is
//    applied to the fp32 scores; the per-token v scale is folded into the
//    exponent (P' = exp2(s + log2(v_scale) - m), all weights in (0, 1]) and
//    P' enters the second product as two f16 parts (hi + lo), so the result
//    keeps fp32-level accuracy like the reference's all-fp32 kernel: FP8
//    activation quantisation downstream turns fp16-level attention errors
//    into visible output differences. P' changes from the accumulator layout
//    to the operand layout with movmatrix (an in-register 8x8 transpose).
//  * Online softmax in the exp2 domain, one running-max update per pair of
//    16-token tiles; warps of a CTA interleave tiles and are merged through
//    shared memory at the end. Long contexts with
//    few sequences are split over CTAs (flash-decoding); partial (m, l, o)
//    rows go to a workspace and a second kernel merges them.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kStages = 4;                               // tiles in flight per warp
constexpr int kTileBytes = 16 * kD;                      // one operand of a 16-token tile
constexpr int kStageBytes = 2 * kTileBytes + 2 * 16 * 4;  // K, V, k scales, v scales
constexpr int kSmemBytes = kWarps * kStages * kStageBytes;
static_assert(kSmemBytes >= (kWarps * 8 * (kD + 4) + 2 * kWarps * 8) * 4, "merge buffers alias the stages");
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kPScaleLog2 = 14.f;       // P' scaled into [0, 2^14] for its f16 hi/lo split
constexpr float kPUnscale = 1.f / 16384.f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Position of 16-byte chunk j of tile row r: j ^ swz(r). Makes both read
// patterns conflict free: K reads rows {2p, 2p+1} x chunks {0..3} (or {4..7})
// per quarter warp, V reads rows {0, 2, 4, 6} (+1, +8) x a chunk pair.
__device__ __forceinline__ int swz(int r) { return (r & 6) ^ ((r & 1) << 2); }

struct DecodeArgs {
  const __half* q;            // [B, Hq, D]
  const uint8_t* k_cache;     // [NB, BS, Hkv, D]
  const uint8_t* v_cache;
  const float* k_scale;       // [NB, BS, Hkv]
  const float* v_scale;
  const int32_t* seqlens;     // [B]
  const int32_t* block_tables;  // [B, max_blocks]
  __half* out;                // [B, Hq, D]
  float* ws_o;                // [B, Hq, S, D]   (S > 1 only)
  float* ws_ml;               // [B, Hq, S, 2]
  int B, Hq, Hkv, block_size, max_blocks, splits;
  int bs_log2;                // log2(block_size) when it is a power of two, else -1
  float scale_log2;           // softmax_scale * log2(e)
};

__global__ void __launch_bounds__(kWarps * 32, 3) decode_kernel(DecodeArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  pdl_wait();
  pdl_trigger();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int L = a.seqlens[b];
  const int ntiles = (L + 15) >> 4;
  const int tps = (ntiles + a.splits - 1) / a.splits;
  const int t_begin = split * tps;
  const int t_end = min(ntiles, t_begin + tps);

  // Q fragment: head g of this group, d = 64j + 16c + [0,16).
  uint32_t qf[2][8];
  {
    const bool valid = g < G;
    const __half* qrow = a.q + ((int64_t)b * a.Hq + kvh * G + (valid ? g : 0)) * kD;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 u0 = valid ? *reinterpret_cast<const uint4*>(qrow + 64 * j + 16 * c) : make_uint4(0, 0, 0, 0);
      uint4 u1 = valid ? *reinterpret_cast<const uint4*>(qrow + 64 * j + 16 * c + 8) : make_uint4(0, 0, 0, 0);
      qf[j][0] = u0.x; qf[j][1] = u0.y; qf[j][2] = u0.z; qf[j][3] = u0.w;
      qf[j][4] = u1.x; qf[j][5] = u1.y; qf[j][6] = u1.z; qf[j][7] = u1.w;
    }
  }

  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};  // heads 2c, 2c+1
  float l_run[2] = {0.f, 0.f};              // per-thread partial sums (reduced over g at the end)

  const int64_t tok_stride = (int64_t)a.Hkv * kD;  // bytes between consecutive tokens of a page
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;
  unsigned char* wsm = smem + warp * (kStages * kStageBytes);  // this warp's ring
  const uint32_t wsm_u32 = smem_u32(wsm);
  const int first = t_begin + warp;
  const int n_my = first < t_end ? (t_end - first + kWarps - 1) / kWarps : 0;

  // Copy tile number k of this warp (all lanes) into stage k % kStages. The 16
  // tokens of a tile never cross a page (block_size % 16 == 0), and every tile
  // starts below L, so its page is in the table and all 16 rows are in memory.
  // Per-lane constants of the copies: chunk (r, j) = (q >> 3, q & 7) for q = lane + 32 i,
  // and the scale row of this lane (k scales in lanes 0-15, v scales in 16-31).
  uint32_t so[4], go[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = lane + 32 * i, r = q >> 3, j = q & 7;
    so[i] = (uint32_t)(r * 128 + ((j ^ swz(r)) << 4));
    go[i] = (uint32_t)(r * tok_stride + 16 * j);
  }
  const float* sbase = (lane < 16 ? a.k_scale : a.v_scale) + (int64_t)(lane & 15) * a.Hkv + kvh;
  const uint32_t s_off = (uint32_t)(2 * kTileBytes + (lane >> 4) * 64 + (lane & 15) * 4);
  const uint8_t* kc = a.k_cache + (int64_t)kvh * kD;
  const uint8_t* vc = a.v_cache + (int64_t)kvh * kD;
  const int bs_shift = a.bs_log2;
  auto issue = [&](int k) {
    const int p0 = (first + k * kWarps) << 4;
    const int page = bs_shift >= 0 ? p0 >> bs_shift : p0 / a.block_size;
    const int64_t tok0 = (int64_t)__ldg(bt + page) * a.block_size + (p0 - page * a.block_size);
    const uint8_t* kb = kc + tok0 * tok_stride;
    const uint8_t* vb = vc + tok0 * tok_stride;
    const uint32_t st = wsm_u32 + (uint32_t)((k % kStages) * kStageBytes);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      cp_async16(st + so[i], kb + go[i]);
      cp_async16(st + kTileBytes + so[i], vb + go[i]);
    }
    cp_async4(st + s_off, sbase + tok0 * a.Hkv);
  };
#pragma unroll
  for (int k = 0; k < kStages; ++k) {
    if (k < n_my) issue(k);
    cp_async_commit();  // one group per tile slot, empty or not
  }

  auto ld = [](const unsigned char* t, int r, int j) {
    return *reinterpret_cast<const uint4*>(t + r * 128 + ((j ^ swz(r)) << 4));
  };
  // S^T = K . Q^T for the tile in ring slot `slot`: s[0], s[1] = token g, heads 2c, 2c+1;
  // s[2], s[3] = token g + 8 (raw dot products, before the k scale).
  auto scores = [&](int slot, float (&sc)[4]) {
    const unsigned char* sk = wsm + slot * kStageBytes;
    const uint4 k0a = ld(sk, g, c), k0b = ld(sk, g, 4 + c);  // K rows g, g+8: chunks c and 4 + c
    const uint4 k1a = ld(sk, g + 8, c), k1b = ld(sk, g + 8, 4 + c);
    const uint32_t kw0[8] = {k0a.x, k0a.y, k0a.z, k0a.w, k0b.x, k0b.y, k0b.z, k0b.w};
    const uint32_t kw1[8] = {k1a.x, k1a.y, k1a.z, k1a.w, k1b.x, k1b.y, k1b.z, k1b.w};
    sc[0] = sc[1] = sc[2] = sc[3] = 0.f;
#pragma unroll
    for (int st = 0; st < 8; ++st) {
      const int j = st >> 2, w = st & 3;
      const uint32_t r0 = e4m3x2_to_f16x2((uint16_t)(kw0[st] & 0xffff));
      const uint32_t r2 = e4m3x2_to_f16x2((uint16_t)(kw0[st] >> 16));
      const uint32_t r1 = e4m3x2_to_f16x2((uint16_t)(kw1[st] & 0xffff));
      const uint32_t r3 = e4m3x2_to_f16x2((uint16_t)(kw1[st] >> 16));
      mma16816(sc, r0, r1, r2, r3, qf[j][2 * w], qf[j][2 * w + 1]);
    }
  };
  // O^T += V^T . P'^T for the tile in ring slot `slot`, V rows past the end zeroed.
  auto accumulate = [&](int slot, int p0, uint32_t pb0, uint32_t pb1, uint32_t pc0, uint32_t pc1) {
    const unsigned char* sv = wsm + slot * kStageBytes + kTileBytes;
    uint4 v0 = ld(sv, 2 * c, g), v1 = ld(sv, 2 * c + 1, g);  // V rows 2c, 2c+1, 2c+8, 2c+9: chunk g
    uint4 v2 = ld(sv, 2 * c + 8, g), v3 = ld(sv, 2 * c + 9, g);
    if (p0 + 16 > L) {  // stale bytes past the end can never reach the product
      if (p0 + 2 * c >= L) v0 = make_uint4(0, 0, 0, 0);
      if (p0 + 2 * c + 1 >= L) v1 = make_uint4(0, 0, 0, 0);
      if (p0 + 2 * c + 8 >= L) v2 = make_uint4(0, 0, 0, 0);
      if (p0 + 2 * c + 9 >= L) v3 = make_uint4(0, 0, 0, 0);
    }
    const uint32_t va[4] = {v0.x, v0.y, v0.z, v0.w};
    const uint32_t vb[4] = {v1.x, v1.y, v1.z, v1.w};
    const uint32_t vc[4] = {v2.x, v2.y, v2.z, v2.w};
    const uint32_t vd[4] = {v3.x, v3.y, v3.z, v3.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int w = i >> 1;
      // bytes 2i, 2i+1 of the 16-byte chunks -> (row 2c, row 2c+1) pairs
      const uint32_t sel = (i & 1) ? 0x7362u : 0x5140u;
      const uint32_t lo = prmt(va[w], vb[w], sel);  // {R0[2i], R1[2i], R0[2i+1], R1[2i+1]}
      const uint32_t hi = prmt(vc[w], vd[w], sel);
      const uint32_t a0 = e4m3x2_to_f16x2((uint16_t)(lo & 0xffff));
      const uint32_t a1 = e4m3x2_to_f16x2((uint16_t)(lo >> 16));
      const uint32_t a2 = e4m3x2_to_f16x2((uint16_t)(hi & 0xffff));
      const uint32_t a3 = e4m3x2_to_f16x2((uint16_t)(hi >> 16));
      mma16816(acc[i], a0, a1, a2, a3, pb0, pb1);
      mma16816(acc[i], a0, a1, a2, a3, pc0, pc1);
    }
  };

  // Two tiles (k, k + 1) per iteration: one running-max update, one rescale of
  // the accumulators and one set of shuffles serve 32 tokens.
  for (int k = 0; k < n_my; k += 2) {
    cp_async_wait<kStages - 2>();  // this lane's copies of tiles k, k + 1 have landed
    __syncwarp();                  // ... and every other lane's
    const bool has1 = k + 1 < n_my;
    const int slot0 = k % kStages, slot1 = (k + 1) % kStages;
    const int pa = (first + k * kWarps) << 4, pb = (first + (k + 1) * kWarps) << 4;
    float sA[4], sB[4];
    scores(slot0, sA);
    if (has1) scores(slot1, sB);
    const float* ksA = reinterpret_cast<const float*>(wsm + slot0 * kStageBytes + 2 * kTileBytes);
    const float* ksB = reinterpret_cast<const float*>(wsm + slot1 * kStageBytes + 2 * kTileBytes);
    // token validity; the second tile counts as empty when this warp has no tile k + 1
    const bool a0 = pa + g < L, a1 = pa + g + 8 < L;
    const bool b0 = has1 && pb + g < L, b1 = has1 && pb + g + 8 < L;
    sA[0] = a0 ? sA[0] * ksA[g] * a.scale_log2 : -INFINITY;
    sA[1] = a0 ? sA[1] * ksA[g] * a.scale_log2 : -INFINITY;
    sA[2] = a1 ? sA[2] * ksA[g + 8] * a.scale_log2 : -INFINITY;
    sA[3] = a1 ? sA[3] * ksA[g + 8] * a.scale_log2 : -INFINITY;
    sB[0] = b0 ? sB[0] * ksB[g] * a.scale_log2 : -INFINITY;
    sB[1] = b0 ? sB[1] * ksB[g] * a.scale_log2 : -INFINITY;
    sB[2] = b1 ? sB[2] * ksB[g + 8] * a.scale_log2 : -INFINITY;
    sB[3] = b1 ? sB[3] * ksB[g + 8] * a.scale_log2 : -INFINITY;

    // Fold the per-token v scale into the exponent: w = p * v_scale = exp2(s + log2(v_scale) - m),
    // with the running max m taken over s + log2(v_scale), so every weight is in (0, 1] and its
    // f16 hi/lo split (below) keeps ~22 bits. The denominator sums exp2(s - m) in fp32.
    const float lvA0 = a0 ? lg2(ksA[16 + g]) : 0.f, lvA1 = a1 ? lg2(ksA[16 + g + 8]) : 0.f;
    const float lvB0 = b0 ? lg2(ksB[16 + g]) : 0.f, lvB1 = b1 ? lg2(ksB[16 + g + 8]) : 0.f;
    const float wA[4] = {sA[0] + lvA0, sA[1] + lvA0, sA[2] + lvA1, sA[3] + lvA1};
    const float wB[4] = {sB[0] + lvB0, sB[1] + lvB0, sB[2] + lvB1, sB[3] + lvB1};
    float tmax0 = fmaxf(fmaxf(wA[0], wA[2]), fmaxf(wB[0], wB[2]));
    float tmax1 = fmaxf(fmaxf(wA[1], wA[3]), fmaxf(wB[1], wB[3]));
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, o));
      tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, o));
    }
    const float mn0 = fmaxf(m_run[0], tmax0), mn1 = fmaxf(m_run[1], tmax1);
    // Tile k always holds token pa < L, so mn is finite here.
    const float al0 = ex2(m_run[0] - mn0), al1 = ex2(m_run[1] - mn1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    l_run[0] = l_run[0] * al0 + ((ex2(sA[0] - mn0) + ex2(sA[2] - mn0)) + (ex2(sB[0] - mn0) + ex2(sB[2] - mn0)));
    l_run[1] = l_run[1] * al1 + ((ex2(sA[1] - mn1) + ex2(sA[3] - mn1)) + (ex2(sB[1] - mn1) + ex2(sB[3] - mn1)));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[i][0] *= al0; acc[i][1] *= al1;
      acc[i][2] *= al0; acc[i][3] *= al1;
    }
    // P'^T operands, as f16 hi + lo parts, transposed to the B layout. The weights are
    // scaled by 2^kPScaleLog2 (undone in the final division) so that lo stays a normal
    // f16 for every weight that matters (P' >= 2^-16).
    auto pmat = [&](const float (&w)[4], uint32_t& pb0, uint32_t& pb1, uint32_t& pc0, uint32_t& pc1) {
      const float q00 = ex2(w[0] - mn0 + kPScaleLog2), q01 = ex2(w[1] - mn1 + kPScaleLog2);
      const float q10 = ex2(w[2] - mn0 + kPScaleLog2), q11 = ex2(w[3] - mn1 + kPScaleLog2);
      const uint32_t h0 = pack_h2(q00, q01), h1 = pack_h2(q10, q11);
      const float2 h0f = h2_to_f2(h0), h1f = h2_to_f2(h1);
      const uint32_t l0 = pack_h2(q00 - h0f.x, q01 - h0f.y), l1 = pack_h2(q10 - h1f.x, q11 - h1f.y);
      pb0 = movmatrix_trans(h0);
      pb1 = movmatrix_trans(h1);
      pc0 = movmatrix_trans(l0);
      pc1 = movmatrix_trans(l1);
    };
    uint32_t pb0, pb1, pc0, pc1;
    pmat(wA, pb0, pb1, pc0, pc1);
    accumulate(slot0, pa, pb0, pb1, pc0, pc1);
    if (has1) {
      pmat(wB, pb0, pb1, pc0, pc1);
      accumulate(slot1, pb, pb0, pb1, pc0, pc1);
    }
    __syncwarp();  // every lane is done with both slots: they may be refilled
    if (k + kStages < n_my) issue(k + kStages);
    cp_async_commit();
    if (k + 1 + kStages < n_my) issue(k + 1 + kStages);
    cp_async_commit();
  }

  // ---- merge warps ---------------------------------------------------------
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], o);
    l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], o);
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with its ring: reuse it for the merge
  float(*sm_o)[8][kD + 4] = reinterpret_cast<float(*)[8][kD + 4]>(smem);
  float(*sm_m)[8] = reinterpret_cast<float(*)[8]>(smem + sizeof(float) * kWarps * 8 * (kD + 4));
  float(*sm_l)[8] = sm_m + kWarps;
  if (g == 0) {
    sm_m[warp][2 * c] = m_run[0];
    sm_m[warp][2 * c + 1] = m_run[1];
    sm_l[warp][2 * c] = l_run[0];
    sm_l[warp][2 * c + 1] = l_run[1];
  }
  // acc[i][0..1]: d = 16g + 2i, heads 2c, 2c+1; acc[i][2..3]: d = 16g + 2i + 1.
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sm_o[warp][2 * c][16 * g + 2 * i] = acc[i][0];
    sm_o[warp][2 * c + 1][16 * g + 2 * i] = acc[i][1];
    sm_o[warp][2 * c][16 * g + 2 * i + 1] = acc[i][2];
    sm_o[warp][2 * c + 1][16 * g + 2 * i + 1] = acc[i][3];
  }
  __syncthreads();
  // Thread t handles (head = t / 16, d = 8 * (t % 16) .. +8) for heads < G.
  for (int item = threadIdx.x; item < G * 16; item += blockDim.x) {
    const int h = item >> 4, d0 = (item & 15) * 8;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w][h]);
    float Lsum = 0.f, o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float wt = (sm_m[w][h] == -INFINITY) ? 0.f : ex2(sm_m[w][h] - M);
      Lsum += sm_l[w][h] * wt;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] += sm_o[w][h][d0 + e] * wt;
    }
    const int hq = kvh * G + h;
    if (a.splits == 1) {
      const float inv = (L > 0 && Lsum > 0.f) ? kPUnscale / Lsum : 0.f;
      uint4 packed;
      packed.x = pack_h2(o[0] * inv, o[1] * inv);
      packed.y = pack_h2(o[2] * inv, o[3] * inv);
      packed.z = pack_h2(o[4] * inv, o[5] * inv);
      packed.w = pack_h2(o[6] * inv, o[7] * inv);
      *reinterpret_cast<uint4*>(a.out + ((int64_t)b * a.Hq + hq) * kD + d0) = packed;
    } else {
      const int64_t row = ((int64_t)b * a.Hq + hq) * a.splits + split;
      float* dst = a.ws_o + row * kD + d0;
      *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4], o[5], o[6], o[7]);
      if (d0 == 0) {
        a.ws_ml[row * 2] = M;
        a.ws_ml[row * 2 + 1] = Lsum;
      }
    }
  }
}

// Merge split partials: one CTA per (sequence, q head), one thread per d.
__global__ void __launch_bounds__(kD) decode_merge_kernel(const float* __restrict__ ws_o,
                                                          const float* __restrict__ ws_ml,
                                                          const int32_t* __restrict__ seqlens, int Hq, int splits,
                                                          __half* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y, hq = blockIdx.x, d = threadIdx.x;
  const int64_t row0 = ((int64_t)b * Hq + hq) * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ws_ml[(row0 + s) * 2]);
  float Lsum = 0.f, o = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = ws_ml[(row0 + s) * 2];
    const float wt = (m == -INFINITY) ? 0.f : ex2(m - M);
    Lsum += ws_ml[(row0 + s) * 2 + 1] * wt;
    o += ws_o[(row0 + s) * kD + d] * wt;
  }
  const float r = (seqlens[b] > 0 && Lsum > 0.f) ? o * kPUnscale / Lsum : 0.f;
  out[((int64_t)b * Hq + hq) * kD + d] = __float2half_rn(r);
}

}  // namespace

int decode_num_splits(int B, int Hkv, int max_blocks, int block_size, int num_sms) {
  const int ctas = B * Hkv;
  const int target = num_sms * 4;
  if (ctas >= target) return 1;
  const int max_ctx = max_blocks * block_size;
  // at least 8 tiles (128 tokens) per split so each warp has work
  const int max_split = max(1, (max_ctx + 127) / 128);
  int s = (target + ctas - 1) / ctas;
  return min(s, min(max_split, 256));
}

size_t decode_workspace_bytes(int B, int Hq, int splits) {
  if (splits <= 1) return 0;
  return (size_t)B * Hq * splits * (kD + 2) * sizeof(float);
}

cudaError_t launch_decode_attention(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                                    const float* v_scale, const int32_t* seqlens, const int32_t* block_tables,
                                    void* out, int B, int Hq, int Hkv, int head_dim, int block_size, int max_blocks,
                                    float softmax_scale, int splits, void* workspace, cudaStream_t stream) {
  if (head_dim != kD || Hq % Hkv != 0 || Hq / Hkv > 8 || block_size % 16 != 0 || splits < 1)
    return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  DecodeArgs a;
  a.q = (const __half*)q;
  a.k_cache = (const uint8_t*)k_cache;
  a.v_cache = (const uint8_t*)v_cache;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.seqlens = seqlens;
  a.block_tables = block_tables;
  a.out = (__half*)out;
  a.ws_o = (float*)workspace;
  a.ws_ml = splits > 1 ? (float*)workspace + (size_t)B * Hq * splits * kD : nullptr;
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.block_size = block_size;
  a.bs_log2 = (block_size & (block_size - 1)) == 0 ? __builtin_ctz((unsigned)block_size) : -1;
  a.max_blocks = max_blocks;
  a.splits = splits;
  a.scale_log2 = softmax_scale * kLog2e;
  dim3 grid(splits, Hkv, B);
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  cudaError_t e = launch_kernel(decode_kernel, grid, dim3(kWarps * 32), kSmemBytes, stream, a);
  if (e != cudaSuccess || splits <= 1) return e;
  return launch_kernel(decode_merge_kernel, dim3(Hq, B), dim3(kD), 0, stream, (const float*)a.ws_o,
                       (const float*)a.ws_ml, seqlens, Hq, splits, (__half*)out);
}

// ---------------------------------------------------------------------------
// Allocation-free variant (ms_paged_decode_fp8_noalloc).
//
// Some callers cannot allocate device memory at the point where they run
// attention: code running inside another framework's allocator or memory
// pool, embedders that forbid cudaMalloc after start-up, or callers whose
// only handle is a stream. For them the context-split partials live in a
// fixed buffer compiled into the library. Every GPU that loads the library
// holds this buffer (kNoAllocScratchBytes) until the process exits. All calls
// on a device share it: calls that overlap on the GPU (two streams, or two
// host threads) race on it and must be serialised by the caller. Nothing in
// it needs to start at zero: each call writes every partial it later reads.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = 4u << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];
}  // namespace

size_t decode_noalloc_scratch_bytes() { return kNoAllocScratchBytes; }

// Device address of the built-in scratch on the current device. Host code
// cannot use the symbol itself (it names a host-side stand-in), so the
// address is looked up with that device current and cached per device and
// CUDA context: after a context is destroyed and recreated (cudaDeviceReset)
// the next call looks it up again. A look-up (the first call on a device, or
// the first after a reset) must not happen during stream capture.
cudaError_t decode_noalloc_scratch(void** ptr) {
  typedef CUresult (*CtxFn)(CUcontext*);
  static std::mutex mu;
  static void* addr[64] = {};
  static CUcontext ctx_of[64] = {};
  static CtxFn ctx_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      ctx_fn = reinterpret_cast<CtxFn>(f);
  });
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (ctx_fn == nullptr) return cudaErrorUnknown;
  CUcontext ctx = nullptr;
  if (ctx_fn(&ctx) != CUDA_SUCCESS) return cudaErrorUnknown;
  std::lock_guard<std::mutex> g(mu);
  if (ctx == nullptr || addr[dev] == nullptr || ctx_of[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // also makes the device's context current
    if (e != cudaSuccess) return e;
    if (ctx_fn(&ctx) != CUDA_SUCCESS) return cudaErrorUnknown;
    addr[dev] = p;
    ctx_of[dev] = ctx;
  }
  *ptr = addr[dev];
  return cudaSuccess;
}

}  // namespace ms
