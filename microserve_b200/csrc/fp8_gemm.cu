// FP8 e4m3 W8A8 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   Y[m, n] = fp16( (sum_k Xq[m,k] * Wq[n,k]) * sx[m] * sw[n] )   (+ bias[n], rounded again)
//
// This is the reference's `_fp8_mm` + `FP8DynamicLinear.forward`
// (microserve/layers/fp8_linear.py:26-45, :64-80): fp32 accumulation of exact
// e4m3 products, per-token-row x per-output-channel dequant in the epilogue.
//
// Layout: Xq [M, K] and Wq [N, K] are both K-contiguous ("TN"). The kernel
// computes the transposed product D[n, m] = Wq . Xq^T, so the weight matrix is
// the MMA's M operand (128 rows per tile) and the tokens are its N operand
// (BN = 32..256 columns). Decode batches (M <= 256 tokens) then fill one
// tile's N and the kernel streams the weights once; prefill uses the same
// tile shape over more token tiles.
//
// Per CTA: warp 0 issues TMA loads (128B-swizzled, K-major) into a ring of
// shared-memory stages of CH 128-byte K chunks each (one TMA box per operand
// per stage); warp 1 owns the TMEM accumulator and issues tcgen05.mma
// (kind::f8f6f4, 128 x BN x 32 per instruction, 4 per chunk); warps 2-5 drain
// TMEM with tcgen05.ld and apply the dequant epilogue. The kernel is
// persistent: whole tiles round-robin when they fill the SMs evenly, else
// stream-K (the tiles x K-steps work split evenly over at most one CTA per SM,
// tiles shared by two CTAs summed in-kernel from fp32 partials in the caller's
// workspace), so there is no wave quantisation and no separate reduction pass.
// Programmatic dependent launch: the weight loads of the first stage and the
// CTA prologue may overlap the preceding grid; everything that reads its
// results (activations, token scales, workspace, output) waits for it.
//
// Two more tile shapes: 256 weight rows x 256 tokens on one SM (fp8_gemm_wide_kernel,
// two M = 128 MMAs sharing each token stage) and, opt-in (ms_set_pair_tiles), 256
// weight rows x BN tokens on a pair of SMs (fp8_gemm_pair_kernel, tcgen05 cta_group::2).
// Every kernel also takes fp16 operands (kind::f16, K counted in bytes, no scales) for
// the LM head (ms_f16_gemm).
//
// Every wait is bounded (common.cuh: mbar_wait); on a timeout the kernel
// records a device status, skips the rest and still frees its TMEM.
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"
#include "tp_rows.cuh"

namespace ms {
namespace {

constexpr int kBM = 128;          // weight rows per tile (MMA M)
constexpr int kChunk = 128;       // K bytes per swizzle span (one 128B-swizzled tile row)
constexpr int kThreads = 192;     // 6 warps

struct GemmArgs {
  int M, N, K;
  int KT;       // K steps of CH chunks
  int tiles_m;  // token tiles
  int64_t T;    // output tiles
  int64_t U;    // work units = tiles * KT
  int G;        // CTAs (persistent, one per SM at most)
  int dp;       // 1: whole tiles round-robin (no K split); 0: stream-K or split-K
  int splits;   // split-K: CTAs per tile (CTA c = tile c / splits, K part c % splits); 0 otherwise
  const float* sx;
  const float* sw;
  const __half* bias;
  __half* y;
  float* ws;   // [G][BN][kBM] fp32 partial tiles (stream-K fixup)
  int* flags;  // [G] partial-ready flags; zero before and after every launch
  int tma_y;   // 1: the output tensor map is valid (N % 8 == 0, y 16-byte aligned)
  int f16;     // 1: fp16 operands (kind::f16; K counted in bytes, sx / sw null = 1)
  // Row-parallel push (tensor parallelism, rp_R > 0): instead of y, output row m
  // goes to rank m / rp_R's receive slot [b][rp_rank][m mod rp_R] (b = the parity
  // of the epoch word *rp_ctrl), over NVLink for the other ranks (tp_rows.cuh).
  __half* rp_recv[kTpMaxWorld];
  const int* rp_ctrl;
  int64_t rp_half, rp_src;  // elements of one parity set / of one source's slots
  int rp_R, rp_rank;
  // rp_tail: after its tiles, every CTA also does the tensor-parallel row work
  // (reduce + residual + RMSNorm + FP8, gather; tp_rows.cuh) for the row indices
  // j = CTA, CTA + grid, ... < R, so the whole row-parallel linear + all-reduce +
  // norm is this one kernel. Needs every CTA of the grid resident (grid <= SMs).
  int rp_tail, rp_nvt;
  TpRows tail;
};

// BN: token columns per tile (MMA N). CH: 128-byte K chunks per pipeline stage.
// With CH = 2 the operands are described by 3D tensor maps (chunk, row, byte)
// so ONE TMA box brings two chunks (e.g. 32 KB of weights): TMA throughput per
// SM is bounded by boxes per second, not bytes, for boxes up to 32 KB.
template <int BN, int CH>
struct Cfg {
  static constexpr int kChunkA = kBM * kChunk;  // one K chunk of the weight tile (16 KB)
  static constexpr int kChunkB = BN * kChunk;   // one K chunk of the token tile
  static constexpr int kABytes = CH * kChunkA;
  static constexpr int kStageBytes = CH * (kChunkA + kChunkB);
  static constexpr int kAccCols = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));  // TMEM columns
  static constexpr int kTmemCols = 2 * kAccCols;  // two accumulators (double buffer)
  static constexpr int kSxBytes = 2 * BN * 4;     // token scales of the current tile, double-buffered
  static constexpr int kRowsBytes = 2 * BN * 8;   // row-parallel push: destination of each token row
  static constexpr int kBarBytes = 256;
  static constexpr int kFit = (227 * 1024 - 1024 - kBarBytes - kSxBytes - kRowsBytes) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + kBarBytes + kSxBytes + kRowsBytes;
  // tcgen05 instruction descriptor: D=f32, A=B=e4m3, both K-major, N=BN, M=128.
  static constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
  static_assert(kStages >= 2, "shared memory budget");
  static_assert(BN % 16 == 0 && BN <= 256, "MMA N");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);  // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                   // layout: SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint32_t dst, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint32_t dst, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Bulk tensor store of a staged output tile (shared -> global), then wait until
// it is complete. One thread.
__device__ __forceinline__ void tma_store_2d_wait(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(src)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The tensor-parallel row work at the end of a row-parallel GEMM (rp_tail): runs on
// all threads of the CTA once its tiles are pushed; the stage buffers are free by
// then and hold the staged row (smem >= H * 2 + 256 bytes).
template <int NVT, int WB>
__device__ __noinline__ void rowpar_tail(const TpRows& a, unsigned char* smem) {
  H8* srow = reinterpret_cast<H8*>(smem);
  float* red_ss = reinterpret_cast<float*>(smem + a.H * 2);
  float* red_max = red_ss + kMaxRowWarps;
  int* s_e = reinterpret_cast<int*>(red_max + 32);
  // no CTA can advance the epoch before this one arrives, so this is the call's epoch
  if (threadIdx.x == 0) *s_e = *reinterpret_cast<volatile int*>(a.ctrl);
  __syncthreads();
  const int e = *s_e, b = e & 1;
  const uint64_t limit = wait_limit_ns();
  bool fail = false;
  for (int j = blockIdx.x; j < a.R && !fail; j += gridDim.x)
    if (a.rank * a.R + j < a.M) fail = !tp_reduce_row<NVT, WB>(a, j, b, limit, srow, red_ss, red_max);
  for (int j = blockIdx.x; j < a.R && !fail; j += gridDim.x) fail = !tp_collect_rows<NVT, WB>(a, j, b, limit);
  fail = __syncthreads_or(fail) != 0;
  if (threadIdx.x == 0) tp_finish_call(a, fail, e);
}

// Row-parallel destination of output row m (rank m / R's receive slot for this rank).
__device__ __forceinline__ __half* rp_row(const GemmArgs& a, int m, int b) {
  const int owner = m / a.rp_R;
  return a.rp_recv[owner] + (int64_t)b * a.rp_half + a.rp_rank * a.rp_src + (int64_t)(m - owner * a.rp_R) * a.N;
}
// A pushed value never has the receive slots' "not yet written" pattern (0xFFFF, a NaN).
__device__ __forceinline__ __half rp_out(__half h) {
  return __half_as_ushort(h) == 0xFFFFu ? __ushort_as_half((unsigned short)0x7FFFu) : h;
}

// Output of 16 token columns of one weight row n: y = fp16(fp16(v * sx * sw[n]) + bias[n]).
// With `stage` the values go to a shared-memory tile [tokens][128 rows] fp16 (the
// CTA then writes the tile with one bulk tensor store); without, straight to y
// with one 2-byte store per token (64 bytes per warp instruction).
__device__ __forceinline__ void out16(const GemmArgs& args, const float* v, const float* sx, float swn, float bn,
                                      int m0, int c0, int cols, int n, __half* stage, int row,
                                      __half* const* rows = nullptr) {
  const float4* sxv = reinterpret_cast<const float4*>(sx + c0);
  float sc[16];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float4 f = sxv[g];
    sc[4 * g] = f.x;
    sc[4 * g + 1] = f.y;
    sc[4 * g + 2] = f.z;
    sc[4 * g + 3] = f.w;
  }
  __half r[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) r[j] = __float2half_rn(v[j] * sc[j] * swn);
  if (args.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = __float2half_rn(__half2float(r[j]) + bn);
  }
  if (stage != nullptr) {
#pragma unroll
    for (int j = 0; j < 16; ++j) stage[(c0 + j) * kBM + row] = r[j];
    return;
  }
  if (n >= args.N) return;
  if (rows != nullptr) {  // row-parallel push: each token row to its owner's slot
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < cols) rows[c0 + j][n] = rp_out(r[j]);
    return;
  }
  const int64_t N = args.N;
  __half* yp = args.y + (int64_t)(m0 + c0) * N + n;
  if (c0 + 16 <= cols) {
#pragma unroll
    for (int j = 0; j < 16; ++j) yp[j * N] = r[j];
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < cols) yp[j * N] = r[j];
  }
}

// One stage of an operand: CH chunks starting at K step k, rows from `row`.
template <int CH>
__device__ __forceinline__ void load_stage(const CUtensorMap* map, uint32_t dst, uint64_t* bar, int k, int row) {
  if constexpr (CH == 1) {
    tma_load_2d(map, dst, bar, k * kChunk, row);
  } else {
    tma_load_3d(map, dst, bar, 0, row, k * CH);
  }
}

// fp16 operands: the same 32 bytes of K per instruction (16 elements), and the
// same instruction descriptor (format code 0 is f16 for kind::f16, e4m3 for
// kind::f8f6f4).
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void umma_f8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Epilogue warps only (4 warps, 128 threads): named barrier 1.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// First work unit of CTA c under the even partition of U units over G CTAs.
__device__ __forceinline__ int64_t unit_begin(int64_t c, int64_t U, int G) { return c * U / G; }

// The work of one CTA as a sequence of segments (tile t, K steps [kb, ke)).
// Data-parallel mode: whole tiles cta, cta + G, ...; stream-K mode: the
// CTA's contiguous range of the U = T * KT units, cut at tile boundaries.
struct SegIter {
  int64_t u, u_end, t_dp;
  int64_t T;
  int KT, G, dp, splits, cta;
  __device__ SegIter(const GemmArgs& a, int cta_)
      : u(unit_begin(cta_, a.U, a.G)), u_end(unit_begin(cta_ + 1, a.U, a.G)), t_dp(cta_), T(a.T), KT(a.KT),
        G(a.G), dp(a.dp), splits(a.splits), cta(cta_) {}
  __device__ bool next(int64_t& t, int& kb, int& ke) {
    if (splits > 0) {  // one segment: K part (cta % splits) of tile cta / splits
      if (t_dp < 0) return false;
      t = cta / splits;
      const int j = cta % splits;
      kb = (int)((int64_t)j * KT / splits);
      ke = (int)((int64_t)(j + 1) * KT / splits);
      t_dp = -1;
      return true;
    }
    if (dp) {
      if (t_dp >= T) return false;
      t = t_dp;
      kb = 0;
      ke = KT;
      t_dp += G;
      return true;
    }
    if (u >= u_end) return false;
    t = u / KT;
    kb = (int)(u - t * KT);
    ke = (int)((int64_t)KT < kb + (u_end - u) ? (int64_t)KT : kb + (u_end - u));
    u += ke - kb;
    return true;
  }
};

// K-loop start offset of a whole-tile segment: different weight tiles begin at
// different K so the CTAs of a wave spread their activation reads over L2.
__device__ __forceinline__ int k_rotation(const GemmArgs& a, int64_t t, int kb, int ke) {
  if (!a.dp || ke - kb < 2) return 0;
  return (int)(((t / a.tiles_m) * 5) % (ke - kb));
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Split-K epilogue (all 128 epilogue threads of a CTA). The `splits` CTAs of a
// tile each hold a K part in TMEM. Every CTA stores its fp32 partial
// (column-major [BN][128], 8 KB per 16 columns) to its workspace slot and
// arrives on the tile's counter; once all parts are in, each CTA reduces a
// different slice of 16-column chunks: one thread brings that slice of every
// partial into shared memory with bulk copies (the pipeline stages are idle:
// one tile per CTA), then each thread sums its row over the parts in a fixed
// order, applies the dequant scales and stores. The counter goes to 2 *
// splits (arrive, then done) and the last CTA resets it to zero.
template <int BN, int CH>
__device__ __forceinline__ void split_epilogue(const GemmArgs& args, uint32_t acc, int64_t t, int m0, int cols, int n,
                                               bool n_ok, float swn, float bn, const float* sx, float* my_ws,
                                               unsigned char* smem, uint64_t* red_full, uint64_t* acc_empty, int et,
                                               int row, __half* const* rows) {
  using C = Cfg<BN, CH>;
  const int S = args.splits;
  for (int c0 = 0; c0 < BN; c0 += 16) {
    float v[16];
    tmem_ld16(acc + (uint32_t)c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) my_ws[(int64_t)(c0 + j) * kBM + row] = v[j];
  }
  // These stores are read back by bulk copies (the async proxy), in this CTA and
  // in the tile's other CTAs: order them for that proxy, then GPU-wide.
  asm volatile("fence.proxy.async.global;" ::: "memory");
  __threadfence();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  mbar_arrive(acc_empty);
  constexpr int kChunks = BN / 16;
  const int part = (int)(blockIdx.x % S);
  const int per = (kChunks + S - 1) / S;
  const int q0 = min(kChunks, part * per), q1 = min(kChunks, q0 + per);
  int* cnt = args.flags + t;
  epi_sync();  // every partial store of this CTA precedes the release below
  if (et == 0) {
    atomicAdd(cnt, 1);
    const uint64_t t0 = global_ns();
    uint32_t spins = 0;
    while (ld_acquire(cnt) < S) {
      if ((++spins & 255u) == 0 && global_ns() - t0 > wait_limit_ns()) {
        set_device_status(kStatusMbarTimeout);
        break;
      }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the bulk copies below read other CTAs' stores
    const uint32_t bytes = (uint32_t)(S * (q1 - q0)) * 16u * kBM * 4u;
    mbar_arrive_expect_tx(red_full, bytes);
    const float* base = args.ws + (int64_t)(t * S) * BN * kBM;
    for (int p = 0; p < S; ++p)
      for (int q = q0; q < q1; ++q)
        bulk_g2s(smem_u32(smem + (size_t)(p * per + (q - q0)) * 16 * kBM * 4),
                 base + (int64_t)p * BN * kBM + (int64_t)q * 16 * kBM, 16u * kBM * 4u, red_full);
  }
  static_assert(C::kStages * C::kStageBytes >= (kChunks + 8) * 16 * kBM * 4, "split-K slices fit the stages");
  const bool ok = mbar_wait(red_full, 0);
  const float* red = reinterpret_cast<const float*>(smem);
  for (int q = q0; ok && q < q1; ++q) {
    const int c0 = q * 16;
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
    for (int p = 0; p < S; ++p) {
      const float* src = red + (size_t)(p * per + (q - q0)) * 16 * kBM + row;
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += src[j * kBM];
    }
    if (!n_ok || c0 >= cols) continue;
    __half r[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = __float2half_rn(v[j] * sx[c0 + j] * swn);
    if (args.bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 16; ++j) r[j] = __float2half_rn(__half2float(r[j]) + bn);
    }
    if (rows != nullptr) {  // row-parallel push
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c0 + j < cols) rows[c0 + j][n] = rp_out(r[j]);
      continue;
    }
    __half* yp = args.y + (int64_t)(m0 + c0) * args.N + n;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < cols) yp[(int64_t)j * args.N] = r[j];
  }
  epi_sync();  // every thread is past its wait on the counter's first phase
  if (et == 0) {
    if (atomicAdd(cnt, 1) == 2 * S - 1) *cnt = 0;  // last of the 2 * splits arrivals
  }
}

// Persistent GEMM, data-parallel or stream-K. In stream-K mode the U = tiles *
// KT work units (one K step of one 128 x BN output tile) are split evenly over
// G CTAs; each CTA walks its contiguous range tile by tile ("segments"). A
// segment that starts at k = 0 owns its tile: when the tile continues in later
// CTAs, the owner adds their fp32 partials (ws, flagged ready) before the
// epilogue. A segment that starts mid-tile stores its partial and raises its
// flag. The accumulator is double-buffered in TMEM so a tile's epilogue
// overlaps the next tile's main loop.
//
// Roles: warp 0 lane 0 issues TMA, warp 1 owns TMEM and lane 0 issues MMAs,
// warps 2-5 are the epilogue (TMEM lane quarter = warp % 4). The other lanes
// of warps 0-1 wait at __syncwarp so every warp reaches the final block
// barrier converged (a partially arrived warp would count as arrived).
template <int BN, int CH, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ GemmArgs args) {
  using C = Cfg<BN, CH>;
  static_assert(C::kStages * C::kStageBytes >= BN * kBM * 2, "staged output tile fits the stages");
  // The 128B swizzle atoms need 1024-byte alignment. The dynamic window is only
  // guaranteed 16-byte aligned (it follows any static shared memory), so align by
  // hand; declaring the array __align__(1024) would let the compiler fold the
  // adjustment below to zero.
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* red_full = acc_empty + 2;       // split-K: partial slices landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_full + 1);
  float* s_sx = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes + C::kBarBytes);  // [2][BN]
  __half** s_rows = reinterpret_cast<__half**>(smem + C::kStages * C::kStageBytes + C::kBarBytes + C::kSxBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int KT = args.KT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(red_full, 1);
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int i = 0;  // stage counter across segments
      SegIter it(args, cta);
      int64_t t;
      int kb, ke;
      bool ok = true, waited = false;
      while (ok && it.next(t, kb, ke)) {
        const int n0 = (int)(t / args.tiles_m) * kBM;
        const int m0 = (int)(t % args.tiles_m) * BN;
        const int nk = ke - kb, rot = k_rotation(args, t, kb, ke);
        for (int j = 0; j < nk; ++j, ++i) {
          const int s = i % C::kStages;
          const uint32_t ph = (uint32_t)(i / C::kStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u)) {
            ok = false;
            break;
          }
          const int k = kb + (j + rot) % nk;
          unsigned char* sa = smem + s * C::kStageBytes;
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          // weights never depend on the preceding grid: stream them before waiting for it
          // (requesting every free stage's weights before the wait measured slower: the
          // first stage's activations then queue behind them)
          load_stage<CH>(&tmap_w, smem_u32(sa), &full[s], k, n0);
          if (!waited) {
            pdl_wait();
            waited = true;
          }
          load_stage<CH>(&tmap_x, smem_u32(sa + C::kABytes), &full[s], k, m0);
        }
      }
      pdl_trigger();  // every load of this CTA is issued
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int i = 0, seg = 0;
      SegIter it(args, cta);
      int64_t t;
      int kb, ke;
      while (it.next(t, kb, ke)) {
        const int b = seg & 1;
        if (!mbar_wait(&acc_empty[b], (((uint32_t)seg >> 1) & 1u) ^ 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + (uint32_t)(b * C::kAccCols);
        bool ok = true;
        for (int j = 0; j < ke - kb; ++j, ++i) {
          const int s = i % C::kStages;
          const uint32_t ph = (uint32_t)(i / C::kStages) & 1u;
          if (!mbar_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(smem + s * C::kStageBytes);
          const uint32_t b_addr = a_addr + C::kABytes;
          // The start-address field of a descriptor is (address >> 4) in 14 bits and
          // shared addresses stay below 2^18, so stepping through the stage is a
          // constant add to the stage's first descriptor: the single issuing thread
          // keeps up with the tensor core on small token tiles.
          const uint64_t da0 = smem_desc_sw128(a_addr), db0 = smem_desc_sw128(b_addr);
#pragma unroll
          for (int c = 0; c < CH; ++c) {
#pragma unroll
            for (int kk = 0; kk < kChunk / 32; ++kk) {
              const uint64_t da = da0 + (uint64_t)((c * C::kChunkA + kk * 32) >> 4);
              const uint64_t db = db0 + (uint64_t)((c * C::kChunkB + kk * 32) >> 4);
              const uint32_t accum = (j > 0 || c > 0 || kk > 0) ? 1u : 0u;
              if constexpr (F16)
                umma_f16(acc, da, db, C::kIdesc, accum);
              else
                umma_f8(acc, da, db, C::kIdesc, accum);
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
        ++seg;
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5 -> TMEM lane quarters 2,3,0,1) ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;  // row within the 128-row weight tile
    const int et = threadIdx.x - 64;
    float* my_ws = args.ws + (int64_t)cta * BN * kBM;
    pdl_wait();  // token scales come from the preceding grid; the workspace may be in use until it ends
    // row-parallel push: the receive-slot parity of this call (the epoch word is
    // advanced by the tensor-parallel op that precedes this GEMM in the stream)
    const int rp_b = args.rp_R > 0 ? (*reinterpret_cast<const volatile int*>(args.rp_ctrl) & 1) : 0;
    int seg = -1;
    SegIter it(args, cta);
    int64_t t;
    int kb, ke;
    while (it.next(t, kb, ke)) {
      ++seg;
      const int n = (int)(t / args.tiles_m) * kBM + row;
      const int m0 = (int)(t % args.tiles_m) * BN;
      const int b = seg & 1;
      const int cols = min(BN, args.M - m0);  // valid token columns of this tile
      const bool owner = kb == 0;
      const bool n_ok = n < args.N;
      float swn = 0.f, bn = 0.f;
      if (owner || args.splits > 0) {
        // scales are inputs: fetch them while the tile is still accumulating
        for (int j = et; j < cols; j += 128) {
          s_sx[b * BN + j] = args.sx != nullptr ? args.sx[m0 + j] : 1.f;
          if (args.rp_R > 0) s_rows[b * BN + j] = rp_row(args, m0 + j, rp_b);
        }
        swn = n_ok ? (args.sw != nullptr ? args.sw[n] : 1.f) : 0.f;
        bn = (n_ok && args.bias != nullptr) ? __half2float(args.bias[n]) : 0.f;
      }
      if (!mbar_wait(&acc_full[b], ((uint32_t)seg >> 1) & 1u)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc = tmem + (uint32_t)(b * C::kAccCols) + ((uint32_t)(q * 32) << 16);

      if (args.splits > 0) {
        split_epilogue<BN, CH>(args, acc, t, m0, cols, n, n_ok, swn, bn, s_sx + b * BN, my_ws, smem, red_full,
                               acc_empty + b, et, row, args.rp_R > 0 ? s_rows + b * BN : nullptr);
        continue;
      }
      if (!owner) {
        // partial segment: hand the fp32 tile to the owner (column-major: coalesced per warp)
        for (int c0 = 0; c0 < cols; c0 += 16) {
          float v[16];
          tmem_ld16(acc + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) my_ws[(int64_t)(c0 + j) * kBM + row] = v[j];
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&acc_empty[b]);
        epi_sync();  // all partial stores precede the release below (release is cumulative)
        if (et == 0) st_release(&args.flags[cta], 1);
        continue;
      }

      // owner: contributors are the CTAs whose ranges begin inside this tile
      const int64_t tile_end = (t + 1) * (int64_t)KT;
      int c_first = cta + 1, c_last = cta;
      if (ke < KT) {
        while (c_last + 1 < args.G && unit_begin(c_last + 1, args.U, args.G) < tile_end) ++c_last;
        if (et == 0) {
          const uint64_t t0 = global_ns();
          for (int c = c_first; c <= c_last; ++c) {
            uint32_t spins = 0;
            while (ld_acquire(&args.flags[c]) == 0) {
              if ((++spins & 255u) == 0 && global_ns() - t0 > wait_limit_ns()) {
                set_device_status(kStatusMbarTimeout);
                break;
              }
            }
          }
        }
      }
      // The CTA's last segment: its loads have landed and its MMAs are done, so the
      // stage buffers are free to hold the output tile for one bulk tensor store.
      __half* stage = nullptr;
      if (args.tma_y) {
        SegIter rest = it;
        int64_t t2;
        int kb2, ke2;
        if (!rest.next(t2, kb2, ke2)) stage = reinterpret_cast<__half*>(smem);
      }
      epi_sync();  // s_sx filled; contributors' partials visible
      for (int c0 = 0; c0 < cols; c0 += 16) {
        float v[16];
        tmem_ld16(acc + (uint32_t)c0, v);
        for (int c = c_first; c <= c_last; c += 4) {
          // up to four contributors' loads in flight before any add
          float w4[4][16];
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            if (c + d <= c_last) {
              const float* w = args.ws + (int64_t)(c + d) * BN * kBM + (int64_t)c0 * kBM + row;
#pragma unroll
              for (int j = 0; j < 16; ++j) w4[d][j] = w[(int64_t)j * kBM];
            }
          }
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            if (c + d <= c_last) {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] += w4[d][j];
            }
          }
        }
        out16(args, v, s_sx + b * BN, swn, bn, m0, c0, cols, n, stage, row,
              args.rp_R > 0 ? s_rows + b * BN : nullptr);
      }
      if (stage != nullptr) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // staged tile -> the bulk store
        epi_sync();
        if (et == 0) tma_store_2d_wait(&tmap_y, smem_u32(stage), (int)(t / args.tiles_m) * kBM, m0);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&acc_empty[b]);
      if (c_last >= c_first) {
        epi_sync();  // every thread has read the partials
        if (et == 0)
          for (int c = c_first; c <= c_last; ++c) args.flags[c] = 0;
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
  if (args.rp_tail) {  // this CTA's tiles are all pushed: its share of the row work
    __syncwarp();
    const int wb = tp_world_bound(args.tail.world);
#define MS_TAIL(N, W) \
  if (args.rp_nvt == N && wb == W) rowpar_tail<N, W>(args.tail, smem);
    MS_TAIL(1, 2) MS_TAIL(1, 4) MS_TAIL(1, 8)
    MS_TAIL(2, 2) MS_TAIL(2, 4) MS_TAIL(2, 8)
    MS_TAIL(3, 2) MS_TAIL(3, 4) MS_TAIL(3, 8)
    MS_TAIL(4, 2) MS_TAIL(4, 4) MS_TAIL(4, 8)
#undef MS_TAIL
  }
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Arrive (release, cluster scope) on a barrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Every thread of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// 2-SM tiles (tcgen05 cta_group::2) for prefill-sized M: a cluster of two CTAs
// computes a 256 weight-row x 256 token output tile with ONE MMA per K step of
// 32 bytes. Each CTA loads half of each operand into its own shared memory (128
// weight rows, 128 tokens: a stage is 2 x 32 KB per CTA instead of 96 KB for a
// 128 x 256 tile on one SM), the leader CTA (cluster rank 0) issues the MMAs,
// which read both CTAs' halves, and each CTA's TMEM receives its 128 weight rows
// x 256 tokens. So every output needs half the L2 -> SM bytes of the one-SM
// tile (per-SM ingest bounds the one-SM kernel). Each CTA's TMA
// loads bring only its own half, from this GPU's memory; their completion is
// counted on the leader's barrier (.cta_group::2). Tiles are dealt whole to the
// pairs, with double-buffered accumulators as in fp8_gemm_kernel.
//   full[s]     leader only: both CTAs' loads of stage s landed (armed by the leader
//               with both halves' bytes)
//   empty[s]    each CTA: the MMAs reading stage s are done (a commit to each CTA)
//   acc_full[b] each CTA: accumulator b complete (a commit to each CTA)
//   acc_empty[b] leader: both CTAs' epilogues have drained accumulator b
//               (128 local + 128 remote arrivals)
constexpr int kPairBN = 256;                          // tokens per prefill tile (128 per CTA)
constexpr int kPairRows = 2 * kBM;                    // weight rows per tile (128 per CTA)
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;        // shared address of the same object in rank 0
template <int BN, int CH>
struct PairCfg {
  static constexpr int kABytes = CH * kBM * kChunk;                // this CTA's weight rows
  static constexpr int kStageBytes = kABytes + CH * (BN / 2) * kChunk;  // + this CTA's BN / 2 tokens
  static constexpr int kBarBytes = 256;
  static constexpr int kSxBytes = 2 * BN * 4;
  static constexpr int kAccCols = BN <= 64 ? 64 : (BN <= 128 ? 128 : 256);  // TMEM columns per accumulator
  static constexpr int kFit = (227 * 1024 - 1024 - kBarBytes - kSxBytes) / kStageBytes;
  static constexpr int kStages = kFit > 6 ? 6 : kFit;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + kBarBytes + kSxBytes;
  // D=f32, A=B=e4m3 (or f16 for kind::f16), K-major, N=BN, M=256
  static constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kPairRows >> 4) << 24);
  static_assert(kStages >= 2, "shared memory budget");
  static_assert(BN % 32 == 0 && BN <= 256, "each CTA's token half: whole 8-row swizzle atoms, MMA N <= 256");
};

__device__ __forceinline__ void tma_load_pair_2d(const CUtensorMap* map, uint32_t dst, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_pair_3d(const CUtensorMap* map, uint32_t dst, uint32_t bar, int c0, int c1,
                                                 int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
template <int CH>
__device__ __forceinline__ void load_pair_stage(const CUtensorMap* map, uint32_t dst, uint32_t bar, int k, int row) {
  if constexpr (CH == 1) {
    tma_load_pair_2d(map, dst, bar, k * kChunk, row);
  } else {
    tma_load_pair_3d(map, dst, bar, 0, row, k * CH);
  }
}
template <bool F16>
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  if constexpr (F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accum));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accum));
  }
}
// Completion of this thread's earlier MMAs arrives on the barrier at the same
// shared offset in both CTAs of the pair (one commit per CTA).
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  const uint32_t local = smem_u32(bar);
  uint32_t peer;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 1;" : "=r"(peer) : "r"(local));
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(local) : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer) : "memory");
}

template <int BN, int CH, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                         const __grid_constant__ GemmArgs args) {
  using C = PairCfg<BN, CH>;
  extern __shared__ __align__(16) unsigned char smem_raw[];  // aligned by hand, see fp8_gemm_kernel
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* s_sx = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes + C::kBarBytes);  // [2][256]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_ctarank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int KT = args.KT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * 128);
    }
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
  }
  if (warp == 1) {  // the same warp in both CTAs allocates the pair's accumulators
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * C::kAccCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other

  if (warp == 0) {
    if (lane == 0) {  // TMA producer (both CTAs: this CTA's halves)
      int i = 0;
      bool ok = true, waited = false;
      for (int64_t t = pair; ok && t < args.T; t += pairs) {
        const int n0 = (int)(t / args.tiles_m) * kPairRows + rank * kBM;
        const int m0 = (int)(t % args.tiles_m) * BN + rank * (BN / 2);
        for (int k = 0; k < KT; ++k, ++i) {
          const int s = i % C::kStages;
          if (!mbar_wait(&empty[s], ((uint32_t)(i / C::kStages) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::kStageBytes);
          const uint32_t bar = smem_u32(&full[s]) & kPeerBitMask;  // the leader's full[s]
          const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
          load_pair_stage<CH>(&tmap_w, sa, bar, k, n0);
          if (!waited) {
            pdl_wait();
            waited = true;
          }
          load_pair_stage<CH>(&tmap_x, sa + C::kABytes, bar, k, m0);
        }
      }
      pdl_trigger();
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // MMA issuer: the leader only
      int i = 0, tile = 0;
      for (int64_t t = pair; t < args.T; t += pairs, ++tile) {
        const int b = tile & 1;
        if (!mbar_wait(&acc_empty[b], (((uint32_t)tile >> 1) & 1u) ^ 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + (uint32_t)(b * C::kAccCols);
        bool ok = true;
        for (int k = 0; k < KT; ++k, ++i) {
          const int s = i % C::kStages;
          if (!mbar_wait(&full[s], (uint32_t)(i / C::kStages) & 1u)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(smem + s * C::kStageBytes);
          const uint64_t da0 = smem_desc_sw128(a_addr), db0 = smem_desc_sw128(a_addr + C::kABytes);
#pragma unroll
          for (int c = 0; c < CH; ++c) {
#pragma unroll
            for (int kk = 0; kk < kChunk / 32; ++kk) {
              const uint64_t da = da0 + (uint64_t)((c * kBM * kChunk + kk * 32) >> 4);
              const uint64_t db = db0 + (uint64_t)((c * (BN / 2) * kChunk + kk * 32) >> 4);
              umma_pair<F16>(acc, da, db, C::kIdesc, (k > 0 || c > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[b]);
      }
    }
    __syncwarp();
  } else {  // epilogue: warps 2..5 -> TMEM lane quarters 2, 3, 0, 1 of this CTA's 128 rows
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int et = threadIdx.x - 64;
    const uint32_t leader_acc_empty = smem_u32(acc_empty) & kPeerBitMask;
    pdl_wait();
    int tile = 0;
    for (int64_t t = pair; t < args.T; t += pairs, ++tile) {
      const int b = tile & 1;
      const int n = (int)(t / args.tiles_m) * kPairRows + rank * kBM + row;
      const int m0 = (int)(t % args.tiles_m) * BN;
      const int cols = min(BN, args.M - m0);
      for (int j = et; j < cols; j += 128) s_sx[b * BN + j] = args.sx != nullptr ? args.sx[m0 + j] : 1.f;
      const bool n_ok = n < args.N;
      const float swn = n_ok ? (args.sw != nullptr ? args.sw[n] : 1.f) : 0.f;
      const float bn = (n_ok && args.bias != nullptr) ? __half2float(args.bias[n]) : 0.f;
      if (!mbar_wait(&acc_full[b], ((uint32_t)tile >> 1) & 1u)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      epi_sync();  // s_sx filled
      const uint32_t acc = tmem + (uint32_t)(b * C::kAccCols) + ((uint32_t)(q * 32) << 16);
      for (int c0 = 0; c0 < cols; c0 += 16) {
        float v[16];
        tmem_ld16(acc + (uint32_t)c0, v);
        out16(args, v, s_sx + b * BN, swn, bn, m0, c0, cols, n, nullptr, row);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      epi_sync();  // every thread has read s_sx[b] and accumulator b
      mbar_arrive_remote(leader_acc_empty + (uint32_t)(b * 8));
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  // nothing of either CTA is touched by the other after this point
  cluster_sync_all();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * C::kAccCols));
  }
  cluster_sync_all();  // both CTAs have released the pair's accumulators before either exits
}

// Wide tiles for decode batches of 129..256 tokens with many weight tiles (the
// gate/up projection): 256 weight rows x 256 tokens per tile, computed as two
// M = 128 MMAs that share every activation stage. The activations are read once
// per 256 weight rows (half the L2 -> SM bytes of 128-row tiles) and a stage is
// two 32 KB TMA boxes (weights, activations). The two accumulators fill TMEM
// (512 columns), so a tile's epilogue overlaps only the next tile's loads, not
// its MMAs. Whole tiles dealt round-robin; 128-byte K steps (2D maps).
constexpr int kWideRows = 256;
constexpr int kWideBN = 256;
constexpr int kWideStages = 3;
constexpr int kWideABytes = kWideRows * kChunk;                  // 32 KB of weights
constexpr int kWideStageBytes = kWideABytes + kWideBN * kChunk;  // + 32 KB of activations
constexpr int kWideBarBytes = 128;
constexpr int kWideSmem = kWideStages * kWideStageBytes + 1024 + kWideBarBytes + kWideBN * 4;
constexpr uint32_t kWideIdesc = (1u << 4) | ((uint32_t)(kWideBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
static_assert(kWideSmem <= 227 * 1024, "shared memory budget");
static_assert(2 * kWideBN * kBM * 2 <= kWideStages * kWideStageBytes, "staged output tile fits the stages");

template <bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_wide_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                         const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ GemmArgs args) {
  extern __shared__ __align__(16) unsigned char smem_raw[];  // aligned by hand, see fp8_gemm_kernel
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWideStages * kWideStageBytes);
  uint64_t* empty = full + kWideStages;
  uint64_t* acc_full = empty + kWideStages;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  float* s_sx = reinterpret_cast<float*>(smem + kWideStages * kWideStageBytes + kWideBarBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = args.KT;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWideStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int i = 0;
      bool ok = true, waited = false;
      for (int64_t t = blockIdx.x; ok && t < args.T; t += args.G) {
        const int n0 = (int)(t / args.tiles_m) * kWideRows;
        const int m0 = (int)(t % args.tiles_m) * kWideBN;
        for (int k = 0; k < KT; ++k, ++i) {
          const int s = i % kWideStages;
          if (!mbar_wait(&empty[s], ((uint32_t)(i / kWideStages) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          unsigned char* sa = smem + s * kWideStageBytes;
          mbar_arrive_expect_tx(&full[s], kWideStageBytes);
          tma_load_2d(&tmap_w, smem_u32(sa), &full[s], k * kChunk, n0);
          if (!waited) {
            pdl_wait();
            waited = true;
          }
          tma_load_2d(&tmap_x, smem_u32(sa + kWideABytes), &full[s], k * kChunk, m0);
        }
      }
      pdl_trigger();
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      int i = 0, tile = 0;
      for (int64_t t = blockIdx.x; t < args.T; t += args.G, ++tile) {
        if (!mbar_wait(acc_empty, ((uint32_t)tile & 1u) ^ 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        bool ok = true;
        for (int k = 0; k < KT; ++k, ++i) {
          const int s = i % kWideStages;
          if (!mbar_wait(&full[s], (uint32_t)(i / kWideStages) & 1u)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(smem + s * kWideStageBytes);
          const uint32_t b_addr = a_addr + kWideABytes;
          const uint64_t da0 = smem_desc_sw128(a_addr), db0 = smem_desc_sw128(b_addr);  // see fp8_gemm_kernel
#pragma unroll
          for (int kk = 0; kk < kChunk / 32; ++kk) {
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              const uint64_t da = da0 + (uint64_t)((mt * kBM * kChunk + kk * 32) >> 4);
              const uint64_t db = db0 + (uint64_t)((kk * 32) >> 4);
              const uint32_t accum = (k > 0 || kk > 0) ? 1u : 0u;
              if constexpr (F16)
                umma_f16(tmem + (uint32_t)(mt * kWideBN), da, db, kWideIdesc, accum);
              else
                umma_f8(tmem + (uint32_t)(mt * kWideBN), da, db, kWideIdesc, accum);
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
    }
    __syncwarp();
  } else {  // epilogue: warps 2..5 -> TMEM lane quarters 2, 3, 0, 1
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int et = threadIdx.x - 64;
    const int64_t N = args.N;
    pdl_wait();
    int tile = 0;
    for (int64_t t = blockIdx.x; t < args.T; t += args.G, ++tile) {
      const int n0 = (int)(t / args.tiles_m) * kWideRows;
      const int m0 = (int)(t % args.tiles_m) * kWideBN;
      const int cols = min(kWideBN, args.M - m0);
      epi_sync();  // the previous tile's readers of s_sx are done
      for (int j = et; j < cols; j += 128) s_sx[j] = args.sx != nullptr ? args.sx[m0 + j] : 1.f;
      float swn[2], bn[2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int n = n0 + mt * kBM + row;
        swn[mt] = n < N ? (args.sw != nullptr ? args.sw[n] : 1.f) : 0.f;
        bn[mt] = (n < N && args.bias != nullptr) ? __half2float(args.bias[n]) : 0.f;
      }
      if (!mbar_wait(acc_full, (uint32_t)tile & 1u)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // The CTA's last tile: every load has landed and every MMA is done, so the
      // stage buffers hold the two 128-row halves of the output tile ([256 tokens]
      // [128 rows] fp16 each) for two bulk tensor stores.
      const bool staged = args.tma_y && t + args.G >= args.T;
      epi_sync();  // s_sx filled
#pragma unroll 1
      for (int mt = 0; mt < 2; ++mt) {
        const int n = n0 + mt * kBM + row;
        const uint32_t acc = tmem + (uint32_t)(mt * kWideBN) + ((uint32_t)(q * 32) << 16);
        __half* stage = staged ? reinterpret_cast<__half*>(smem + (size_t)mt * kWideBN * kBM * 2) : nullptr;
        for (int c0 = 0; c0 < cols; c0 += 16) {
          float v[16];
          tmem_ld16(acc + (uint32_t)c0, v);
          out16(args, v, s_sx, swn[mt], bn[mt], m0, c0, cols, n, stage, row);
        }
      }
      if (staged) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // staged tile -> the bulk stores
        epi_sync();
        if (et == 0) {
          for (int mt = 0; mt < 2; ++mt)
            if (n0 + mt * kBM < N)
              tma_store_2d_wait(&tmap_y, smem_u32(smem + (size_t)mt * kWideBN * kBM * 2), n0 + mt * kBM, m0);
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(acc_empty);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// CUDA-core FP8 GEMM for shapes the TMA path cannot describe (K % 16 != 0).
// One thread per output element; used only for tiny irregular layers.
__global__ void fp8_gemm_simt_kernel(const uint8_t* __restrict__ xq, const uint8_t* __restrict__ wq, int M, int N,
                                     int K, const float* __restrict__ sx, const float* __restrict__ sw,
                                     const __half* __restrict__ bias, __half* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) acc += e4m3_to_f32(xq[(int64_t)m * K + k]) * e4m3_to_f32(wq[(int64_t)n * K + k]);
  __half r = __float2half_rn(acc * sx[m] * sw[n]);
  if (bias != nullptr) r = __float2half_rn(__half2float(r) + __half2float(bias[n]));
  y[(int64_t)m * N + n] = r;
}

// ---------------------------------------------------------------------------
// Host side: tensor-map encoding (driver entry point, cached), tile choice.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  int64_t rows, cols;
  int box_rows, ch;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows && ch == o.ch;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) * 31) ^
           (std::hash<int64_t>()(k.cols) * 131) ^ (size_t)k.box_rows * 7 ^ (size_t)k.ch * 1009;
  }
};

// K-major e4m3 matrix [rows, cols] (cols contiguous), 128-byte swizzle.
//  ch == 1: 2D map (byte, row), box = [box_rows, 128 bytes]; cols need only be a
//           multiple of 16 (out-of-range K reads as zero).
//  ch == 2: 3D map (byte within a 128-byte chunk, row, chunk) with strides
//           (cols, 128), box = [2 chunks][box_rows][128 bytes]: one box is two
//           consecutive K-chunk tiles, each laid out exactly as a 2D box. Needs
//           cols % 128 == 0 (a chunk past K reads as zero).
bool make_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int box_rows, int ch) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{ptr, rows, cols, box_rows, ch};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  CUresult r;
  if (ch == 0) {
    // fp16 output y [rows = tokens, cols = N], box = [box_rows tokens][128 weight rows], no swizzle
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBM, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    r = enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (ch == 1) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols};
    cuuint32_t box[2] = {(cuuint32_t)kChunk, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    if (cols % kChunk != 0) return false;
    cuuint64_t dims[3] = {(cuuint64_t)kChunk, (cuuint64_t)rows, (cuuint64_t)(cols / kChunk)};
    cuuint64_t strides[2] = {(cuuint64_t)cols, (cuuint64_t)kChunk};
    cuuint32_t box[3] = {(cuuint32_t)kChunk, (cuuint32_t)box_rows, (cuuint32_t)ch};
    cuuint32_t estr[3] = {1, 1, 1};
    r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return true;
}

template <int BN, int CH, bool F16>
cudaError_t launch_tc_kind(const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& my, const GemmArgs& args,
                           cudaStream_t stream) {
  using C = Cfg<BN, CH>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel<BN, CH, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  // Stream-K owners wait for later CTAs' partials, so all G <= SM-count CTAs
  // (one per SM) must become resident. The preceding grid never waits on this
  // one, so its SMs free up; the next grid cannot start before every CTA here
  // has triggered (after issuing its last load), i.e. before all are resident.
  return launch_kernel(fp8_gemm_kernel<BN, CH, F16>, dim3(args.G), dim3(kThreads), C::kSmemBytes, stream, mw, mx,
                       my, args);
}

template <int BN, int CH>
cudaError_t launch_tc(const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& my, const GemmArgs& args,
                      cudaStream_t stream) {
  return args.f16 ? launch_tc_kind<BN, CH, true>(mw, mx, my, args, stream)
                  : launch_tc_kind<BN, CH, false>(mw, mx, my, args, stream);
}

template <int BN, int CH, bool F16>
cudaError_t launch_pair_kind(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& args, cudaStream_t stream) {
  using C = PairCfg<BN, CH>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fp8_gemm_pair_kernel<BN, CH, F16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  if (args.G % 2 != 0) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(args.G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;  // the two CTAs of a tile: one pair of SMs
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl_enabled.load(std::memory_order_relaxed) ? 2 : 1;
  MS_COUNT_LAUNCH();
  return cudaLaunchKernelEx(&cfg, fp8_gemm_pair_kernel<BN, CH, F16>, mw, mx, args);
}

template <int BN>
cudaError_t launch_pair_bn(int ch, bool f16, const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& args,
                           cudaStream_t stream) {
  if (ch == 2)
    return f16 ? launch_pair_kind<BN, 2, true>(mw, mx, args, stream)
               : launch_pair_kind<BN, 2, false>(mw, mx, args, stream);
  return f16 ? launch_pair_kind<BN, 1, true>(mw, mx, args, stream) : launch_pair_kind<BN, 1, false>(mw, mx, args, stream);
}

template <int BN>
cudaError_t launch_bn(int ch, const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& my,
                      const GemmArgs& args, cudaStream_t stream) {
  return ch == 2 ? launch_tc<BN, 2>(mw, mx, my, args, stream) : launch_tc<BN, 1>(mw, mx, my, args, stream);
}

constexpr size_t kFlagBytes = 1024;  // per-CTA partial-ready flags at the start of the workspace
constexpr int kMinUnitsPerCta = 4;

struct Plan {
  int bn, ch, ctas, dp, splits, wide, pair;
};

// Tile shape and scheduling for an M x N x K problem (rules fitted to B200
// measurements of the decode and prefill shapes of the Qwen3 family):
//  * Decode batches whose weight tiles are fewer than half the SMs (qkv, o and
//    down projections) when M <= 128, or when K is long (>= 24 steps, the down
//    projection) for M <= 256: split-K. One token tile of BN = M rounded
//    up to 32/64/96/128/192/256, `splits` = SMs / weight tiles (<= 8) CTAs per
//    tile, each streaming 1/splits of K once; the partials are reduced in a
//    balanced way (each CTA finishes a slice of the tile). With 129..256 tokens
//    and 8..23 K steps (few weight tiles: the q/k/v shards of tensor parallelism)
//    4 K parts over 64-token tiles instead (128-token tiles when 64-token ones
//    would fill more than 2/3 of the SMs).
//  * 129..256 tokens with more 128-row weight tiles than SMs (the gate/up
//    projection): 256 x 256 tiles of fp8_gemm_wide_kernel, dealt whole.
//  * Other decode shapes: BN = M up to 128; for 129..256 tokens the smallest of
//    64/96/128-token tiles whose tile count fits one wave; whole tiles dealt
//    round-robin over the SMs.
// Every CTA writes its last output tile through shared memory with a bulk
// tensor store when N % 8 == 0 (earlier tiles' epilogues overlap the next main
// loop and keep direct stores).
//  * M > 256 (prefill): 256-token tiles; whole tiles when they fill the SMs
//    evenly, else stream-K over tiles x K-steps.
Plan make_plan(int M, int N, int K, int num_sms, bool allow_pair = true) {
  Plan p{256, (K % kChunk == 0) ? 2 : 1, 1, 0, 0, 0, 0};
  const int64_t tiles_n = (N + kBM - 1) / kBM;
  const int64_t pairs = num_sms / 2;
  if (M > 128 && M <= 256 && tiles_n > num_sms && allow_pair && K >= 2048 && pairs >= 1) {
    // e.g. gate/up at 256 tokens: 256 x 256 tiles on SM pairs, over all SMs (8B gate/up
    // 30.6 us in two waves of 74 pairs vs 34.0 us for the one-SM 256 x 256 tiles on 96
    // SMs below; B200)
    const int64_t T2 = (N + kPairRows - 1) / kPairRows;
    p.pair = 1;
    p.dp = 1;
    p.bn = 256;
    p.ctas = (int)(2 * (T2 < pairs ? T2 : pairs));
    return p;
  }
  if (M > 128 && M <= 256 && tiles_n > num_sms) {  // e.g. gate/up: 256-row x 256-token tiles
    const int64_t T = (N + kWideRows - 1) / kWideRows;
    p.wide = 1;
    p.dp = 1;
    p.ch = 1;
    p.bn = kWideBN;
    p.ctas = (int)(T < num_sms ? T : num_sms);
    return p;
  }
  const int64_t steps = (K + kChunk * p.ch - 1) / (kChunk * p.ch);
  if (M <= 256) {
    const int full = M <= 32 ? 32 : M <= 64 ? 64 : M <= 96 ? 96 : M <= 128 ? 128 : M <= 192 ? 192 : 256;
    const int64_t s = num_sms / tiles_n;
    // For 128 < M <= 256 the 256-token tile's partials (128 KB each) cost more
    // than they save unless K is long or 128-token tiles dealt whole would leave
    // three quarters of the SMs idle (the small shards of tensor parallelism).
    const int64_t dp_tiles = tiles_n * ((M + kBM - 1) / kBM);
    if (s >= 2 && steps >= 2 && (M <= 128 || steps >= 24 || 4 * dp_tiles < num_sms)) {
      if (M > 128 && steps < 24 && steps >= 8) {
        // few weight tiles (the q/k/v shard of tensor parallelism): 4 K parts over
        // narrower token tiles (256 x 768 x 4096: 64-token tiles 8.0 us vs one
        // 256-token tile in 8 parts 10.8 us; 256 x 1536 x 4096: 128-token tiles 9.7
        // vs 11.9 us, B200 sweep); 64-token tiles while they fill at most 2/3 of the SMs
        const int64_t t64 = tiles_n * ((M + 63) / 64);
        p.bn = 3 * 4 * t64 <= 2 * (int64_t)num_sms ? 64 : 128;
        p.splits = 4;
        p.ctas = (int)(tiles_n * ((M + p.bn - 1) / p.bn) * p.splits);
        return p;
      }
      p.bn = full;
      // every K part must hold at least one step: an empty part would hand over an
      // accumulator the MMA never wrote
      int64_t sp = s < steps ? s : steps;
      p.splits = (int)(sp < 8 ? sp : 8);
      p.ctas = (int)(tiles_n * p.splits);
      return p;
    }
  }
  if (M > 256 && allow_pair && K <= 8192) {
    // prefill: 256 x 256 tiles on SM pairs (fp8_gemm_pair_kernel) when they fill the
    // pairs evenly (B200, 8192 tokens: q/k/v 192.9 vs 223.3 us for one-SM tiles, o and
    // gate/up within 1 %, the 12288-long K of down 417 vs 395 us, so not for long K)
    const int64_t T2 = ((N + kPairRows - 1) / kPairRows) * ((M + kPairBN - 1) / kPairBN);
    const int64_t waves2 = (T2 + pairs - 1) / pairs;
    if (pairs >= 1 && T2 >= pairs && (double)T2 / ((double)waves2 * pairs) >= 0.9) {
      p.pair = 1;
      p.dp = 1;
      p.bn = kPairBN;
      p.ctas = (int)(2 * pairs);
      return p;
    }
  }
  if (M <= 32) p.bn = 32;
  else if (M <= 64) p.bn = 64;
  else if (M <= 96) p.bn = 96;
  else if (M <= 128) p.bn = 128;
  else if (M <= 256) {
    // the smallest token tile whose tiles still fit one wave: more CTAs share the
    // weight streams (qkv at 256 tokens: 144 CTAs of 96 tokens, 12.1 vs 12.9 us;
    // o: 128 CTAs of 64 tokens, 11.5 vs 12.4 us)
    p.bn = 128;
    if (tiles_n * ((M + 63) / 64) <= num_sms) p.bn = 64;
    else if (tiles_n * ((M + 95) / 96) <= num_sms) p.bn = 96;
  }
  const int64_t tiles_m = (M + p.bn - 1) / p.bn;
  const int64_t T = tiles_n * tiles_m;
  const bool decode = M <= 256 && M > 64;
  if (decode && (2 * T >= num_sms || steps <= 16)) {
    p.dp = 1;
    p.ctas = (int)(T < num_sms ? T : num_sms);
    const int64_t T2 = ((N + kPairRows - 1) / kPairRows) * ((M + 95) / 96);
    if (M > 128 && allow_pair && K >= 2048 && T2 <= pairs) {
      // 256 weight rows x 96 tokens on SM pairs, one wave (each SM loads 48 tokens:
      // qkv at 256 tokens 12.7 vs 13.7 us, o 11.7 vs 12.3 us; B200)
      p.pair = 1;
      p.bn = 96;
      p.ctas = (int)(2 * T2);
    }
    return p;
  }
  const int64_t waves = (T + num_sms - 1) / num_sms;
  if (T >= num_sms && (double)T / ((double)waves * num_sms) >= 0.9) {
    p.dp = 1;
    p.ctas = num_sms;
    return p;
  }
  int64_t g = T * steps / kMinUnitsPerCta;
  if (g < 1) g = 1;
  if (g > num_sms) g = num_sms;
  if (g > (int64_t)(kFlagBytes / sizeof(int))) g = kFlagBytes / sizeof(int);
  p.ctas = (int)g;
  return p;
}

}  // namespace

void gemm_plan(int M, int N, int K, int num_sms, int* out) {
  if (K % 16 != 0) {  // CUDA-core kernel: one thread per output, 128-column blocks
    out[0] = 0;
    out[1] = (int)((N + 127) / 128) * M;
    out[2] = out[3] = out[5] = out[6] = 0;
    out[4] = 1;
    return;
  }
  const Plan p = make_plan(M, N, K, num_sms, g_pair_tiles_enabled.load(std::memory_order_relaxed) != 0);
  out[0] = p.bn;
  out[1] = p.ctas;
  out[2] = p.splits;
  out[3] = p.wide;
  out[4] = p.dp;
  out[5] = p.ch;
  out[6] = p.pair;
}

size_t gemm_workspace_bytes(int M, int N, int K, int num_sms) {
  if (K % 16 != 0 || M <= 0) return 0;
  // the plan of a plain call, and of a row-parallel call (no SM pairs) of the same shape
  size_t need = 0;
  for (int allow_pair = 0; allow_pair < 2; ++allow_pair) {
    const Plan p = make_plan(M, N, K, num_sms, allow_pair != 0);
    const size_t b = p.dp ? 0 : kFlagBytes + (size_t)p.ctas * p.bn * kBM * sizeof(float);
    need = b > need ? b : need;
  }
  return need;
}

cudaError_t launch_fp8_gemm(const void* xq, const float* sx, const void* wq, const float* sw, const void* bias,
                            void* y, int M, int N, int K, void* workspace, size_t workspace_bytes, int num_sms,
                            cudaStream_t stream, const TpRows* rp, bool* tail, bool f16) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (f16 && (K % 16 != 0 || rp != nullptr)) return cudaErrorInvalidValue;
  if (rp != nullptr && (K % 16 != 0 || rp->H != N || rp->M != M)) return cudaErrorInvalidValue;
  if (K % 16 != 0) {
    dim3 grid((N + 127) / 128, M);
    return launch_kernel(fp8_gemm_simt_kernel, grid, dim3(128), 0, stream, (const uint8_t*)xq, (const uint8_t*)wq, M,
                         N, K, sx, sw, (const __half*)bias, (__half*)y);
  }
  // (row-parallel push and the tensor-parallel tail are written for one-SM tiles)
  const Plan p = make_plan(M, N, K, num_sms, rp == nullptr && g_pair_tiles_enabled.load(std::memory_order_relaxed));
  const int bn = p.bn;
  if (!p.dp && (gemm_workspace_bytes(M, N, K, num_sms) > workspace_bytes || workspace == nullptr))
    return cudaErrorInvalidValue;
  CUtensorMap mw, mx, my;
  // The bulk store of a CTA's last output tile needs 16-byte aligned rows of y
  // (and a local y: pushed rows leave through plain stores).
  const bool tma_y = rp == nullptr && N % 8 == 0 && ((uintptr_t)y & 15) == 0 && make_map(&my, y, M, N, bn, 0);
  if (!tma_y) memset(&my, 0, sizeof(my));
  if (p.pair) {
    if (!make_map(&mw, wq, N, K, kBM, p.ch) || !make_map(&mx, xq, M, K, p.bn / 2, p.ch))
      return cudaErrorInvalidValue;
    GemmArgs args = {};
    args.M = M;
    args.N = N;
    args.K = K;
    args.KT = (K + kChunk * p.ch - 1) / (kChunk * p.ch);
    args.tiles_m = (M + p.bn - 1) / p.bn;
    args.T = (int64_t)((N + kPairRows - 1) / kPairRows) * args.tiles_m;
    args.G = p.ctas;
    args.dp = 1;
    args.sx = sx;
    args.sw = sw;
    args.bias = (const __half*)bias;
    args.y = (__half*)y;
    args.f16 = f16 ? 1 : 0;
    switch (p.bn) {
      case 64: return launch_pair_bn<64>(p.ch, f16, mw, mx, args, stream);
      case 96: return launch_pair_bn<96>(p.ch, f16, mw, mx, args, stream);
      case 128: return launch_pair_bn<128>(p.ch, f16, mw, mx, args, stream);
      case 256: return launch_pair_bn<256>(p.ch, f16, mw, mx, args, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  if (p.wide) {
    if (rp != nullptr) return cudaErrorInvalidValue;  // row-parallel outputs are never that wide
    if (!make_map(&mw, wq, N, K, kWideRows, 1) || !make_map(&mx, xq, M, K, kWideBN, 1)) return cudaErrorInvalidValue;
    GemmArgs args = {};
    args.M = M;
    args.N = N;
    args.K = K;
    args.KT = (K + kChunk - 1) / kChunk;
    args.tiles_m = (M + kWideBN - 1) / kWideBN;
    args.T = (int64_t)((N + kWideRows - 1) / kWideRows) * args.tiles_m;
    args.U = args.T * args.KT;
    args.G = p.ctas;
    args.dp = 1;
    args.tma_y = tma_y ? 1 : 0;
    args.f16 = f16 ? 1 : 0;
    args.sx = sx;
    args.sw = sw;
    args.bias = (const __half*)bias;
    args.y = (__half*)y;
    if (f16) {
      static const cudaError_t attr =
          cudaFuncSetAttribute(fp8_gemm_wide_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWideSmem);
      if (attr != cudaSuccess) return attr;
      return launch_kernel(fp8_gemm_wide_kernel<true>, dim3(args.G), dim3(kThreads), kWideSmem, stream, mw, mx, my,
                           args);
    }
    static const cudaError_t attr =
        cudaFuncSetAttribute(fp8_gemm_wide_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWideSmem);
    if (attr != cudaSuccess) return attr;
    return launch_kernel(fp8_gemm_wide_kernel<false>, dim3(args.G), dim3(kThreads), kWideSmem, stream, mw, mx, my,
                         args);
  }
  if (!make_map(&mw, wq, N, K, kBM, p.ch) || !make_map(&mx, xq, M, K, bn, p.ch)) return cudaErrorInvalidValue;
  GemmArgs args = {};
  if (rp != nullptr) {
    for (int r = 0; r < rp->world; ++r) args.rp_recv[r] = rp->recv[r];
    args.rp_ctrl = rp->ctrl;
    args.rp_half = rp->recv_half;
    args.rp_src = rp->recv_src;
    args.rp_R = rp->R;
    args.rp_rank = rp->rank;
    // the row work in the GEMM's own tail: every CTA resident (all plans here use at
    // most one CTA per SM), at most two owned rows per CTA, the canonical RMSNorm
    // layout (32 W threads) and a row (<= 4 vectors per thread) within 192 threads
    const int nv = N / 8;
    if (tail != nullptr && *tail) {
      *tail = p.ctas <= num_sms && rp->R <= 2 * p.ctas && 32 * row_warps(nv) <= kThreads && nv <= 4 * kThreads;
      if (*tail) {
        args.rp_tail = 1;
        args.rp_nvt = (nv + kThreads - 1) / kThreads;
        args.tail = *rp;
      }
    }
  } else if (tail != nullptr) {
    *tail = false;
  }
  args.M = M;
  args.N = N;
  args.K = K;
  args.KT = (K + kChunk * p.ch - 1) / (kChunk * p.ch);
  args.tiles_m = (M + bn - 1) / bn;
  args.T = (int64_t)((N + kBM - 1) / kBM) * args.tiles_m;
  args.U = args.T * args.KT;
  args.G = p.ctas;
  args.dp = p.dp;
  args.splits = p.splits;
  args.tma_y = tma_y ? 1 : 0;
  args.f16 = f16 ? 1 : 0;
  if (p.splits > args.KT) return cudaErrorInvalidValue;  // a K part without steps
  args.sx = sx;
  args.sw = sw;
  args.bias = (const __half*)bias;
  args.y = (__half*)y;
  args.flags = p.dp ? nullptr : (int*)workspace;
  args.ws = p.dp ? nullptr : (float*)((char*)workspace + kFlagBytes);
  switch (bn) {
    case 32: return launch_bn<32>(p.ch, mw, mx, my, args, stream);
    case 64: return launch_bn<64>(p.ch, mw, mx, my, args, stream);
    case 96: return launch_bn<96>(p.ch, mw, mx, my, args, stream);
    case 128: return launch_bn<128>(p.ch, mw, mx, my, args, stream);
    case 192: return launch_bn<192>(p.ch, mw, mx, my, args, stream);
    default: return launch_bn<256>(p.ch, mw, mx, my, args, stream);
  }
}

}  // namespace ms
