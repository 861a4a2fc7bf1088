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
// shared-memory stages; warp 1 owns the TMEM accumulator and issues
// tcgen05.mma (kind::f8f6f4, 128 x BN x 32 per instruction, 4 per 128-byte K
// step); warps 2-5 drain TMEM with tcgen05.ld and apply the dequant epilogue.
// Small tile counts split K over CTAs: each split writes an fp32 partial and a
// second kernel reduces the partials and applies the epilogue.
//
// Every wait is bounded (common.cuh: mbar_wait); on a timeout the kernel
// records a device status, skips the rest and still frees its TMEM.
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kBM = 128;       // weight rows per tile (MMA M)
constexpr int kBK = 128;       // K bytes per stage (one 128B swizzle span)
constexpr int kThreads = 192;  // 6 warps

struct GemmArgs {
  int M, N, K;
  int k_tiles_per_split;
  int k_tiles;
  const float* sx;
  const float* sw;
  const __half* bias;
  __half* y;
  float* ws;  // split partials [splits, M, N] (splits > 1)
};

template <int BN>
struct Cfg {
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
  // tcgen05 instruction descriptor: D=f32, A=B=e4m3, both K-major, N=BN, M=128.
  static constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
};

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);         // start address
  d |= (uint64_t)1 << 16;                           // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                           // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                           // layout: SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint32_t dst, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
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

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    GemmArgs args) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment required by the 128B swizzle atoms.
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* done = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM;
  const int m0 = blockIdx.y * BN;
  const int split = blockIdx.z;
  const int kt0 = split * args.k_tiles_per_split;
  const int kt1 = min(args.k_tiles, kt0 + args.k_tiles_per_split);
  const int nk = kt1 - kt0;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
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
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kStages;
        const uint32_t ph = (uint32_t)(i / C::kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u)) {
          s_abort = 1;
          break;
        }
        unsigned char* sa = smem + s * C::kStageBytes;
        mbar_arrive_expect_tx(&full[s], C::kStageBytes);
        const int kc = (kt0 + i) * kBK;
        tma_load_2d(&tmap_w, smem_u32(sa), &full[s], kc, n0);
        tma_load_2d(&tmap_x, smem_u32(sa + C::kABytes), &full[s], kc, m0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kStages;
        const uint32_t ph = (uint32_t)(i / C::kStages) & 1u;
        if (!mbar_wait(&full[s], ph)) {
          ok = false;
          s_abort = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_addr = smem_u32(smem + s * C::kStageBytes);
        const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 32; ++kk) {
          umma_f8(tmem, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), C::kIdesc,
                  (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(done);
    }
  } else {
    // Epilogue warps 2..5 -> TMEM lane quarters 2,3,0,1.
    const int q = warp & 3;
    const int n = n0 + q * 32 + lane;
    bool ok = (nk > 0) ? mbar_wait(done, 0) : true;
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const bool n_ok = n < args.N;
      const float swn = (n_ok && args.ws == nullptr) ? args.sw[n] : 0.f;
      const float bn = (n_ok && args.bias != nullptr) ? __half2float(args.bias[n]) : 0.f;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        if (m0 + c0 >= args.M) break;
        float v[16];
        if (nk > 0) {
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
        if (!n_ok) continue;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c0 + j;
          if (m < args.M) {
            if (args.ws != nullptr) {
              args.ws[((int64_t)split * args.M + m) * args.N + n] = v[j];
            } else {
              __half r = __float2half_rn(v[j] * args.sx[m] * swn);
              if (args.bias != nullptr) r = __float2half_rn(__half2float(r) + bn);
              args.y[(int64_t)m * args.N + n] = r;
            }
          }
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
}

// Sum split partials and apply the dequant epilogue. 4 outputs per thread.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                     const float* __restrict__ sx, const float* __restrict__ sw,
                                     const __half* __restrict__ bias, __half* __restrict__ y) {
  const int64_t total = (int64_t)M * N;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < total;
       i += (int64_t)gridDim.x * blockDim.x * 4) {
    float4 acc = *reinterpret_cast<const float4*>(ws + i);
    for (int s = 1; s < splits; ++s) {
      float4 p = *reinterpret_cast<const float4*>(ws + (int64_t)s * total + i);
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    const int m = (int)(i / N);
    const int n = (int)(i % N);
    const float a[4] = {acc.x, acc.y, acc.z, acc.w};
    __half r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      r[j] = __float2half_rn(a[j] * sx[m] * sw[n + j]);
      if (bias != nullptr) r[j] = __float2half_rn(__half2float(r[j]) + __half2float(bias[n + j]));
    }
    *reinterpret_cast<__half2*>(y + i) = __halves2half2(r[0], r[1]);
    *reinterpret_cast<__half2*>(y + i + 2) = __halves2half2(r[2], r[3]);
  }
}

// CUDA-core FP8 GEMM for shapes the TMA path cannot describe (K % 16 != 0).
// One thread per output element; used only for tiny irregular layers.
__global__ void fp8_gemm_simt_kernel(const uint8_t* __restrict__ xq, const uint8_t* __restrict__ wq, int M, int N,
                                     int K, const float* __restrict__ sx, const float* __restrict__ sw,
                                     const __half* __restrict__ bias, __half* __restrict__ y) {
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
  int box_rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) * 31) ^
           (std::hash<int64_t>()(k.cols) * 131) ^ (size_t)k.box_rows * 7;
  }
};

// 2D K-major e4m3 matrix [rows, cols] (cols contiguous), box = [box_rows, 128 bytes], 128B swizzle.
bool make_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{ptr, rows, cols, box_rows};
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
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return true;
}

template <int BN>
cudaError_t launch_tc(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& args, dim3 grid,
                      cudaStream_t stream) {
  using C = Cfg<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  fp8_gemm_kernel<BN><<<grid, kThreads, C::kSmemBytes, stream>>>(mw, mx, args);
  MS_COUNT_LAUNCH();
  return cudaGetLastError();
}

int choose_bn(int M) {
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

}  // namespace

void gemm_plan(int M, int N, int K, int num_sms, int* bn_out, int* splits_out) {
  const int bn = choose_bn(M);
  const int tiles = ((N + kBM - 1) / kBM) * ((M + bn - 1) / bn);
  const int k_tiles = (K + kBK - 1) / kBK;
  int splits = 1;
  if (tiles * 2 <= num_sms) {
    splits = num_sms / tiles;
    const int max_splits = k_tiles / 4 > 0 ? k_tiles / 4 : 1;  // >= 4 K steps per split
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    // balance: equal K steps per split
    const int per = (k_tiles + splits - 1) / splits;
    splits = (k_tiles + per - 1) / per;
  }
  *bn_out = bn;
  *splits_out = splits;
}

size_t gemm_workspace_bytes(int M, int N, int K, int num_sms) {
  int bn, splits;
  if (K % 16 != 0) return 0;
  gemm_plan(M, N, K, num_sms, &bn, &splits);
  return splits > 1 ? (size_t)splits * M * N * sizeof(float) : 0;
}

cudaError_t launch_fp8_gemm(const void* xq, const float* sx, const void* wq, const float* sw, const void* bias,
                            void* y, int M, int N, int K, void* workspace, size_t workspace_bytes, int num_sms,
                            cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (K % 16 != 0 || N % 4 != 0) {
    dim3 grid((N + 127) / 128, M);
    fp8_gemm_simt_kernel<<<grid, 128, 0, stream>>>((const uint8_t*)xq, (const uint8_t*)wq, M, N, K, sx, sw,
                                                    (const __half*)bias, (__half*)y);
    MS_COUNT_LAUNCH();
    return cudaGetLastError();
  }
  int bn, splits;
  gemm_plan(M, N, K, num_sms, &bn, &splits);
  const size_t need = splits > 1 ? (size_t)splits * M * N * sizeof(float) : 0;
  if (need > workspace_bytes) return cudaErrorInvalidValue;
  CUtensorMap mw, mx;
  if (!make_map(&mw, wq, N, K, kBM) || !make_map(&mx, xq, M, K, bn)) return cudaErrorInvalidValue;
  GemmArgs args;
  args.M = M;
  args.N = N;
  args.K = K;
  args.k_tiles = (K + kBK - 1) / kBK;
  args.k_tiles_per_split = (args.k_tiles + splits - 1) / splits;
  args.sx = sx;
  args.sw = sw;
  args.bias = (const __half*)bias;
  args.y = (__half*)y;
  args.ws = splits > 1 ? (float*)workspace : nullptr;
  dim3 grid((N + kBM - 1) / kBM, (M + bn - 1) / bn, splits);
  cudaError_t e;
  switch (bn) {
    case 32: e = launch_tc<32>(mw, mx, args, grid, stream); break;
    case 64: e = launch_tc<64>(mw, mx, args, grid, stream); break;
    case 128: e = launch_tc<128>(mw, mx, args, grid, stream); break;
    default: e = launch_tc<256>(mw, mx, args, grid, stream); break;
  }
  if (e != cudaSuccess || splits == 1) return e;
  const int64_t total = (int64_t)M * N;
  int blocks = (int)((total / 4 + 255) / 256);
  if (blocks > num_sms * 8) blocks = num_sms * 8;
  splitk_reduce_kernel<<<blocks, 256, 0, stream>>>((const float*)workspace, splits, M, N, sx, sw,
                                                    (const __half*)bias, (__half*)y);
  MS_COUNT_LAUNCH();
  return cudaGetLastError();
}

}  // namespace ms
