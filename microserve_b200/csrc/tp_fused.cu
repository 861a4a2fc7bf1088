// Tensor-parallel all-reduce fused with the residual add, RMSNorm and FP8 row
// quantisation that follow every row-parallel linear of the decoder layer
// (o_proj -> post_attention_layernorm, down_proj -> next input_layernorm), over
// NVLink peer memory (CUDA IPC mappings; plain loads and stores, no multicast).
// The row work, its data flow and why no flag or fence is needed are described
// in tp_rows.cuh; this file holds the standalone kernel (push + reduce +
// collect in one launch, or reduce + collect when the row-parallel GEMM already
// pushed its tiles) and the buffer layout.
#include "common.cuh"
#include "kernels.h"
#include "rowops.cuh"
#include "tp_rows.cuh"

namespace ms {

namespace {

constexpr int kTpThreads = 512;

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

// NVT: 16-byte vectors of an fp16 row per thread (ceil(H / 8 / blockDim)); WB: a
// bound on the ranks (2, 4 or 8) that sizes the loads kept in flight. The grid
// has at most one CTA per SM, so every CTA of every rank is resident at once; CTA c
// handles the row indices j = c, c + gridDim, ... < R and issues all of its pushes
// before its first wait.
template <int NVT, int WB>
__global__ void __launch_bounds__(kTpThreads) tp_rowpar_norm_kernel(TpRows a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];  // the owned row after the residual add, [H] fp16
  H8* srow = reinterpret_cast<H8*>(smem_raw);
  __shared__ float red_ss[kMaxRowWarps];
  __shared__ float red_max[32];
  pdl_wait();
  const int e = *reinterpret_cast<volatile int*>(a.ctrl);
  const int b = e & 1;
  const uint64_t limit = wait_limit_ns();
  pdl_trigger();
  if (!a.pushed)
    for (int j = blockIdx.x; j < a.R; j += gridDim.x) tp_push_rows(a, j, b);
  bool fail = false;
  for (int j = blockIdx.x; j < a.R && !fail; j += gridDim.x)
    if (a.rank * a.R + j < a.M) fail = !tp_reduce_row<NVT, WB>(a, j, b, limit, srow, red_ss, red_max);
  for (int j = blockIdx.x; j < a.R && !fail; j += gridDim.x) fail = !tp_collect_rows<NVT, WB>(a, j, b, limit);
  fail = __syncthreads_or(fail) != 0;
  if (threadIdx.x == 0) tp_finish_call(a, fail, e);
}

}  // namespace

TpLayout tp_layout(int world, int64_t H, int64_t max_rows) {
  TpLayout l;
  const int64_t rc = (max_rows + world - 1) / world;
  int64_t off = 0;
  l.partial = off;
  off = align256(off + max_rows * H * 2);
  l.recv = off;  // [2][world][rc][H] fp16
  off = align256(off + 2 * (int64_t)world * rc * H * 2);
  l.grq = off;  // [2][max_rows][H] e4m3
  off = align256(off + 2 * max_rows * H);
  l.grs = off;  // [2][max_rows] fp32
  off = align256(off + 2 * max_rows * 4);
  l.grh = off;  // [2][max_rows][H] fp16
  off = align256(off + 2 * max_rows * H * 2);
  l.ctrl = off;  // control words: the end of the area peers write
  off = align256(off + 256);
  l.outq = off;  // [max_rows][H] e4m3
  off = align256(off + max_rows * H);
  l.outs = off;  // [max_rows] fp32
  off = align256(off + max_rows * 4);
  l.outh = off;  // [max_rows][H] fp16
  off = align256(off + max_rows * H * 2);
  l.total = off;
  return l;
}

TpRows tp_rows_args(void* const* bases, int rank, int world, int64_t H, int64_t max_rows, int M) {
  const TpLayout l = tp_layout(world, H, max_rows);
  const int64_t rc = (max_rows + world - 1) / world;
  TpRows a = {};
  for (int p = 0; p < world; ++p) {
    char* base = static_cast<char*>(bases[p]);
    a.recv[p] = reinterpret_cast<__half*>(base + l.recv);
    a.grq[p] = reinterpret_cast<uint8_t*>(base + l.grq);
    a.grs[p] = reinterpret_cast<float*>(base + l.grs);
    a.grh[p] = reinterpret_cast<__half*>(base + l.grh);
  }
  char* me = static_cast<char*>(bases[rank]);
  a.partial = reinterpret_cast<const __half*>(me + l.partial);
  a.outq = reinterpret_cast<uint8_t*>(me + l.outq);
  a.outs = reinterpret_cast<float*>(me + l.outs);
  a.outh = reinterpret_cast<__half*>(me + l.outh);
  a.ctrl = reinterpret_cast<int*>(me + l.ctrl);
  a.recv_src = rc * H;
  a.recv_half = (int64_t)world * rc * H;
  a.g_half = max_rows;
  a.rank = rank;
  a.world = world;
  a.M = M;
  a.H = (int)H;
  a.R = (M + world - 1) / world;
  a.W = row_warps((int)(H / 8));
  return a;
}

cudaError_t launch_tp_buffer_init(void* base, int world, int64_t H, int64_t max_rows, cudaStream_t stream) {
  const TpLayout l = tp_layout(world, H, max_rows);
  cudaError_t e = cudaMemsetAsync(base, 0xFF, (size_t)l.ctrl, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(static_cast<char*>(base) + l.ctrl, 0, (size_t)(l.total - l.ctrl), stream);
  return e;
}

cudaError_t launch_tp_allreduce_rmsnorm_fp8(void* const* bases, int rank, int world, int64_t H, int64_t max_rows,
                                            void* residual, const void* weight, int M, float eps, int want_h,
                                            int pushed, int num_sms, cudaStream_t stream) {
  if (num_sms < 1 || world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || H % 16 != 0 || H > 16384 ||
      M > max_rows)
    return cudaErrorInvalidValue;
  if (M <= 0) return cudaSuccess;
  TpRows a = tp_rows_args(bases, rank, world, H, max_rows, M);
  a.residual = static_cast<__half*>(residual);
  a.weight = static_cast<const __half*>(weight);
  a.want_h = want_h ? 1 : 0;
  a.pushed = pushed ? 1 : 0;
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
  const int wb = tp_world_bound(world);
#define MS_TP_OP(N, W)                   \
  if (nvt == N && wb == W)               \
    return launch_kernel(tp_rowpar_norm_kernel<N, W>, grid, dim3(T), smem, stream, a);
  MS_TP_OP(1, 2) MS_TP_OP(1, 4) MS_TP_OP(1, 8)
  MS_TP_OP(2, 2) MS_TP_OP(2, 4) MS_TP_OP(2, 8)
  MS_TP_OP(3, 2) MS_TP_OP(3, 4) MS_TP_OP(3, 8)
  MS_TP_OP(4, 2) MS_TP_OP(4, 4) MS_TP_OP(4, 8)
#undef MS_TP_OP
  return cudaErrorInvalidValue;
}

}  // namespace ms
