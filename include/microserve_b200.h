/*
 * microserve-b200: C ABI of the B200 (sm_100a) FP8 decoder-layer kernels.
 *
 * Every entry point takes raw device pointers, explicit sizes and a
 * cudaStream_t passed as `void*`, enqueues its kernels on that stream and
 * returns without synchronising. None allocates device memory: callers own
 * every buffer, including the scratch `workspace` some kernels need (query
 * its size with the matching *_workspace_size function). All entry points are
 * CUDA-graph capturable.
 *
 * Return codes: MS_OK (0) or a negative MS_ERR_* code; ms_last_error() then
 * returns a message (thread-local). Tensor layouts are row-major and
 * contiguous unless a stride argument says otherwise; fp16 is IEEE half,
 * fp8 is e4m3 ("float8_e4m3fn"), scales are fp32.
 *
 * FP8 encoding (bit-exact with the reference):
 *   scale = max(amax, 1e-8) * fl32(1/448);  code = e4m3_rn_satfinite(clamp(x / scale, -448, 448))
 *   (the reference writes `/ 448`; its Triton kernels and torch's CUDA division evaluate
 *   that as a multiply by the fp32 reciprocal, which is what its GPU outputs show)
 *
 * Each declaration names the reference interface it replaces
 * (gssg1/microserve, path:line).
 */
#ifndef MICROSERVE_B200_H_
#define MICROSERVE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MS_OK 0
#define MS_ERR_INVALID (-1)     /* bad argument: null pointer, negative or unsupported size */
#define MS_ERR_UNSUPPORTED (-2) /* shape outside what the kernels implement (e.g. head_dim != 128) */
#define MS_ERR_CUDA (-3)        /* a CUDA runtime call failed; see ms_last_error() */
#define MS_ERR_WORKSPACE (-4)   /* workspace smaller than the *_workspace_size result */

/* Library version (major * 10000 + minor * 100 + patch). */
int ms_version(void);

/* Message for the last non-zero return code on this thread. */
const char* ms_last_error(void);

/* Number of kernel launches the library has issued from this process (host
 * counter; a CUDA-graph replay re-runs captured launches without calling the
 * library, so it is counted once, at capture). */
int64_t ms_launch_count(void);

/* Programmatic dependent launch (no reference counterpart; a launch setting of
 * this library). When enabled (the default) every kernel is launched with
 * programmatic stream serialization allowed: it may start its prologue (and,
 * for the GEMM, its weight loads) while the preceding kernel in the stream
 * finishes, and waits for that kernel before touching any data it could
 * produce or consume. Returns the previous setting. Process-wide. */
int ms_set_pdl(int enable);

/* GEMM schedules on pairs of SMs (tcgen05 cta_group::2 clusters; no reference
 * counterpart): off by default; when enabled, 129..256-token and prefill shapes
 * may use them (ms_fp8_gemm_plan reports plan[6] = 1), otherwise every GEMM uses
 * one-SM tiles. The engine enables them on one GPU when Config.gemm_pair_tiles
 * is set. Returns the previous setting. Process-wide. */
int ms_set_pair_tiles(int enable);

/* Reads and clears the device status word of the current device. Kernels
 * that wait on barriers give up after a bounded time, record a non-zero code
 * there (1 = tensor-core pipeline timeout, 2 = peer timeout) and return.
 * Synchronises `stream`. */
int ms_get_device_status(int* status, void* stream);

/* Per-row dynamic FP8 quantisation of an fp16 matrix.
 *   x [M, K] fp16 with row stride ldx (elements) -> xq [M, K] e4m3, sx [M] fp32.
 * Replaces `_quantize_fp8_rows` (microserve/layers/fp8_linear.py:14-23). The
 * same call quantises weights offline with one scale per output channel
 * (microserve/layers/fp8_linear.py:49-56, FP8DynamicLinear.__init__). */
int ms_quantize_rows_fp8(const void* x, int64_t ldx, int64_t M, int64_t K, void* xq, float* sx, void* stream);

/* W8A8 FP8 GEMM with per-row x per-channel dequant:
 *   y [M, N] fp16 = fp16((xq [M,K] . wq [N,K]^T) * sx[m] * sw[n]) (+ bias[n], fp16 add)
 * Replaces `_fp8_mm` and FP8DynamicLinear.forward
 * (microserve/layers/fp8_linear.py:26-45, :64-80). bias may be NULL.
 * workspace: at least ms_fp8_gemm_workspace_size(M, N, K) bytes (may be 0). */
size_t ms_fp8_gemm_workspace_size(int64_t M, int64_t N, int64_t K);

/* The schedule ms_fp8_gemm uses for M x N x K on a GPU with `sms` SMs (host
 * only, no GPU needed; for inspection and tests): plan[0] token-tile width BN
 * (0 = the CUDA-core kernel for K % 16 != 0), plan[1] CTAs, plan[2] K parts
 * per weight tile (split-K; 0 otherwise), plan[3] 1 for 256-row x 256-token
 * tiles, plan[4] 1 for whole tiles (0: split-K or stream-K), plan[5] 128-byte
 * K chunks per pipeline stage, plan[6] 1 for 256 x 256 tiles on pairs of SMs
 * (tcgen05 cta_group::2; plan must hold 7 ints). No reference counterpart (the reference's
 * `_fp8_mm` grid is fixed, microserve/layers/fp8_linear.py:75-77). */
int ms_fp8_gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int* plan);
int ms_fp8_gemm(const void* xq, const float* sx, const void* wq, const float* sw, const void* bias, void* y,
                int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* fp16 GEMM on the same tcgen05 kernels (kind::f16): y [M, N] fp16 = fp16(x [M, K] .
 * w [N, K]^T), fp32 accumulation, both operands K-contiguous and 16-byte aligned,
 * K % 8 == 0. Replaces the LM head's F.linear (microserve/layers/embed_head.py:35-36,
 * ParallelLMHead.forward; the vocab-parallel slice of it under tensor parallelism).
 * workspace: at least ms_f16_gemm_workspace_size(M, N, K) bytes (may be 0). */
size_t ms_f16_gemm_workspace_size(int64_t M, int64_t N, int64_t K);
int ms_f16_gemm(const void* x, const void* w, void* y, int64_t M, int64_t N, int64_t K, void* workspace,
                size_t workspace_bytes, void* stream);

/* RMSNorm over rows of H (H % 16 == 0, H <= 32768), optionally fused with the residual
 * add and an FP8 quantisation of the output:
 *   residual == NULL: y = fp16(fp16(x * rsqrt(mean(x^2) + eps)) * weight)
 *   residual != NULL: r = fp16(x + residual) -> residual_out; y = norm(r)
 *   y (may be NULL) fp16 [M, H]; yq/sy (may be NULL) = ms_quantize_rows_fp8(y)
 * Replaces RMSNorm.forward with `_rmsnorm_kernel` / `_residual_rmsnorm_kernel`
 * (microserve/layers/layernorm.py:7-42, :59-85). residual_out may alias residual. */
int ms_rmsnorm(const void* x, const void* residual, const void* weight, int64_t M, int64_t H, float eps,
               void* residual_out, void* y, void* yq, float* sy, void* stream);

/* SiLU-and-mul over gu [M, 2I] (gate | up), I % 16 == 0, I <= 32768:
 *   a = fp16(fp16(silu(gate)) * up) -> out [M, I] (may be NULL); aq/sa (may be NULL) its FP8 rows.
 * Replaces SiluAndMul (microserve/layers/activation.py:5-8) followed by
 * `_quantize_fp8_rows` of down_proj's input (microserve/layers/fp8_linear.py:71-73). */
int ms_silu_mul(const void* gu, int64_t M, int64_t I, void* out, void* aq, float* sa, void* stream);

/* FP8 KV-cache store: per (token, kv head) scale + e4m3 codes scattered to slots.
 *   k, v [T, kv_heads, head_dim] fp16; slots [T] int64 (negative = skip)
 *   k_cache, v_cache [num_blocks, block_size, kv_heads, head_dim] e4m3
 *   k_scale, v_scale [num_blocks, block_size, kv_heads] fp32
 * Replaces store_fp8_kvcache (microserve/layers/fp8_kv_cache.py:11-61). head_dim must be 128. */
int ms_store_kv_fp8(const void* k, const void* v, int64_t T, int kv_heads, int head_dim, const int64_t* slots,
                    void* k_cache, void* v_cache, float* k_scale, float* v_scale, void* stream);

/* Attention prologue of Qwen3Attention.forward fused in one pass over the QKV
 * projection output qkv [T, (q_heads + 2 kv_heads) * head_dim] fp16:
 * per-head q/k RMSNorm (skipped when q_norm_w == NULL), neox RoPE from fp16
 * tables cos/sin [max_position, head_dim / 2] at positions [T] int64, then
 *   q_out [T, q_heads, head_dim] fp16,
 *   k_out / v_out [T, kv_heads, head_dim] fp16 (each may be NULL),
 *   FP8 store of k and v into the cache at slots (skipped when slots == NULL).
 * Replaces microserve/models/qwen3.py:44-53 (q/k norm: layers/layernorm.py:82-85,
 * RoPE: layers/rotary_embedding.py:24-31) and the store of attention.py:41-43. */
int ms_qkv_post(const void* qkv, int64_t T, int q_heads, int kv_heads, int head_dim, const void* q_norm_w,
                const void* k_norm_w, float eps, const int64_t* positions, const void* cos_tab, const void* sin_tab,
                const int64_t* slots, void* q_out, void* k_out, void* v_out, void* k_cache, void* v_cache,
                float* k_scale, float* v_scale, void* stream);

/* Paged FP8-KV decode attention, one query token per sequence.
 *   q [B, Hq, head_dim] fp16; seqlens [B] int32; block_tables [B, max_blocks] int32
 *   caches as in ms_store_kv_fp8; out [B, Hq, head_dim] fp16 (0 for seqlens == 0)
 * Hq % Hkv == 0, Hq / Hkv <= 8, head_dim == 128, block_size % 16 == 0.
 * Replaces fp8_decode_attention (microserve/layers/fp8_decode_attention.py:8-101).
 * workspace: ms_paged_decode_workspace_size(...) bytes (0 when no context split is used). */
size_t ms_paged_decode_workspace_size(int B, int Hq, int Hkv, int max_blocks, int block_size);
int ms_paged_decode_fp8(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                        const float* v_scale, const int32_t* seqlens, const int32_t* block_tables, void* out, int B,
                        int Hq, int Hkv, int head_dim, int block_size, int max_blocks, float softmax_scale,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ms_paged_decode_fp8 without a workspace argument and without any allocation.
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory where attention runs (inside another framework's memory pool,
 * embedders that forbid cudaMalloc after start-up, callers holding only a
 * stream). The context-split partials go to a 4 MiB buffer built into the
 * library, which every GPU that loads the library keeps until exit; batches
 * needing more return MS_ERR_UNSUPPORTED (use ms_paged_decode_fp8). The first
 * call on a device (and the first after the device's context was destroyed and
 * recreated, e.g. by cudaDeviceReset) looks up the buffer's device address, so
 * make it before any stream capture. All calls on a device share the buffer:
 * calls that overlap on the GPU race and must be serialised by the caller. */
int ms_paged_decode_fp8_noalloc(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                                const float* v_scale, const int32_t* seqlens, const int32_t* block_tables, void* out,
                                int B, int Hq, int Hkv, int head_dim, int block_size, int max_blocks,
                                float softmax_scale, void* stream);

/* Causal chunked-prefill attention over the paged FP8 cache, any number of
 * sequences: sequence s has queries q[cu_q[s] .. cu_q[s+1]) at positions
 * kv_lens[s] - q_len_s .. kv_lens[s] - 1 and attends to its first kv_lens[s]
 * cached tokens (which must already hold this chunk's keys/values).
 *   q, out [total_q, Hq, head_dim] fp16; cu_q [num_seqs + 1] int32; kv_lens [num_seqs] int32
 *   block_tables [num_seqs, max_blocks] int32; block_size % 64 == 0
 * Replaces fp8_chunk_prefill_attention
 * (microserve/layers/fp8_chunk_prefill_attention.py:8-109; one sequence per call there). */
int ms_paged_prefill_fp8(const void* q, const void* k_cache, const void* v_cache, const float* k_scale,
                         const float* v_scale, const int32_t* block_tables, const int32_t* cu_q,
                         const int32_t* kv_lens, void* out, int num_seqs, int64_t total_q, int Hq, int Hkv,
                         int head_dim, int block_size, int max_blocks, float softmax_scale, void* stream);

/* Causal varlen prefill attention over fresh fp16 q, k, v (first chunk of
 * each sequence): q, out [total, Hq, head_dim]; k, v [total, Hkv, head_dim];
 * cu [num_seqs + 1] int32 (same offsets for queries and keys).
 * Replaces the FP8-KV PREFILL branch's flash_attn_varlen_func call
 * (microserve/layers/attention.py:49-55). */
int ms_varlen_prefill(const void* q, const void* k, const void* v, const int32_t* cu, void* out, int num_seqs,
                      int64_t total, int Hq, int Hkv, int head_dim, float softmax_scale, void* stream);

/* Greedy token selection: idx[m] = argmax_v x[m, v] over fp16 logits rows
 * (row stride ldx elements), the first index of the maximum, NaN above every
 * number, -0.0 equal to +0.0; vmax (may be NULL) receives the maximum as fp32
 * (for merging vocab-parallel shards). Replaces the greedy branch of `_sample`
 * (microserve/engine/model_runner.py:33-34, torch.argmax). The workspace
 * (ms_argmax_workspace_size bytes) must be zeroed before its first use and
 * used for this entry point only (per-row counters at its start return to zero
 * after every call). M <= 16384. */
size_t ms_argmax_workspace_size(int64_t M);
int ms_argmax_rows(const void* x, int64_t M, int64_t V, int64_t ldx, int64_t* idx, float* vmax, void* workspace,
                   size_t workspace_bytes, void* stream);

/* ---- tensor parallel over NVLink peer memory (no reference counterpart for the
 * plumbing; the fused op replaces dist.all_reduce + add/RMSNorm + act quant) ----
 *
 * ms_ipc_handle: CUDA IPC handle (64 bytes) of the allocation holding `ptr` and
 * ptr's offset inside it; ms_ipc_open maps a peer's handle in this process
 * (base to close later, ptr = base + offset); ms_ipc_close unmaps. */
int ms_ipc_handle(const void* ptr, void* handle, int64_t* offset);
int ms_ipc_open(const void* handle, int64_t offset, void** base_out, void** ptr_out);
int ms_ipc_close(void* base);

/* Byte offsets inside one rank's communication buffer for the fused op below
 * (world ranks, hidden size H, at most max_rows rows per call):
 *   offsets[0] partial  [max_rows, H] fp16  this rank's row-parallel output, when
 *                                           the GEMM does not push its tiles itself
 *   offsets[1] out_q    [max_rows, H] e4m3  the normalised rows of the last call (FP8 codes)
 *   offsets[2] out_s    [max_rows] fp32     their scales
 *   offsets[3] out_h    [max_rows, H] fp16  the normalised rows of the last want_fp16 call
 *   offsets[4] total bytes.
 * The rest of the buffer holds the receive slots peers write (internal).
 * No reference counterpart (plumbing of the op below). */
int ms_tp_layout(int world, int64_t hidden, int64_t max_rows, int64_t* offsets);

/* Puts one rank's buffer (ms_tp_layout total bytes, 256-byte aligned) in its
 * initial state: every byte 0xFF ("not yet written") except the control words
 * (zero). Call once per rank, before the buffer is shared, with the stream
 * synchronised before any peer's first call. */
int ms_tp_buffer_init(void* base, int world, int64_t hidden, int64_t max_rows, void* stream);

/* Row-parallel all-reduce + residual add + RMSNorm + FP8 row quantisation, one
 * kernel per rank. bases[p] = rank p's communication buffer as mapped in this
 * process (CUDA IPC; bases[rank] is the local one). The rank's row-parallel
 * output [M, H] fp16 is read from its partial area, or - with pushed != 0 - is
 * already in the receive slots because ms_fp8_gemm_rowpar wrote it there. With
 * R = ceil(M / world), rank r owns rows [r R, (r + 1) R): it sums those rows of
 * every rank's output in rank order (fp32, rounded to fp16 once), adds its
 * residual rows (updated in place, fp16), normalises them (weight [H] fp16, eps)
 * and sends codes + scales (with want_fp16: fp16 rows) to every rank; on the
 * GPU the call ends once all M rows are in this rank's out area. Rows of the
 * residual that the rank does not own are neither read nor written. Readiness
 * is carried by the data (no flags); every wait is bounded (ms_set_wait_limit)
 * and a wait that runs out records status 2 (peer timeout, ms_get_device_status),
 * after which the buffers of the whole group must be re-initialised. Every rank
 * makes the same sequence of calls with the same M.
 * Replaces RowParallelLinear's dist.all_reduce (microserve/layers/linear.py:70-77)
 * + the add/RMSNorm that follows (layers/layernorm.py:22-42) + the next FP8
 * activation quantisation (layers/fp8_linear.py:14-23).
 * world <= 8, H % 16 == 0, H <= 16384, 0 <= M <= max_rows. */
int ms_tp_allreduce_rmsnorm_fp8(void* const* bases, int rank, int world, int64_t hidden, int64_t max_rows,
                                void* residual, const void* weight, int64_t M, float eps, int want_fp16, int pushed,
                                void* stream);

/* The row-parallel FP8 GEMM of tensor parallelism (o_proj, down_proj) with its
 * output pushed to the ranks that own the rows: Y = fp16((Xq . Wq^T) * sx * sw)
 * as ms_fp8_gemm (xq [M, K], wq [N, K] this rank's K shard, N = the hidden size
 * of the buffers), except that each output row m is written - by the GEMM's
 * epilogue, tile by tile, as tiles finish - into the receive slot of rank
 * m / ceil(M / world) in that rank's communication buffer (bases as for
 * ms_tp_allreduce_rmsnorm_fp8), so the transfer overlaps the GEMM. Follow it
 * with ms_tp_allreduce_rmsnorm_fp8(..., pushed = 1) on the same stream.
 * workspace: ms_fp8_gemm_workspace_size(M, N, K) bytes. Replaces the GEMM of
 * RowParallelLinear (microserve/layers/linear.py:70-77; F.linear, or
 * FP8DynamicLinear.forward when quantised, layers/fp8_linear.py:64-80) and the
 * transfer half of its dist.all_reduce. */
int ms_fp8_gemm_rowpar(const void* xq, const float* sx, const void* wq, const float* sw, int64_t M, int64_t N,
                       int64_t K, void* workspace, size_t workspace_bytes, void* const* bases, int rank, int world,
                       int64_t max_rows, void* stream);

/* ms_fp8_gemm_rowpar + ms_tp_allreduce_rmsnorm_fp8(..., pushed = 1) as ONE kernel
 * per rank: the row-parallel FP8 GEMM pushes its output rows to their owners from
 * its epilogue, then each CTA, once its tiles are out, reduces its share of this
 * rank's rows (rank order, fp32), adds the residual, normalises (weight, eps),
 * quantises and sends the rows to every rank (codes + scales, or fp16 rows with
 * want_fp16) - outputs and semantics exactly those of the two calls, in the out
 * areas of ms_tp_layout. When the row work does not fit the GEMM's tail (hidden
 * > 6144, or more than two owned rows per GEMM CTA - prefill-sized M) the call
 * launches the two kernels instead. Replaces RowParallelLinear + its
 * dist.all_reduce (microserve/layers/linear.py:70-77; FP8DynamicLinear.forward,
 * layers/fp8_linear.py:64-80) + the add/RMSNorm after it (layers/layernorm.py:22-42)
 * + the next activation quantisation (layers/fp8_linear.py:14-23). */
int ms_fp8_gemm_rowpar_ar_rmsnorm(const void* xq, const float* sx, const void* wq, const float* sw, int64_t M,
                                  int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* const* bases,
                                  int rank, int world, int64_t max_rows, void* residual, const void* weight,
                                  float eps, int want_fp16, void* stream);

/* Upper bound, in nanoseconds, of every in-kernel wait on the current device
 * (peer data, pipeline barriers); default 4e9. A wait that runs out records a
 * device status and the kernel returns. Set it outside stream capture; it
 * applies to launches made after the call. No reference counterpart (the
 * reference has only host asserts, microserve/engine/llm.py:43-49). */
int ms_set_wait_limit(uint64_t ns);

/* Per-row absolute maximum of fp16 rows: amax[m] = max_k |x[m, k]| (fp32).
 * With ms_quantize_rows_fp8_amax it gives the exact row scales of a K-sharded
 * activation (an all-reduce max of amax between the two calls): the scale the
 * reference computes over the full row (microserve/layers/fp8_linear.py:20). */
int ms_row_amax(const void* x, int64_t ldx, int64_t M, int64_t K, float* amax, void* stream);

/* ms_quantize_rows_fp8 with the row amax given (scale = max(amax[m], 1e-8)
 * * fl32(1/448)) instead of taken over the K columns passed. */
int ms_quantize_rows_fp8_amax(const void* x, int64_t ldx, int64_t M, int64_t K, const float* amax, void* xq,
                              float* sx, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MICROSERVE_B200_H_ */
