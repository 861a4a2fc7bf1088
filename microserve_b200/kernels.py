"""Torch-tensor wrappers around the C ABI (one function per entry point).

These check dtypes/shapes the way the reference's wrappers assert them, pass
raw pointers and the current stream to the library and return torch tensors.
Every function requires CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

import threading

import torch

from microserve_b200 import _lib
from microserve_b200._lib import check, ptr, stream_ptr

FP8 = torch.float8_e4m3fn


def _cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (microserve-b200 has no CPU path)")


class _Workspace(threading.local):
    """Per-thread, per-device scratch buffers for kernels that need one, one
    buffer per kernel family ("gemm", "decode").

    The GEMM buffer starts zeroed: its first bytes hold tile flags that every
    GEMM call leaves at zero again. Buffers grow on demand outside CUDA-graph
    capture; inside a capture they must already be large enough (reserve()
    before capturing)."""

    def __init__(self):
        self.buf: dict[tuple[int, str], torch.Tensor] = {}
        # Buffers replaced by a larger one stay alive: captured CUDA graphs may
        # still hold their addresses.
        self.retired: list[torch.Tensor] = []

    def get(self, nbytes: int, device: torch.device, name: str = "decode") -> torch.Tensor | None:
        if nbytes == 0:
            return None
        idx = device.index if device.index is not None else torch.cuda.current_device()
        cur = self.buf.get((idx, name))
        if cur is None or cur.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    f"{name} workspace of {nbytes} bytes needed during CUDA-graph capture; reserve it first")
            if cur is not None:
                self.retired.append(cur)
            cur = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self.buf[(idx, name)] = cur
        return cur

    def reserve(self, nbytes: int, device: torch.device, name: str = "decode") -> None:
        self.get(nbytes, device, name)


workspace = _Workspace()


def quantize_rows_fp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [M, K] fp16 (unit stride on K) -> (xq [M, K] e4m3, sx [M] fp32)."""
    _cuda(x, "x")
    if x.dtype != torch.float16:
        raise ValueError("quantize_rows_fp8 requires fp16 input")
    x2 = x if x.dim() == 2 else x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, K = x2.shape
    xq = torch.empty((M, K), dtype=FP8, device=x.device)
    sx = torch.empty((M,), dtype=torch.float32, device=x.device)
    check(_lib.load().ms_quantize_rows_fp8(ptr(x2), x2.stride(0), M, K, ptr(xq), ptr(sx), stream_ptr()),
          "ms_quantize_rows_fp8")
    return xq, sx


def row_amax(x: torch.Tensor) -> torch.Tensor:
    """x [M, K] fp16 -> amax [M] fp32, the per-row absolute maximum."""
    _cuda(x, "x")
    if x.dtype != torch.float16:
        raise ValueError("row_amax requires fp16 input")
    x2 = x if x.dim() == 2 else x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, K = x2.shape
    amax = torch.empty((M,), dtype=torch.float32, device=x.device)
    check(_lib.load().ms_row_amax(ptr(x2), x2.stride(0), M, K, ptr(amax), stream_ptr()), "ms_row_amax")
    return amax


def quantize_rows_fp8_amax(x: torch.Tensor, amax: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_rows_fp8 with the row amax given (scale = max(amax, 1e-8) * fl32(1/448))."""
    _cuda(x, "x")
    if x.dtype != torch.float16 or amax.dtype != torch.float32:
        raise ValueError("quantize_rows_fp8_amax requires fp16 rows and fp32 amax")
    x2 = x if x.dim() == 2 else x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, K = x2.shape
    if amax.shape != (M,):
        raise ValueError("amax must have one entry per row")
    xq = torch.empty((M, K), dtype=FP8, device=x.device)
    sx = torch.empty((M,), dtype=torch.float32, device=x.device)
    check(_lib.load().ms_quantize_rows_fp8_amax(ptr(x2), x2.stride(0), M, K, ptr(amax), ptr(xq), ptr(sx),
                                                stream_ptr()), "ms_quantize_rows_fp8_amax")
    return xq, sx


def fp8_gemm(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
             bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """y [M, N] fp16 = fp16((xq . wq^T) * sx[:, None] * sw[None, :]) (+ bias)."""
    _cuda(xq, "xq")
    M, K = xq.shape
    N = wq.shape[0]
    if wq.shape[1] != K or xq.dtype != FP8 or wq.dtype != FP8:
        raise ValueError("fp8_gemm: expected e4m3 xq [M, K] and wq [N, K]")
    if not (xq.is_contiguous() and wq.is_contiguous()):
        raise ValueError("fp8_gemm: operands must be contiguous")
    y = out if out is not None else torch.empty((M, N), dtype=torch.float16, device=xq.device)
    lib = _lib.load()
    nbytes = lib.ms_fp8_gemm_workspace_size(M, N, K)
    ws = workspace.get(nbytes, xq.device, "gemm")
    check(lib.ms_fp8_gemm(ptr(xq), ptr(sx), ptr(wq), ptr(sw), ptr(bias), ptr(y), M, N, K, ptr(ws),
                          0 if ws is None else ws.numel(), stream_ptr()), "ms_fp8_gemm")
    return y


def f16_gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """y [M, N] fp16 = x [M, K] . w [N, K]^T with fp32 accumulation (the LM head's
    F.linear) on this library's tcgen05 GEMM."""
    _cuda(x, "x")
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K or x.dtype != torch.float16 or w.dtype != torch.float16:
        raise ValueError("f16_gemm: expected fp16 x [M, K] and w [N, K]")
    if not (x.is_contiguous() and w.is_contiguous()):
        raise ValueError("f16_gemm: operands must be contiguous")
    y = out if out is not None else torch.empty((M, N), dtype=torch.float16, device=x.device)
    lib = _lib.load()
    ws = workspace.get(lib.ms_f16_gemm_workspace_size(M, N, K), x.device, "gemm")
    check(lib.ms_f16_gemm(ptr(x), ptr(w), ptr(y), M, N, K, ptr(ws), 0 if ws is None else ws.numel(), stream_ptr()),
          "ms_f16_gemm")
    return y


def fp8_gemm_rowpar(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, bases, rank: int,
                    world: int, max_rows: int) -> None:
    """Row-parallel FP8 GEMM whose output rows go to their owners' receive slots in
    the tensor-parallel buffers `bases` (ms_fp8_gemm_rowpar)."""
    _cuda(xq, "xq")
    M, K = xq.shape
    N = wq.shape[0]
    if wq.shape[1] != K or xq.dtype != FP8 or wq.dtype != FP8:
        raise ValueError("fp8_gemm_rowpar: expected e4m3 xq [M, K] and wq [N, K]")
    if not (xq.is_contiguous() and wq.is_contiguous()):
        raise ValueError("fp8_gemm_rowpar: operands must be contiguous")
    lib = _lib.load()
    ws = workspace.get(lib.ms_fp8_gemm_workspace_size(M, N, K), xq.device, "gemm")
    check(lib.ms_fp8_gemm_rowpar(ptr(xq), ptr(sx), ptr(wq), ptr(sw), M, N, K, ptr(ws), 0 if ws is None else ws.numel(),
                                 bases, rank, world, max_rows, stream_ptr()), "ms_fp8_gemm_rowpar")


def fp8_gemm_rowpar_ar_rmsnorm(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, bases,
                               rank: int, world: int, max_rows: int, residual: torch.Tensor, weight: torch.Tensor,
                               eps: float, want_fp16: bool) -> None:
    """Row-parallel FP8 GEMM + all-reduce + residual + RMSNorm + FP8 (or fp16) rows in one
    kernel over the tensor-parallel buffers `bases` (ms_fp8_gemm_rowpar_ar_rmsnorm)."""
    _cuda(xq, "xq")
    M, K = xq.shape
    N = wq.shape[0]
    if wq.shape[1] != K or xq.dtype != FP8 or wq.dtype != FP8:
        raise ValueError("fp8_gemm_rowpar_ar_rmsnorm: expected e4m3 xq [M, K] and wq [N, K]")
    if not (xq.is_contiguous() and wq.is_contiguous()):
        raise ValueError("fp8_gemm_rowpar_ar_rmsnorm: operands must be contiguous")
    lib = _lib.load()
    ws = workspace.get(lib.ms_fp8_gemm_workspace_size(M, N, K), xq.device, "gemm")
    check(lib.ms_fp8_gemm_rowpar_ar_rmsnorm(ptr(xq), ptr(sx), ptr(wq), ptr(sw), M, N, K, ptr(ws),
                                            0 if ws is None else ws.numel(), bases, rank, world, max_rows,
                                            ptr(residual), ptr(weight), float(eps), 1 if want_fp16 else 0,
                                            stream_ptr()), "ms_fp8_gemm_rowpar_ar_rmsnorm")


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
            want_fp16: bool = True, want_fp8: bool = False):
    """(residual +) RMSNorm with optional fp16 and FP8 outputs.

    Returns (y | None, yq | None, sy | None, residual_out | None)."""
    _cuda(x, "x")
    H = x.shape[-1]
    x2 = x.reshape(-1, H)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    dev = x.device
    r2 = None
    rout = None
    if residual is not None:
        r2 = residual.reshape(-1, H)
        if not r2.is_contiguous():
            r2 = r2.contiguous()
        rout = torch.empty_like(x2)
    y = torch.empty_like(x2) if want_fp16 else None
    yq = torch.empty((M, H), dtype=FP8, device=dev) if want_fp8 else None
    sy = torch.empty((M,), dtype=torch.float32, device=dev) if want_fp8 else None
    check(_lib.load().ms_rmsnorm(ptr(x2), ptr(r2), ptr(weight), M, H, float(eps), ptr(rout), ptr(y), ptr(yq),
                                 ptr(sy), stream_ptr()), "ms_rmsnorm")
    return y, yq, sy, rout


def silu_mul(gu: torch.Tensor, want_fp16: bool = True, want_fp8: bool = False):
    """gu [M, 2I] -> (a [M, I] fp16 | None, aq | None, sa | None)."""
    _cuda(gu, "gu")
    g2 = gu.reshape(-1, gu.shape[-1])
    if not g2.is_contiguous():
        g2 = g2.contiguous()
    M, I2 = g2.shape
    I = I2 // 2
    out = torch.empty((M, I), dtype=torch.float16, device=gu.device) if want_fp16 else None
    aq = torch.empty((M, I), dtype=FP8, device=gu.device) if want_fp8 else None
    sa = torch.empty((M,), dtype=torch.float32, device=gu.device) if want_fp8 else None
    check(_lib.load().ms_silu_mul(ptr(g2), M, I, ptr(out), ptr(aq), ptr(sa), stream_ptr()), "ms_silu_mul")
    return out, aq, sa


def store_kv_fp8(key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping) -> None:
    T, Hkv, D = key.shape
    check(_lib.load().ms_store_kv_fp8(ptr(key), ptr(value), T, Hkv, D, ptr(slot_mapping), ptr(k_cache),
                                      ptr(v_cache), ptr(k_scale), ptr(v_scale), stream_ptr()), "ms_store_kv_fp8")


def qkv_post(qkv: torch.Tensor, q_heads: int, kv_heads: int, head_dim: int, positions: torch.Tensor,
             cos_tab: torch.Tensor, sin_tab: torch.Tensor, q_norm_w: torch.Tensor | None,
             k_norm_w: torch.Tensor | None, eps: float, slots: torch.Tensor | None = None,
             caches: tuple | None = None, want_kv: bool = False):
    """Fused q/k norm + RoPE (+ FP8 KV store). Returns (q, k | None, v | None)."""
    T = qkv.shape[0]
    dev = qkv.device
    q = torch.empty((T, q_heads, head_dim), dtype=torch.float16, device=dev)
    k = torch.empty((T, kv_heads, head_dim), dtype=torch.float16, device=dev) if want_kv else None
    v = torch.empty((T, kv_heads, head_dim), dtype=torch.float16, device=dev) if want_kv else None
    kc = vc = ks = vs = None
    if caches is not None:
        kc, vc, ks, vs = caches
    check(_lib.load().ms_qkv_post(ptr(qkv), T, q_heads, kv_heads, head_dim, ptr(q_norm_w), ptr(k_norm_w),
                                  float(eps), ptr(positions), ptr(cos_tab), ptr(sin_tab),
                                  ptr(slots) if caches is not None else None, ptr(q), ptr(k), ptr(v), ptr(kc),
                                  ptr(vc), ptr(ks), ptr(vs), stream_ptr()), "ms_qkv_post")
    return q, k, v


def decode_workspace_bytes(B: int, Hq: int, Hkv: int, max_blocks: int, block_size: int) -> int:
    return _lib.load().ms_paged_decode_workspace_size(B, Hq, Hkv, max_blocks, block_size)


def paged_decode_fp8(query, k_cache, v_cache, k_scale, v_scale, cache_seqlens, block_tables,
                     softmax_scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    B, Hq, D = query.shape
    NB, BS, Hkv, D2 = k_cache.shape
    max_blocks = block_tables.shape[1]
    o = out if out is not None else torch.empty_like(query)
    lib = _lib.load()
    nbytes = lib.ms_paged_decode_workspace_size(B, Hq, Hkv, max_blocks, BS)
    ws = workspace.get(nbytes, query.device)
    check(lib.ms_paged_decode_fp8(ptr(query), ptr(k_cache), ptr(v_cache), ptr(k_scale), ptr(v_scale),
                                  ptr(cache_seqlens), ptr(block_tables), ptr(o), B, Hq, Hkv, D, BS, max_blocks,
                                  float(softmax_scale), ptr(ws), 0 if ws is None else ws.numel(), stream_ptr()),
          "ms_paged_decode_fp8")
    return o


def paged_prefill_fp8(query, k_cache, v_cache, k_scale, v_scale, block_tables, cu_q, kv_lens,
                      softmax_scale: float) -> torch.Tensor:
    T, Hq, D = query.shape
    NB, BS, Hkv, _ = k_cache.shape
    o = torch.empty_like(query)
    num_seqs = cu_q.shape[0] - 1
    check(_lib.load().ms_paged_prefill_fp8(ptr(query), ptr(k_cache), ptr(v_cache), ptr(k_scale), ptr(v_scale),
                                           ptr(block_tables), ptr(cu_q), ptr(kv_lens), ptr(o), num_seqs, T, Hq,
                                           Hkv, D, BS, block_tables.shape[1], float(softmax_scale), stream_ptr()),
          "ms_paged_prefill_fp8")
    return o


def varlen_prefill(q, k, v, cu, softmax_scale: float) -> torch.Tensor:
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    o = torch.empty_like(q)
    check(_lib.load().ms_varlen_prefill(ptr(q), ptr(k), ptr(v), ptr(cu), ptr(o), cu.shape[0] - 1, T, Hq, Hkv, D,
                                        float(softmax_scale), stream_ptr()), "ms_varlen_prefill")
    return o


def argmax_rows(x: torch.Tensor, want_max: bool = False):
    """Row-wise argmax of fp16 logits [M, V] (unit stride on V): int64 indices
    (first index of the maximum, NaN highest, torch.argmax's rule) and, if
    want_max, the fp32 maxima."""
    _cuda(x, "x")
    if x.dtype != torch.float16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("argmax_rows: expected fp16 [M, V] with unit stride on V")
    M, V = x.shape
    idx = torch.empty(M, dtype=torch.int64, device=x.device)
    vmax = torch.empty(M, dtype=torch.float32, device=x.device) if want_max else None
    lib = _lib.load()
    ws = workspace.get(lib.ms_argmax_workspace_size(M), x.device, "argmax")
    check(lib.ms_argmax_rows(ptr(x), M, V, x.stride(0), ptr(idx), ptr(vmax), ptr(ws),
                             0 if ws is None else ws.numel(), stream_ptr()), "ms_argmax_rows")
    return (idx, vmax) if want_max else idx
