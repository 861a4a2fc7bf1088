"""The library's ops registered with torch.library (namespace ``microserve_b200``).

Each op runs the CUDA kernel through the C ABI (via ``microserve_b200.kernels``)
and has a fake implementation that gives the output shapes and dtypes without a
GPU, so torch's tracers (FakeTensor, ``make_fx``, ``torch.compile``) and CUDA-graph
capture treat them as opaque ops of known outputs. Ops that write the paged KV
cache declare those arguments as mutated.

The model in this package calls ``microserve_b200.kernels`` directly (no
dispatcher hop on the decode path); these ops are the surface for callers that
compose with torch, e.g. the reference's layers replaced op by op:

    reference call site (microserve/...)                 op
    layers/fp8_linear.py:71-73  _quantize_fp8_rows       quantize_rows_fp8
    layers/fp8_linear.py:75-79  _fp8_mm (+ bias)         fp8_gemm
    layers/layernorm.py:59-85   RMSNorm.forward          rmsnorm / add_rmsnorm (+ _fp8)
    layers/activation.py:5-8    SiluAndMul               silu_mul (+ _fp8)
    layers/fp8_kv_cache.py:42-61 store_fp8_kvcache       store_kv_fp8
    models/qwen3.py:44-53       q/k norm + RoPE (+store) qkv_post_decode / qkv_post_prefill
    layers/fp8_decode_attention.py:60-101                paged_decode_fp8
    layers/fp8_chunk_prefill_attention.py:77-109         paged_prefill_fp8
    layers/attention.py:49-55   flash_attn_varlen_func   varlen_prefill
    engine/model_runner.py:33-34 greedy torch.argmax     argmax_rows
"""
from __future__ import annotations

from typing import Optional

import torch
from torch.library import custom_op

from microserve_b200 import kernels

FP8 = torch.float8_e4m3fn
_NS = "microserve_b200"


def _rows(x: torch.Tensor) -> int:
    return x.numel() // x.shape[-1]


# ------------------------------------------------------------------ FP8 linear
@custom_op(f"{_NS}::quantize_rows_fp8", mutates_args=())
def quantize_rows_fp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [..., K] fp16 -> (xq [M, K] e4m3, sx [M] fp32), one dynamic scale per row."""
    return kernels.quantize_rows_fp8(x)


@quantize_rows_fp8.register_fake
def _(x):
    M, K = _rows(x), x.shape[-1]
    return x.new_empty((M, K), dtype=FP8), x.new_empty((M,), dtype=torch.float32)


@custom_op(f"{_NS}::fp8_gemm", mutates_args=())
def fp8_gemm(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
             bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y [M, N] fp16 = fp16((xq . wq^T) * sx * sw) (+ bias)."""
    return kernels.fp8_gemm(xq, sx, wq, sw, bias)


@fp8_gemm.register_fake
def _(xq, sx, wq, sw, bias=None):
    return xq.new_empty((xq.shape[0], wq.shape[0]), dtype=torch.float16)


# ------------------------------------------------------------------ RMSNorm
@custom_op(f"{_NS}::rmsnorm", mutates_args=())
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """y = fp16(fp16(x * rsqrt(mean(x^2) + eps)) * weight), rows of x [M, H]."""
    return kernels.rmsnorm(x, weight, eps)[0]


@rmsnorm.register_fake
def _(x, weight, eps):
    return x.new_empty((_rows(x), x.shape[-1]))


@custom_op(f"{_NS}::add_rmsnorm", mutates_args=())
def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """r = fp16(x + residual); returns (rmsnorm(r), r)."""
    y, _, _, r = kernels.rmsnorm(x, weight, eps, residual)
    return y, r


@add_rmsnorm.register_fake
def _(x, residual, weight, eps):
    shape = (_rows(x), x.shape[-1])
    return x.new_empty(shape), x.new_empty(shape)


@custom_op(f"{_NS}::rmsnorm_fp8", mutates_args=())
def rmsnorm_fp8(x: torch.Tensor, weight: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm fused with the next linear's row quantisation: (yq e4m3, sy fp32)."""
    _, yq, sy, _ = kernels.rmsnorm(x, weight, eps, want_fp16=False, want_fp8=True)
    return yq, sy


@rmsnorm_fp8.register_fake
def _(x, weight, eps):
    M = _rows(x)
    return x.new_empty((M, x.shape[-1]), dtype=FP8), x.new_empty((M,), dtype=torch.float32)


@custom_op(f"{_NS}::add_rmsnorm_fp8", mutates_args=())
def add_rmsnorm_fp8(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                    eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """r = fp16(x + residual); returns (yq, sy) of rmsnorm(r) and r."""
    _, yq, sy, r = kernels.rmsnorm(x, weight, eps, residual, want_fp16=False, want_fp8=True)
    return yq, sy, r


@add_rmsnorm_fp8.register_fake
def _(x, residual, weight, eps):
    M, H = _rows(x), x.shape[-1]
    return (x.new_empty((M, H), dtype=FP8), x.new_empty((M,), dtype=torch.float32), x.new_empty((M, H)))


# ------------------------------------------------------------------ SiLU * mul
@custom_op(f"{_NS}::silu_mul", mutates_args=())
def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """gu [M, 2I] (gate | up) -> fp16(fp16(silu(gate)) * up) [M, I]."""
    return kernels.silu_mul(gu)[0]


@silu_mul.register_fake
def _(gu):
    return gu.new_empty((_rows(gu), gu.shape[-1] // 2))


@custom_op(f"{_NS}::silu_mul_fp8", mutates_args=())
def silu_mul_fp8(gu: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """SiLU * mul fused with down_proj's row quantisation: (aq e4m3 [M, I], sa fp32 [M])."""
    _, aq, sa = kernels.silu_mul(gu, want_fp16=False, want_fp8=True)
    return aq, sa


@silu_mul_fp8.register_fake
def _(gu):
    M = _rows(gu)
    return gu.new_empty((M, gu.shape[-1] // 2), dtype=FP8), gu.new_empty((M,), dtype=torch.float32)


# ------------------------------------------------------------------ KV cache
_CACHES = ("k_cache", "v_cache", "k_scale", "v_scale")


@custom_op(f"{_NS}::store_kv_fp8", mutates_args=_CACHES)
def store_kv_fp8(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 k_scale: torch.Tensor, v_scale: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Per (token, kv head) scale + e4m3 codes of key/value [T, Hkv, D] scattered to slot_mapping."""
    kernels.store_kv_fp8(key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping)


@store_kv_fp8.register_fake
def _(key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping):
    return None


@custom_op(f"{_NS}::qkv_post_decode", mutates_args=_CACHES)
def qkv_post_decode(qkv: torch.Tensor, positions: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor,
                    q_norm_w: Optional[torch.Tensor], k_norm_w: Optional[torch.Tensor], slots: torch.Tensor,
                    k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
                    q_heads: int, kv_heads: int, head_dim: int, eps: float) -> torch.Tensor:
    """One pass over the QKV output: q/k RMSNorm, RoPE, FP8 K/V store; returns q [T, Hq, D]."""
    q, _, _ = kernels.qkv_post(qkv, q_heads, kv_heads, head_dim, positions, cos_tab, sin_tab, q_norm_w,
                               k_norm_w, eps, slots, (k_cache, v_cache, k_scale, v_scale), want_kv=False)
    return q


@qkv_post_decode.register_fake
def _(qkv, positions, cos_tab, sin_tab, q_norm_w, k_norm_w, slots, k_cache, v_cache, k_scale, v_scale,
      q_heads, kv_heads, head_dim, eps):
    return qkv.new_empty((qkv.shape[0], q_heads, head_dim))


@custom_op(f"{_NS}::qkv_post_prefill", mutates_args=_CACHES)
def qkv_post_prefill(qkv: torch.Tensor, positions: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor,
                     q_norm_w: Optional[torch.Tensor], k_norm_w: Optional[torch.Tensor], slots: torch.Tensor,
                     k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
                     q_heads: int, kv_heads: int, head_dim: int,
                     eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """As qkv_post_decode, also returning the fp16 k and v (first-chunk prefill attention)."""
    return kernels.qkv_post(qkv, q_heads, kv_heads, head_dim, positions, cos_tab, sin_tab, q_norm_w, k_norm_w,
                            eps, slots, (k_cache, v_cache, k_scale, v_scale), want_kv=True)


@qkv_post_prefill.register_fake
def _(qkv, positions, cos_tab, sin_tab, q_norm_w, k_norm_w, slots, k_cache, v_cache, k_scale, v_scale,
      q_heads, kv_heads, head_dim, eps):
    T = qkv.shape[0]
    return (qkv.new_empty((T, q_heads, head_dim)), qkv.new_empty((T, kv_heads, head_dim)),
            qkv.new_empty((T, kv_heads, head_dim)))


# ------------------------------------------------------------------ attention
@custom_op(f"{_NS}::paged_decode_fp8", mutates_args=())
def paged_decode_fp8(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor,
                     v_scale: torch.Tensor, cache_seqlens: torch.Tensor, block_tables: torch.Tensor,
                     softmax_scale: float) -> torch.Tensor:
    """Decode attention of query [B, Hq, D] over each sequence's paged FP8 K/V."""
    return kernels.paged_decode_fp8(query, k_cache, v_cache, k_scale, v_scale, cache_seqlens, block_tables,
                                    softmax_scale)


@paged_decode_fp8.register_fake
def _(query, k_cache, v_cache, k_scale, v_scale, cache_seqlens, block_tables, softmax_scale):
    return torch.empty_like(query)


@custom_op(f"{_NS}::paged_prefill_fp8", mutates_args=())
def paged_prefill_fp8(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor,
                      v_scale: torch.Tensor, block_tables: torch.Tensor, cu_q: torch.Tensor, kv_lens: torch.Tensor,
                      softmax_scale: float) -> torch.Tensor:
    """Causal attention of new tokens query [T, Hq, D] over prefix + themselves in the paged FP8 cache."""
    return kernels.paged_prefill_fp8(query, k_cache, v_cache, k_scale, v_scale, block_tables, cu_q, kv_lens,
                                     softmax_scale)


@paged_prefill_fp8.register_fake
def _(query, k_cache, v_cache, k_scale, v_scale, block_tables, cu_q, kv_lens, softmax_scale):
    return torch.empty_like(query)


@custom_op(f"{_NS}::varlen_prefill", mutates_args=())
def varlen_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                   softmax_scale: float) -> torch.Tensor:
    """Causal varlen attention over fresh fp16 q [T, Hq, D], k, v [T, Hkv, D]."""
    return kernels.varlen_prefill(q, k, v, cu_seqlens, softmax_scale)


@varlen_prefill.register_fake
def _(q, k, v, cu_seqlens, softmax_scale):
    return torch.empty_like(q)


# ------------------------------------------------------------------ sampling
@custom_op(f"{_NS}::argmax_rows", mutates_args=())
def argmax_rows(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token per row of fp16 logits [M, V]: first index of the maximum, NaN highest."""
    return kernels.argmax_rows(logits)


@argmax_rows.register_fake
def _(logits):
    return logits.new_empty((logits.shape[0],), dtype=torch.int64)


OPS = ("quantize_rows_fp8", "fp8_gemm", "rmsnorm", "add_rmsnorm", "rmsnorm_fp8", "add_rmsnorm_fp8", "silu_mul",
       "silu_mul_fp8", "store_kv_fp8", "qkv_post_decode", "qkv_post_prefill", "paged_decode_fp8",
       "paged_prefill_fp8", "varlen_prefill", "argmax_rows")
