"""Paged attention layer (microserve/layers/attention.py:23-85), FP8 KV cache.

The runner injects k_cache / v_cache / k_scale_cache / v_scale_cache /
kv_cache_dtype as plain attributes (microserve/engine/model_runner.py:111-122).
forward(q, k, v) stores k/v into the cache and then, by context mode:
  DECODE        -> paged FP8 decode attention
  PREFILL       -> causal varlen attention over the fresh fp16 q, k, v
  CHUNK_PREFILL -> causal attention over the cache (every sequence of the
                   batch in one launch; the reference handles one)
forward_cached(q, k, v) is the same without the store, for callers whose
prologue kernel already wrote the cache (the fused Qwen3 layer).
Only the FP8 e4m3 cache is implemented.
"""
import torch
from torch import nn

from microserve_b200 import kernels
from microserve_b200.layers.fp8_kv_cache import store_fp8_kvcache
from microserve_b200.utils.context import AttentionMode, get_context


class Attention(nn.Module):
    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])
        self.k_scale_cache = self.v_scale_cache = None
        self.kv_cache_dtype = "fp8_e4m3"

    def _check_cache(self):
        assert self.k_cache.numel(), "k_cache not injected: the runner must allocate the KV cache first"
        if self.kv_cache_dtype != "fp8_e4m3":
            raise NotImplementedError("microserve-b200 implements the FP8 e4m3 KV cache only")

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        self._check_cache()
        ctx = get_context()
        store_fp8_kvcache(k, v, self.k_cache, self.v_cache, self.k_scale_cache, self.v_scale_cache,
                          ctx.slot_mapping)
        return self.forward_cached(q, k, v)

    def forward_cached(self, q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        self._check_cache()
        ctx = get_context()
        if ctx.mode is AttentionMode.DECODE:
            return kernels.paged_decode_fp8(q, self.k_cache, self.v_cache, self.k_scale_cache, self.v_scale_cache,
                                            ctx.cache_seqlens, ctx.block_tables, self.scale, out=out)
        if ctx.mode is AttentionMode.PREFILL:
            return kernels.varlen_prefill(q, k, v, ctx.cu_seqlens_q, self.scale)
        if ctx.mode is AttentionMode.CHUNK_PREFILL:
            return kernels.paged_prefill_fp8(q, self.k_cache, self.v_cache, self.k_scale_cache, self.v_scale_cache,
                                             ctx.block_tables, ctx.cu_seqlens_q, ctx.cache_seqlens, self.scale)
        raise RuntimeError(f"unsupported attention mode: {ctx.mode}")
