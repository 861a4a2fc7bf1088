"""Decode attention over the paged FP8 KV cache
(microserve/layers/fp8_decode_attention.py:62-101). `block_n` is accepted for
signature compatibility; the kernel's tiling is fixed (16-token tiles, GQA
heads grouped, context split chosen from the batch shape)."""
import torch

from microserve_b200 import kernels


def fp8_decode_attention(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         k_scale_cache: torch.Tensor, v_scale_cache: torch.Tensor, cache_seqlens: torch.Tensor,
                         block_tables: torch.Tensor, softmax_scale: float, block_n: int | None = None,
                         out: torch.Tensor | None = None) -> torch.Tensor:
    query = query.contiguous()
    cache_seqlens = cache_seqlens.contiguous()
    block_tables = block_tables.contiguous()
    batch_size, num_q_heads, head_dim = query.shape
    num_kv_heads = k_cache.shape[2]
    assert query.dtype == torch.float16
    assert k_cache.dtype == v_cache.dtype == torch.float8_e4m3fn
    assert k_scale_cache.dtype == v_scale_cache.dtype == torch.float32
    assert cache_seqlens.dtype == torch.int32
    assert block_tables.dtype == torch.int32
    assert num_q_heads % num_kv_heads == 0
    assert head_dim == k_cache.shape[3]
    return kernels.paged_decode_fp8(query, k_cache, v_cache, k_scale_cache, v_scale_cache, cache_seqlens,
                                    block_tables, softmax_scale, out=out)
