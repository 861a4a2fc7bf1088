"""Causal chunked-prefill attention over the paged FP8 KV cache
(microserve/layers/fp8_chunk_prefill_attention.py:70-109), plus the
multi-sequence form used by the runner (the reference runs one sequence per
launch). `block_m` / `block_n` are accepted for signature compatibility."""
import torch

from microserve_b200 import kernels


def fp8_chunk_prefill_attention(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                k_scale_cache: torch.Tensor, v_scale_cache: torch.Tensor,
                                block_table: torch.Tensor, prefix_len: int, softmax_scale: float,
                                block_m: int | None = None, block_n: int | None = None) -> torch.Tensor:
    query = query.contiguous()
    block_table = block_table.contiguous().view(1, -1).to(torch.int32)
    query_len, num_q_heads, head_dim = query.shape
    num_kv_heads = k_cache.shape[2]
    assert query.dtype == torch.float16
    assert k_cache.dtype == v_cache.dtype == torch.float8_e4m3fn
    assert k_scale_cache.dtype == v_scale_cache.dtype == torch.float32
    assert num_q_heads % num_kv_heads == 0
    assert head_dim == k_cache.shape[3]
    meta = torch.tensor([0, query_len, prefix_len + query_len], dtype=torch.int32).to(query.device,
                                                                                       non_blocking=True)
    return kernels.paged_prefill_fp8(query, k_cache, v_cache, k_scale_cache, v_scale_cache, block_table,
                                     meta[:2], meta[2:], softmax_scale)


def fp8_varlen_chunk_prefill_attention(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                       k_scale_cache: torch.Tensor, v_scale_cache: torch.Tensor,
                                       block_tables: torch.Tensor, cu_seqlens_q: torch.Tensor,
                                       kv_lens: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    """Every sequence of a chunked-prefill batch in one launch: sequence s has
    queries cu_seqlens_q[s]:cu_seqlens_q[s+1] and kv_lens[s] cached tokens."""
    return kernels.paged_prefill_fp8(query.contiguous(), k_cache, v_cache, k_scale_cache, v_scale_cache,
                                     block_tables.contiguous(), cu_seqlens_q, kv_lens, softmax_scale)
