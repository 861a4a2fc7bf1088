"""FP8 e4m3 paged KV-cache store (microserve/layers/fp8_kv_cache.py:42-61)."""
import torch

from microserve_b200 import kernels

FP8_MAX = 448.0


def store_fp8_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      k_scale_cache: torch.Tensor, v_scale_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    key = key.contiguous()
    value = value.contiguous()
    slot_mapping = slot_mapping.contiguous()
    if slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.long()
    num_tokens, num_kv_heads, head_dim = key.shape
    assert value.shape == key.shape
    assert key.dtype == torch.float16
    assert k_cache.dtype == v_cache.dtype == torch.float8_e4m3fn
    assert k_scale_cache.dtype == v_scale_cache.dtype == torch.float32
    assert k_cache.shape[2:] == (num_kv_heads, head_dim)
    assert k_scale_cache.shape == k_cache.shape[:-1]
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    kernels.store_kv_fp8(key, value, k_cache, v_cache, k_scale_cache, v_scale_cache, slot_mapping)
