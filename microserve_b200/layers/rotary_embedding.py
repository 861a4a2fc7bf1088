"""Neox-style rotary embedding (microserve/layers/rotary_embedding.py:4-41).

The fp32 cos/sin tables are built exactly as the reference builds them (on
the host, in fp32, emb = cat(freqs, freqs)); the kernel reads their fp16
casts (the reference casts per call, :26-27), and since the two halves of
`emb` are equal only the first head_dim/2 columns are kept.
"""
import torch
from torch import nn

from microserve_b200 import kernels


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


class RotaryEmbedding(nn.Module):
    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float) -> None:
        super().__init__()
        self.head_size = head_size
        assert rotary_dim == head_size
        # built on the host even when the model is constructed under a CUDA device context,
        # so the tables are the reference's CPU-computed values
        cpu = torch.device("cpu")
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32, device=cpu) / rotary_dim))
        t = torch.arange(max_position_embeddings, dtype=torch.float32, device=cpu)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1)
        cos = emb.cos().unsqueeze_(1)
        sin = emb.sin().unsqueeze_(1)
        self.register_buffer("cos_cache", cos, persistent=False)
        self.register_buffer("sin_cache", sin, persistent=False)
        half = rotary_dim // 2
        self.register_buffer("cos_half16", cos[:, 0, :half].to(torch.float16).contiguous(), persistent=False)
        self.register_buffer("sin_half16", sin[:, 0, :half].to(torch.float16).contiguous(), persistent=False)

    def _apply(self, fn, recurse=True):
        # keep the fp32 tables fp32 and the fp16 tables fp16 under model.to(dtype)
        out = super()._apply(fn, recurse)
        if self.cos_cache.dtype != torch.float32:
            self.cos_cache = self.cos_cache.float()
            self.sin_cache = self.sin_cache.float()
        if self.cos_half16.dtype != torch.float16:
            self.cos_half16 = self.cos_half16.half()
            self.sin_half16 = self.sin_half16.half()
        return out

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor
                ) -> tuple[torch.Tensor, torch.Tensor]:
        """q [T, Hq, D], k [T, Hkv, D] fp16 -> rotated (q, k), via the fused prologue kernel."""
        T, Hq, D = query.shape[0], query.shape[-2], query.shape[-1]
        Hkv = key.shape[-2]
        q2 = query.reshape(T, Hq * D)
        k2 = key.reshape(T, Hkv * D)
        packed = torch.cat([q2, k2, k2], dim=1).contiguous()
        q, k, _ = kernels.qkv_post(packed, Hq, Hkv, D, positions.contiguous(), self.cos_half16, self.sin_half16,
                                   None, None, 0.0, want_kv=True)
        return q.view(query.shape), k.view(key.shape)


_ROPE_CACHE: dict = {}


def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float) -> RotaryEmbedding:
    key = (head_size, rotary_dim, max_position, base)
    if key not in _ROPE_CACHE:
        _ROPE_CACHE[key] = RotaryEmbedding(head_size, rotary_dim, max_position, base)
    return _ROPE_CACHE[key]
