"""CPU oracle for the FP8 decoder-layer path - TEST INFRASTRUCTURE ONLY.

A plain-PyTorch (CPU, fp16 storage / fp32 math) restatement of the
reference's FP8 path, used by tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / --impl reference legs as the checker. The product path
(microserve_b200) never imports this module.

Each function cites the reference lines it restates (gssg1/microserve,
path:line). The FP8 formulas are those of the reference's Triton kernels,
written the way the reference's own tests restate them (tests/test_fp8.py:25-28,
tests/test_fp8_kv_attention.py:30-36,63-70,96-105).

Pinning: tests/golden/ holds vectors produced by running the reference
itself - its CPU-runnable modules in this container (make_golden.py) and its
Triton kernels on a B200 (make_golden_gpu.py) - and tests/test_oracle_cpu.py
and tests/test_reference_golden.py check this module against them.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

FP8_MAX = 448.0
E4M3 = torch.float8_e4m3fn
# The reference writes `max(amax, 1e-8) / 448`, but both places that evaluate it on the GPU
# (its Triton kernels and torch's CUDA tensor-by-scalar division) multiply by the fp32
# reciprocal; tests/golden/reference_gpu.pt (the reference's own outputs) pins that.
INV_FP8_MAX = torch.tensor(1.0 / FP8_MAX, dtype=torch.float32)


def fp8_scale(amax: torch.Tensor) -> torch.Tensor:
    """Per-row scale of the reference's FP8 encode (fp8_linear.py:20, :52; fp8_kv_cache.py:34-35)."""
    return amax.float().clamp_min(1e-8) * INV_FP8_MAX


# ---------------------------------------------------------------- FP8 linear
def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row dynamic quant (microserve/layers/fp8_linear.py:14-23)."""
    xf = x.float()
    s = fp8_scale(xf.abs().amax(dim=-1))
    q = (xf / s[..., None]).clamp(-FP8_MAX, FP8_MAX).to(E4M3)
    return q, s


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Offline per-output-channel weight quant (microserve/layers/fp8_linear.py:51-54)."""
    wf = w.detach().float()
    s = fp8_scale(wf.abs().amax(dim=1))
    q = (wf / s[:, None]).clamp(-FP8_MAX, FP8_MAX).to(E4M3)
    return q, s


def fp8_gemm(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
             bias: torch.Tensor | None = None) -> torch.Tensor:
    """(Xq . Wq^T) * sx * sw -> fp16 (microserve/layers/fp8_linear.py:40-45, tests/test_fp8.py:27-28)."""
    y = (F.linear(xq.float(), wq.float()) * sx[:, None] * sw[None, :]).half()
    if bias is not None:
        y = y + bias.half()
    return y


def fp8_linear(x: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, bias=None) -> torch.Tensor:
    """FP8DynamicLinear.forward (microserve/layers/fp8_linear.py:64-80)."""
    xq, sx = quantize_rows(x.reshape(-1, x.shape[-1]))
    return fp8_gemm(xq, sx, wq, sw, bias).view(*x.shape[:-1], wq.shape[0])


# ------------------------------------------------------------- elementwise
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """RMSNorm torch path (microserve/layers/layernorm.py:55-57, 82-85)."""
    def norm(v):
        var = v.float().pow(2).mean(dim=-1, keepdim=True)
        return v * torch.rsqrt(var + eps)
    if residual is None:
        return norm(x.float()).to(x.dtype) * w
    y = (x.float() + residual.float()).to(x.dtype)
    return norm(y.float()).to(y.dtype) * w, y


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    """SiluAndMul (microserve/layers/activation.py:5-8)."""
    a, b = x.chunk(2, -1)
    return F.silu(a) * b


def rope_tables(head_dim: int, max_position: int, base: float) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin caches [max_pos, 1, D] fp32 (microserve/layers/rotary_embedding.py:13-20)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().unsqueeze_(1), emb.sin().unsqueeze_(1)


def _rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def rope(positions, q, k, cos_cache, sin_cache):
    """RotaryEmbedding.forward (microserve/layers/rotary_embedding.py:24-31)."""
    cos = cos_cache[positions].to(q.dtype)
    sin = sin_cache[positions].to(q.dtype)
    return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


# ------------------------------------------------------------- FP8 KV cache
def store_kv(k, v, k_cache, v_cache, k_scale, v_scale, slots) -> None:
    """store_fp8_kvcache (microserve/layers/fp8_kv_cache.py:24-39): per (token, head)
    scale = max(amax_d, 1e-8)*fl32(1/448), codes = e4m3(clamp(x/scale)), scattered to slot."""
    bs = k_cache.shape[1]
    for src, cache, sc in ((k, k_cache, k_scale), (v, v_cache, v_scale)):
        xf = src.float()
        s = fp8_scale(xf.abs().amax(dim=-1))
        q = (xf / s[..., None]).clamp(-FP8_MAX, FP8_MAX).to(E4M3)
        blk, off = slots // bs, slots % bs
        cache[blk, off] = q
        sc[blk, off] = s


def gather_kv(cache, scale, table, length):
    """Dequantised [length, Hkv, D] fp32 rows of one sequence (tests/test_fp8_kv_attention.py:30-36)."""
    bs = cache.shape[1]
    pos = torch.arange(length)
    blk = table[pos // bs].long()
    off = pos % bs
    return cache[blk, off].float() * scale[blk, off][..., None]


def decode_attention(q, k_cache, v_cache, k_scale, v_scale, seqlens, block_tables, sm_scale):
    """fp8_decode_attention reference math (tests/test_fp8_kv_attention.py:63-70); 0 for empty rows
    (microserve/layers/fp8_decode_attention.py:58)."""
    B, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    head_map = torch.arange(Hq) // (Hq // Hkv)
    out = torch.zeros(B, Hq, D, dtype=torch.float32)
    for b in range(B):
        L = int(seqlens[b])
        if L == 0:
            continue
        kk = gather_kv(k_cache, k_scale, block_tables[b], L)[:, head_map]
        vv = gather_kv(v_cache, v_scale, block_tables[b], L)[:, head_map]
        s = torch.einsum("hd,lhd->hl", q[b].float(), kk) * sm_scale
        out[b] = torch.einsum("hl,lhd->hd", s.softmax(-1), vv)
    return out.half()


def decode_attention_grouped(q, k_cache, v_cache, k_scale, v_scale, seqlens, block_tables, sm_scale):
    """decode_attention with the q heads of each kv head grouped instead of K/V copied
    per q head (the same math, about twice as fast on the host cores; used where the
    oracle is timed, pinned to decode_attention by tests/test_oracle_cpu.py)."""
    B, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    G = Hq // Hkv
    out = torch.zeros(B, Hq, D, dtype=torch.float32)
    for b in range(B):
        L = int(seqlens[b])
        if L == 0:
            continue
        kk = gather_kv(k_cache, k_scale, block_tables[b], L)
        vv = gather_kv(v_cache, v_scale, block_tables[b], L)
        s = torch.einsum("hgd,lhd->hgl", q[b].float().view(Hkv, G, D), kk) * sm_scale
        out[b] = torch.einsum("hgl,lhd->hgd", s.softmax(-1), vv).reshape(Hq, D)
    return out.half()


def chunk_prefill_attention(q, k_cache, v_cache, k_scale, v_scale, table, prefix_len, sm_scale):
    """Single-sequence causal chunk attention over the cache
    (tests/test_fp8_kv_attention.py:96-105; kernel microserve/layers/fp8_chunk_prefill_attention.py:8-67)."""
    Q, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    head_map = torch.arange(Hq) // (Hq // Hkv)
    total = prefix_len + Q
    kk = gather_kv(k_cache, k_scale, table, total)[:, head_map]
    vv = gather_kv(v_cache, v_scale, table, total)[:, head_map]
    s = torch.einsum("qhd,lhd->hql", q.float(), kk) * sm_scale
    vis = torch.arange(total)[None, :] <= (prefix_len + torch.arange(Q))[:, None]
    s = s.masked_fill(~vis[None], float("-inf"))
    return torch.einsum("hql,lhd->qhd", s.softmax(-1), vv).half()


def varlen_prefill(q, k, v, cu, sm_scale):
    """Causal attention per sequence on fresh fp16 q, k, v (the FP8-KV PREFILL branch,
    microserve/layers/attention.py:49-55: flash_attn_varlen_func, causal=True)."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    head_map = torch.arange(Hq) // (Hq // Hkv)
    out = torch.zeros(T, Hq, D, dtype=torch.float32)
    for s0, s1 in zip(cu[:-1].tolist(), cu[1:].tolist()):
        n = s1 - s0
        qq, kk, vv = q[s0:s1].float(), k[s0:s1, head_map].float(), v[s0:s1, head_map].float()
        s = torch.einsum("qhd,khd->hqk", qq, kk) * sm_scale
        mask = torch.ones(n, n, dtype=torch.bool).tril()
        s = s.masked_fill(~mask[None], float("-inf"))
        out[s0:s1] = torch.einsum("hqk,khd->qhd", s.softmax(-1), vv)
    return out.half()


# ------------------------------------------------------------ decoder layer
class LayerWeights:
    """FP8 weights of one Qwen3 decoder layer (codes + per-channel scales) and its norms."""

    def __init__(self, qkv, o, gate_up, down, in_norm, post_norm, q_norm, k_norm):
        self.qkv, self.o, self.gate_up, self.down = qkv, o, gate_up, down  # (wq, sw) pairs
        self.in_norm, self.post_norm, self.q_norm, self.k_norm = in_norm, post_norm, q_norm, k_norm


def decoder_layer(lw: LayerWeights, positions, hidden, residual, *, Hq, Hkv, D, eps, cos_cache, sin_cache,
                  mode: str, caches, slots, seqlens=None, block_tables=None, cu=None, prefix_len=None,
                  grouped_attention: bool = False):
    """Qwen3DecoderLayer.forward with FP8 linears and the FP8 KV cache
    (microserve/models/qwen3.py:42-54,65-66,91-100; attention.py:36-61).
    mode: "decode" | "prefill" | "chunk" (chunk: one sequence, block_tables[0], prefix_len).
    grouped_attention: decode attention through decode_attention_grouped (same math)."""
    if residual is None:
        h, residual = rmsnorm(hidden, lw.in_norm, eps), hidden
    else:
        h, residual = rmsnorm(hidden, lw.in_norm, eps, residual)
    qkv = fp8_linear(h, *lw.qkv)
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    q = q.reshape(-1, Hq, D)
    k = k.reshape(-1, Hkv, D)
    v = v.reshape(-1, Hkv, D)
    q = rmsnorm(q, lw.q_norm, eps)
    k = rmsnorm(k, lw.k_norm, eps)
    q, k = rope(positions, q, k, cos_cache, sin_cache)
    kc, vc, ks, vs = caches
    store_kv(k, v, kc, vc, ks, vs, slots)
    scale = D ** -0.5
    if mode == "decode":
        attend = decode_attention_grouped if grouped_attention else decode_attention
        o = attend(q, kc, vc, ks, vs, seqlens, block_tables, scale)
    elif mode == "prefill":
        o = varlen_prefill(q, k, v, cu, scale)
    elif mode == "chunk":
        o = chunk_prefill_attention(q, kc, vc, ks, vs, block_tables[0], prefix_len, scale)
    else:
        raise RuntimeError(f"unsupported attention mode: {mode}")
    h = fp8_linear(o.reshape(-1, Hq * D), *lw.o)
    h, residual = rmsnorm(h, lw.post_norm, eps, residual)
    h = fp8_linear(silu_mul(fp8_linear(h, *lw.gate_up)), *lw.down)
    return h, residual


def slot_mapping(block_table: list[int], positions: list[int], block_size: int) -> list[int]:
    """slot = table[p // bs] * bs + p % bs (microserve/engine/model_runner.py:135-137)."""
    return [block_table[p // block_size] * block_size + p % block_size for p in positions]


def block_table_rows(tables: list[list[int]]) -> torch.Tensor:
    """int32 rows padded with -1 (microserve/engine/model_runner.py:208-216)."""
    width = max(len(t) for t in tables)
    out = torch.full((len(tables), width), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        out[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    return out


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "math", "torch", "F")]
