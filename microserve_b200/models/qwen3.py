"""Qwen3 decoder (microserve/models/qwen3.py), tensor-parallel, with a fused
FP8 forward.

Module tree, parameter names and `packed_modules_mapping` are the
reference's, so checkpoints load the same way. Two forwards exist:

* the module path (each submodule's forward, like the reference), used when
  the linears are not FP8-quantised;
* the fused FP8 path (Qwen3DecoderLayer.forward_fp8), used once
  quantize_fp8_linears() ran and the KV cache is FP8. Per layer it launches:
    1. (residual +) RMSNorm -> FP8 rows              (input_layernorm + qkv act quant)
    2. FP8 GEMM  qkv                                  (qkv_proj)
    3. q/k RMSNorm + RoPE + FP8 KV store              (qwen3.py:49-53, attention.py:41-43)
    4. attention (decode / prefill / chunk)           (attention.py:44-60)
    5. FP8 row quant of o + FP8 GEMM o_proj
    6. residual + RMSNorm -> FP8 rows                 (post_attention_layernorm + act quant)
    7. FP8 GEMM gate_up
    8. SiLU*mul -> FP8 rows                           (act_fn + down_proj act quant)
    9. FP8 GEMM down_proj
  With tensor parallelism over peer memory, 5+6 and 9+(the next layer's 1, or
  the final norm) are each ONE kernel: the row-parallel GEMM pushes its output
  rows to the ranks that own them and then sums, adds, normalises and gathers
  (Qwen3DecoderLayer.forward_tp).
  Every intermediate rounding matches the reference's module path: each
  fused FP8 producer quantises exactly the fp16 tensor the reference would
  have materialised and then quantised.
"""
import torch
from torch import nn

from microserve_b200 import kernels
from microserve_b200.layers.activation import SiluAndMul
from microserve_b200.layers.attention import Attention
from microserve_b200.layers.embed_head import ParallelLMHead, VocabParallelEmbedding
from microserve_b200.layers.fp8_linear import FP8DynamicLinear
from microserve_b200.layers.layernorm import RMSNorm
from microserve_b200.layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
from microserve_b200.layers.rotary_embedding import get_rope
from microserve_b200.utils import dist as tp
from microserve_b200.utils.context import AttentionMode, get_context


def tp_quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """FP8 rows of a row-parallel linear's input (the attention output for o_proj,
    SiLU*mul for down_proj), which is sharded along K under tensor parallelism.
    The reference scales each row by its amax over the FULL K
    (microserve/layers/fp8_linear.py:20). By default each rank scales its shard
    by the shard's own amax (no communication; equal to the reference at TP=1).
    With exact activation scales (utils.dist.set_exact_act_scale) the ranks
    all-reduce the row amax (max of M floats) first, so every code equals the
    single-GPU code."""
    if tp.tp_size() == 1 or not tp.exact_act_scale():
        return kernels.quantize_rows_fp8(x)
    amax = tp.all_reduce_max_(kernels.row_amax(x))
    return kernels.quantize_rows_fp8_amax(x, amax)


class Qwen3Attention(nn.Module):
    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, max_position: int,
                 head_dim: int | None = None, rms_norm_eps: float = 1e-6, qkv_bias: bool = False,
                 rope_theta: float = 1000000.0, fused_rmsnorm: bool = True) -> None:
        super().__init__()
        size = tp.tp_size()
        self.total_num_heads = num_heads
        self.total_num_kv_heads = num_kv_heads
        self.num_heads = num_heads // size
        self.num_kv_heads = num_kv_heads // size
        self.head_dim = head_dim or hidden_size // num_heads
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.scaling = self.head_dim ** -0.5
        self.rms_norm_eps = rms_norm_eps
        self.qkv_proj = QKVParallelLinear(hidden_size, self.head_dim, num_heads, num_kv_heads, bias=qkv_bias)
        self.o_proj = RowParallelLinear(num_heads * self.head_dim, hidden_size, bias=False)
        self.rotary_emb = get_rope(self.head_dim, self.head_dim, max_position, rope_theta)
        self.attn = Attention(self.num_heads, self.head_dim, self.scaling, self.num_kv_heads)
        self.has_qk_norm = not qkv_bias
        if not qkv_bias:
            self.q_norm = RMSNorm(self.head_dim, eps=rms_norm_eps, use_triton=fused_rmsnorm)
            self.k_norm = RMSNorm(self.head_dim, eps=rms_norm_eps, use_triton=fused_rmsnorm)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
        qkv = self.qkv_proj(hidden_states)
        q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
        q = q.reshape(-1, self.num_heads, self.head_dim)
        k = k.reshape(-1, self.num_kv_heads, self.head_dim)
        v = v.reshape(-1, self.num_kv_heads, self.head_dim)
        if self.has_qk_norm:
            q = self.q_norm(q)
            k = self.k_norm(k)
        q, k = self.rotary_emb(positions, q, k)
        o = self.attn(q, k, v)
        return self.o_proj(o.reshape(-1, self.num_heads * self.head_dim))

    def forward_fp8(self, positions: torch.Tensor, xq: torch.Tensor, sx: torch.Tensor, tpf=None, norm=None,
                    residual: torch.Tensor | None = None):
        """Fused FP8 path; xq/sx are the FP8 rows of the normed hidden states. With
        tpf (tensor parallel, utils.tp_fused.TpFused) o_proj is one kernel with the
        all-reduce, the residual add and `norm` (the post-attention RMSNorm): it
        returns the FP8 rows (xq, sx) of the next input instead of o_proj's output."""
        ctx = get_context()
        attn = self.attn
        qkv = self.qkv_proj.forward_fp8(xq, sx)
        want_kv = ctx.mode is AttentionMode.PREFILL
        q, k, v = kernels.qkv_post(
            qkv, self.num_heads, self.num_kv_heads, self.head_dim, positions, self.rotary_emb.cos_half16,
            self.rotary_emb.sin_half16, self.q_norm.weight if self.has_qk_norm else None,
            self.k_norm.weight if self.has_qk_norm else None, self.rms_norm_eps, ctx.slot_mapping,
            (attn.k_cache, attn.v_cache, attn.k_scale_cache, attn.v_scale_cache), want_kv=want_kv)
        o = attn.forward_cached(q, k, v)
        oq, so = tp_quantize_rows(o.view(-1, self.q_size))
        if tpf is not None:
            return tpf.rowpar_gemm_norm(oq, so, self.o_proj.weight_fp8, self.o_proj.weight_scale, residual,
                                        norm.weight, norm.eps)
        return self.o_proj.forward_fp8(oq, so)


class Qwen3MLP(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int, hidden_act: str) -> None:
        super().__init__()
        self.gate_up_proj = MergedColumnParallelLinear(hidden_size, [intermediate_size] * 2, bias=False)
        self.down_proj = RowParallelLinear(intermediate_size, hidden_size, bias=False)
        assert hidden_act == "silu"
        self.act_fn = SiluAndMul()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(self.act_fn(self.gate_up_proj(x)))

    def forward_fp8(self, xq: torch.Tensor, sx: torch.Tensor, tpf=None, norm=None,
                    residual: torch.Tensor | None = None, want_fp16: bool = False):
        """With tpf (tensor parallel) down_proj is one kernel with the all-reduce, the
        residual add and `norm` (the next layer's input RMSNorm or the final norm): it
        returns the next FP8 rows (xq, sx), or with want_fp16 the normalised fp16 rows."""
        gu = self.gate_up_proj.forward_fp8(xq, sx)
        if tp.exact_act_scale():
            a, _, _ = kernels.silu_mul(gu, want_fp16=True, want_fp8=False)
            aq, sa = tp_quantize_rows(a)
        else:
            aq, sa = self.act_fn.forward_fp8(gu)
        if tpf is not None:
            return tpf.rowpar_gemm_norm(aq, sa, self.down_proj.weight_fp8, self.down_proj.weight_scale, residual,
                                        norm.weight, norm.eps, want_fp16=want_fp16)
        return self.down_proj.forward_fp8(aq, sa)


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, config) -> None:
        super().__init__()
        fused = getattr(config, "_microserve_fused_rmsnorm", True)
        self.self_attn = Qwen3Attention(
            hidden_size=config.hidden_size,
            num_heads=config.num_attention_heads,
            num_kv_heads=config.num_key_value_heads,
            max_position=config.max_position_embeddings,
            rms_norm_eps=config.rms_norm_eps,
            qkv_bias=getattr(config, "attention_bias", False),
            head_dim=getattr(config, "head_dim", None),
            rope_theta=getattr(config, "rope_theta", 1000000.0),
            fused_rmsnorm=fused,
        )
        self.mlp = Qwen3MLP(hidden_size=config.hidden_size, intermediate_size=config.intermediate_size,
                            hidden_act=config.hidden_act)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps, use_triton=fused)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps, use_triton=fused)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor,
                residual: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
        if residual is None:
            hidden_states, residual = self.input_layernorm(hidden_states), hidden_states
        else:
            hidden_states, residual = self.input_layernorm(hidden_states, residual)
        hidden_states = self.self_attn(positions, hidden_states)
        hidden_states, residual = self.post_attention_layernorm(hidden_states, residual)
        hidden_states = self.mlp(hidden_states)
        return hidden_states, residual

    def forward_fp8(self, positions: torch.Tensor, hidden_states: torch.Tensor,
                    residual: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
        """Fused FP8 layer (one GPU, or tensor parallel with NCCL all-reduces)."""
        if residual is None:
            xq, sx, _ = self.input_layernorm.forward_fp8(hidden_states)
            residual = hidden_states
        else:
            xq, sx, residual = self.input_layernorm.forward_fp8(hidden_states, residual)
        h = self.self_attn.forward_fp8(positions, xq, sx)
        xq, sx, residual = self.post_attention_layernorm.forward_fp8(h, residual)
        return self.mlp.forward_fp8(xq, sx), residual

    def forward_tp(self, positions: torch.Tensor, xq: torch.Tensor, sx: torch.Tensor, residual: torch.Tensor,
                   tpf, next_norm, final: bool):
        """Fused FP8 layer, tensor parallel over peer memory (utils.tp_fused.TpFused):
        xq/sx are this layer's normalised input rows; o_proj and down_proj each run as
        one kernel with the all-reduce, the residual add (this rank's rows of
        `residual`, updated in place) and the norm that follows them - the
        post-attention norm, then `next_norm` (the next layer's input norm, or the
        final norm when `final`, which returns fp16 rows instead of FP8 ones)."""
        xq, sx = self.self_attn.forward_fp8(positions, xq, sx, tpf=tpf, norm=self.post_attention_layernorm,
                                            residual=residual)
        return self.mlp.forward_fp8(xq, sx, tpf=tpf, norm=next_norm, residual=residual, want_fp16=final)


class Qwen3Model(nn.Module):
    def __init__(self, config) -> None:
        super().__init__()
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def _fp8_ready(self) -> bool:
        a = self.layers[0].self_attn
        return isinstance(a.qkv_proj, FP8DynamicLinear) and a.attn.kv_cache_dtype == "fp8_e4m3"

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        hidden_states = self.embed_tokens(input_ids)
        fused = self._fp8_ready()
        tpf = getattr(self, "tp_fused", None) if fused else None
        if tpf is not None:
            # tensor parallel: the embedding rows are complete on every rank; from there on
            # each row-parallel linear carries the all-reduce and the norm after it
            residual = hidden_states
            xq, sx, _ = self.layers[0].input_layernorm.forward_fp8(hidden_states)
            last = len(self.layers) - 1
            for i, layer in enumerate(self.layers):
                nxt = self.norm if i == last else self.layers[i + 1].input_layernorm
                out = layer.forward_tp(positions, xq, sx, residual, tpf, nxt, final=(i == last))
                if i < last:
                    xq, sx = out
            return out
        residual = None
        for layer in self.layers:
            if fused:
                hidden_states, residual = layer.forward_fp8(positions, hidden_states, residual)
            else:
                hidden_states, residual = layer(positions, hidden_states, residual)
        return self.norm(hidden_states, residual)[0]


class Qwen3ForCausalLM(nn.Module):
    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", 0),
        "up_proj": ("gate_up_proj", 1),
    }

    def __init__(self, config, fused_rmsnorm: bool = True) -> None:
        super().__init__()
        config._microserve_fused_rmsnorm = fused_rmsnorm
        self.config = config
        self.model = Qwen3Model(config)
        self.lm_head = ParallelLMHead(config.vocab_size, config.hidden_size)
        if getattr(config, "tie_word_embeddings", False):
            self.lm_head.weight.data = self.model.embed_tokens.weight.data

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids, positions)

    def compute_logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return self.lm_head(hidden_states)
