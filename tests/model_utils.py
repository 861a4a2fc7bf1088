"""Helpers shared by the model-level tests: small Qwen3 configs and an oracle
forward (CPU) that reads the GPU model's own FP8 weights."""
from __future__ import annotations

import torch

from oracle import fp8_decoder as O


def qwen3_config(layers=2, hidden=1024, heads=16, kv_heads=8, inter=3072, vocab=4096, max_pos=40960, tie=True):
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
                       num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=128,
                       max_position_embeddings=max_pos, rms_norm_eps=1e-6, tie_word_embeddings=tie,
                       hidden_act="silu", attention_bias=False)


class OracleModel:
    """CPU restatement of Qwen3ForCausalLM's FP8 forward with its own FP8 KV cache."""

    def __init__(self, model, num_blocks: int, block_size: int = 256):
        cfg = model.config
        self.Hq, self.Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.Hq
        self.eps = cfg.rms_norm_eps
        self.embed = model.model.embed_tokens.weight.detach().cpu()
        self.lm_head = model.lm_head.weight.detach().cpu()
        self.final_norm = model.model.norm.weight.detach().cpu()
        self.layers = []
        for layer in model.model.layers:
            a, m = layer.self_attn, layer.mlp

            def wp(lin):
                return lin.weight_fp8.detach().cpu(), lin.weight_scale.detach().cpu()
            self.layers.append(O.LayerWeights(wp(a.qkv_proj), wp(a.o_proj), wp(m.gate_up_proj), wp(m.down_proj),
                                              layer.input_layernorm.weight.detach().cpu(),
                                              layer.post_attention_layernorm.weight.detach().cpu(),
                                              a.q_norm.weight.detach().cpu(), a.k_norm.weight.detach().cpu()))
        self.cos, self.sin = O.rope_tables(self.D, cfg.max_position_embeddings, getattr(cfg, "rope_theta", 1e6))
        self.block_size = block_size
        shape = (num_blocks + 1, block_size, self.Hkv, self.D)
        self.caches = [[torch.zeros(shape, dtype=torch.float8_e4m3fn), torch.zeros(shape, dtype=torch.float8_e4m3fn),
                        torch.ones(shape[:-1]), torch.ones(shape[:-1])] for _ in self.layers]

    def forward(self, ids, positions, mode, slots, **kw):
        h = torch.nn.functional.embedding(ids, self.embed)
        residual = None
        for lw, caches in zip(self.layers, self.caches):
            h, residual = O.decoder_layer(lw, positions, h, residual, Hq=self.Hq, Hkv=self.Hkv, D=self.D,
                                          eps=self.eps, cos_cache=self.cos, sin_cache=self.sin, mode=mode,
                                          caches=caches, slots=slots, **kw)
        return O.rmsnorm(h, self.final_norm, self.eps, residual)[0]

    def logits(self, hidden):
        return (hidden.float() @ self.lm_head.float().T).half()
