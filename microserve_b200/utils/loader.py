"""Checkpoint loading through the layers' weight_loader hooks
(microserve/utils/loader.py:11-29), plus seeded random ("dummy") weights.

Dummy weights are generated per parameter from a generator seeded with
(seed, parameter name), at the FULL (unsharded) checkpoint shape, and pass
through the same weight_loader hooks as real checkpoint tensors, so every
tensor-parallel size sees the same model. Linear and embedding weights are
N(0, 0.02); RMSNorm weights keep their init of 1.
"""
from __future__ import annotations

import os
import zlib
from glob import glob

import torch
from torch import nn


def default_weight_loader(param: nn.Parameter, loaded_weight: torch.Tensor):
    param.data.copy_(loaded_weight)


def _route(model: nn.Module, weight_name: str):
    """(param, shard_id | None) for a checkpoint tensor name."""
    for packed_name, (param_name, shard_id) in getattr(model, "packed_modules_mapping", {}).items():
        if packed_name in weight_name:
            return model.get_parameter(weight_name.replace(packed_name, param_name)), shard_id
    return model.get_parameter(weight_name), None


def _load_one(model: nn.Module, name: str, tensor: torch.Tensor) -> None:
    param, shard_id = _route(model, name)
    loader = getattr(param, "weight_loader", default_weight_loader)
    if shard_id is None:
        loader(param, tensor)
    else:
        loader(param, tensor, shard_id)


def load_model(model: nn.Module, path: str) -> None:
    from safetensors import safe_open
    files = sorted(glob(os.path.join(path, "*.safetensors")))
    assert files, f"no safetensors found under {path}"
    for file in files:
        with safe_open(file, "pt", "cpu") as f:
            for weight_name in f.keys():
                _load_one(model, weight_name, f.get_tensor(weight_name))


def checkpoint_shapes(cfg) -> dict[str, tuple[int, ...]]:
    """Checkpoint tensor names and full shapes of a Qwen3 config (HF naming)."""
    h, V, I = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size
    D = getattr(cfg, "head_dim", None) or h // cfg.num_attention_heads
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    out: dict[str, tuple[int, ...]] = {"model.embed_tokens.weight": (V, h), "model.norm.weight": (h,)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        out.update({
            p + "self_attn.q_proj.weight": (Hq * D, h),
            p + "self_attn.k_proj.weight": (Hkv * D, h),
            p + "self_attn.v_proj.weight": (Hkv * D, h),
            p + "self_attn.o_proj.weight": (h, Hq * D),
            p + "self_attn.q_norm.weight": (D,),
            p + "self_attn.k_norm.weight": (D,),
            p + "mlp.gate_proj.weight": (I, h),
            p + "mlp.up_proj.weight": (I, h),
            p + "mlp.down_proj.weight": (h, I),
            p + "input_layernorm.weight": (h,),
            p + "post_attention_layernorm.weight": (h,),
        })
    if not getattr(cfg, "tie_word_embeddings", False):
        out["lm_head.weight"] = (V, h)
    return out


def dummy_tensor(name: str, shape: tuple[int, ...], seed: int, device, dtype=torch.float16) -> torch.Tensor:
    if len(shape) == 1:  # norm weights
        return torch.ones(shape, dtype=dtype, device=device)
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF)
    return torch.empty(shape, dtype=torch.float32, device=device).normal_(0.0, 0.02, generator=g).to(dtype)


def load_dummy(model: nn.Module, cfg, seed: int, device) -> None:
    for name, shape in checkpoint_shapes(cfg).items():
        _load_one(model, name, dummy_tensor(name, shape, seed, device))
