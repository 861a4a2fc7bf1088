"""The model-level parity cases: seeded synthetic Qwen3 checkpoints and prompts
that both the reference's engine (tests/golden/make_golden_engine.py, run once on
a B200) and this repository's engine (tests/test_engine_reference_gpu.py) load
and run greedily. Everything is regenerated from seeds, so only the reference's
outputs are stored (tests/golden/reference_engine.pt).

Cases:
  "small"  3 decoder layers of Qwen3-0.6B shape (hidden 1024, 16 q / 8 kv heads,
           head_dim 128, MLP 3072), vocabulary 8192, tied embeddings - logits of
           every step are stored;
  "0.6b"   the full Qwen3-0.6B shape of BASELINE config 2 (28 layers, vocabulary
           151936, tied embeddings) - greedy tokens only.
Weights: N(0, 0.02) for linears and embeddings, 1 for RMSNorm weights (the
workload's synthetic initialisation), fp16, generated per tensor from
(seed, name) by microserve_b200.utils.loader.dummy_tensor on the GPU.
"""
from __future__ import annotations

import os
import random

CASES = {
    "small": dict(layers=3, vocab=8192, prompt_lens=(37, 100, 250, 300), steps=32, logits=True),
    "0.6b": dict(layers=28, vocab=151936, prompt_lens=(37, 100, 250, 300), steps=32, logits=False),
}
SEED = 0


def hf_config(case: str):
    from transformers import Qwen3Config
    c = CASES[case]
    return Qwen3Config(vocab_size=c["vocab"], hidden_size=1024, intermediate_size=3072,
                       num_hidden_layers=c["layers"], num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                       max_position_embeddings=40960, rms_norm_eps=1e-6, tie_word_embeddings=True,
                       hidden_act="silu", attention_bias=False, torch_dtype="float16")


def write_checkpoint(case: str, path: str) -> str:
    """config.json + model.safetensors of the case under `path` (created); returns path."""
    import torch
    from safetensors.torch import save_file
    from microserve_b200.utils.loader import checkpoint_shapes, dummy_tensor
    os.makedirs(path, exist_ok=True)
    cfg = hf_config(case)
    cfg.save_pretrained(path)
    # generated on the GPU when there is one (the fixture maker and the GPU tests run on
    # the same B200 image, so the same Philox streams), else on the host
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    tensors = {name: dummy_tensor(name, shape, SEED, dev).cpu().contiguous()
               for name, shape in checkpoint_shapes(cfg).items()}
    # The tied head is written out as its own tensor: the reference converts its
    # model with .to(dtype) after tying (microserve/engine/model_runner.py:56-57),
    # which gives lm_head its own storage, so a checkpoint without lm_head.weight
    # leaves the reference's head uninitialised. Both engines load it from here.
    if cfg.tie_word_embeddings:
        tensors["lm_head.weight"] = tensors["model.embed_tokens.weight"].clone()
    save_file(tensors, os.path.join(path, "model.safetensors"))
    del tensors
    torch.cuda.empty_cache() if torch.cuda.is_available() else None
    return path


def prompts(case: str) -> list[list[int]]:
    c = CASES[case]
    rng = random.Random(1234)
    return [[rng.randrange(100, c["vocab"]) for _ in range(n)] for n in c["prompt_lens"]]


ENGINE_KW = dict(max_num_seqs=8, max_num_batched_tokens=1024, max_model_len=2048, num_kvcache_blocks=32,
                 quantization="fp8_dynamic", kv_cache_dtype="fp8_e4m3")
