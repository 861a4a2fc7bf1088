"""Engine configuration: the reference's fields and checks
(microserve/Config.py:4-38) plus
  tensor_parallel_size - GPUs per model replica (one process per GPU, group
                         set up by the launcher, see utils/dist.py);
  tp_fused_collective  - with tensor parallelism on the FP8 path, sum the
                         row-parallel outputs with this library's peer-memory
                         kernel fused with add + RMSNorm + FP8 quantisation
                         (utils/tp_fused.py) instead of NCCL all-reduce;
  tp_fused_gemm        - with the fused collective: each row-parallel GEMM
                         pushes its rows to their owners and does the
                         reduce / norm itself (one kernel); False: the GEMM
                         writes its partial locally and a second kernel does
                         the rest;
  tp_exact_act_scale   - with tensor parallelism, scale each row-parallel
                         input row (o_proj, down_proj) by its amax over the
                         full row, as a single GPU does (one all-reduce max of
                         a float per row), instead of the local shard's amax;
  gemm_pair_tiles      - on one GPU, let the FP8 / fp16 GEMMs use tiles on
                         pairs of SMs (tcgen05 cta_group::2) where they are
                         faster (129..256 tokens, prefill);
  load_format          - "safetensors" (model_dir holds the checkpoint) or
                         "dummy" (seeded N(0, 0.02) random weights of the
                         shape in model_dir/config.json or `hf_config`);
  hf_config            - a transformers config object used instead of
                         reading model_dir/config.json.
The FP8 e4m3 KV cache is the only cache this engine implements, so it is the
default here; fp16 activations are required by the FP8 path (as in the
reference).
"""
import os
from dataclasses import dataclass, field

import torch


@dataclass
class Config:
    model_dir: str = "~/huggingface/Qwen3-0.6B"
    block_size: int = 256
    num_kvcache_blocks: int = 0
    gpu_memory_utilization: float = 0.90
    max_num_seqs: int = 32
    max_num_batched_tokens: int = 4096
    max_model_len: int = 4096
    eos_token_id: int | None = None
    dtype: torch.dtype = field(default=torch.float16)
    seed: int = 0
    enforce_eager: bool = False
    fused_rmsnorm: bool = True
    quantization: str | None = "fp8_dynamic"
    kv_cache_dtype: str = "fp8_e4m3"
    scheduler_policy: str = "mixed"
    tensor_parallel_size: int = 1
    tp_fused_collective: bool = True
    tp_fused_gemm: bool = False
    tp_exact_act_scale: bool = False
    gemm_pair_tiles: bool = False
    load_format: str = "safetensors"
    hf_config: object = None

    def __post_init__(self):
        self.model_dir = os.path.expanduser(self.model_dir)
        assert self.block_size > 0 and self.block_size % 256 == 0, "block_size must be a multiple of 256"
        assert 0 < self.gpu_memory_utilization <= 1.0
        assert self.quantization in (None, "fp8_dynamic"), "unsupported quantization"
        assert self.kv_cache_dtype in ("fp16", "fp8_e4m3"), "unsupported KV cache dtype"
        if self.kv_cache_dtype == "fp8_e4m3":
            assert self.dtype == torch.float16, "FP8 KV cache currently requires FP16 model dtype"
        assert self.scheduler_policy in ("mixed", "prefill_first"), "unsupported scheduler policy"
        assert self.tensor_parallel_size >= 1
        assert self.load_format in ("safetensors", "dummy"), "unsupported load_format"
