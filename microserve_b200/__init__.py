"""microserve-b200: B200-native (sm_100a) FP8 decoder-layer path for microserve.

Layout mirrors the reference package (microserve/):
  layers/   the operator surface (linear, FP8 linear, RMSNorm, attention, ...)
  models/   Qwen3 (module path + fused FP8 path)
  engine/   LLMEngine, scheduler, block manager, model runner (CUDA graphs)
  utils/    attention context, checkpoint loader, tensor-parallel state
  csrc/     CUDA kernels and the C ABI (include/microserve_b200.h)
  kernels.py / _lib.py   torch wrappers and the ctypes binding of the C ABI
"""
__version__ = "0.1.0"
