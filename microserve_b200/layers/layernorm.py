"""RMSNorm with the reference's interface (microserve/layers/layernorm.py:44-85).

forward(x) -> y and forward(x, residual) -> (y, residual') with
residual' = fp16(x + residual) and y = fp16(fp16(v * rsqrt(mean(v^2) + eps)) * w),
computed by the library's row kernel for every input (strided inputs are
made contiguous first; the norm is per row). `use_triton` is accepted for
signature compatibility and ignored: there is one implementation.
forward_fp8 additionally emits the FP8 rows (and scales) of y for the next
FP8 GEMM, which is what the fused decoder layer uses.
"""
import torch
from torch import nn

from microserve_b200 import kernels


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6, use_triton: bool = True) -> None:
        super().__init__()
        self.eps = eps
        self.use_triton = use_triton
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None
                ) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
        if x.dtype != torch.float16 or not x.is_cuda:
            raise ValueError("RMSNorm requires CUDA FP16 input")
        y, _, _, r = kernels.rmsnorm(x, self.weight, self.eps, residual)
        if residual is None:
            return y.view(x.shape)
        return y.view(x.shape), r.view(x.shape)

    def forward_fp8(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        """Returns (yq [M, H] e4m3, sy [M] fp32, residual' or None)."""
        _, yq, sy, r = kernels.rmsnorm(x, self.weight, self.eps, residual, want_fp16=False, want_fp8=True)
        return yq, sy, r
