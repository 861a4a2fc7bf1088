"""SiLU-and-mul (microserve/layers/activation.py:5-8): silu(x[:, :I]) * x[:, I:]."""
import torch
from torch import nn

from microserve_b200 import kernels


class SiluAndMul(nn.Module):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != torch.float16 or not x.is_cuda:
            raise ValueError("SiluAndMul requires CUDA FP16 input")
        out, _, _ = kernels.silu_mul(x)
        return out.view(*x.shape[:-1], x.shape[-1] // 2)

    def forward_fp8(self, x: torch.Tensor):
        """Returns (aq e4m3, sa fp32): the FP8 rows of silu(gate) * up."""
        _, aq, sa = kernels.silu_mul(x, want_fp16=False, want_fp8=True)
        return aq, sa
