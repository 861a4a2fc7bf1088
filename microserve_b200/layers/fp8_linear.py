"""Dynamic FP8 e4m3 W8A8 linear (the reference's microserve/layers/fp8_linear.py).

FP8DynamicLinear(source) quantises the source weight once, per output channel
(scale = max(amax_row, 1e-8) * fl32(1/448), :49-56: the reference writes
`/ 448`, which torch evaluates on the GPU as a multiply by the fp32 reciprocal), and its forward quantises the
activation rows dynamically (:14-23) and runs the tcgen05 FP8 GEMM with the
per-row x per-channel dequant epilogue (:26-45). Weight quantisation runs on
the GPU through the library's row quantiser (the same formula).

Tensor parallelism follows the source layer's mode: column-parallel layers
hold whole rows, so their scales are the single-GPU ones; a row-parallel
layer quantises its column shard with the scale of the full row
(LinearBase.full_row_amax) and sums its partial outputs over the group.
"""
import torch
from torch import nn

from microserve_b200 import kernels
from microserve_b200.layers.linear import LinearBase
from microserve_b200.utils import dist as tp

FP8_MAX = 448.0  # largest finite value of torch.float8_e4m3fn
INV_FP8_MAX = 1.0 / FP8_MAX  # applied in fp32, as torch applies `/ 448` on the GPU


class FP8DynamicLinear(nn.Module):
    def __init__(self, source: LinearBase):
        super().__init__()
        w = source.weight.detach()
        if not w.is_cuda:
            raise ValueError("FP8DynamicLinear quantises on the GPU: move the model to CUDA first")
        w16 = w.to(torch.float16).contiguous()
        if source.full_row_amax is not None:
            scales = source.full_row_amax.float().clamp_min(1e-8) * INV_FP8_MAX
            packed = (w16.float() / scales[:, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
        elif w.dtype == torch.float16:
            packed, scales = kernels.quantize_rows_fp8(w16)
        else:  # fp32 master weights: the reference's formula on the original values
            wf = w.float()
            scales = wf.abs().amax(dim=1).clamp_min(1e-8) * INV_FP8_MAX
            packed = (wf / scales[:, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
        self.register_buffer("weight_fp8", packed.contiguous())
        self.register_buffer("weight_scale", scales.contiguous())
        if source.bias is None:
            self.register_buffer("bias", None)
        else:
            self.register_buffer("bias", source.bias.detach().to(torch.float16).clone())
        self.in_features = w.shape[1]
        self.out_features = w.shape[0]
        self.tp_mode = getattr(source, "tp_mode", "replicated")
        self.tp_rank = getattr(source, "tp_rank", 0)
        self.tp_size = getattr(source, "tp_size", 1)

    def _bias_here(self):
        # a row-parallel bias is added once, by rank 0, before the sum
        if self.bias is None or (self.tp_mode == "row" and self.tp_rank != 0):
            return None
        return self.bias

    def forward_fp8(self, xq: torch.Tensor, sx: torch.Tensor, reduce: bool = True,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """GEMM on an already-quantised activation (fused producers). A row-parallel
        layer sums its output over the group unless reduce=False (the fused
        tensor-parallel op then reads the partial from `out`)."""
        y = kernels.fp8_gemm(xq, sx, self.weight_fp8, self.weight_scale, self._bias_here(), out=out)
        if reduce and self.tp_mode == "row":
            tp.all_reduce_(y)
        return y

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != torch.float16 or not x.is_cuda:
            raise ValueError("fp8_dynamic requires CUDA FP16 input activations")
        x2 = x.reshape(-1, self.in_features)
        xq, sx = kernels.quantize_rows_fp8(x2)
        y = self.forward_fp8(xq, sx)
        return y.view(*x.shape[:-1], self.out_features)


def quantize_fp8_linears(model: nn.Module) -> int:
    """Replace every LinearBase child with an FP8DynamicLinear; return the count."""
    count = 0
    for parent in model.modules():
        for name, child in list(parent.named_children()):
            if isinstance(child, LinearBase):
                setattr(parent, name, FP8DynamicLinear(child))
                count += 1
    return count
