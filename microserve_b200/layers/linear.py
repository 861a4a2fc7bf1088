"""Linear layers with the reference's names, constructors and weight loaders
(microserve/layers/linear.py:5-77), made tensor-parallel.

With tp_size == 1 every class holds the full [out, in] weight exactly as the
reference does. With tp_size == t:
  * QKVParallelLinear / MergedColumnParallelLinear shard the output rows
    (q/k/v heads, gate/up rows) - column parallel, no communication;
  * RowParallelLinear shards the input columns and sums partial outputs over
    the group (the FP8 path fuses that sum into its GEMM epilogue);
  * ReplicatedLinear keeps everything.
Each loader receives the full checkpoint tensor and keeps its own shard.
RowParallelLinear also records the per-output-channel amax over the FULL
input width, so the FP8 per-channel weight scale equals the single-GPU one
(microserve/layers/fp8_linear.py:51-52 computes it over the whole row).

The unquantised forward is a plain fp16 F.linear; the serving path is the
FP8 one (fp8_linear.FP8DynamicLinear).
"""
import torch
import torch.nn.functional as F
from torch import nn

from microserve_b200.utils import dist as tp


class LinearBase(nn.Module):
    tp_mode = "replicated"  # "replicated" | "column" | "row"

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__()
        self.input_size = input_size
        self.output_size = output_size
        self.tp_rank = tp.tp_rank()
        self.tp_size = tp.tp_size()
        in_local, out_local = self._local_shape(input_size, output_size)
        self.weight = nn.Parameter(torch.empty(out_local, in_local))
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(out_local))
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)
        self.full_row_amax: torch.Tensor | None = None

    def _local_shape(self, input_size: int, output_size: int) -> tuple[int, int]:
        return input_size, output_size

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param.data.copy_(loaded_weight)

    def reset_parameters(self):
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight, self.bias)


class ReplicatedLinear(LinearBase):
    """Full weight on every rank."""


def _shard(n: int, size: int, what: str) -> int:
    if n % size:
        raise ValueError(f"{what}={n} is not divisible by tensor-parallel size {size}")
    return n // size


class RowParallelLinear(LinearBase):
    """Input columns sharded over the TP group; outputs summed over it."""

    tp_mode = "row"

    def _local_shape(self, input_size, output_size):
        return _shard(input_size, self.tp_size, "input_size"), output_size

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        if param is self.bias or loaded_weight.dim() == 1:
            param.data.copy_(loaded_weight)
            return
        if self.tp_size > 1:
            self.full_row_amax = loaded_weight.detach().float().abs().amax(dim=1).to(param.device)
        k = param.shape[1]
        param.data.copy_(loaded_weight.narrow(1, self.tp_rank * k, k))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x, self.weight, self.bias if self.tp_rank == 0 else None)
        return tp.all_reduce_(y)


class MergedColumnParallelLinear(LinearBase):
    """[gate; up] rows, each sharded over the TP group (local [gate_r; up_r])."""

    tp_mode = "column"

    def __init__(self, input_size: int, output_sizes: list[int], bias: bool = False):
        self.output_sizes = output_sizes
        super().__init__(input_size, sum(output_sizes), bias)

    def _local_shape(self, input_size, output_size):
        return input_size, sum(_shard(s, self.tp_size, "output size") for s in self.output_sizes)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: int):
        local = [s // self.tp_size for s in self.output_sizes]
        offset = sum(local[:loaded_shard_id])
        size = local[loaded_shard_id]
        src = loaded_weight.narrow(0, self.tp_rank * size, size)
        param.data.narrow(0, offset, size).copy_(src)


class QKVParallelLinear(LinearBase):
    """Rows [q (Hq*D); k (Hkv*D); v (Hkv*D)], heads sharded over the TP group."""

    tp_mode = "column"

    def __init__(self, hidden_size: int, head_size: int, total_num_heads: int, total_num_kv_heads: int,
                 bias: bool = False):
        self.head_size = head_size
        self.total_num_heads = total_num_heads
        self.total_num_kv_heads = total_num_kv_heads
        size = tp.tp_size()
        self.num_heads = _shard(total_num_heads, size, "num_heads")
        self.num_kv_heads = _shard(total_num_kv_heads, size, "num_kv_heads")
        output_size = (total_num_heads + 2 * total_num_kv_heads) * head_size
        super().__init__(hidden_size, output_size, bias)

    def _local_shape(self, input_size, output_size):
        return input_size, (self.num_heads + 2 * self.num_kv_heads) * self.head_size

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: str):
        assert loaded_shard_id in ("q", "k", "v")
        D = self.head_size
        if loaded_shard_id == "q":
            size, offset = self.num_heads * D, 0
        elif loaded_shard_id == "k":
            size, offset = self.num_kv_heads * D, self.num_heads * D
        else:
            size, offset = self.num_kv_heads * D, (self.num_heads + self.num_kv_heads) * D
        src = loaded_weight.narrow(0, self.tp_rank * size, size)
        param.data.narrow(0, offset, size).copy_(src)
