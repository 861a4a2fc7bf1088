"""Token embedding and LM head (microserve/layers/embed_head.py:5-36).

Single GPU: plain fp16 embedding lookup and LM-head projection (fp16 operands,
fp32 accumulation, on this library's tcgen05 GEMM), as in the reference. Under tensor parallelism both are vocab-parallel: each rank holds
vocab rows [r*V/t, (r+1)*V/t); the embedding sums the masked lookups over the
group, and the head returns this rank's logits slice (the runner's greedy
sampler reduces (max, index) pairs across ranks instead of gathering logits).
"""
import torch
import torch.nn.functional as F
from torch import nn

from microserve_b200.utils import dist as tp


class VocabParallelEmbedding(nn.Module):
    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.tp_rank, self.tp_size = tp.tp_rank(), tp.tp_size()
        self.shard = (num_embeddings + self.tp_size - 1) // self.tp_size
        self.vocab_start = self.tp_rank * self.shard
        rows = min(self.shard, num_embeddings - self.vocab_start)
        self.weight = nn.Parameter(torch.empty(rows, embedding_dim))
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param.data.copy_(loaded_weight.narrow(0, self.vocab_start, param.shape[0]))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_size == 1:
            return F.embedding(x, self.weight)
        local = x - self.vocab_start
        mask = (local >= 0) & (local < self.weight.shape[0])
        y = F.embedding(local.clamp(0, self.weight.shape[0] - 1), self.weight)
        y = y * mask.unsqueeze(-1).to(y.dtype)
        return tp.all_reduce_(y)


class ParallelLMHead(VocabParallelEmbedding):
    def __init__(self, num_embeddings: int, embedding_dim: int, bias: bool = False):
        assert not bias
        super().__init__(num_embeddings, embedding_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Logits of this rank's vocab slice (the full vocab when tp_size == 1): the
        library's fp16 tcgen05 GEMM on the GPU (host tensors: the CPU tests of the
        tensor-parallel logic)."""
        if x.is_cuda:
            from microserve_b200 import kernels
            return kernels.f16_gemm(x.contiguous(), self.weight)
        return F.linear(x, self.weight)
