"""Tensor-parallel process group state.

One process per GPU. `init_tensor_parallel()` records the group every
TP-aware layer uses; with no group (the default) tp_size == 1 and every layer
behaves exactly like the reference's single-GPU layers.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_GROUP = None
_RANK = 0
_SIZE = 1
_EXACT_ACT_SCALE = False
_ORDERED_SUM = False


def init_tensor_parallel(group=None) -> None:
    """Use `group` (default: the world) for tensor parallelism."""
    global _GROUP, _RANK, _SIZE
    if not dist.is_initialized():
        raise RuntimeError("torch.distributed must be initialised before init_tensor_parallel()")
    _GROUP = group if group is not None else dist.group.WORLD
    _RANK = dist.get_rank(_GROUP)
    _SIZE = dist.get_world_size(_GROUP)


def reset_tensor_parallel() -> None:
    global _GROUP, _RANK, _SIZE, _EXACT_ACT_SCALE, _ORDERED_SUM
    _GROUP, _RANK, _SIZE, _EXACT_ACT_SCALE, _ORDERED_SUM = None, 0, 1, False, False


def set_ordered_sum(enable: bool) -> None:
    """For checks: all_reduce_ of fp16 tensors as an all-gather and an fp32 sum in rank
    order, rounded to fp16 once - the arithmetic of the fused peer-memory collective -
    instead of NCCL's reduction, whose order and intermediate fp16 roundings depend on
    the algorithm it picks (identical to it for two ranks, where a + b = b + a)."""
    global _ORDERED_SUM
    _ORDERED_SUM = bool(enable)


def set_exact_act_scale(enable: bool) -> None:
    """Row-parallel activation scales from the full row (an all-reduce max of one
    float per row before each o_proj / down_proj quantisation) instead of the
    local shard: FP8 codes identical to TP=1, one small collective more."""
    global _EXACT_ACT_SCALE
    _EXACT_ACT_SCALE = bool(enable)


def exact_act_scale() -> bool:
    return _EXACT_ACT_SCALE and _SIZE > 1


def tp_rank() -> int:
    return _RANK


def tp_size() -> int:
    return _SIZE


def tp_group():
    return _GROUP


def all_reduce_(x: torch.Tensor) -> torch.Tensor:
    """In-place sum over the TP group (identity when tp_size == 1)."""
    if _SIZE > 1:
        if _ORDERED_SUM and x.dtype == torch.float16:
            parts = [torch.empty_like(x, memory_format=torch.contiguous_format) for _ in range(_SIZE)]
            dist.all_gather(parts, x.contiguous(), group=_GROUP)
            acc = parts[0].float()
            for part in parts[1:]:
                acc += part.float()
            x.copy_(acc.half())
        else:
            dist.all_reduce(x, group=_GROUP)
    return x


def all_reduce_max_(x: torch.Tensor) -> torch.Tensor:
    if _SIZE > 1:
        dist.all_reduce(x, op=dist.ReduceOp.MAX, group=_GROUP)
    return x


def tp_argmax(local_logits: torch.Tensor, vocab_start: int) -> torch.Tensor:
    """Greedy token over a vocab-parallel logits slice [B, V_local]: the global
    argmax with the smallest index winning ties (torch.argmax's rule), from an
    all-gather of one (max, index) pair per row instead of the logits."""
    if local_logits.is_cuda and local_logits.dtype == torch.float16:
        from microserve_b200 import kernels
        local_idx, local_max = kernels.argmax_rows(local_logits, want_max=True)
    else:  # host tensors (the gloo tests of this logic)
        local_max, local_idx = local_logits.float().max(dim=-1)
    if _SIZE == 1:
        return local_idx
    local_idx = local_idx + vocab_start
    pair = torch.stack([local_max, local_idx.to(torch.float64).float()], dim=-1)
    gathered = [torch.empty_like(pair) for _ in range(_SIZE)]
    dist.all_gather(gathered, pair, group=_GROUP)
    allp = torch.stack(gathered, dim=0)  # [t, B, 2]; ranks hold ascending vocab ranges
    best = allp[..., 0].argmax(dim=0)    # first (lowest) rank with the max value
    return allp[..., 1].gather(0, best.unsqueeze(0)).squeeze(0).to(torch.int64)
