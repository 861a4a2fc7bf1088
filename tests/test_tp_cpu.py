"""Tensor-parallel host logic on CPU: two gloo ranks check the sharded weight
loaders, the row-parallel sum, the vocab-parallel embedding and the
distributed greedy argmax against single-process results."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F


def _worker(rank, world, init_file, errq):
    try:
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
        from microserve_b200.layers.embed_head import ParallelLMHead, VocabParallelEmbedding
        from microserve_b200.layers.linear import (MergedColumnParallelLinear, QKVParallelLinear,
                                                   RowParallelLinear)
        from microserve_b200.utils import dist as tp
        tp.init_tensor_parallel()
        g = torch.Generator().manual_seed(0)
        H, D, Hq, Hkv, I, V = 64, 16, 4, 2, 48, 37
        wq, wk, wv = (torch.randn(Hq * D, H, generator=g), torch.randn(Hkv * D, H, generator=g),
                      torch.randn(Hkv * D, H, generator=g))
        wgate, wup = torch.randn(I, H, generator=g), torch.randn(I, H, generator=g)
        wo = torch.randn(H, Hq * D, generator=g)
        emb = torch.randn(V, H, generator=g)
        x = torch.randn(5, H, generator=g)

        qkv = QKVParallelLinear(H, D, Hq, Hkv)
        for sid, w in (("q", wq), ("k", wk), ("v", wv)):
            qkv.weight.weight_loader(qkv.weight, w, sid)
        hq, hk = Hq // world, Hkv // world
        exp = torch.cat([wq[rank * hq * D:(rank + 1) * hq * D], wk[rank * hk * D:(rank + 1) * hk * D],
                         wv[rank * hk * D:(rank + 1) * hk * D]])
        assert torch.equal(qkv.weight.data, exp)

        gu = MergedColumnParallelLinear(H, [I, I])
        gu.weight.weight_loader(gu.weight, wgate, 0)
        gu.weight.weight_loader(gu.weight, wup, 1)
        i2 = I // world
        assert torch.equal(gu.weight.data, torch.cat([wgate[rank * i2:(rank + 1) * i2], wup[rank * i2:(rank + 1) * i2]]))

        o = RowParallelLinear(Hq * D, H)
        o.weight.weight_loader(o.weight, wo)
        k2 = Hq * D // world
        assert torch.equal(o.weight.data, wo[:, rank * k2:(rank + 1) * k2])
        assert torch.equal(o.full_row_amax, wo.abs().amax(dim=1))  # FP8 scales from the full row
        xin = torch.randn(5, Hq * D, generator=torch.Generator().manual_seed(1))
        y = o(xin[:, rank * k2:(rank + 1) * k2])
        assert torch.allclose(y, F.linear(xin, wo), atol=1e-4)

        e = VocabParallelEmbedding(V, H)
        e.weight.weight_loader(e.weight, emb)
        ids = torch.tensor([0, 5, 18, 19, 36])
        assert torch.allclose(e(ids), F.embedding(ids, emb))

        head = ParallelLMHead(V, H)
        head.weight.weight_loader(head.weight, emb)
        logits = head(x)
        full = F.linear(x, emb)
        assert torch.equal(tp.tp_argmax(logits, head.vocab_start), full.argmax(-1))
        # ties across ranks resolve to the smallest index, like torch.argmax
        tie = torch.zeros(3, head.weight.shape[0])
        tie[:, 0] = 1.0
        assert tp.tp_argmax(tie, head.vocab_start).tolist() == [0, 0, 0]
        dist.barrier()
        dist.destroy_process_group()
    except Exception as ex:  # report to the parent
        import traceback
        errq.put(f"rank {rank}: {ex}\n{traceback.format_exc()}")
        raise
    # gloo's worker threads can abort the interpreter's normal teardown ("terminate called
    # without an active exception") after a clean destroy; every check has passed here.
    os._exit(0)


def test_tensor_parallel_layers_two_gloo_ranks(tmp_path):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    init_file = tmp_path / "pg_init"
    procs = [ctx.Process(target=_worker, args=(r, 2, str(init_file), errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, "\n".join(errs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def _ordered_sum_worker(rank, world, init_file, errq):
    try:
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
        from microserve_b200.utils import dist as tp
        tp.init_tensor_parallel()
        parts = [(torch.randn(3, 40, generator=torch.Generator().manual_seed(p)) * 10 ** p).half()
                 for p in range(world)]
        acc = torch.zeros(3, 40)
        for p in range(world):  # fp32, rank order, one rounding at the end
            acc = acc + parts[p].float()
        x = parts[rank].clone()
        tp.set_ordered_sum(True)
        assert tp.all_reduce_(x) is x
        assert torch.equal(x, acc.half())
        tp.set_ordered_sum(False)
        y = tp.all_reduce_(torch.ones(4, dtype=torch.float32))  # other dtypes: the plain all-reduce
        assert torch.equal(y, torch.full((4,), float(world)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as ex:
        import traceback
        errq.put(f"rank {rank}: {ex}\n{traceback.format_exc()}")
        raise
    os._exit(0)


def test_ordered_sum_is_the_rank_order_fp32_sum_four_gloo_ranks(tmp_path):
    """The reference all-reduce of bench.py's tensor-parallel parity check: an fp32 sum in
    rank order rounded to fp16 once, on every rank (4 ranks, magnitudes 1..1000 so that
    another order would round differently)."""
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    procs = [ctx.Process(target=_ordered_sum_worker, args=(r, 4, str(tmp_path / "pg"), errq)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, "\n".join(errs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
