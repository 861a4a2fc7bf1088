"""Seeded inputs of the reference-GPU golden cases (tests/golden/reference_gpu.pt).

Every input is produced on the CPU from a fixed torch.Generator seed, so the
fixture only stores the reference's outputs; make_golden_gpu.py (on the box)
and the tests rebuild the same inputs from here. KV caches are filled with
the oracle's FP8 store, which the "store" case pins bit-exactly to the
reference's Triton store.
"""
from __future__ import annotations

import torch

from oracle import fp8_decoder as O

BS, D = 256, 128
SCALE = D ** -0.5


def _g(seed):
    return torch.Generator().manual_seed(seed)


def store_case():
    """64 tokens x 2 kv heads scattered over 2 blocks, mixed magnitudes, one all-zero head."""
    g = _g(101)
    k = (torch.randn(64, 2, D, generator=g) * torch.logspace(-3, 1, 64)[:, None, None]).half()
    v = torch.randn(64, 2, D, generator=g).half()
    k[7, 1].zero_()
    slots = torch.randperm(2 * BS, generator=g)[:64].long()
    return k, v, slots, 2


def _filled(seed, lengths, tables, hkv, scale=0.2):
    g = _g(seed)
    nb = max(max(t) for t in tables) + 1
    kc = torch.zeros(nb, BS, hkv, D, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    ks = torch.ones(nb, BS, hkv)
    vs = torch.ones_like(ks)
    keys = torch.randn(sum(lengths), hkv, D, generator=g).half() * scale
    vals = torch.randn(sum(lengths), hkv, D, generator=g).half() * scale
    slots = sum((O.slot_mapping(t, list(range(L)), BS) for t, L in zip(tables, lengths)), [])
    O.store_kv(keys, vals, kc, vc, ks, vs, torch.tensor(slots))
    return [kc, vc, ks, vs]


def decode_case():
    """The geometry of the reference's tests/test_fp8_kv_attention.py:39-73."""
    lengths = [1, 73, 300]
    tables = [[0, 1], [2, 3], [4, 5]]
    caches = _filled(201, lengths, tables, 8)
    q = torch.randn(3, 16, D, generator=_g(202)).half() * 0.2
    return caches, q, torch.tensor(lengths, dtype=torch.int32), torch.tensor(tables, dtype=torch.int32)


def chunk_case():
    """tests/test_fp8_kv_attention.py:76-108 geometry: prefix 273 + 31 queries, table [1, 0]."""
    caches = _filled(301, [304], [[1, 0]], 4)
    q = torch.randn(31, 8, D, generator=_g(302)).half() * 0.2
    return caches, q, torch.tensor([[1, 0]], dtype=torch.int32), 273


def linear_case():
    g = _g(401)
    w = (torch.randn(384, 256, generator=g) * 0.02).half()
    x = torch.randn(17, 256, generator=g).half()
    x[3].zero_()
    return w, x


def rmsnorm_case():
    g = _g(501)
    x = torch.randn(17, 1024, generator=g).half()
    r = torch.randn(17, 1024, generator=g).half()
    w = (1 + 0.1 * torch.randn(1024, generator=g)).half()
    return x, r, w


def varlen_case():
    g = _g(601)
    lens = [1, 9, 30]
    T = sum(lens)
    q = torch.randn(T, 8, D, generator=g).half() * 0.5
    k = torch.randn(T, 4, D, generator=g).half() * 0.5
    v = torch.randn(T, 4, D, generator=g).half()
    cu = torch.tensor([0, 1, 10, 40], dtype=torch.int32)
    return q, k, v, cu
