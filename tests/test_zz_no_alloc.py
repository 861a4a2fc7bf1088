"""The allocation-free decode entry point (ms_paged_decode_fp8_noalloc).

It serves callers that cannot allocate device memory where attention runs
(inside another framework's memory pool, embedders that forbid cudaMalloc
after start-up, callers holding only a stream): the context-split partials
go to a buffer built into the library instead of a caller workspace. This
test calls it through the C ABI twice in a row, on a batch whose context is
split (so the built-in buffer is really used), and checks each result
against ms_paged_decode_fp8 with a caller workspace, within the decode
tolerance the other tests use (0.004; the two paths run the same kernel and
in practice agree exactly). The file name sorts last so a stop-at-first-
failure run has already run every other test; it also passes on its own in
a fresh process, where its first call performs the per-device set-up.
"""
import ctypes

import pytest
import torch

from oracle import fp8_decoder as O

pytestmark = pytest.mark.gpu

BS, D = 256, 128


def _case(seed, lengths, hq, hkv):
    g = torch.Generator().manual_seed(seed)
    nblk = [(L + BS - 1) // BS for L in lengths]
    perm = torch.randperm(sum(nblk), generator=g).tolist()
    tables, o = [], 0
    for n in nblk:
        tables.append(perm[o:o + n])
        o += n
    kc = torch.zeros(sum(nblk), BS, hkv, D, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    ks = torch.ones(sum(nblk), BS, hkv)
    vs = torch.ones_like(ks)
    keys = torch.randn(sum(lengths), hkv, D, generator=g).half() * 0.3
    vals = torch.randn(sum(lengths), hkv, D, generator=g).half()
    slots = sum((O.slot_mapping(t, list(range(L)), BS) for t, L in zip(tables, lengths)), [])
    O.store_kv(keys, vals, kc, vc, ks, vs, torch.tensor(slots))
    q = torch.randn(len(lengths), hq, D, generator=g).half() * 0.3
    dev = "cuda"
    return (q.to(dev), kc.to(dev), vc.to(dev), ks.to(dev), vs.to(dev),
            torch.tensor(lengths, dtype=torch.int32, device=dev), O.block_table_rows(tables).to(dev))


def _noalloc(lib, q, kc, vc, ks, vs, lens, bt):
    from microserve_b200._lib import check, stream_ptr
    out = torch.empty_like(q)
    B, Hq, _ = q.shape
    check(lib.ms_paged_decode_fp8_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ks.data_ptr(), vs.data_ptr(),
                                          lens.data_ptr(), bt.data_ptr(), out.data_ptr(), B, Hq, kc.shape[2], D, BS,
                                          bt.shape[1], ctypes.c_float(D ** -0.5), stream_ptr()),
          "ms_paged_decode_fp8_noalloc")
    return out


def test_noalloc_decode_matches_workspace_entry_point_twice():
    from microserve_b200 import _lib, kernels
    lib = _lib.load()
    cases = [(21, [3000, 700], 32, 8), (22, [5000, 90, 1500], 16, 8)]
    for seed, lengths, hq, hkv in cases:
        args = _case(seed, lengths, hq, hkv)
        q, kc, vc, ks, vs, lens, bt = args
        # the batch is split over CTAs, so the built-in scratch is used
        assert kernels.decode_workspace_bytes(q.shape[0], hq, hkv, bt.shape[1], BS) > 0
        got = _noalloc(lib, *args)
        ref = kernels.paged_decode_fp8(q, kc, vc, ks, vs, lens, bt, D ** -0.5)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got.float() - ref.float()).abs().max().item() < 0.004
    assert _lib.device_status() == 0


def test_noalloc_rejects_batches_beyond_its_buffer():
    from microserve_b200 import _lib, kernels
    lib = _lib.load()
    dev = "cuda"
    Hq, Hkv, nblk = 64, 8, 64
    # the first batch size (on this device's SM count) whose context split needs
    # more scratch than the 4 MiB built-in buffer holds
    B = next((b for b in range(1, 4096) if kernels.decode_workspace_bytes(b, Hq, Hkv, nblk, BS) > 4 << 20), None)
    assert B is not None
    q = torch.zeros(B, Hq, D, dtype=torch.float16, device=dev)
    kc = torch.zeros(1, BS, Hkv, D, dtype=torch.float8_e4m3fn, device=dev)
    ks = torch.ones(1, BS, Hkv, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    bt = torch.zeros(B, nblk, dtype=torch.int32, device=dev)
    rc = lib.ms_paged_decode_fp8_noalloc(q.data_ptr(), kc.data_ptr(), kc.data_ptr(), ks.data_ptr(), ks.data_ptr(),
                                         lens.data_ptr(), bt.data_ptr(), q.data_ptr(), B, Hq, Hkv, D, BS, nblk,
                                         ctypes.c_float(1.0), 0)
    assert rc == _lib.MS_ERR_UNSUPPORTED
    assert b"built-in buffer" in lib.ms_last_error()
