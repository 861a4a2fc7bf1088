"""Failure detection of the fused tensor-parallel op on one GPU, without any GPU
fault: the op runs as rank 0 of a two-rank group whose "rank 1" is a second,
local buffer that nothing ever writes. Rank 0's wait for rank 1's rows must run
out after the (shortened) wait limit, record status 2 (peer timeout), leave the
epoch where it was and return - the context stays usable - and the host check
the engine runs after every step must raise."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

H, ROWS = 1024, 8


def _buffer(lib, world):
    from microserve_b200._lib import check, stream_ptr
    from microserve_b200.utils.tp_fused import layout
    lay = layout(world, H, ROWS)
    buf = torch.empty(lay["total"] + 256, dtype=torch.uint8, device="cuda")
    base = (buf.data_ptr() + 255) // 256 * 256
    check(lib.ms_tp_buffer_init(base, world, H, ROWS, stream_ptr()), "ms_tp_buffer_init")
    return buf, base, lay


def test_peer_that_never_answers_times_out_and_is_reported():
    import time
    from microserve_b200 import _lib
    from microserve_b200._lib import DeviceWaitTimeout, check, stream_ptr
    lib = _lib.load()
    assert _lib.device_status() == 0
    mine, base0, lay = _buffer(lib, 2)
    silent, base1, _ = _buffer(lib, 2)
    g = torch.Generator(device="cuda").manual_seed(0)
    part = torch.randn(ROWS, H, device="cuda", generator=g).half()
    torch.cuda.synchronize()
    off = base0 - mine.data_ptr()
    mine[off + lay["partial"]:off + lay["partial"] + part.numel() * 2].copy_(part.view(-1).view(torch.uint8))
    residual = torch.randn(ROWS, H, device="cuda", generator=g).half()
    weight = torch.ones(H, device="cuda", dtype=torch.float16)
    bases = (C.c_void_p * 2)(base0, base1)
    _lib.set_wait_limit(0.05)
    try:
        t0 = time.perf_counter()
        check(lib.ms_tp_allreduce_rmsnorm_fp8(bases, 0, 2, H, ROWS, residual.data_ptr(), weight.data_ptr(), ROWS,
                                              C.c_float(1e-6), 0, 0, stream_ptr()), "ms_tp_allreduce_rmsnorm_fp8")
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        _lib.set_wait_limit(4.0)
    assert elapsed < 2.0, elapsed  # ended by the 50 ms limit, not by the default 4 s one

    with pytest.raises(DeviceWaitTimeout, match="peer"):
        _lib.raise_on_device_status("tensor-parallel step")
    assert _lib.device_status() == 0  # read-and-clear
    # the context is still usable
    x = torch.randn(4, 1024, device="cuda").half()
    assert torch.isfinite(x.float().sum())
