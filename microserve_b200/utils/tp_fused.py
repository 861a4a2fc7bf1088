"""Peer buffers for the fused tensor-parallel op (ms_tp_allreduce_rmsnorm_fp8).

Each rank allocates one device buffer holding
  partial   [R, H] fp16     this rank's row-parallel output (read by every rank)
  gather_q  2 x [R, H] e4m3 FP8 rows written by every rank (two halves: the op
                            before attention and the op before the MLP alternate,
                            so a rank never overwrites rows a peer may still read)
  gather_s  2 x [R] fp32    their row scales
  gather_h  [R, H] fp16     normalised fp16 rows (the final norm, for the LM head)
  flags     [2 * world] i32 ready / done flags written by every rank
  ctrl      [2] i32         this rank's epoch and block-arrival counter
(R = the most rows one forward can hold), exports it with a CUDA IPC handle,
gathers the handles over the process group and maps every peer's buffer. The
pointers are fixed for the life of the model, so the op is CUDA-graph safe.

The replaced reference path: RowParallelLinear's dist.all_reduce
(microserve/layers/linear.py:70-77) followed by RMSNorm's residual add + norm
(layers/layernorm.py:22-42) and the next FP8DynamicLinear's row quantisation
(layers/fp8_linear.py:14-23).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from microserve_b200 import _lib
from microserve_b200._lib import check, stream_ptr
from microserve_b200.utils import dist as tp

FP8 = torch.float8_e4m3fn


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class TpFused:
    def __init__(self, max_rows: int, hidden: int, device: torch.device):
        self.world, self.rank = tp.tp_size(), tp.tp_rank()
        if not 1 < self.world <= 8:
            raise ValueError("TpFused needs 2..8 ranks")
        if hidden % 8 != 0 or hidden > 16384:
            raise ValueError("TpFused needs hidden % 8 == 0 and hidden <= 16384")
        self.R, self.H, self.device = max_rows, hidden, device
        R, H, W = max_rows, hidden, self.world
        off, lay = 0, {}
        for name, nbytes in (("partial", R * H * 2), ("q0", R * H), ("q1", R * H), ("s0", R * 4), ("s1", R * 4),
                             ("h", R * H * 2), ("flags", 2 * W * 4), ("ctrl", 8)):
            lay[name] = off
            off = _align(off + nbytes)
        self.layout = lay
        self.buf = torch.zeros(off, dtype=torch.uint8, device=device)
        lib = _lib.load()
        handle = (C.c_ubyte * 64)()
        offset = C.c_int64(0)
        check(lib.ms_ipc_handle(self.buf.data_ptr(), handle, C.byref(offset)), "ms_ipc_handle")
        mine = (bytes(handle), int(offset.value))
        allh: list = [None] * W
        dist.all_gather_object(allh, mine, group=tp.tp_group())
        self._opened: list[int] = []
        bases = []
        for p, (h, o) in enumerate(allh):
            if p == self.rank:
                bases.append(self.buf.data_ptr())
                continue
            hb = (C.c_ubyte * 64).from_buffer_copy(h)
            base, ptr = C.c_void_p(), C.c_void_p()
            check(lib.ms_ipc_open(hb, o, C.byref(base), C.byref(ptr)), "ms_ipc_open")
            self._opened.append(base.value)
            bases.append(ptr.value)
        self.bases = bases

        def arr(name):
            a = (C.c_void_p * W)()
            for p in range(W):
                a[p] = bases[p] + lay[name]
            return a
        self.p_partial = arr("partial")
        self.p_q = [arr("q0"), arr("q1")]
        self.p_s = [arr("s0"), arr("s1")]
        self.p_h = arr("h")
        self.p_flags = arr("flags")
        self.p_ctrl = C.c_void_p(self.buf.data_ptr() + lay["ctrl"])
        torch.cuda.synchronize(device)
        dist.barrier(group=tp.tp_group())  # every rank mapped every buffer before the first op

    def _view(self, name: str, dtype: torch.dtype, shape: tuple[int, ...]) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= d
        o = self.layout[name]
        return self.buf[o:o + n * torch.empty((), dtype=dtype).element_size()].view(dtype).view(*shape)

    def partial(self, rows: int) -> torch.Tensor:
        """This rank's row-parallel output buffer [rows, H] fp16 (the GEMM's `out`)."""
        if rows > self.R:
            raise ValueError(f"TpFused holds {self.R} rows, {rows} requested")
        return self._view("partial", torch.float16, (self.R, self.H))[:rows]

    def allreduce_norm_fp8(self, rows: int, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                           half: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Sum the ranks' partial outputs, add the residual (rows owned by this rank
        are updated in place), RMSNorm, FP8 row quantisation; every rank receives all
        rows: returns (xq [rows, H] e4m3, sx [rows] fp32)."""
        self._launch(rows, residual, weight, eps, half, with_h=False)
        q = self._view(f"q{half}", FP8, (self.R, self.H))[:rows]
        s = self._view(f"s{half}", torch.float32, (self.R,))[:rows]
        return q, s

    def allreduce_norm_fp16(self, rows: int, residual: torch.Tensor, weight: torch.Tensor, eps: float
                            ) -> torch.Tensor:
        """As allreduce_norm_fp8, returning the normalised fp16 rows [rows, H] (the final norm)."""
        self._launch(rows, residual, weight, eps, 0, with_h=True)
        return self._view("h", torch.float16, (self.R, self.H))[:rows]

    def _launch(self, rows, residual, weight, eps, half, with_h):
        if rows > self.R:
            raise ValueError(f"TpFused holds {self.R} rows, {rows} requested")
        if residual.shape != (rows, self.H) or residual.dtype != torch.float16 or not residual.is_contiguous():
            raise ValueError("residual must be a contiguous fp16 [rows, H] tensor")
        lib = _lib.load()
        check(lib.ms_tp_allreduce_rmsnorm_fp8(self.p_partial, self.p_q[half], self.p_s[half],
                                              self.p_h if with_h else None, self.p_flags, self.p_ctrl,
                                              residual.data_ptr(), weight.data_ptr(), self.rank, self.world, rows,
                                              self.H, float(eps), stream_ptr()),
              "ms_tp_allreduce_rmsnorm_fp8")

    def close(self) -> None:
        lib = _lib.load()
        for b in self._opened:
            lib.ms_ipc_close(b)
        self._opened = []
