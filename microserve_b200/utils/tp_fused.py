"""Peer buffers for the fused tensor-parallel op (ms_tp_allreduce_rmsnorm_fp8).

Each rank allocates one device buffer whose layout the library defines
(ms_tp_layout): this rank's row-parallel output (`partial`, the GEMM's out),
receive slots its peers write, and the gather areas every owner writes its
normalised rows into (FP8 codes + scales, or fp16 rows for the final norm).
The buffer is put in its initial state (ms_tp_buffer_init: "not yet written"
pattern), exported with a CUDA IPC handle, the handles are gathered over the
process group and every peer's buffer is mapped. The pointers are fixed for
the life of the model, so the op is CUDA-graph safe.

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
_PARTS = ("partial", "outq", "outs", "outh", "total")


def layout(world: int, hidden: int, max_rows: int) -> dict[str, int]:
    """Byte offsets of one rank's buffer (the library's layout)."""
    off = (C.c_int64 * 5)()
    check(_lib.load().ms_tp_layout(world, hidden, max_rows, off), "ms_tp_layout")
    return dict(zip(_PARTS, list(off)))


class TpFused:
    def __init__(self, max_rows: int, hidden: int, device: torch.device, fused_gemm: bool = True):
        self.fused_gemm = fused_gemm
        self.world, self.rank = tp.tp_size(), tp.tp_rank()
        if not 1 < self.world <= 8:
            raise ValueError("TpFused needs 2..8 ranks")
        if hidden % 16 != 0 or hidden > 16384:
            raise ValueError("TpFused needs hidden % 16 == 0 and hidden <= 16384")
        self.R, self.H, self.device = max_rows, hidden, device
        W = self.world
        lib = _lib.load()
        self.layout = layout(W, hidden, max_rows)
        self.buf = torch.empty(self.layout["total"] + 256, dtype=torch.uint8, device=device)
        self.base = (self.buf.data_ptr() + 255) // 256 * 256  # the library wants 256-byte alignment
        check(lib.ms_tp_buffer_init(self.base, W, hidden, max_rows, stream_ptr()), "ms_tp_buffer_init")
        torch.cuda.synchronize(device)
        handle = (C.c_ubyte * 64)()
        offset = C.c_int64(0)
        check(lib.ms_ipc_handle(self.base, handle, C.byref(offset)), "ms_ipc_handle")
        mine = (bytes(handle), int(offset.value))
        allh: list = [None] * W
        dist.all_gather_object(allh, mine, group=tp.tp_group())
        self._opened: list[int] = []
        self.bases = (C.c_void_p * W)()
        for p, (h, o) in enumerate(allh):
            if p == self.rank:
                self.bases[p] = self.base
                continue
            hb = (C.c_ubyte * 64).from_buffer_copy(h)
            base, ptr = C.c_void_p(), C.c_void_p()
            check(lib.ms_ipc_open(hb, o, C.byref(base), C.byref(ptr)), "ms_ipc_open")
            self._opened.append(base.value)
            self.bases[p] = ptr.value
        torch.cuda.synchronize(device)
        dist.barrier(group=tp.tp_group())  # every rank mapped every buffer before the first op

    def _view(self, name: str, dtype: torch.dtype, shape: tuple[int, ...]) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= d
        o = self.base - self.buf.data_ptr() + self.layout[name]
        return self.buf[o:o + n * torch.empty((), dtype=dtype).element_size()].view(dtype).view(*shape)

    def partial(self, rows: int) -> torch.Tensor:
        """This rank's row-parallel output buffer [rows, H] fp16 (the GEMM's `out`)."""
        if rows > self.R:
            raise ValueError(f"TpFused holds {self.R} rows, {rows} requested")
        return self._view("partial", torch.float16, (self.R, self.H))[:rows]

    def rowpar_gemm(self, xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor) -> None:
        """The row-parallel FP8 GEMM (o_proj / down_proj shard) with each output row
        pushed by the GEMM's epilogue to the rank that owns it (ms_fp8_gemm_rowpar);
        the next allreduce_norm_* call takes pushed=True."""
        from microserve_b200 import kernels
        M, K = xq.shape
        if wq.shape != (self.H, K):
            raise ValueError(f"rowpar_gemm: weight must be [{self.H}, {K}]")
        if M > self.R:
            raise ValueError(f"TpFused holds {self.R} rows, {M} requested")
        kernels.fp8_gemm_rowpar(xq, sx, wq, sw, self.bases, self.rank, self.world, self.R)

    def rowpar_gemm_norm(self, xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                         residual: torch.Tensor, weight: torch.Tensor, eps: float, want_fp16: bool = False):
        """Row-parallel FP8 GEMM + all-reduce + residual add + RMSNorm + FP8 quantisation:
        returns (xq [rows, H] e4m3, sx [rows] fp32) of the normalised rows, or with
        want_fp16 the fp16 rows [rows, H]. With fused_gemm one kernel
        (ms_fp8_gemm_rowpar_ar_rmsnorm); otherwise the GEMM pushes each output row to the
        rank that owns it (ms_fp8_gemm_rowpar) and ms_tp_allreduce_rmsnorm_fp8 does the
        rest on the pushed rows (B200, 256 rows: 26.6 vs 27.7 us at TP=2 and 24.4 vs
        26.0 us at TP=8 for a local partial + the op pushing it; the same bits)."""
        from microserve_b200 import kernels
        M, K = xq.shape
        if wq.shape != (self.H, K):
            raise ValueError(f"rowpar_gemm_norm: weight must be [{self.H}, {K}]")
        self._check(M, residual)
        if not self.fused_gemm:
            self.rowpar_gemm(xq, sx, wq, sw)
            if want_fp16:
                return self.allreduce_norm_fp16(M, residual, weight, eps, pushed=True)
            return self.allreduce_norm_fp8(M, residual, weight, eps, pushed=True)
        kernels.fp8_gemm_rowpar_ar_rmsnorm(xq, sx, wq, sw, self.bases, self.rank, self.world, self.R, residual,
                                           weight, eps, want_fp16)
        if want_fp16:
            return self._view("outh", torch.float16, (self.R, self.H))[:M]
        return (self._view("outq", FP8, (self.R, self.H))[:M], self._view("outs", torch.float32, (self.R,))[:M])

    def allreduce_norm_fp8(self, rows: int, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                           pushed: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
        """Sum the ranks' partial outputs (in `partial`, or already pushed by
        rowpar_gemm), add the residual (rows owned by this rank are updated in place),
        RMSNorm, FP8 row quantisation; every rank receives all rows: returns
        (xq [rows, H] e4m3, sx [rows] fp32)."""
        self._launch(rows, residual, weight, eps, want_h=False, pushed=pushed)
        q = self._view("outq", FP8, (self.R, self.H))[:rows]
        s = self._view("outs", torch.float32, (self.R,))[:rows]
        return q, s

    def allreduce_norm_fp16(self, rows: int, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                            pushed: bool = False) -> torch.Tensor:
        """As allreduce_norm_fp8, returning the normalised fp16 rows [rows, H] (the final norm)."""
        self._launch(rows, residual, weight, eps, want_h=True, pushed=pushed)
        return self._view("outh", torch.float16, (self.R, self.H))[:rows]

    def _check(self, rows, residual):
        if rows > self.R:
            raise ValueError(f"TpFused holds {self.R} rows, {rows} requested")
        if residual.shape != (rows, self.H) or residual.dtype != torch.float16 or not residual.is_contiguous():
            raise ValueError("residual must be a contiguous fp16 [rows, H] tensor")

    def _launch(self, rows, residual, weight, eps, want_h, pushed):
        self._check(rows, residual)
        check(_lib.load().ms_tp_allreduce_rmsnorm_fp8(self.bases, self.rank, self.world, self.H, self.R,
                                                      residual.data_ptr(), weight.data_ptr(), rows, float(eps),
                                                      1 if want_h else 0, 1 if pushed else 0, stream_ptr()),
              "ms_tp_allreduce_rmsnorm_fp8")

    def close(self) -> None:
        lib = _lib.load()
        for b in self._opened:
            lib.ms_ipc_close(b)
        self._opened = []
