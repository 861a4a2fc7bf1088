"""ctypes binding of the C ABI in include/microserve_b200.h.

The library is built in-tree (microserve_b200/libmicroserve_b200.so, see
build.py). There is no fallback: if the library is missing or fails to load,
every op raises. Tensors cross the boundary as raw pointers
(`tensor.data_ptr()`) and the current CUDA stream as `void*`.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmicroserve_b200.so"

vp, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t
fp = C.POINTER(C.c_float)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "ms_version": (i32, []),
    "ms_last_error": (C.c_char_p, []),
    "ms_launch_count": (i64, []),
    "ms_set_pdl": (i32, [i32]),
    "ms_set_pair_tiles": (i32, [i32]),
    "ms_argmax_workspace_size": (sz, [i64]),
    "ms_ipc_handle": (i32, [vp, vp, C.POINTER(C.c_int64)]),
    "ms_ipc_open": (i32, [vp, i64, C.POINTER(vp), C.POINTER(vp)]),
    "ms_ipc_close": (i32, [vp]),
    "ms_tp_layout": (i32, [i32, i64, i64, C.POINTER(C.c_int64)]),
    "ms_tp_buffer_init": (i32, [vp, i32, i64, i64, vp]),
    "ms_tp_allreduce_rmsnorm_fp8": (i32, [vp, i32, i32, i64, i64, vp, vp, i64, f32, i32, i32, vp]),
    "ms_set_wait_limit": (i32, [C.c_uint64]),
    "ms_fp8_gemm_rowpar": (i32, [vp, vp, vp, vp, i64, i64, i64, vp, sz, vp, i32, i32, i64, vp]),
    "ms_fp8_gemm_rowpar_ar_rmsnorm": (i32, [vp, vp, vp, vp, i64, i64, i64, vp, sz, vp, i32, i32, i64, vp, vp, f32,
                                           i32, vp]),
    "ms_row_amax": (i32, [vp, i64, i64, i64, vp, vp]),
    "ms_quantize_rows_fp8_amax": (i32, [vp, i64, i64, i64, vp, vp, vp, vp]),
    "ms_argmax_rows": (i32, [vp, i64, i64, i64, vp, vp, vp, sz, vp]),
    "ms_get_device_status": (i32, [C.POINTER(C.c_int), vp]),
    "ms_quantize_rows_fp8": (i32, [vp, i64, i64, i64, vp, vp, vp]),
    "ms_fp8_gemm_workspace_size": (sz, [i64, i64, i64]),
    "ms_fp8_gemm_plan": (i32, [i64, i64, i64, i32, C.POINTER(C.c_int)]),
    "ms_f16_gemm_workspace_size": (C.c_size_t, [i64, i64, i64]),
    "ms_f16_gemm": (i32, [vp, vp, vp, i64, i64, i64, vp, C.c_size_t, vp]),
    "ms_fp8_gemm": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, vp, sz, vp]),
    "ms_rmsnorm": (i32, [vp, vp, vp, i64, i64, f32, vp, vp, vp, vp, vp]),
    "ms_silu_mul": (i32, [vp, i64, i64, vp, vp, vp, vp]),
    "ms_store_kv_fp8": (i32, [vp, vp, i64, i32, i32, vp, vp, vp, vp, vp, vp]),
    "ms_qkv_post": (i32, [vp, i64, i32, i32, i32, vp, vp, f32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "ms_paged_decode_workspace_size": (sz, [i32, i32, i32, i32, i32]),
    "ms_paged_decode_fp8": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32, vp, sz, vp]),
    "ms_paged_decode_fp8_noalloc": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32, vp]),
    "ms_paged_prefill_fp8": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i64, i32, i32, i32, i32, i32, f32, vp]),
    "ms_varlen_prefill": (i32, [vp, vp, vp, vp, vp, i32, i64, i32, i32, i32, f32, vp]),
}

MS_ERR_INVALID, MS_ERR_UNSUPPORTED, MS_ERR_CUDA, MS_ERR_WORKSPACE = -1, -2, -3, -4

_lib: C.CDLL | None = None


class KernelLibraryMissing(RuntimeError):
    pass


def load() -> C.CDLL:
    """Load (once) and return the kernel library; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise KernelLibraryMissing(
            f"{LIB_PATH} not found: build it with `python -m microserve_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def check(rc: int, what: str) -> None:
    """Map a non-zero return code to the reference's error types."""
    if rc == 0:
        return
    msg = load().ms_last_error().decode(errors="replace")
    if rc in (MS_ERR_INVALID, MS_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def device_status() -> int:
    """Read and clear the device status word (non-zero = a bounded wait timed out)."""
    s = C.c_int(0)
    check(load().ms_get_device_status(C.byref(s), stream_ptr()), "ms_get_device_status")
    return s.value


STATUS_NAMES = {1: "a pipeline barrier wait timed out", 2: "a peer (tensor-parallel rank) did not answer in time"}


class DeviceWaitTimeout(RuntimeError):
    """A bounded in-kernel wait ran out (ms_get_device_status != 0): results of
    the step are invalid; with tensor parallelism the group must be rebuilt."""


def raise_on_device_status(where: str) -> None:
    """Read (and clear) the device status word; raise DeviceWaitTimeout if set."""
    s = device_status()
    if s != 0:
        raise DeviceWaitTimeout(f"{where}: device status {s} ({STATUS_NAMES.get(s, 'unknown')})")


def set_wait_limit(seconds: float) -> None:
    """Upper bound of every in-kernel wait on the current device (default 4 s)."""
    check(load().ms_set_wait_limit(max(1, int(seconds * 1e9))), "ms_set_wait_limit")
