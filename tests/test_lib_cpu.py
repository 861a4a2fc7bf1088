"""CPU-side checks of the C ABI library: it loads, and it exports exactly the
entry points include/microserve_b200.h declares (no GPU needed)."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    text = (ROOT / "include" / "microserve_b200.h").read_text()
    return sorted(set(re.findall(r"\b(ms_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "ms_fp8_gemm" in names and "ms_paged_decode_fp8" in names and len(names) >= 12


def test_library_exports_every_declared_symbol():
    from microserve_b200 import _lib
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_lib.SIGNATURES) == set(_declared())
    assert lib.ms_version() >= 100


def test_workspace_queries_without_gpu():
    from microserve_b200 import _lib
    lib = _lib.load()
    assert lib.ms_fp8_gemm_workspace_size(0, 10, 10) == 0
    assert lib.ms_paged_decode_workspace_size(256, 32, 8, 8, 256) == 0  # 2048 CTAs: no split


def test_bad_arguments_are_rejected_without_launch():
    from microserve_b200 import _lib
    lib = _lib.load()
    assert lib.ms_fp8_gemm(None, None, None, None, None, None, 4, 4, 4, None, 0, None) == _lib.MS_ERR_INVALID
    assert b"null" in lib.ms_last_error()
    assert lib.ms_store_kv_fp8(None, None, 1, 8, 64, None, None, None, None, None, None) == _lib.MS_ERR_UNSUPPORTED
