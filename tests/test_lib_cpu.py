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


def test_f16_gemm_arguments_are_checked_without_launch():
    """ms_f16_gemm (the LM head's GEMM) rejects bad sizes, null pointers and K % 8 != 0
    before touching the GPU; its workspace query is host-only."""
    from microserve_b200 import _lib
    lib = _lib.load()
    assert lib.ms_f16_gemm(None, None, None, 4, 4, 0, None, 0, None) == _lib.MS_ERR_INVALID
    assert lib.ms_f16_gemm(None, None, None, 4, 4, 8, None, 0, None) == _lib.MS_ERR_INVALID
    assert b"null" in lib.ms_last_error()
    assert lib.ms_f16_gemm(8, 8, 8, 4, 4, 12, None, 0, None) == _lib.MS_ERR_UNSUPPORTED
    assert lib.ms_f16_gemm(None, None, None, 0, 4, 8, None, 0, None) == 0  # nothing to do
    assert lib.ms_f16_gemm_workspace_size(256, 4096, 4096) >= 0


def _plan(M, N, K, sms=148):
    import ctypes as C
    from microserve_b200 import _lib
    out = (C.c_int * 7)()
    assert _lib.load().ms_fp8_gemm_plan(M, N, K, sms, out) == 0
    p = dict(zip(("bn", "ctas", "splits", "wide", "dp", "ch", "pair"), list(out)))
    return p if p.pop("pair") == 0 else dict(p, pair=1)


def test_gemm_schedules_of_the_8b_decode_and_prefill_shapes():
    """The FP8 GEMM planner's choices for the bench's Qwen3-8B shapes on 148 SMs
    (the rules in csrc/fp8_gemm.cu make_plan; timings behind them in
    profiles/fp8_gemm_qwen3-8b_m256.md), with one-SM tiles (the default) and with the
    SM-pair schedules turned on (ms_set_pair_tiles)."""
    from microserve_b200 import _lib
    lib = _lib.load()
    # decode, 256 tokens: qkv / o whole tiles of 96 / 64 tokens, one wave each
    assert _plan(256, 6144, 4096) == dict(bn=96, ctas=144, splits=0, wide=0, dp=1, ch=2)
    assert _plan(256, 4096, 4096) == dict(bn=64, ctas=128, splits=0, wide=0, dp=1, ch=2)
    # gate_up: 96 tiles of 256 weight rows x 256 tokens
    assert _plan(256, 24576, 4096) == dict(bn=256, ctas=96, splits=0, wide=1, dp=1, ch=1)
    # down (long K): split-K, 32 weight tiles x 4 K parts
    assert _plan(256, 4096, 12288) == dict(bn=256, ctas=128, splits=4, wide=0, dp=0, ch=2)
    # tensor-parallel q/k/v shards at 256 tokens: 4 K parts over 64- / 128-token tiles
    assert _plan(256, 768, 4096) == dict(bn=64, ctas=96, splits=4, wide=0, dp=0, ch=2)
    assert _plan(256, 1536, 4096) == dict(bn=128, ctas=96, splits=4, wide=0, dp=0, ch=2)
    # one token: split-K with a 32-token tile, 3 K parts per weight tile
    assert _plan(1, 6144, 4096) == dict(bn=32, ctas=144, splits=3, wide=0, dp=0, ch=2)
    # prefill: 256-token tiles, whole tiles when they fill the SMs evenly
    p = _plan(8192, 4096, 4096)
    assert p["bn"] == 256 and p["dp"] == 1 and p["ctas"] == 148
    # K % 16 != 0: the CUDA-core kernel
    assert _plan(3, 70, 50)["bn"] == 0

    prev = lib.ms_set_pair_tiles(1)
    try:
        # decode, 256 tokens: qkv / o as 256 weight rows x 96 tokens on SM pairs, one wave each
        assert _plan(256, 6144, 4096) == dict(bn=96, ctas=144, splits=0, wide=0, dp=1, ch=2, pair=1)
        assert _plan(256, 4096, 4096) == dict(bn=96, ctas=96, splits=0, wide=0, dp=1, ch=2, pair=1)
        # gate_up: 96 tiles of 256 weight rows x 256 tokens on the 74 SM pairs
        assert _plan(256, 24576, 4096) == dict(bn=256, ctas=148, splits=0, wide=0, dp=1, ch=2, pair=1)
        # short K: one-SM tiles as before; down keeps split-K
        assert _plan(256, 4096, 1024) == dict(bn=64, ctas=128, splits=0, wide=0, dp=1, ch=2)
        assert _plan(256, 24576, 1024) == dict(bn=256, ctas=96, splits=0, wide=1, dp=1, ch=1)
        assert _plan(256, 4096, 12288) == dict(bn=256, ctas=128, splits=4, wide=0, dp=0, ch=2)
        # prefill: 256 x 256 tiles on SM pairs when they fill the pairs evenly (512 tiles, 6.9 waves)
        assert _plan(8192, 4096, 4096) == dict(bn=256, ctas=148, splits=0, wide=0, dp=1, ch=2, pair=1)
        assert _plan(8192, 24576, 4096)["pair"] == 1 and _plan(8192, 6144, 4096)["pair"] == 1
        # too few tiles for the pairs (64 tiles), or a long K: one-SM tiles
        assert "pair" not in _plan(1024, 4096, 4096) and "pair" not in _plan(8192, 4096, 12288)
    finally:
        lib.ms_set_pair_tiles(prev)


def test_pair_tile_schedules_are_opt_in():
    """Off by default: every shape has a one-SM schedule until ms_set_pair_tiles(1);
    turning it off again restores them."""
    from microserve_b200 import _lib
    lib = _lib.load()
    for M, N, K in ((256, 6144, 4096), (256, 24576, 4096), (8192, 4096, 4096)):
        assert "pair" not in _plan(M, N, K), (M, N, K)
    prev = lib.ms_set_pair_tiles(1)
    assert prev == 0
    try:
        assert _plan(256, 6144, 4096)["pair"] == 1
    finally:
        lib.ms_set_pair_tiles(0)
    assert "pair" not in _plan(256, 6144, 4096)


def test_gemm_schedules_keep_cooperating_ctas_resident():
    """Split-K and stream-K CTAs wait for one another, so those schedules never
    launch more CTAs than SMs; no K part is empty."""
    for sms in (132, 148):
        for M in (1, 16, 64, 100, 128, 160, 200, 256, 300, 1024, 4096):
            for N, K in ((768, 4096), (4096, 512), (6144, 4096), (4096, 12288), (24576, 4096), (1000, 1040)):
                p = _plan(M, N, K, sms)
                if not p["dp"]:
                    assert p["ctas"] <= sms, (M, N, K, sms, p)
                if p["splits"]:
                    steps = -(-K // (128 * p["ch"]))
                    assert 2 <= p["splits"] <= steps, (M, N, K, sms, p)
