"""Parity of every CUDA kernel (through the C ABI) with the CPU oracle.

Tolerances: bit-exact for FP8 codes, scales, the residual stream and every
integer; the reference's own test tolerances elsewhere
(tests/test_fp8.py: 0.002 for the 50->70 GEMM; tests/test_fp8_kv_attention.py:
0.004 decode, 0.006 chunk prefill; tests/test_fused_rmsnorm.py: 1e-3).
"""
import math

import pytest
import torch

from oracle import fp8_decoder as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib_loaded():
    from microserve_b200 import _lib
    _lib.load()
    yield
    assert _lib.device_status() == 0, "a kernel recorded a timeout"


def _codes(t):
    return t.view(torch.uint8)


# ------------------------------------------------------------------ quantisation
@pytest.mark.parametrize("shape", [(1, 50), (3, 50), (17, 50), (16, 1024), (256, 4096), (7, 12288), (2, 25600)])
def test_quantize_rows_bit_exact(shape):
    from microserve_b200 import kernels
    torch.manual_seed(0)
    x = torch.randn(shape, dtype=torch.float16) * 3
    x[0].zero_()  # all-zero row -> scale 1e-8 / 448
    x[-1, ::7] = -0.0  # negative zeros encode as 0x80
    q, s = kernels.quantize_rows_fp8(x.to(DEV))
    qr, sr = O.quantize_rows(x)
    assert torch.equal(s.cpu(), sr)
    assert torch.equal(_codes(q.cpu()), _codes(qr))


def test_weight_quant_matches_reference_formula():
    from microserve_b200.layers.fp8_linear import FP8DynamicLinear
    from microserve_b200.layers.linear import ReplicatedLinear
    torch.manual_seed(0)
    fp = ReplicatedLinear(50, 70).half()
    with torch.no_grad():
        fp.weight.normal_(0, 0.02)
    wq_ref, sw_ref = O.quantize_weight(fp.weight.float())
    q = FP8DynamicLinear(fp.cuda())
    assert torch.equal(q.weight_scale.cpu(), sw_ref)
    assert torch.equal(_codes(q.weight_fp8.cpu()), _codes(wq_ref))


# ------------------------------------------------------------------ GEMM
def test_fp8_linear_reference_case():
    """The reference's own FP8 GEMM check (tests/test_fp8.py:12-29)."""
    from microserve_b200.layers.fp8_linear import FP8DynamicLinear
    from microserve_b200.layers.linear import ReplicatedLinear
    torch.manual_seed(0)
    fp = ReplicatedLinear(50, 70).half().cuda()
    with torch.no_grad():
        fp.weight.normal_(0, 0.02)
    quant = FP8DynamicLinear(fp)
    for m in (1, 3, 17):
        x = torch.randn(m, 50, device=DEV, dtype=torch.float16)
        if m == 3:
            x[0].zero_()
        actual = quant(x)
        assert torch.isfinite(actual).all()
        assert (torch.nn.functional.linear(x, fp.weight) - actual).abs().max().item() < 0.1
        xq, sx = O.quantize_rows(x.cpu())
        ref = O.fp8_gemm(xq, sx, quant.weight_fp8.cpu(), quant.weight_scale.cpu())
        assert (ref - actual.cpu()).abs().max().item() < 0.002


GEMM_SHAPES = [
    (1, 6144, 4096), (16, 4096, 4096), (64, 24576, 1024), (100, 1024, 3072), (256, 6144, 4096),
    (256, 4096, 12288), (256, 5120, 3200), (300, 2048, 1024), (1024, 4096, 4096), (4096, 6144, 4096),
    (8, 4096, 512), (33, 96, 160),
    # token tiles of 96 / 192 columns, an odd number of 128-byte K chunks, K % 128 != 0
    (96, 4096, 4096), (150, 2048, 4096), (200, 384, 1280), (256, 1024, 1040), (129, 640, 4224),
    # 256-row x 256-token tiles (129..256 tokens, more 128-row weight tiles than SMs), ragged last tile;
    # the 8B gate/up projection first; (160, 40000, 640) deals two tiles to some CTAs
    (256, 24576, 4096), (256, 24576, 1024), (200, 19000, 512), (160, 40000, 640), (129, 24576, 272),
    # tensor-parallel shards: few weight tiles at 256 tokens (split-K over 64- and 128-token tiles, a ragged
    # last token tile, and one 256-token tile in 8 parts)
    (256, 768, 4096), (256, 1536, 4096), (200, 768, 4096), (129, 1536, 2048), (256, 768, 2048), (256, 4096, 512),
    # 129..256 tokens dealt as 64- / 96-token tiles (o and qkv projections at 256 tokens, a ragged last tile)
    (256, 4096, 4096), (160, 4096, 2048),
    # N % 8 != 0: rows of y not 16-byte aligned, so the last tile is stored directly (no bulk store)
    (64, 1001, 512), (256, 6150, 1024), (200, 19001, 512), (700, 1003, 1024),
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_fp8_gemm_vs_oracle(M, N, K):
    from microserve_b200 import kernels
    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).half()
    w = (torch.randn(N, K, generator=g) * 0.02).half()
    xq, sx = O.quantize_rows(x)
    wq, sw = O.quantize_weight(w)
    y = kernels.fp8_gemm(xq.to(DEV), sx.to(DEV), wq.to(DEV), sw.to(DEV)).cpu()
    ref = O.fp8_gemm(xq, sx, wq, sw)
    # identical products, fp32 sums in a different order: within 2 fp16 ulps of the magnitude
    tol = 2e-3 * max(1.0, ref.abs().max().item())
    err = (y.float() - ref.float()).abs().max().item()
    assert err <= tol, (err, tol)
    assert O.rel_l2(y, ref) < 1e-3


def test_fp8_gemm_sequence_no_stale_state():
    """Shapes whose weight tiles are split over several CTAs along K (fewer steps
    than spare SMs), run back to back with fresh data after other GEMM kernels:
    every K part must be computed in the current call (tensor memory and the
    workspace keep values between kernels)."""
    from microserve_b200 import kernels
    shapes = [(33, 96, 256), (33, 96, 160), (8, 4096, 512), (33, 128, 160), (64, 96, 160), (33, 96, 288),
              (256, 4096, 4096), (33, 96, 160), (256, 24576, 1024), (1, 4096, 4096), (200, 19000, 512),
              (33, 96, 1040)]
    for i, (M, N, K) in enumerate(shapes):
        g = torch.Generator().manual_seed(1000 + i)
        x = torch.randn(M, K, generator=g).half()
        w = (torch.randn(N, K, generator=g) * 0.02).half()
        xq, sx = O.quantize_rows(x)
        wq, sw = O.quantize_weight(w)
        y = kernels.fp8_gemm(xq.to(DEV), sx.to(DEV), wq.to(DEV), sw.to(DEV)).cpu()
        ref = O.fp8_gemm(xq, sx, wq, sw)
        tol = 2e-3 * max(1.0, ref.abs().max().item())
        assert (y.float() - ref.float()).abs().max().item() <= tol, (M, N, K)


PAIR_GEMM_SHAPES = [
    # prefill-sized tiles on SM pairs (tcgen05 cta_group::2, 256 x 256 per pair): 2-chunk stages; ragged M,
    # N and K % 128 != 0 (1-chunk stages); 96 weight tiles; one K step per tile
    (8192, 4096, 4096), (8000, 4000, 1040), (2048, 24576, 1024), (4096, 9472, 256),
    # 129..256 tokens: 256 weight rows x 96 tokens (qkv / o; a ragged token tile), 256 x 256 over all pairs
    (256, 6144, 4096), (200, 4096, 2048), (256, 24576, 4096),
]


@pytest.mark.parametrize("M,N,K", PAIR_GEMM_SHAPES)
def test_fp8_gemm_on_sm_pairs(M, N, K):
    """Shapes the planner gives to the SM-pair kernel, against an fp32 product of the
    dequantised operands on the GPU (the oracle's arithmetic: exact products, fp32
    sums, per-row x per-channel scales); with a bias on the first shape."""
    import ctypes as C
    from microserve_b200 import _lib, kernels
    lib = _lib.load()
    prev = lib.ms_set_pair_tiles(1)
    try:
        plan = (C.c_int * 7)()
        assert lib.ms_fp8_gemm_plan(M, N, K, torch.cuda.get_device_properties(0).multi_processor_count,
                                    plan) == 0 and plan[6] == 1, list(plan)
        g = torch.Generator(device=DEV).manual_seed(M + N + K)
        xq, sx = kernels.quantize_rows_fp8(torch.randn(M, K, generator=g, device=DEV).half())
        wq, sw = kernels.quantize_rows_fp8((torch.randn(N, K, generator=g, device=DEV) * 0.02).half())
        bias = torch.randn(N, generator=g, device=DEV).half() if M == 8192 else None
        y = kernels.fp8_gemm(xq, sx, wq, sw, bias)
        torch.cuda.synchronize()
    finally:
        lib.ms_set_pair_tiles(prev)
    ref = (xq.float() @ wq.float().t()) * sx[:, None] * sw[None, :]
    if bias is not None:
        ref = ref.half().float() + bias.float()
    tol = 2e-3 * max(1.0, ref.abs().max().item())
    assert (y.float() - ref).abs().max().item() <= tol
    assert (y.float() - ref).norm().item() <= 1e-3 * ref.norm().item()


F16_GEMM_SHAPES = [
    # the LM head at 256 sequences: the full Qwen3 vocabulary, and its vocab-parallel shard at TP = 8
    (256, 151936, 4096), (256, 18992, 4096),
    # one and a few rows (decode of small batches), split-K shards, a prefill-sized M (stream-K / whole tiles),
    # prefill on SM pairs
    (1, 18992, 4096), (7, 1000, 64), (64, 24576, 1024), (256, 768, 4096), (300, 2048, 1024), (1024, 4096, 4096),
    (4096, 8192, 2048),
    # 256-row x 256-token tiles with a ragged last tile; N % 8 != 0 (no bulk store); K % 64 != 0
    (200, 19000, 512), (37, 1001, 520), (129, 24576, 272),
]


def test_f16_gemm_on_sm_pairs():
    """The LM head's fp16 GEMM with the SM-pair schedule on (256 x 256 tiles over all
    pairs; kind::f16 with cta_group::2) against an fp32 product."""
    from microserve_b200 import _lib, kernels
    lib = _lib.load()
    g = torch.Generator(device=DEV).manual_seed(11)
    for M, N, K in ((256, 151936, 4096), (4096, 8192, 2048)):
        x = torch.randn(M, K, generator=g, device=DEV).half()
        w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).half()
        prev = lib.ms_set_pair_tiles(1)
        try:
            y = kernels.f16_gemm(x, w)
            torch.cuda.synchronize()
        finally:
            lib.ms_set_pair_tiles(prev)
        ref = x.float() @ w.float().t()
        tol = 2e-3 * max(1.0, ref.abs().max().item())
        assert (y.float() - ref).abs().max().item() <= tol, (M, N, K)


@pytest.mark.parametrize("M,N,K", F16_GEMM_SHAPES)
def test_f16_gemm_vs_fp32(M, N, K):
    """The LM head's fp16 GEMM (ms_f16_gemm, kind::f16 on the tcgen05 kernels) against an
    fp32 product of the same fp16 operands, and against torch's F.linear (the reference's
    call, microserve/layers/embed_head.py:35-36)."""
    from microserve_b200 import kernels
    g = torch.Generator(device=DEV).manual_seed(M * 3 + N + K)
    x = torch.randn(M, K, generator=g, device=DEV).half()
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).half()
    y = kernels.f16_gemm(x, w)
    ref = x.float() @ w.float().t()
    # exact products, fp32 sums in another order, one rounding to fp16: within 2 fp16 ulps
    tol = 2e-3 * max(1.0, ref.abs().max().item())
    assert (y.float() - ref).abs().max().item() <= tol
    lin = torch.nn.functional.linear(x, w)
    assert (y.float() - lin.float()).abs().max().item() <= tol
    assert (y.float() - ref).norm().item() <= 1e-3 * ref.norm().item()


@pytest.mark.parametrize("M,N,K", [(5, 384, 256), (200, 19000, 256), (200, 19000, 512)])
def test_fp8_gemm_bias(M, N, K):
    from microserve_b200 import kernels
    torch.manual_seed(3)
    x = torch.randn(M, K).half()
    w = (torch.randn(N, K) * 0.05).half()
    b = torch.randn(N).half()
    xq, sx = O.quantize_rows(x)
    wq, sw = O.quantize_weight(w)
    y = kernels.fp8_gemm(xq.cuda(), sx.cuda(), wq.cuda(), sw.cuda(), b.cuda()).cpu()
    ref = O.fp8_gemm(xq, sx, wq, sw, b)
    assert (y.float() - ref.float()).abs().max().item() < 4e-3


# ------------------------------------------------------------------ RMSNorm / SiLU
@pytest.mark.parametrize("rows", [1, 17, 511])
def test_rmsnorm_reference_case(rows):
    """tests/test_fused_rmsnorm.py:6-24: residual bit-exact, output within 1e-3."""
    from microserve_b200.layers.layernorm import RMSNorm
    torch.manual_seed(0)
    x = torch.randn(rows, 1024, dtype=torch.float16)
    r = torch.randn_like(x)
    w = (1 + 0.1 * torch.randn(1024)).half()
    norm = RMSNorm(1024).half().cuda()
    norm.weight.data.copy_(w)
    y, rr = norm(x.cuda(), r.cuda())
    ey, er = O.rmsnorm(x, w, 1e-6, r)
    assert torch.equal(rr.cpu(), er)
    torch.testing.assert_close(y.cpu(), ey, atol=1e-3, rtol=1e-3)
    y0 = norm(x.cuda())
    torch.testing.assert_close(y0.cpu(), O.rmsnorm(x, w, 1e-6), atol=1e-3, rtol=1e-3)
    # FP8 epilogue == row quantisation of the kernel's own fp16 output
    yq, sy, rr2 = norm.forward_fp8(x.cuda(), r.cuda())
    q2, s2 = O.quantize_rows(y.cpu())
    assert torch.equal(sy.cpu(), s2) and torch.equal(_codes(yq.cpu()), _codes(q2))
    assert torch.equal(rr2.cpu(), er)


@pytest.mark.parametrize("M,I", [(1, 3072), (64, 12288), (9, 25600)])
def test_silu_mul(M, I):
    from microserve_b200 import kernels
    torch.manual_seed(1)
    gu = torch.randn(M, 2 * I, dtype=torch.float16) * 2
    out, aq, sa = kernels.silu_mul(gu.cuda(), want_fp16=True, want_fp8=True)
    ref = O.silu_mul(gu)
    torch.testing.assert_close(out.cpu(), ref, atol=2e-3, rtol=2e-3)
    q2, s2 = O.quantize_rows(out.cpu())
    assert torch.equal(sa.cpu(), s2) and torch.equal(_codes(aq.cpu()), _codes(q2))


# ------------------------------------------------------------------ KV cache
BS, HQ, HKV, D = 256, 16, 8, 128


def _alloc(nb, hkv=HKV):
    k = torch.zeros(nb, BS, hkv, D, dtype=torch.float8_e4m3fn)
    ks = torch.ones(nb, BS, hkv, dtype=torch.float32)
    return k, k.clone(), ks, ks.clone()


def test_store_kv_bit_exact():
    from microserve_b200.layers.fp8_kv_cache import store_fp8_kvcache
    torch.manual_seed(5)
    T = 300
    k = torch.randn(T, HKV, D, dtype=torch.float16) * 0.2
    v = torch.randn(T, HKV, D, dtype=torch.float16)
    k[3, 2].zero_()
    slots = torch.randperm(4 * BS)[:T].long()
    ref = _alloc(4)
    O.store_kv(k, v, *ref, slots)
    got = [t.cuda() for t in _alloc(4)]
    store_fp8_kvcache(k.cuda(), v.cuda(), *got, slots.cuda())
    for a, b in zip(got, ref):
        a = a.cpu()
        assert torch.equal(a.view(torch.uint8) if a.dtype == torch.float8_e4m3fn else a,
                           b.view(torch.uint8) if b.dtype == torch.float8_e4m3fn else b)


def test_qkv_post_norm_rope_store():
    from microserve_b200 import kernels
    from microserve_b200.layers.rotary_embedding import RotaryEmbedding
    torch.manual_seed(6)
    T, Hq, Hkv = 37, 32, 8
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, dtype=torch.float16)
    qw = (1 + 0.1 * torch.randn(D)).half()
    kw = (1 + 0.1 * torch.randn(D)).half()
    pos = torch.randint(0, 4000, (T,)).long()
    slots = torch.randperm(2 * BS)[:T].long()
    rope = RotaryEmbedding(D, D, 4096, 1e6).cuda()
    caches = [t.cuda() for t in _alloc(2, Hkv)]
    q, k, v = kernels.qkv_post(qkv.cuda(), Hq, Hkv, D, pos.cuda(), rope.cos_half16, rope.sin_half16, qw.cuda(),
                               kw.cuda(), 1e-6, slots.cuda(), caches, want_kv=True)
    cos, sin = O.rope_tables(D, 4096, 1e6)
    rq, rk, rv = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    rq = O.rmsnorm(rq.reshape(T, Hq, D), qw, 1e-6)
    rk = O.rmsnorm(rk.reshape(T, Hkv, D), kw, 1e-6)
    rq, rk = O.rope(pos, rq, rk, cos, sin)
    torch.testing.assert_close(q.cpu(), rq, atol=4e-3, rtol=4e-3)
    torch.testing.assert_close(k.cpu(), rk, atol=4e-3, rtol=4e-3)
    assert torch.equal(v.cpu(), rv.reshape(T, Hkv, D))
    ref = _alloc(2, Hkv)
    O.store_kv(k.cpu(), v.cpu(), *ref, slots)  # store of the kernel's own k/v: bit-exact
    for a, b in zip(caches, ref):
        a = a.cpu()
        if a.dtype == torch.float8_e4m3fn:
            a, b = a.view(torch.uint8), b.view(torch.uint8)
        assert torch.equal(a, b)


def test_rope_no_norm_matches_reference_math():
    from microserve_b200.layers.rotary_embedding import RotaryEmbedding
    torch.manual_seed(7)
    T, Hq, Hkv = 9, 16, 8
    q = torch.randn(T, Hq, D, dtype=torch.float16)
    k = torch.randn(T, Hkv, D, dtype=torch.float16)
    pos = torch.randint(0, 30000, (T,)).long()
    rope = RotaryEmbedding(D, D, 32768, 1e6).cuda()
    gq, gk = rope(pos.cuda(), q.cuda(), k.cuda())
    cos, sin = O.rope_tables(D, 32768, 1e6)
    rq, rk = O.rope(pos, q, k, cos, sin)
    assert torch.equal(gq.cpu(), rq) and torch.equal(gk.cpu(), rk)  # fp16 ops, identical rounding


# ------------------------------------------------------------------ attention
def _fill_cache(lengths, tables, hkv=HKV, nb=None, seed=1, scale=0.2):
    torch.manual_seed(seed)
    nb = nb or (max(max(t) for t in tables) + 1)
    caches = _alloc(nb, hkv)
    keys, vals, slots = [], [], []
    for b, L in enumerate(lengths):
        keys.append(torch.randn(L, hkv, D, dtype=torch.float16) * scale)
        vals.append(torch.randn(L, hkv, D, dtype=torch.float16) * scale)
        slots += O.slot_mapping(tables[b], list(range(L)), BS)
    O.store_kv(torch.cat(keys), torch.cat(vals), *caches, torch.tensor(slots))
    return caches


@pytest.mark.parametrize("lengths,hq,hkv,tables", [
    ([38, 301, 514], 16, 8, [[0], [1, 2], [3, 4, 5]]),
    ([301, 701], 16, 8, [[0, 1], [2, 3, 4]]),
    ([600, 900, 3], 32, 8, [[5, 1, 0], [2, 3, 4, 6], [7]]),
])
def test_decode_attention_fixed_tables(lengths, hq, hkv, tables):
    from microserve_b200.layers.fp8_decode_attention import fp8_decode_attention
    caches = _fill_cache(lengths, tables, hkv=hkv, seed=13, scale=0.8)
    bt = O.block_table_rows(tables)
    torch.manual_seed(10)
    q = torch.randn(len(lengths), hq, D, dtype=torch.float16)
    got = fp8_decode_attention(q.cuda(), *[c.cuda() for c in caches], torch.tensor(lengths, dtype=torch.int32).cuda(),
                               bt.cuda(), D ** -0.5).cpu()
    ref = O.decode_attention(q, *caches, torch.tensor(lengths), bt, D ** -0.5)
    for b in range(len(lengths)):
        assert O.rel_l2(got[b], ref[b]) < 1e-3, (b, O.rel_l2(got[b], ref[b]))
    # fp32-level accuracy (the reference decode kernel is all-fp32): against an fp64
    # evaluation, outputs are the correctly rounded fp16 value or 1 ulp off, rarely.
    head_map = torch.arange(hq) // (hq // hkv)
    for b, L in enumerate(lengths):
        kk = O.gather_kv(caches[0], caches[2], bt[b], L)[:, head_map].double()
        vv = O.gather_kv(caches[1], caches[3], bt[b], L)[:, head_map].double()
        sc = torch.einsum("hd,lhd->hl", q[b].double(), kk) * D ** -0.5
        exact = torch.einsum("hl,lhd->hd", sc.softmax(-1), vv)
        rounded = exact.half()
        ulp = (rounded.float().abs() * 2.0 ** -10).clamp_min(2.0 ** -24)
        err = (got[b].float() - exact.float()).abs()
        assert (err <= ulp).all(), (b, (err / ulp).max().item())
        assert (got[b] != rounded).float().mean().item() < 0.02, (b, (got[b] != rounded).float().mean().item())


@pytest.mark.parametrize("lengths,hq,hkv", [
    ([1, 73, 300], 16, 8),            # tests/test_fp8_kv_attention.py:39-73
    ([0, 5, 256, 257, 1000], 32, 8),  # empty row, page edges
    ([2047, 33, 512, 1], 64, 8),      # G = 8
    ([8000], 32, 8),                  # one long sequence: context split + merge
    ([4100, 17], 16, 2),
])
def test_decode_attention(lengths, hq, hkv):
    from microserve_b200.layers.fp8_decode_attention import fp8_decode_attention
    nblk = [max(1, (L + BS - 1) // BS) for L in lengths]
    perm = torch.randperm(sum(nblk), generator=torch.Generator().manual_seed(4)).tolist()
    tables, o = [], 0
    for n in nblk:
        tables.append(perm[o:o + n])
        o += n
    caches = _fill_cache(lengths, tables, hkv=hkv)
    bt = O.block_table_rows(tables)
    torch.manual_seed(9)
    q = torch.randn(len(lengths), hq, D, dtype=torch.float16) * 0.2
    scale = D ** -0.5
    got = fp8_decode_attention(q.cuda(), *[c.cuda() for c in caches], torch.tensor(lengths, dtype=torch.int32).cuda(),
                               bt.cuda(), scale).cpu()
    ref = O.decode_attention(q, *caches, torch.tensor(lengths), bt, scale)
    assert torch.isfinite(got).all()
    err = (got.float() - ref.float()).abs().max().item()
    assert err < 0.004, err
    for b, L in enumerate(lengths):
        if L == 0:
            assert torch.all(got[b] == 0)


def test_chunk_prefill_reference_case():
    """tests/test_fp8_kv_attention.py:76-108: prefix 273 + 31 queries, table [1, 0]."""
    from microserve_b200.layers.fp8_chunk_prefill_attention import fp8_chunk_prefill_attention
    torch.manual_seed(2)
    prefix, ql = 273, 31
    total = prefix + ql
    table = torch.tensor([[1, 0]], dtype=torch.int32)
    caches = _alloc(2)
    key = torch.randn(total, HKV, D, dtype=torch.float16) * 0.2
    value = torch.randn_like(key)
    slots = torch.tensor(O.slot_mapping([1, 0], list(range(total)), BS))
    O.store_kv(key, value, *caches, slots)
    q = torch.randn(ql, HQ, D, dtype=torch.float16) * 0.2
    got = fp8_chunk_prefill_attention(q.cuda(), *[c.cuda() for c in caches], table.cuda(), prefix,
                                      D ** -0.5).cpu()
    ref = O.chunk_prefill_attention(q, *caches, table[0], prefix, D ** -0.5)
    assert torch.isfinite(got).all()
    assert (got.float() - ref.float()).abs().max().item() < 0.006


@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8), (64, 8)])
def test_chunk_prefill_multi_sequence(hq, hkv):
    from microserve_b200.layers.fp8_chunk_prefill_attention import fp8_varlen_chunk_prefill_attention
    seqs = [(273, 31), (0, 64), (500, 1), (256, 200)]  # (prefix, query) per sequence
    tables, nb = [], 0
    for p, qn in seqs:
        n = (p + qn + BS - 1) // BS
        tables.append(list(range(nb, nb + n))[::-1])
        nb += n
    caches = _fill_cache([p + qn for p, qn in seqs], tables, hkv=hkv, nb=nb, seed=3)
    torch.manual_seed(8)
    qs = [torch.randn(qn, hq, D, dtype=torch.float16) * 0.2 for _, qn in seqs]
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([qn for _, qn in seqs]), 0)), dtype=torch.int32)
    kv = torch.tensor([p + qn for p, qn in seqs], dtype=torch.int32)
    bt = O.block_table_rows(tables)
    got = fp8_varlen_chunk_prefill_attention(torch.cat(qs).cuda(), *[c.cuda() for c in caches], bt.cuda(),
                                             cu.cuda(), kv.cuda(), D ** -0.5).cpu()
    for i, (p, qn) in enumerate(seqs):
        ref = O.chunk_prefill_attention(qs[i], *caches, bt[i], p, D ** -0.5)
        err = (got[cu[i]:cu[i + 1]].float() - ref.float()).abs().max().item()
        assert err < 0.006, (i, err)


def test_varlen_prefill_fresh_kv():
    from microserve_b200 import kernels
    torch.manual_seed(11)
    lens = [1, 31, 64, 200, 5]
    T = sum(lens)
    q = torch.randn(T, 32, D, dtype=torch.float16) * 0.5
    k = torch.randn(T, 8, D, dtype=torch.float16) * 0.5
    v = torch.randn(T, 8, D, dtype=torch.float16)
    cu = torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist(), dtype=torch.int32)
    got = kernels.varlen_prefill(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), D ** -0.5).cpu()
    ref = O.varlen_prefill(q, k, v, cu, D ** -0.5)
    assert (got.float() - ref.float()).abs().max().item() < 0.006


# ------------------------------------------------------------------ greedy sampling
@pytest.mark.parametrize("M,V,pad", [(257, 151936, 0), (3, 1001, 7), (64, 75968, 0)])
def test_argmax_rows_matches_torch(M, V, pad):
    """Greedy pick of `_sample` (model_runner.py:33-34): torch.argmax semantics, incl.
    first index on ties, NaN counted as the maximum and -0.0 == +0.0."""
    from microserve_b200 import kernels
    g = torch.Generator().manual_seed(M + V)
    full = (torch.randn(M, V + pad, generator=g) * 4).half()
    x = full[:, :V]
    x[0, 5] = x[0, 900] = 60.0            # tie: first index wins
    x[1].fill_(-1.0)
    x[1, 17] = float("nan")               # NaN is the maximum
    x[2].fill_(-1.0)
    x[2, 3] = -0.0
    x[2, 4] = 0.0                         # -0.0 == +0.0: index 3
    if M > 3:
        x[3].fill_(float("-inf"))         # all -inf: index 0
    xd = full.cuda()[:, :V]
    idx, vmax = kernels.argmax_rows(xd, want_max=True)
    ref = x.float().argmax(dim=-1)
    assert torch.equal(idx.cpu(), ref)
    vm = vmax.cpu()
    exp = x.float().gather(1, ref[:, None]).squeeze(1)
    assert torch.equal(torch.isnan(vm), torch.isnan(exp))
    ok = ~torch.isnan(exp)
    assert torch.equal(vm[ok], exp[ok])
    # a second call reuses the (self-resetting) workspace counters
    assert torch.equal(kernels.argmax_rows(xd).cpu(), ref)
