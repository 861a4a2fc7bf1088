"""The torch.library ops (microserve_b200/library.py) without a GPU: every op
is registered, its fake implementation gives the output shapes and dtypes of the
CUDA kernel's outputs, and a decoder-layer slice traces (make_fx, fake tensors)
into a graph whose nodes are these ops."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import microserve_b200.library as L

ops = torch.ops.microserve_b200
FP8 = torch.float8_e4m3fn
M, H, I, HQ, HKV, D, NB, BS = 16, 1024, 3072, 16, 8, 128, 6, 256


def _cuda(*shape, dtype=torch.float16):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def test_every_op_is_registered():
    for name in L.OPS:
        assert hasattr(ops, name), name


def test_fake_outputs_match_the_kernels_shapes():
    with FakeTensorMode():
        x = _cuda(M, H)
        xq, sx = ops.quantize_rows_fp8(x)
        assert (xq.shape, xq.dtype, sx.shape, sx.dtype) == ((M, H), FP8, (M,), torch.float32)
        wq, sw = _cuda(3 * H, H, dtype=FP8), _cuda(3 * H, dtype=torch.float32)
        y = ops.fp8_gemm(xq, sx, wq, sw, None)
        assert (y.shape, y.dtype, y.device.type) == ((M, 3 * H), torch.float16, "cuda")
        w = _cuda(H)
        assert ops.rmsnorm(x, w, 1e-6).shape == (M, H)
        yy, rr = ops.add_rmsnorm(x, x, w, 1e-6)
        assert yy.shape == rr.shape == (M, H)
        yq, sy = ops.rmsnorm_fp8(x, w, 1e-6)
        assert (yq.dtype, sy.shape) == (FP8, (M,))
        yq, sy, rr = ops.add_rmsnorm_fp8(x, x, w, 1e-6)
        assert (yq.shape, yq.dtype, sy.shape, rr.shape) == ((M, H), FP8, (M,), (M, H))
        gu = _cuda(M, 2 * I)
        assert ops.silu_mul(gu).shape == (M, I)
        aq, sa = ops.silu_mul_fp8(gu)
        assert (aq.shape, aq.dtype, sa.shape) == ((M, I), FP8, (M,))

        kc, vc = _cuda(NB, BS, HKV, D, dtype=FP8), _cuda(NB, BS, HKV, D, dtype=FP8)
        ks, vs = _cuda(NB, BS, HKV, dtype=torch.float32), _cuda(NB, BS, HKV, dtype=torch.float32)
        slots = _cuda(M, dtype=torch.int64)
        assert ops.store_kv_fp8(_cuda(M, HKV, D), _cuda(M, HKV, D), kc, vc, ks, vs, slots) is None
        qkv = _cuda(M, (HQ + 2 * HKV) * D)
        pos = _cuda(M, dtype=torch.int64)
        cos, sin = _cuda(4096, D // 2), _cuda(4096, D // 2)
        qn, kn = _cuda(D), _cuda(D)
        q = ops.qkv_post_decode(qkv, pos, cos, sin, qn, kn, slots, kc, vc, ks, vs, HQ, HKV, D, 1e-6)
        assert q.shape == (M, HQ, D)
        q, k, v = ops.qkv_post_prefill(qkv, pos, cos, sin, None, None, slots, kc, vc, ks, vs, HQ, HKV, D, 1e-6)
        assert (q.shape, k.shape, v.shape) == ((M, HQ, D), (M, HKV, D), (M, HKV, D))

        B = 4
        qd = _cuda(B, HQ, D)
        o = ops.paged_decode_fp8(qd, kc, vc, ks, vs, _cuda(B, dtype=torch.int32), _cuda(B, 3, dtype=torch.int32),
                                 D ** -0.5)
        assert (o.shape, o.dtype) == ((B, HQ, D), torch.float16)
        qp = _cuda(M, HQ, D)
        o = ops.paged_prefill_fp8(qp, kc, vc, ks, vs, _cuda(2, 3, dtype=torch.int32), _cuda(3, dtype=torch.int32),
                                  _cuda(2, dtype=torch.int32), D ** -0.5)
        assert o.shape == (M, HQ, D)
        o = ops.varlen_prefill(qp, _cuda(M, HKV, D), _cuda(M, HKV, D), _cuda(3, dtype=torch.int32), D ** -0.5)
        assert o.shape == (M, HQ, D)
        idx = ops.argmax_rows(_cuda(M, 151936))
        assert (idx.shape, idx.dtype) == ((M,), torch.int64)


def test_decoder_layer_slice_traces_into_library_ops():
    """norm -> QKV GEMM -> ... -> MLP, traced with fake tensors: the graph holds the
    library's ops (opaque to the tracer) with the kernels' output shapes."""
    def mlp_block(hidden, residual, norm_w, wq_gu, sw_gu, wq_down, sw_down):
        xq, sx, residual = ops.add_rmsnorm_fp8(hidden, residual, norm_w, 1e-6)
        gu = ops.fp8_gemm(xq, sx, wq_gu, sw_gu, None)
        aq, sa = ops.silu_mul_fp8(gu)
        return ops.fp8_gemm(aq, sa, wq_down, sw_down, None), residual

    with FakeTensorMode():
        args = (_cuda(M, H), _cuda(M, H), _cuda(H), _cuda(2 * I, H, dtype=FP8), _cuda(2 * I, dtype=torch.float32),
                _cuda(H, I, dtype=FP8), _cuda(H, dtype=torch.float32))
        gm = make_fx(mlp_block, tracing_mode="fake")(*args)
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert sum("microserve_b200.fp8_gemm" in t for t in targets) == 2, targets
    assert any("add_rmsnorm_fp8" in t for t in targets) and any("silu_mul_fp8" in t for t in targets), targets
    outs = [n for n in gm.graph.nodes if n.op == "output"][0].args[0]
    assert tuple(outs[0].meta["val"].shape) == (M, H)
