"""Generate tests/golden/reference_gpu.pt by running the reference's own GPU
kernels (its Triton kernels and its flash-attn call) on a B200.

The reference package must be importable (installed offline into
baseline/_ref with pip --no-index --no-deps --target baseline/_ref); this
script is run once on a GPU box:

    PYTHONPATH=baseline/_ref python tests/golden/make_golden_gpu.py out.pt

Inputs are regenerated from fixed CPU seeds by tests/golden/gpu_cases.py, so
only the reference's outputs are stored. Nothing in the test suite, smoke()
or bench.py runs the reference; they read the committed file.
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

from tests.golden import gpu_cases as C  # noqa: E402


def main(out_path: str) -> None:
    from microserve.layers.fp8_chunk_prefill_attention import fp8_chunk_prefill_attention
    from microserve.layers.fp8_decode_attention import fp8_decode_attention
    from microserve.layers.fp8_kv_cache import store_fp8_kvcache
    from microserve.layers.fp8_linear import FP8DynamicLinear
    from microserve.layers.layernorm import RMSNorm
    from microserve.layers.linear import ReplicatedLinear

    dev = "cuda"
    out = {}

    # store_fp8_kvcache (layers/fp8_kv_cache.py)
    k, v, slots, nb = C.store_case()
    kc = torch.zeros(nb, C.BS, k.shape[1], C.D, dtype=torch.float8_e4m3fn, device=dev)
    vc = torch.zeros_like(kc)
    ks = torch.ones(nb, C.BS, k.shape[1], device=dev)
    vs = torch.ones_like(ks)
    store_fp8_kvcache(k.to(dev), v.to(dev), kc, vc, ks, vs, slots.to(dev))
    sl = slots.to(dev)
    out["store"] = dict(k_codes=kc.view(-1, k.shape[1], C.D)[sl].view(torch.uint8).cpu(),
                        v_codes=vc.view(-1, k.shape[1], C.D)[sl].view(torch.uint8).cpu(),
                        k_scale=ks.view(-1, k.shape[1])[sl].cpu(), v_scale=vs.view(-1, k.shape[1])[sl].cpu())

    # fp8_decode_attention (layers/fp8_decode_attention.py), the reference test's geometry
    caches, q, lens, bt = C.decode_case()
    caches = [c.to(dev) for c in caches]
    out["decode"] = fp8_decode_attention(q.to(dev), *caches, lens.to(dev), bt.to(dev), C.SCALE).cpu()

    # fp8_chunk_prefill_attention (layers/fp8_chunk_prefill_attention.py)
    caches, q, table, prefix = C.chunk_case()
    caches = [c.to(dev) for c in caches]
    out["chunk"] = fp8_chunk_prefill_attention(q.to(dev), *caches, table.to(dev), prefix, C.SCALE).cpu()

    # FP8DynamicLinear forward (layers/fp8_linear.py: _quantize_fp8_rows + _fp8_mm)
    w, x = C.linear_case()
    lin = ReplicatedLinear(w.shape[1], w.shape[0]).half().to(dev)
    with torch.no_grad():
        lin.weight.copy_(w.to(dev))
    q8 = FP8DynamicLinear(lin)
    out["linear"] = dict(y=q8(x.to(dev)).cpu(), w_codes=q8.weight_fp8.view(torch.uint8).cpu(),
                         w_scale=q8.weight_scale.cpu())

    # fused residual RMSNorm (layers/layernorm.py Triton kernels)
    x, r, wn = C.rmsnorm_case()
    norm = RMSNorm(x.shape[1], use_triton=True).half().to(dev)
    with torch.no_grad():
        norm.weight.copy_(wn.to(dev))
    y, rr = norm(x.to(dev), r.to(dev))
    out["rmsnorm"] = dict(y=y.cpu(), residual_out=rr.cpu(), y_nores=norm(x.to(dev)).cpu())

    # first-chunk prefill: flash_attn_varlen_func on fresh q, k, v (layers/attention.py:49-55)
    try:
        from flash_attn import flash_attn_varlen_func
        q, k, v, cu = C.varlen_case()
        o = flash_attn_varlen_func(q.to(dev), k.to(dev), v.to(dev), cu_seqlens_q=cu.to(dev), cu_seqlens_k=cu.to(dev),
                                   max_seqlen_q=int((cu[1:] - cu[:-1]).max()),
                                   max_seqlen_k=int((cu[1:] - cu[:-1]).max()), softmax_scale=C.SCALE, causal=True)
        out["varlen"] = o.cpu()
    except Exception as ex:  # recorded, not fatal: the restatement then stands alone
        out["varlen_error"] = f"{type(ex).__name__}: {ex}"[:300]

    out["meta"] = dict(torch=str(torch.__version__), device=torch.cuda.get_device_name(),
                       triton=str(__import__("triton").__version__))
    torch.save(out, out_path)
    print("wrote", out_path, {k: (v if isinstance(v, str) else type(v).__name__) for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "reference_gpu.pt")
