"""Generate tests/golden/reference_engine.pt by running the reference's own engine
(microserve.engine.llm.LLMEngine: its Triton FP8 kernels, flash-attn prefill,
eager and CUDA-graph decode) on the seeded synthetic checkpoints of
tests/golden/engine_case.py, greedily, on a B200.

The reference package must be importable (installed offline into baseline/_ref
with pip --no-index --no-deps --target baseline/_ref); run once on a GPU box:

    PYTHONPATH=baseline/_ref:. python tests/golden/make_golden_engine.py OUT.pt SCRATCH_DIR

Recorded per case and decode mode: every sequence's greedy tokens; for the small
case also the logits row each token was taken from (fp16, the reference's own
`_sample` input, microserve/engine/model_runner.py:15-34), for the 0.6B case the
two largest logits of each row. The CPU oracle is also run on each checkpoint
along the reference's token path, and its per-step distance to the reference is
stored: the measured spread between two implementations of the same FP8
arithmetic. Nothing in the test suite, smoke() or bench.py runs the
reference; they read the committed file.
"""
from __future__ import annotations

import shutil
import sys
import time

import torch


def run_reference(case: str, path: str, eager: bool) -> dict:
    import microserve.engine.model_runner as mr
    from microserve.Config import Config
    from microserve.engine.llm import LLMEngine
    from microserve.engine.sequence import SamplingParams
    from tests.golden.engine_case import CASES, ENGINE_KW, prompts

    c = CASES[case]
    seen: dict[int, list] = {}
    original = mr._sample

    def spy(logits, seq):
        token = original(logits, seq)
        seen.setdefault(seq.seq_id, []).append(logits.detach().half().cpu())
        return token

    mr._sample = spy
    try:
        eng = LLMEngine(Config(model_dir=path, enforce_eager=eager, **ENGINE_KW))
        seqs = [eng.add(p, SamplingParams(temperature=0.0), max_tokens=c["steps"]) for p in prompts(case)]
        t0 = time.perf_counter()
        while not eng.is_idle():
            eng.step()
        torch.cuda.synchronize()
        out = {"tokens": [s.completion_token_ids for s in seqs], "seconds": time.perf_counter() - t0}
        # [seqs, steps, V]; kept in the file for the small case only (the 0.6B case keeps
        # the two largest logits of every step: how close each greedy choice was to a tie)
        out["logits"] = torch.stack([torch.stack(seen[s.seq_id]) for s in seqs])
        out["top2"] = out["logits"].float().topk(2, dim=-1).values
        del eng
    finally:
        mr._sample = original
    torch.cuda.empty_cache()
    return out


def oracle_logits(case: str, path: str, forced: list[list[int]]) -> list[torch.Tensor]:
    """The CPU oracle (oracle/fp8_decoder.py) on the same checkpoint and prompts, fed the
    reference's tokens: the logits row of every step, per sequence."""
    from safetensors.torch import load_file
    from oracle import fp8_decoder as O
    from tests.golden.engine_case import CASES, hf_config, prompts
    cfg = hf_config(case)
    w = load_file(f"{path}/model.safetensors")
    L, H, D, Hq, Hkv = cfg.num_hidden_layers, cfg.hidden_size, 128, 16, 8
    layers = []
    for i in range(L):
        p = f"model.layers.{i}."
        qkv = torch.cat([w[p + f"self_attn.{n}_proj.weight"] for n in "qkv"])
        gu = torch.cat([w[p + "mlp.gate_proj.weight"], w[p + "mlp.up_proj.weight"]])
        layers.append(O.LayerWeights(O.quantize_weight(qkv), O.quantize_weight(w[p + "self_attn.o_proj.weight"]),
                                     O.quantize_weight(gu), O.quantize_weight(w[p + "mlp.down_proj.weight"]),
                                     w[p + "input_layernorm.weight"], w[p + "post_attention_layernorm.weight"],
                                     w[p + "self_attn.q_norm.weight"], w[p + "self_attn.k_norm.weight"]))
    embed, final_norm = w["model.embed_tokens.weight"], w["model.norm.weight"]
    cos, sin = O.rope_tables(D, 4096, 1e6)
    bs = 256
    ps = prompts(case)
    steps = CASES[case]["steps"]
    tables = [[2 * i, 2 * i + 1] for i in range(len(ps))]
    caches = [[torch.zeros(2 * len(ps), bs, Hkv, D, dtype=torch.float8_e4m3fn),
               torch.zeros(2 * len(ps), bs, Hkv, D, dtype=torch.float8_e4m3fn),
               torch.ones(2 * len(ps), bs, Hkv), torch.ones(2 * len(ps), bs, Hkv)] for _ in range(L)]

    def forward(ids, pos, slots, **kw):
        h, res = torch.nn.functional.embedding(ids, embed), None
        for lw, c in zip(layers, caches):
            h, res = O.decoder_layer(lw, pos, h, res, Hq=Hq, Hkv=Hkv, D=D, eps=1e-6, cos_cache=cos, sin_cache=sin,
                                     caches=c, slots=slots, **kw)
        h = O.rmsnorm(h, final_norm, 1e-6, res)[0]
        return (h.float() @ embed.float().T).half()

    ids = torch.tensor([t for p in ps for t in p])
    pos = torch.cat([torch.arange(len(p)) for p in ps])
    slots = torch.tensor([v for t, p in zip(tables, ps) for v in O.slot_mapping(t, list(range(len(p))), bs)])
    cu = torch.tensor([0] + [sum(len(p) for p in ps[:i + 1]) for i in range(len(ps))])
    out = [[row] for row in forward(ids, pos, slots, mode="prefill", cu=cu)[cu[1:] - 1]]
    bt = O.block_table_rows(tables)
    for k in range(1, steps):
        pos = torch.tensor([len(p) + k - 1 for p in ps])
        ids = torch.tensor([f[k - 1] for f in forced])
        slots = torch.tensor([t[q // bs] * bs + q % bs for t, q in zip(tables, pos.tolist())])
        rows = forward(ids, pos, slots, mode="decode", seqlens=pos + 1, block_tables=bt)
        for s in range(len(ps)):
            out[s].append(rows[s])
    return [torch.stack(o) for o in out]


def main(out_path: str, scratch: str) -> None:
    from tests.golden.engine_case import CASES, write_checkpoint
    result: dict = {"meta": {"torch": torch.__version__, "gpu": torch.cuda.get_device_name(0)}}
    for case in CASES:
        path = write_checkpoint(case, f"{scratch}/{case}")
        runs = {mode: run_reference(case, path, eager=(mode == "eager")) for mode in ("eager", "graph")}
        agree = [sum(a == b for a, b in zip(x, y)) / len(x)
                 for x, y in zip(runs["eager"]["tokens"], runs["graph"]["tokens"])]
        result[case] = runs
        result["meta"][f"{case}_eager_vs_graph_token_agreement"] = agree
        print(case, "eager vs graph token agreement", agree, flush=True)
        # how far the oracle (CPU restatement) is from the reference engine on the same path
        ref = runs["eager"]["logits"].float()
        orc = torch.stack(oracle_logits(case, path, runs["eager"]["tokens"])).float()
        rel = ((orc - ref).norm(dim=-1) / ref.norm(dim=-1))  # [seqs, steps]
        top2 = ref.topk(2, dim=-1).values
        result["meta"][f"{case}_oracle_vs_reference"] = {
            "rel_l2_per_step": rel, "max_abs_diff_per_step": (orc - ref).abs().amax(-1),
            "argmax_agree": (orc.argmax(-1) == ref.argmax(-1)).float().mean().item(),
            "reference_top1_margin": top2[..., 0] - top2[..., 1]}
        print(case, "oracle vs reference: max rel-L2", rel.max().item(), "median", rel.median().item(),
              "argmax agreement", result["meta"][f"{case}_oracle_vs_reference"]["argmax_agree"], flush=True)
        if not CASES[case]["logits"]:
            for mode in runs:
                del runs[mode]["logits"]
        shutil.rmtree(path, ignore_errors=True)
    torch.save(result, out_path)
    print("wrote", out_path)


if __name__ == "__main__":
    if len(sys.argv) < 3:
        sys.exit("usage: PYTHONPATH=baseline/_ref:. python tests/golden/make_golden_engine.py OUT.pt SCRATCH_DIR")
    main(sys.argv[1], sys.argv[2])
