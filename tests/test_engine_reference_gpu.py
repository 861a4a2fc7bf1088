"""Model-level parity against the reference's own engine (tests/golden/reference_engine.pt,
made by tests/golden/make_golden_engine.py: the reference's LLMEngine with its Triton
FP8 kernels and flash-attn prefill, eager and CUDA-graph decode, on a B200).

Both engines load the same seeded synthetic checkpoint (tests/golden/engine_case.py)
and decode 4 prompts greedily for 32 steps:
  * "small" (3 Qwen3-0.6B-shaped layers, vocabulary 8192): the logits this engine
    computes for every step, fed the reference's tokens (teacher forcing, so both
    follow one token path), against the reference's logits; and the tokens this
    engine chooses when it runs free;
  * "0.6b" (BASELINE config 2's model: 28 layers, vocabulary 151936): free-running
    greedy tokens.
The bar (north star): logits within relative L2 1e-2 of the reference at every step
and identical greedy tokens for the first 32 steps, in eager mode and with CUDA
graphs."""
import pytest
import torch

from tests.golden.engine_case import CASES, ENGINE_KW, prompts, write_checkpoint

pytestmark = pytest.mark.gpu

REF = None


def _ref():
    global REF
    if REF is None:
        from pathlib import Path
        REF = torch.load(Path(__file__).parent / "golden" / "reference_engine.pt", weights_only=False)
    return REF


def _engine(path, eager):
    from microserve_b200.Config import Config
    from microserve_b200.engine.llm import LLMEngine
    return LLMEngine(Config(model_dir=path, load_format="safetensors", enforce_eager=eager, **ENGINE_KW))


def _run(eng, case, forced=None):
    """Greedy generation; with `forced` (per-sequence token lists) every sampled token is
    replaced by the forced one before the next step. Returns (tokens, logits rows)."""
    from microserve_b200.engine.sequence import SamplingParams
    runner = eng.runner
    rows: dict[int, list] = {}
    orig = runner._finish_sampling

    def spy(seqs, logits, greedy):
        out = orig(seqs, logits, greedy)
        for i, s in enumerate(seqs):
            if out[i] is not None:
                rows.setdefault(s.seq_id, []).append(logits[i].detach().half().cpu())
        return out
    runner._finish_sampling = spy
    try:
        steps = CASES[case]["steps"]
        seqs = [eng.add(p, SamplingParams(temperature=0.0), max_tokens=steps) for p in prompts(case)]
        while not eng.is_idle():
            eng.step()
            if forced is not None:
                for s, f in zip(seqs, forced):
                    k = s.num_completion_tokens
                    if k > 0:
                        s.token_ids[-1] = f[k - 1]
    finally:
        runner._finish_sampling = orig
    tokens = [s.completion_token_ids for s in seqs]
    logits = [torch.stack(rows[s.seq_id]) for s in seqs] if rows else None
    return tokens, logits


@pytest.fixture(scope="module")
def small_checkpoint(tmp_path_factory):
    return write_checkpoint("small", str(tmp_path_factory.mktemp("small")))


@pytest.mark.parametrize("mode", ["eager", "graph"])
def test_small_model_logits_and_tokens_match_reference(small_checkpoint, mode):
    ref = _ref()["small"][mode]
    eng = _engine(small_checkpoint, eager=(mode == "eager"))
    _, logits = _run(eng, "small", forced=ref["tokens"])
    ref_logits = _ref()["small"]["eager"]["logits"]
    worst = 0.0
    for s, (got, exp) in enumerate(zip(logits, ref_logits)):
        for k in range(exp.shape[0]):
            rel = ((got[k].float() - exp[k].float()).norm() / exp[k].float().norm()).item()
            worst = max(worst, rel)
            assert rel <= 1e-2, f"sequence {s} step {k}: logits rel-L2 {rel:.3e}"
    free, _ = _run(eng, "small")
    assert free == ref["tokens"], "greedy tokens differ from the reference's"
    print(f"small/{mode}: worst per-step logits rel-L2 {worst:.2e}; 4 x 32 tokens identical")


@pytest.mark.parametrize("mode", ["eager", "graph"])
def test_qwen3_0_6b_greedy_tokens_match_reference(tmp_path, mode):
    path = write_checkpoint("0.6b", str(tmp_path / "ck"))
    eng = _engine(path, eager=(mode == "eager"))
    free, _ = _run(eng, "0.6b")
    ref = _ref()["0.6b"][mode]["tokens"]
    same = [sum(a == b for a, b in zip(x, y)) for x, y in zip(free, ref)]
    assert free == ref, f"greedy tokens differ from the reference's: {same} of 32 identical per sequence"
