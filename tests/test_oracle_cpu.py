"""CPU tests: the oracle against the reference's own outputs (tests/golden/), the
scheduler/block manager against the reference's recorded decisions, and the
runner's host-side batch preparation against the reference formulas."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8_decoder as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def layers():
    return torch.load(GOLDEN / "layers_cpu.pt")


def test_oracle_rmsnorm_matches_reference_module(layers):
    g = layers["rmsnorm"]
    y, r = O.rmsnorm(g["x"], g["weight"], 1e-6, g["residual"])
    assert torch.equal(r, g["residual_out"]) and torch.equal(y, g["y"])
    assert torch.equal(O.rmsnorm(g["x"], g["weight"], 1e-6), g["y_nores"])
    h = layers["head_rmsnorm"]
    assert torch.equal(O.rmsnorm(h["x"], h["weight"], 1e-6), h["y"])


def test_oracle_rope_matches_reference_module(layers):
    g = layers["rope"]
    cos, sin = O.rope_tables(128, 40960, 1e6)
    assert torch.equal(cos[g["positions"]], g["cos"]) and torch.equal(sin[g["positions"]], g["sin"])
    q, k = O.rope(g["positions"], g["q"], g["k"], cos, sin)
    assert torch.equal(q, g["q_out"]) and torch.equal(k, g["k_out"])


def test_oracle_silu_mul_matches_reference_module(layers):
    g = layers["silu_mul"]
    assert torch.equal(O.silu_mul(g["x"]), g["y"])


@pytest.mark.parametrize("name", ["w50x70", "w128x256"])
def test_oracle_weight_quant_vs_reference_module_on_cpu(layers, name):
    """The reference module evaluated on the CPU divides by 448 exactly; on the GPU (where
    the reference quantises) it multiplies by the fp32 reciprocal, which the oracle follows
    (pinned bit-exactly by tests/test_reference_golden.py). The two agree to one ulp in the
    scale and in all but a handful of codes."""
    g = layers["weight_quant_" + name]
    q, s = O.quantize_weight(g["weight"].float())
    assert torch.allclose(s, g["scales"], rtol=2.5e-7, atol=0)
    assert (q.view(torch.uint8) != g["codes"]).float().mean().item() < 1e-3
    exact = g["weight"].float().abs().amax(1).clamp_min(1e-8) / 448.0  # the CPU evaluation
    assert torch.equal(exact, g["scales"])
    assert g["scales"][3].item() == pytest.approx(1e-8 / 448)  # the all-zero channel


def test_oracle_row_quant_round_trip_and_saturation():
    x = torch.tensor([[0.0, 1.0, -2.0, 448.0], [1e-3, -1e-3, 5e-4, 0.0], [0.0, 0.0, 0.0, 0.0]]).half()
    q, s = O.quantize_rows(x)
    assert s[2].item() == pytest.approx(1e-8 / 448)
    back = q.float() * s[:, None]
    assert torch.allclose(back, x.float(), rtol=0.07, atol=0)
    assert q.view(torch.uint8)[0, 3].item() == 0x7E  # 448 = e4m3 max finite


def test_oracle_decode_attention_known_answer():
    """One cached token: attention returns its dequantised value exactly (softmax over one key)."""
    kc = torch.zeros(1, 256, 1, 128, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    ks, vs = torch.ones(1, 256, 1), torch.ones(1, 256, 1)
    k = torch.randn(1, 1, 128).half()
    v = torch.randn(1, 1, 128).half()
    O.store_kv(k, v, kc, vc, ks, vs, torch.tensor([5]))
    q = torch.randn(1, 2, 128).half()
    out = O.decode_attention(q, kc, vc, ks, vs, torch.tensor([6]), torch.tensor([[0]]), 0.1)
    # six visible positions: five zero keys/values (scale 1) and the stored one
    vv = torch.cat([torch.zeros(5, 128), (vc[0, 5, 0].float() * vs[0, 5, 0])[None]])
    kk = torch.cat([torch.zeros(5, 128), (kc[0, 5, 0].float() * ks[0, 5, 0])[None]])
    for h in range(2):
        p = torch.softmax(kk @ q[0, h].float() * 0.1, 0)
        assert torch.allclose(out[0, h].float(), (p[:, None] * vv).sum(0), atol=1e-3)


def test_oracle_grouped_decode_attention_equals_the_loop():
    """The grouped-head decode attention (used where the oracle is timed) computes
    the same thing as the per-head restatement: paged, out-of-order blocks, ragged
    lengths, an empty row, four q heads per kv head."""
    g = torch.Generator().manual_seed(3)
    Hq, Hkv, D, bs = 8, 2, 128, 256
    lens = [300, 0, 17, 520]
    nblk = [(L + bs - 1) // bs or 1 for L in lens]
    perm = torch.randperm(sum(nblk), generator=g).tolist()
    tables, o = [], 0
    for n in nblk:
        tables.append(perm[o:o + n])
        o += n
    kc = torch.randint(0, 120, (sum(nblk), bs, Hkv, D), dtype=torch.uint8, generator=g).view(torch.float8_e4m3fn)
    vc = torch.randint(0, 120, (sum(nblk), bs, Hkv, D), dtype=torch.uint8, generator=g).view(torch.float8_e4m3fn)
    ks = torch.rand(sum(nblk), bs, Hkv, generator=g) * 1e-2
    vs = torch.rand(sum(nblk), bs, Hkv, generator=g) * 1e-2
    q = torch.randn(len(lens), Hq, D, generator=g).half()
    args = (q, kc, vc, ks, vs, torch.tensor(lens), O.block_table_rows(tables), D ** -0.5)
    a, b = O.decode_attention(*args), O.decode_attention_grouped(*args)
    assert (b[1] == 0).all()
    assert (a.float() - b.float()).abs().max().item() < 1e-3


# ------------------------------------------------------------------ scheduler / block manager
def _replay(trace):
    from microserve_b200.engine.scheduler import Scheduler
    from microserve_b200.engine.sequence import Sequence
    p = trace["params"]
    sch = Scheduler(num_kvcache_blocks=p["num_blocks"], block_size=p["block_size"], max_num_seqs=p["max_num_seqs"],
                    max_num_batched_tokens=p["max_batched"], policy=p["policy"], eos_token_id=p["eos"])
    eos, period, bs = p["eos"], p["period"], p["block_size"]
    index, seqs, rounds = {}, [], []
    pending = sorted([tuple(a) for a in trace["arrivals"]], key=lambda a: a[0])
    for rnd in range(len(trace["rounds"])):
        while pending and pending[0][0] <= rnd:
            _, prompt, mt = pending.pop(0)
            s = Sequence(list(prompt), max_tokens=mt)
            index[s.seq_id] = len(seqs)
            seqs.append(s)
            sch.add(s)
        batch = sch.schedule()
        rec = []
        if batch is not None:
            outs = []
            for s in batch:
                p0, n = s.num_computed_tokens, s.num_scheduled_tokens
                bt = list(s.block_table)
                rec.append(dict(seq=index[s.seq_id], computed=p0, scheduled=n, needs_sample=s.needs_sample,
                                gap=s.gap, block_table=bt,
                                slots=O.slot_mapping(bt, list(range(p0, p0 + n)), bs)))
                if not s.needs_sample:
                    outs.append(None)
                    continue
                i, L = index[s.seq_id], len(s.token_ids)
                tok = 1000 + (i * 7 + L) % period
                if eos is not None and (i + L) % 37 == 0:
                    tok = eos
                outs.append(tok)
            sch.postprocess(batch, outs)
        rounds.append(dict(batch=rec, free=sch.block_manager.free_blocks_nums, stats=sch.last_batch_stats))
    finals = [dict(tokens=s.token_ids, status=s.status.name, preemptions=s.preemption_count) for s in seqs]
    return rounds, finals


def _traces():
    with open(GOLDEN / "scheduler_traces.json") as f:
        return json.load(f)


@pytest.mark.parametrize("trace", _traces(), ids=lambda t: t["name"])
def test_scheduler_decisions_match_reference(trace):
    rounds, finals = _replay(trace)
    for i, (got, ref) in enumerate(zip(rounds, trace["rounds"])):
        assert got == ref, f"round {i} differs"
    assert finals == trace["finals"]


def test_block_hash_is_chained_xxhash64_of_int64_tokens():
    import xxhash
    from microserve_b200.engine.block_manager import chain_hash
    toks = [1, 2, 3, 70000]
    h0 = xxhash.xxh64(np.asarray(toks, dtype=np.int64).tobytes()).intdigest()
    assert chain_hash(toks) == h0
    h1 = xxhash.xxh64(h0.to_bytes(8, "little") + np.asarray(toks, dtype=np.int64).tobytes()).intdigest()
    assert chain_hash(toks, h0) == h1


# ------------------------------------------------------------------ runner host-side batch prep
class _Seq:
    def __init__(self, tokens, computed, scheduled, table):
        self.token_ids, self.num_computed_tokens, self.num_scheduled_tokens = tokens, computed, scheduled
        self.block_table = table
        self.num_tokens_with_spec = len(tokens)

    @property
    def gap(self):
        return self.num_tokens_with_spec - self.num_computed_tokens


def _runner():
    from microserve_b200.engine.model_runner import ModelRunner
    r = object.__new__(ModelRunner)
    r.block_size = 256
    r.max_decode_blocks = 8  # max_model_len 2048
    return r


def test_prepare_decode_matches_reference_formulas():
    r = _runner()
    seqs = [_Seq(list(range(300)), 299, 1, [4, 7]), _Seq(list(range(1000, 1513)), 512, 1, [0, 1, 9]),
            _Seq([5], 0, 1, [3])]
    ids, pos, slots, lens, bt = r.prepare_decode(seqs)
    assert ids.tolist() == [299, 1512, 5] and pos.tolist() == [299, 512, 0]
    ref = [O.slot_mapping(s.block_table, [p], 256)[0] for s, p in zip(seqs, [299, 512, 0])]
    assert slots.tolist() == ref and lens.tolist() == [300, 513, 1]
    # decode tables are max_model_len wide (the graphs' width), padded with -1 like the reference's rows
    rows = O.block_table_rows([s.block_table for s in seqs]).numpy()
    assert bt.dtype == np.int32 and bt.shape == (3, 8)
    assert np.array_equal(bt[:, :rows.shape[1]], rows) and (bt[:, rows.shape[1]:] == -1).all()


def test_prepare_prefill_and_chunk_match_reference_formulas():
    r = _runner()
    a = _Seq(list(range(600)), 0, 600, [2, 0, 5])
    b = _Seq(list(range(50)), 0, 50, [1])
    ids, pos, slots, cu = r.prepare_prefill([a, b])
    assert cu.tolist() == [0, 600, 650] and ids.tolist() == list(range(600)) + list(range(50))
    assert slots.tolist() == O.slot_mapping(a.block_table, list(range(600)), 256) + O.slot_mapping([1], list(range(50)), 256)
    c = _Seq(list(range(700)), 292, 8, [3, 4, 6])
    d = _Seq(list(range(900)), 512, 100, [7, 8, 9])
    ids, pos, slots, cu, kv, bt = r.prepare_chunk([c, d])
    assert pos.tolist() == list(range(292, 300)) + list(range(512, 612))
    assert cu.tolist() == [0, 8, 108] and kv.tolist() == [300, 612]
    assert slots.tolist() == O.slot_mapping(c.block_table, list(range(292, 300)), 256) + \
        O.slot_mapping(d.block_table, list(range(512, 612)), 256)
