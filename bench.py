#!/usr/bin/env python
"""Benchmark: Qwen3-8B-shaped FP8 decode throughput.

Workload (synthetic, seeded; no checkpoints or datasets exist offline):
  Qwen3-8B shapes (36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128,
  MLP 12288, vocab 151936), random N(0, 0.02) weights quantised to FP8 e4m3
  per output channel, FP8 e4m3 KV cache in 256-token pages, fp16
  activations; 256 sequences with prompt lengths uniform in [128, 1024]
  (random.Random(0)), greedy decoding, tensor parallel over --gpus.

value (`metric`, device-resident): decode steps of the whole batch (CUDA
  graph replay of embedding -> 36 FP8 decoder layers -> norm -> LM head ->
  greedy argmax) with every step's metadata already in HBM; the argmax of a
  step is the next step's input. tok/s = batch * K / time of K steps.
e2e: the full config-3 job through LLMEngine (add 256 requests of 512 output
  tokens, step() until idle): prompts/metadata go host->device from pinned
  memory and sampled tokens come back every step. tok/s = output tokens /
  elapsed, plus ITL p50 (consecutive token-timestamp deltas).
roofline: the kernel class with the largest share of the decode step (the four
  FP8 GEMMs of a layer, else the decode attention), each launch timed alone on the
  step's own inputs with CUDA events (CUDA-graph replay); algorithmic bytes over
  that time; `traffic` = DRAM bytes of the same launches from ncu captures
  (profiles/roofline_traffic.json).
cpu_baseline: the CPU oracle (a restatement of the reference's FP8 path) on
  the host cores for one decoder layer of the same decode step, scaled to
  the full model.

--impl reference times that CPU restatement alone, whole decode steps of the
same batch (the reference's own kernels are Triton JIT kernels for a GPU; its
FP8 path has no CPU implementation, so the restatement stands in for it).
"""
from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

MODELS = {
    "8b": dict(layers=36, hidden=4096, heads=32, kv_heads=8, inter=12288, vocab=151936, tie=False),
    "0.6b": dict(layers=28, hidden=1024, heads=16, kv_heads=8, inter=3072, vocab=151936, tie=True),
    "32b": dict(layers=64, hidden=5120, heads=64, kv_heads=8, inter=25600, vocab=151936, tie=False),
}
HEAD_DIM = 128
BLOCK = 256
# NVLink: the measured peer-copy bandwidth per direction per GPU on this pool's B200s
# (900 GB/s nominal), the denominator of NVLink-bound fractions.
NVLINK_PEER_GBS = 770.0


def qwen3_cfg(name: str, max_pos: int = 40960):
    from transformers import Qwen3Config
    m = MODELS[name]
    return Qwen3Config(vocab_size=m["vocab"], hidden_size=m["hidden"], intermediate_size=m["inter"],
                       num_hidden_layers=m["layers"], num_attention_heads=m["heads"],
                       num_key_value_heads=m["kv_heads"], head_dim=HEAD_DIM, max_position_embeddings=max_pos,
                       rms_norm_eps=1e-6, tie_word_embeddings=m["tie"], hidden_act="silu", attention_bias=False)


def prompts(n: int, lo: int, hi: int, vocab: int, seed: int = 0) -> list[list[int]]:
    rng = random.Random(seed)
    lens = [rng.randint(lo, hi) for _ in range(n)]
    return [[rng.randrange(100, vocab) for _ in range(L)] for L in lens]


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Clock samples taken DURING the timed region (median SM clock, throttle reasons):
    NVML queries from a thread every 10 ms (read-only), else an nvidia-smi loop.

    The sampler is running before the region opens; every sample is timestamped,
    and only samples between mark_start() and mark_end() count."""

    def __init__(self, index: int, period_ms: int = 25):
        self.index, self.period_ms = index, period_ms
        self.proc, self.lines, self.t0, self.t1 = None, [], None, None
        self._stamped = []

    def __enter__(self):
        import threading
        if self._enter_nvml():
            return self
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        first = threading.Event()

        def reader():
            for line in self.proc.stdout:
                self._stamped.append((time.monotonic(), line))
                first.set()
            first.set()
        self._thread = threading.Thread(target=reader, daemon=True)
        self._thread.start()
        first.wait(timeout=10)
        return self

    def _enter_nvml(self) -> bool:
        """Sample through NVML in a thread (reads only): exact timestamps, a sample every
        10 ms, so even a short timed region holds several. False if NVML is unavailable."""
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception:
            return False
        bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        self._stop = threading.Event()
        self._nvml = nv

        def sampler():
            while not self._stop.is_set():
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                except Exception:
                    break
                flags = ", ".join("Active" if rs & b else "Not Active" for b in bits)
                self._stamped.append((time.monotonic(), f"{sm}, {mx}, {pw:.1f}, {flags}"))
                self._stop.wait(0.01)
        self._thread = threading.Thread(target=sampler, daemon=True)
        self._thread.start()
        self.proc = "nvml"
        return True

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()

    def __exit__(self, *exc):
        if self.proc is None:
            return
        if self.t1 is not None:  # let the sample in flight at the end of the region arrive
            time.sleep(2 * self.period_ms / 1000)
        if self.proc == "nvml":
            self._stop.set()
            self._thread.join(timeout=5)
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass
        else:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._thread.join(timeout=5)
        t0 = self.t0 if self.t0 is not None else 0.0
        t1 = (self.t1 if self.t1 is not None else time.monotonic()) + 1.5 * self.period_ms / 1000
        self.lines = [l for t, l in self._stamped if t0 <= t <= t1 and l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- ours
def build_engine(args, cfg, max_model_len):
    from microserve_b200.Config import Config
    from microserve_b200.engine.llm import LLMEngine
    return LLMEngine(Config(hf_config=cfg, load_format="dummy", quantization="fp8_dynamic",
                            kv_cache_dtype="fp8_e4m3", max_num_seqs=args.batch,
                            max_num_batched_tokens=args.max_batched_tokens, max_model_len=max_model_len,
                            tensor_parallel_size=args.gpus, gpu_memory_utilization=0.9, seed=0,
                            num_kvcache_blocks=args.kv_blocks,
                            tp_fused_collective=not getattr(args, "nccl_allreduce", False),
                            tp_fused_gemm=getattr(args, "tp_one_kernel", False),
                            tp_exact_act_scale=getattr(args, "exact_act_scale", False),
                            gemm_pair_tiles=getattr(args, "pair_tiles", False)))


def sync_all():
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float) -> float:
    if torch.distributed.is_initialized():
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())
    return x


def run_e2e(engine, reqs, out_len):
    """Whole job through LLMEngine; returns (tok/s, itl_p50_ms, elapsed_s, h2d/step, d2h/step, steps)."""
    from microserve_b200.engine.sequence import SamplingParams
    runner = engine.runner
    seqs = [engine.add(r, SamplingParams(temperature=0.0), max_tokens=out_len) for r in reqs]
    h2d0 = runner.host_batch.bytes_uploaded
    sync_all()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record()
    steps = 0
    while not engine.is_idle():
        engine.step()
        steps += 1
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    elapsed = max_over_ranks(max(start.elapsed_time(end) / 1e3, wall))
    out = sum(s.num_completion_tokens for s in seqs)
    itl = [(b - a) * 1e3 for s in seqs for a, b in zip(s.token_timestamps, s.token_timestamps[1:])]
    h2d = (runner.host_batch.bytes_uploaded - h2d0) / max(steps, 1)
    d2h = out * 8 / max(steps, 1)
    return out / elapsed, (statistics.median(itl) if itl else None), elapsed, h2d, d2h, steps


def prefill_batch(engine, reqs):
    """Add `reqs` to the engine and run it until every sequence has been prefilled."""
    from microserve_b200.engine.sequence import SamplingParams
    seqs = [engine.add(r, SamplingParams(temperature=0.0), max_tokens=10 ** 6) for r in reqs]
    while any(s.gap > 1 or s.num_computed_tokens == 0 for s in seqs):
        engine.step()
    return seqs


def decode_metadata(engine, seqs, steps_total, offset=0):
    """Lay out `steps_total` decode steps of metadata for the whole batch in HBM
    (positions, slots, seqlens, tables), starting `offset` tokens after the first
    decode position of each sequence (blocks are allocated as needed; the cache
    content of skipped positions is whatever the pages hold)."""
    runner = engine.runner
    bm = engine.scheduler.block_manager
    B = len(seqs)
    pos = np.zeros((steps_total, B), np.int64)
    slots = np.zeros((steps_total, B), np.int64)
    for i, s in enumerate(seqs):
        p0 = s.num_computed_tokens + offset
        need = (p0 + steps_total - 1) // BLOCK + 1
        while len(s.block_table) < need:
            s.block_table.append(bm._take_free())
        for st in range(steps_total):
            p = p0 + st
            pos[st, i] = p
            slots[st, i] = s.block_table[p // BLOCK] * BLOCK + p % BLOCK
    gv = runner.graph_vars
    width = gv["block_tables"].shape[1]
    bt = np.full((B, width), -1, np.int32)
    for i, s in enumerate(seqs):
        bt[i, :len(s.block_table)] = s.block_table
    ids0 = np.array([s.token_ids[s.num_computed_tokens] for s in seqs], np.int64)
    dev = runner.device
    return dict(seqs=seqs, pos=torch.from_numpy(pos).to(dev), slots=torch.from_numpy(slots).to(dev),
                lens=torch.from_numpy((pos + 1).astype(np.int32)).to(dev), bt=torch.from_numpy(bt).to(dev),
                ids0=torch.from_numpy(ids0).to(dev), ctx0=pos[0] + 1)


@torch.inference_mode()
def decode_step_runner(engine, batch):
    runner = engine.runner
    gv = runner.graph_vars
    B = batch["ids0"].shape[0]
    graph = runner.graphs[B]
    gv["block_tables"][:B].copy_(batch["bt"])
    gv["input_ids"][:B].copy_(batch["ids0"])

    @torch.inference_mode()
    def step(i):
        gv["positions"][:B].copy_(batch["pos"][i])
        gv["slot_mapping"][:B].copy_(batch["slots"][i])
        gv["cache_seqlens"][:B].copy_(batch["lens"][i])
        graph.replay()
        gv["input_ids"][:B].copy_(gv["argmax"][:B])
    return step


def time_kernel(fn, iters=20, warm=3):
    """Device time of one fn() call: `iters` calls captured in a CUDA graph and
    replayed (so host launch overhead is not measured), CUDA events around the replay."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(iters):
            fn()
    graph.replay()  # warm the graph itself
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / 1e3 / iters


@torch.inference_mode()
def kernel_rooflines(engine, batch, step_idx, hbm_peak):
    """Per-kernel achieved HBM bandwidth on the decode step's own inputs: attention over
    layer 0's KV cache (larger than L2), each GEMM cycling through the layers' weights."""
    from microserve_b200 import kernels
    from microserve_b200.utils import dist as tp
    runner = engine.runner
    model = runner.model
    layer = model.model.layers[0]
    attn = layer.self_attn.attn
    B = batch["ids0"].shape[0]
    Hq, Hkv = layer.self_attn.num_heads, layer.self_attn.num_kv_heads
    dev = runner.device
    q = torch.randn(B, Hq, HEAD_DIM, device=dev, dtype=torch.float16) * 0.2
    lens = batch["lens"][step_idx]
    out = torch.empty_like(q)
    t_attn = time_kernel(lambda: kernels.paged_decode_fp8(q, attn.k_cache, attn.v_cache, attn.k_scale_cache,
                                                          attn.v_scale_cache, lens, batch["bt"], HEAD_DIM ** -0.5,
                                                          out=out))
    ctx = lens.double().sum().item()
    attn_bytes = ctx * Hkv * (2 * HEAD_DIM + 2 * 4) + 2 * B * Hq * HEAD_DIM * 2 + B * (4 + 4 * batch["bt"].shape[1])
    res = {"decode_attention": dict(seconds=t_attn, bytes=attn_bytes, per_layer=1)}
    layers = model.model.layers
    lins = {"qkv_proj": [l.self_attn.qkv_proj for l in layers], "o_proj": [l.self_attn.o_proj for l in layers],
            "gate_up_proj": [l.mlp.gate_up_proj for l in layers], "down_proj": [l.mlp.down_proj for l in layers]}
    for name, per_layer in lins.items():
        lin = per_layer[0]
        x = torch.randn(B, lin.in_features, device=dev, dtype=torch.float16)
        xq, sx = kernels.quantize_rows_fp8(x)
        y = torch.empty(B, lin.out_features, device=dev, dtype=torch.float16)
        it = [0]

        def launch():
            # consecutive launches use consecutive layers' weights, as in the decode step,
            # so the weights come from HBM and not from L2
            w = per_layer[it[0] % len(per_layer)]
            kernels.fp8_gemm(xq, sx, w.weight_fp8, w.weight_scale, out=y)
            it[0] += 1
        t = time_kernel(launch)
        byts = lin.out_features * lin.in_features + B * lin.in_features + 2 * B * lin.out_features \
            + 4 * (B + lin.out_features)
        res[name] = dict(seconds=t, bytes=byts, per_layer=1)
    # the row kernels between them, on the step's own shapes (inputs in L2, as in the step)
    H, I = layer.mlp.down_proj.out_features, layer.mlp.down_proj.in_features
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(B, H, device=dev, generator=g).half()
    r = torch.randn(B, H, device=dev, generator=g).half()
    nw = layer.post_attention_layernorm.weight
    eps = layer.post_attention_layernorm.eps
    t = time_kernel(lambda: kernels.rmsnorm(x, nw, eps, r, want_fp16=False, want_fp8=True))
    res["rmsnorm_fp8"] = dict(seconds=t, bytes=B * H * 7 + 4 * B + 2 * H, per_layer=2)
    gu = torch.randn(B, 2 * I, device=dev, generator=g).half()
    t = time_kernel(lambda: kernels.silu_mul(gu, want_fp16=False, want_fp8=True))
    res["silu_mul_fp8"] = dict(seconds=t, bytes=B * 2 * I * 2 + B * I + 4 * B, per_layer=1)
    sa = layer.self_attn
    qkv = torch.randn(B, (Hq + 2 * Hkv) * HEAD_DIM, device=dev, generator=g).half()
    pos, slots = batch["pos"][step_idx], batch["slots"][step_idx]
    t = time_kernel(lambda: kernels.qkv_post(
        qkv, Hq, Hkv, HEAD_DIM, pos, sa.rotary_emb.cos_half16, sa.rotary_emb.sin_half16, sa.q_norm.weight,
        sa.k_norm.weight, sa.rms_norm_eps, slots, (attn.k_cache, attn.v_cache, attn.k_scale_cache,
                                                   attn.v_scale_cache)))
    res["qkv_post"] = dict(seconds=t, bytes=B * (Hq + 2 * Hkv) * HEAD_DIM * 2 + B * Hq * HEAD_DIM * 2
                           + B * Hkv * (2 * HEAD_DIM + 8), per_layer=1)
    o = torch.randn(B, Hq * HEAD_DIM, device=dev, generator=g).half()
    t = time_kernel(lambda: kernels.quantize_rows_fp8(o))
    res["quantize_rows"] = dict(seconds=t, bytes=B * Hq * HEAD_DIM * 3 + 4 * B, per_layer=1)
    # LM head (vocab-parallel shard, fp16 as in the reference)
    head_w = model.lm_head.weight
    hx = torch.randn(B, H, device=dev, generator=g).half()
    t = time_kernel(lambda: model.compute_logits(hx))
    # beside it, the library GEMM the reference calls (torch F.linear -> cuBLAS) on the same operands
    t_lib = time_kernel(lambda: torch.nn.functional.linear(hx, head_w))
    res["lm_head"] = dict(seconds=t, bytes=head_w.numel() * 2 + B * H * 2 + B * head_w.shape[0] * 2, per_layer=0,
                          torch_linear_us=round(t_lib * 1e6, 2))
    tpf = runner.tp_fused
    world = tp.tp_size()
    if world > 1:
        # the fused row-parallel all-reduce + residual + RMSNorm + FP8 (bound by the bytes each
        # rank sends over NVLink: its partial rows to their owners, its codes + scales to every
        # peer) and, for comparison, NCCL's all-reduce of the same fp16 rows
        R = (B + world - 1) // world
        res_rows = torch.randn(B, H, device=dev, generator=g).half()
        w = layer.post_attention_layernorm.weight
        if tpf is not None:
            tpf.partial(B).copy_(torch.randn(B, H, device=dev, generator=g).half())
            sync_all()
            t = time_kernel(lambda: tpf.allreduce_norm_fp8(B, res_rows, w, eps))
            res["tp_allreduce_rmsnorm_fp8"] = dict(seconds=t, bytes=(world - 1) * R * (2 * H + H + 4), per_layer=2,
                                                   bound="nvlink", peak_gbs=NVLINK_PEER_GBS)
        if tpf is not None:
            # o_proj as the decode step runs it: ONE kernel, the row-parallel GEMM pushing its
            # output rows to their owners (the transfer overlaps the GEMM), then reducing,
            # normalising and gathering. Communication hidden = 1 - exposed / standalone, with
            # exposed = fused - (local GEMM + the norm alone) and standalone = op - norm alone.
            o = layer.self_attn.o_proj
            xo = torch.randn(B, o.in_features, device=dev, generator=g).half()
            oq, so = kernels.quantize_rows_fp8(xo)
            sync_all()

            t = time_kernel(lambda: tpf.rowpar_gemm_norm(oq, so, o.weight_fp8, o.weight_scale, res_rows, w, eps))
            op_t = res["tp_allreduce_rmsnorm_fp8"]["seconds"]
            norm_t, gemm_t = res["rmsnorm_fp8"]["seconds"], res["o_proj"]["seconds"]
            exposed = max(0.0, t - gemm_t - norm_t)
            res["tp_o_proj_gemm_allreduce_rmsnorm_fp8"] = dict(
                seconds=t, bytes=(world - 1) * R * (2 * H + H + 4), per_layer=1, bound="nvlink",
                peak_gbs=NVLINK_PEER_GBS,
                comm_hidden_frac=round(1.0 - min(1.0, exposed / max(op_t - norm_t, 1e-9)), 3))
        xr = torch.randn(B, H, device=dev, generator=g).half()
        sync_all()
        t = time_kernel(lambda: torch.distributed.all_reduce(xr, group=tp.tp_group()))
        res["nccl_allreduce"] = dict(seconds=t, bytes=int(2 * (world - 1) / world * B * H * 2), per_layer=0,
                                     bound="nvlink", peak_gbs=NVLINK_PEER_GBS)
        sync_all()
    for v in res.values():
        v["achieved_gbs"] = v["bytes"] / v["seconds"] / 1e9
        v["frac"] = v["achieved_gbs"] / v.get("peak_gbs", hbm_peak)
    return res


GEMM_CLASS = ("qkv_proj", "o_proj", "gate_up_proj", "down_proj")


def measured_traffic():
    """DRAM bytes from ncu captures of the same kernels (profiles/roofline_traffic.json)."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def dominant_roofline(kern, hbm_peak, batch, gpus):
    """Roofline of the kernel class with the largest share of the decode step: the
    four FP8 GEMMs of a layer (one class, weights streamed once each) or the decode
    attention. achieved = algorithmic bytes / CUDA-event time of the launches."""
    gemm_s = sum(kern[k]["seconds"] for k in GEMM_CLASS)
    gemm_b = sum(kern[k]["bytes"] for k in GEMM_CLASS)
    attn = kern["decode_attention"]
    traffic = measured_traffic()
    if gemm_s >= attn["seconds"]:
        name, byts, secs = "fp8_gemm (qkv+o+gate_up+down of one layer)", gemm_b, gemm_s
        t = traffic.get(f"fp8_gemm_layer_b{batch}_tp{gpus}")
        tr = int(t["dram_bytes"]) if t else None
    else:
        name, byts, secs = "decode_attention", attn["bytes"], attn["seconds"]
        r = traffic.get("decode_attention_dram_per_algorithmic_byte")
        tr = int(attn["bytes"] * r["ratio"]) if r else None
    ach = byts / secs / 1e9
    return {"bound": "hbm", "kernel": name, "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(ach / hbm_peak, 4), "traffic": tr, "algorithmic_bytes": int(byts),
            "us": round(secs * 1e6, 2)}


@torch.inference_mode()
def cpu_baseline_layer(engine, batch, step_idx, layers_total, threads=None):
    """Oracle decode of ONE decoder layer and the LM head for the whole batch on the
    host cores (the reference arm's CPU path, with this run's weights and KV cache),
    repeated for ~10 s; the layer time is scaled to the model's layer count."""
    from oracle import fp8_decoder as O
    runner = engine.runner
    model = runner.model
    layer = model.model.layers[0]
    a = layer.self_attn
    if threads:
        torch.set_num_threads(threads)
    B = batch["ids0"].shape[0]

    def wp(lin):  # codes converted to fp32 once (exact), as the reference arm does
        return lin.weight_fp8.cpu().float(), lin.weight_scale.cpu()
    lw = O.LayerWeights(wp(a.qkv_proj), wp(a.o_proj), wp(layer.mlp.gate_up_proj), wp(layer.mlp.down_proj),
                        layer.input_layernorm.weight.cpu(), layer.post_attention_layernorm.weight.cpu(),
                        a.q_norm.weight.cpu(), a.k_norm.weight.cpu())
    bt = batch["bt"].cpu()
    used = sorted({int(b) for b in bt.flatten().tolist() if b >= 0})
    remap = {b: i for i, b in enumerate(used)}
    bt_local = bt.clone().apply_(lambda b: remap.get(b, -1))
    caches = [a.attn.k_cache[used].cpu(), a.attn.v_cache[used].cpu(), a.attn.k_scale_cache[used].cpu(),
              a.attn.v_scale_cache[used].cpu()]
    pos = batch["pos"][step_idx].cpu()
    slots = (bt_local.gather(1, (pos // BLOCK).unsqueeze(1)).squeeze(1).long() * BLOCK + pos % BLOCK)
    cos, sin = O.rope_tables(HEAD_DIM, int(pos.max()) + 1, 1e6)
    hidden = torch.randn(B, model.config.hidden_size, dtype=torch.float16)
    residual = torch.randn_like(hidden)
    head = model.lm_head.weight.cpu().float()
    # repeat the sampled layer and the LM head until ~10 s of CPU work
    layer_t, head_t = [], []
    t_start = time.perf_counter()
    while len(layer_t) < 2 or (time.perf_counter() - t_start < 10.0 and len(layer_t) < 50):
        t0 = time.perf_counter()
        O.decoder_layer(lw, pos, hidden, residual, Hq=a.num_heads, Hkv=a.num_kv_heads, D=HEAD_DIM, eps=1e-6,
                        cos_cache=cos, sin_cache=sin, mode="decode", caches=caches, slots=slots,
                        seqlens=(pos + 1), block_tables=bt_local, grouped_attention=True)
        layer_t.append(time.perf_counter() - t0)
        t1 = time.perf_counter()
        (hidden.float() @ head.T).half().argmax(-1)
        head_t.append(time.perf_counter() - t1)
    t_layer, t_head = statistics.median(layer_t), statistics.median(head_t)
    per_step = t_layer * layers_total + t_head
    return dict(value=B / per_step, unit="tok/s", cores=torch.get_num_threads(), kind="port",
                sample=f"1 of {layers_total} decoder layers and the LM head of one B={B} decode step, "
                       f"median of {len(layer_t)} repetitions, layer time x {layers_total}; "
                       f"oracle/fp8_decoder.py on {torch.get_num_threads()} threads",
                seconds_sampled=round(time.perf_counter() - t_start, 2))


def run_ours(args):
    from microserve_b200 import _lib
    from microserve_b200.utils import dist as tp
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
        tp.init_tensor_parallel()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    lib = _lib.load()
    lib.ms_set_pdl(0 if args.no_pdl else 1)
    cfg = qwen3_cfg(args.model)
    reqs = prompts(args.batch, args.prompt_min, args.prompt_max, cfg.vocab_size)
    steps_total = args.warmup + args.steps
    max_len = args.prompt_max + max(args.output_len, steps_total) + 2 * BLOCK
    engine = build_engine(args, cfg, max_len)
    hbm_peak, peak_kind = peaks()

    result = {}
    if not args.no_e2e:
        # warm-up job (short), then the timed full job
        run_e2e(engine, reqs, 4)
        e2e_tps, itl, e2e_s, h2d, d2h, e2e_steps = run_e2e(engine, reqs, args.output_len)
        result["e2e"] = {"value": round(e2e_tps, 1), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                         "d2h_bytes_per_step": int(d2h), "itl_p50_ms": itl, "elapsed_s": round(e2e_s, 3),
                         "engine_steps": e2e_steps, "output_tokens": args.batch * args.output_len}

    seqs = prefill_batch(engine, reqs)
    batch = decode_metadata(engine, seqs, steps_total)
    parity = tp_parity(engine, batch) if args.gpus > 1 else None
    elapsed, clocks_summary = time_decode_steps(engine, batch, args, lib, local)
    B = args.batch
    value = B * args.steps / elapsed
    ms_step = elapsed / args.steps * 1e3
    # the same K steps at the workload's mean context: config 3's contexts average the
    # prompt-time contexts plus half of the 512 generated tokens
    target = float(batch["ctx0"].mean()) + args.output_len / 2
    offset = max(0, int(round(target - float(batch["ctx0"].mean()) - steps_total / 2)))
    batch_mean = decode_metadata(engine, seqs, steps_total, offset)
    elapsed_mean, _ = time_decode_steps(engine, batch_mean, args, lib, local, sample_clocks=False)

    kern = kernel_rooflines(engine, batch, args.warmup, hbm_peak)
    L = cfg.num_hidden_layers
    roof = dominant_roofline(kern, hbm_peak, B, args.gpus)
    status = _lib.device_status()

    # algorithmic bytes of the whole decode step (per GPU) for context
    ctx = batch["lens"][args.warmup].double().sum().item()
    w_layers = sum(m.weight_fp8.numel() for m in engine.runner.model.modules() if hasattr(m, "weight_fp8"))
    kv_bytes = ctx * L * cfg.num_key_value_heads // args.gpus * (2 * HEAD_DIM + 8)
    head_bytes = engine.runner.model.lm_head.weight.numel() * 2
    step_bytes = w_layers + kv_bytes + head_bytes

    line = {
        "metric": metric_name(args),
        "value": round(value, 1), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 acc, f16 activations",
        "data": "synthetic: random N(0,0.02) weights quantised to FP8, prompts U[128,1024] from random.Random(0)",
        "config": workload_config(args, batch["ctx0"]),
        "setup": {"pdl": not args.no_pdl, "gemm_pair_tiles": bool(args.pair_tiles and args.gpus == 1),
                  "tp_collective": ("nccl all-reduce" if args.nccl_allreduce else
                                    "fused peer-memory all-reduce+rmsnorm+fp8") if args.gpus > 1 else None,
                  "tp_act_scale": "exact (full row)" if args.exact_act_scale else "per shard",
                  "tp_row_parallel": ("one kernel: GEMM pushing rows + reduce/norm tail" if args.tp_one_kernel else
                                      "GEMM pushing rows + separate reduce/norm op") if args.gpus > 1 else None},
        "roofline": dict(roof, peak_kind=f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s"),
        "kernels": {k: {kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in v.items()
                        if kk not in ("seconds", "bytes", "per_layer", "achieved_gbs", "frac")}
                    | {"us": round(v["seconds"] * 1e6, 2), "GBps": round(v["achieved_gbs"], 1),
                       "frac": round(v["frac"], 4)} for k, v in kern.items()},
        "step_roofline": {"algorithmic_bytes": int(step_bytes), "achieved_gbs": round(step_bytes / (ms_step / 1e3) / 1e9, 1),
                          "frac": round(step_bytes / (ms_step / 1e3) / 1e9 / hbm_peak, 4)},
        "decode_step_at_mean_context": {
            "ctx_mean": round(float(batch_mean["lens"][args.warmup:].double().mean()), 1),
            "ms_per_step": round(elapsed_mean / args.steps * 1e3, 4),
            "value": round(B * args.steps / elapsed_mean, 1), "unit": "tok/s"},
        "gpu_launches": int(engine.runner.kernels_per_decode_step.get(B, 0)) * args.steps,
        "clocks": clocks_summary,
        "device_status": status,
    }
    if parity is not None:
        line["tp_parity"] = parity
    line.update(result)
    if rank == 0 and args.gpus == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_layer(engine, batch, args.warmup, L)
    if rank == 0:
        print(json.dumps(line), flush=True)
    engine.runner.release_graphs()
    shutdown_distributed()


@torch.inference_mode()
def time_decode_steps(engine, batch, args, lib, local, sample_clocks=True):
    """W untimed + K timed decode steps (CUDA-graph replays), CUDA events on the
    stream, barrier + synchronize on both sides, max over ranks; clocks sampled
    inside the timed region."""
    step = decode_step_runner(engine, batch)
    steps_total = args.warmup + args.steps
    launches_before = lib.ms_launch_count()
    for i in range(args.warmup):
        step(i)
    sync_all()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with (ClockSampler(local) if sample_clocks else _NoClocks()) as clocks:
        # every rank's sampler is running before any rank starts its clock: a rank that
        # entered the region early would wait in its first step for its peers (each
        # tensor-parallel step synchronises the ranks) and count that wait
        sync_all()
        torch.cuda.nvtx.range_push("decode_timed")
        clocks.mark_start()
        start.record()
        for i in range(args.warmup, steps_total):
            step(i)
        end.record()
        torch.cuda.synchronize()
        clocks.mark_end()
        torch.cuda.nvtx.range_pop()
    sync_all()
    elapsed = max_over_ranks(start.elapsed_time(end) / 1e3)
    assert lib.ms_launch_count() == launches_before, "graph replay must not call the library"
    return elapsed, clocks.summary()


class _NoClocks:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False

    def mark_start(self):
        pass

    def mark_end(self):
        pass

    def summary(self):
        return None


@torch.inference_mode()
def tp_parity(engine, batch):
    """Tensor-parallel correctness on the bench's own batch: one decode step (step 0's
    metadata) through the fused peer-memory collective and again with the same sharded
    weights through the unfused path (RowParallelLinear's all-reduce, then the
    single-GPU RMSNorm kernels), full-vocabulary logits compared. The all-reduce of the
    reference path is an all-gather + fp32 sum in rank order rounded once (the fused
    collective's arithmetic, so the two must agree bit for bit); the NCCL all-reduce,
    whose summation order and fp16 roundings differ at more than two ranks, is
    reported beside it."""
    from microserve_b200.utils import dist as tp
    from microserve_b200.utils.context import AttentionMode, Context, reset_context, set_context
    runner = engine.runner
    model = runner.model
    tpf = model.model.tp_fused
    if tpf is None:
        return {"reference": "n/a (NCCL path is the one timed)"}

    def logits():
        set_context(Context(mode=AttentionMode.DECODE, slot_mapping=batch["slots"][0],
                            cache_seqlens=batch["lens"][0], block_tables=batch["bt"]))
        try:
            h = model(batch["ids0"], batch["pos"][0])
            return runner._full_logits(model.compute_logits(h)).float()
        finally:
            reset_context()
    fused = logits()
    model.model.tp_fused = None
    try:
        tp.set_ordered_sum(True)
        ordered = logits()
        tp.set_ordered_sum(False)
        nccl = logits()
    finally:
        tp.set_ordered_sum(False)
        model.model.tp_fused = tpf
    torch.cuda.synchronize()

    def cmp(ref):
        return (round(((fused - ref).norm() / ref.norm()).item(), 6),
                round((fused.argmax(-1) == ref.argmax(-1)).float().mean().item(), 4))
    rel, agree = cmp(ordered)
    nrel, nagree = cmp(nccl)
    return {"reference": "same weights, unfused: all-gather + rank-order fp32 sum, RMSNorm kernels; one decode step",
            "rows": int(fused.shape[0]), "rel_l2": rel, "token_agree": agree,
            "bitwise_equal": bool(torch.equal(fused, ordered)),
            "nccl_allreduce": {"rel_l2": nrel, "token_agree": nagree}}


def shutdown_distributed(limit_s: float = 60.0) -> None:
    """Barrier, then destroy the process group, bounded: a teardown that does not
    finish within limit_s ends the process (the result line is already printed)."""
    if not torch.distributed.is_initialized():
        return
    import threading
    done = threading.Event()

    def teardown():
        try:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        finally:
            done.set()
    threading.Thread(target=teardown, daemon=True).start()
    if not done.wait(limit_s):
        print("bench: process-group teardown did not finish; exiting", file=sys.stderr, flush=True)
        sys.stdout.flush()
        os._exit(0)


# ------------------------------------------------------------------------ reference
def workload_config(args, ctx0) -> dict:
    """The workload the metric is quoted on (identical in both arms)
    decode steps of the whole batch, contexts growing one token per step from ctx0."""
    ctx0 = np.asarray(ctx0)
    return {"workload": f"Qwen3-{args.model.upper()}-shaped decode step, batch {args.batch}, contexts "
                        f"{int(ctx0.min())}-{int(ctx0.max())} growing 1 token/step",
            "model": f"qwen3-{args.model}", "global_batch": args.batch, "seq_len": int(ctx0.mean()),
            "parallelism": f"tp{args.gpus}", "kv_cache": "fp8_e4m3, 256-token pages",
            "l2": "inputs larger than L2 (weights + KV >> 126 MB); no flush"}


def metric_name(args) -> str:
    """The metric both arms print (BASELINE's headline for the default config 3)."""
    return f"output tok/s Qwen3-{args.model.upper()} FP8 decode (FP8 KV), batch {args.batch}"


def reference_contexts(args) -> list[int]:
    """Context of each sequence at the first decode step: its prompt plus the token
    the prefill sampled (the GPU arm's batch["ctx0"])."""
    return [len(p) + 1 for p in prompts(args.batch, args.prompt_min, args.prompt_max, 1000)]


@torch.inference_mode()
def run_reference(args):
    """The reference's FP8 decode path restated on the CPU (the oracle), timed whole:
    every step is embedding -> all decoder layers -> final norm -> LM head over the
    full batch -> greedy argmax, on this box's host cores, at the GPU arm's contexts.
    Weight codes are converted to fp32 once (e4m3 -> fp32 is exact, so every product
    and sum is the oracle's); the layers share one set of weights and one KV cache
    (each is far larger than the CPU caches, so the cost is that of distinct ones)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import fp8_decoder as O
    m = MODELS[args.model]
    torch.manual_seed(0)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    H, I, Hq, Hkv, L, V = m["hidden"], m["inter"], m["heads"], m["kv_heads"], m["layers"], m["vocab"]

    def lin(n, k):
        wq, sw = O.quantize_weight((torch.randn(n, k) * 0.02).half())
        return wq.float(), sw
    lw = O.LayerWeights(lin((Hq + 2 * Hkv) * HEAD_DIM, H), lin(H, Hq * HEAD_DIM), lin(2 * I, H), lin(H, I),
                        torch.ones(H).half(), torch.ones(H).half(), torch.ones(HEAD_DIM).half(),
                        torch.ones(HEAD_DIM).half())
    ctx0 = reference_contexts(args)
    B = args.batch
    steps_total = args.steps + args.warmup
    nblk = [(c + steps_total) // BLOCK + 1 for c in ctx0]
    tot = sum(nblk)
    kc = torch.randint(0, 120, (tot, BLOCK, Hkv, HEAD_DIM), dtype=torch.uint8).view(torch.float8_e4m3fn)
    vc = torch.randint(0, 120, (tot, BLOCK, Hkv, HEAD_DIM), dtype=torch.uint8).view(torch.float8_e4m3fn)
    ks = torch.rand(tot, BLOCK, Hkv) * 1e-3
    vs = torch.rand(tot, BLOCK, Hkv) * 1e-3
    tables, o = [], 0
    for n in nblk:
        tables.append(list(range(o, o + n)))
        o += n
    bt = O.block_table_rows(tables)
    embed = (torch.randn(V, H) * 0.02).half()
    head = embed.float() if m["tie"] else (torch.randn(V, H) * 0.02).half().float()
    cos, sin = O.rope_tables(HEAD_DIM, max(ctx0) + steps_total + 2, 1e6)
    ids = torch.randint(100, V, (B,))
    times = []
    for it in range(steps_total):
        pos = torch.tensor([c - 1 + it for c in ctx0])
        slots = torch.tensor([tables[b][p // BLOCK] * BLOCK + p % BLOCK for b, p in enumerate(pos.tolist())])
        t0 = time.perf_counter()
        hidden, residual = embed[ids], None
        for _ in range(L):
            hidden, residual = O.decoder_layer(lw, pos, hidden, residual, Hq=Hq, Hkv=Hkv, D=HEAD_DIM, eps=1e-6,
                                               cos_cache=cos, sin_cache=sin, mode="decode",
                                               caches=[kc, vc, ks, vs], slots=slots, seqlens=pos + 1,
                                               block_tables=bt, grouped_attention=True)
        hidden, _ = O.rmsnorm(hidden, torch.ones(H).half(), 1e-6, residual)
        logits = (hidden.float() @ head.T).half()
        ids = logits.argmax(-1)
        dt = time.perf_counter() - t0
        if it >= args.warmup:
            times.append(dt)
        print(f"reference step {it}: {dt:.2f} s", file=sys.stderr, flush=True)
    per_step = statistics.mean(times)
    value = B / per_step
    sample = (f"whole decode steps of the full batch ({B} sequences, {L} decoder layers, LM head over "
              f"{V} tokens, greedy argmax) timed end to end; oracle/fp8_decoder.py (torch CPU) on "
              f"{threads} threads")
    line = {"impl": "reference", "metric": metric_name(args),
            "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 (CPU fp32 math)",
            "data": "synthetic: random N(0,0.02) weights quantised to FP8, prompts U[128,1024] from "
                    "random.Random(0)",
            "config": workload_config(args, ctx0),
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


@torch.inference_mode()
def reference_kernels():
    """The reference's own GPU kernels (Triton), from its offline install in baseline/_ref:
    (fp8_decode_attention, _fp8_mm), or None when that install is absent."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "microserve")):
        return None
    if ref not in sys.path:
        sys.path.insert(0, ref)
    from microserve.layers.fp8_decode_attention import fp8_decode_attention
    from microserve.layers.fp8_linear import _fp8_mm
    return fp8_decode_attention, _fp8_mm


@torch.inference_mode()
def run_tp_rowpar_sweep(args):
    """BASELINE config 5, the fused row-parallel op under torchrun: for each M, the
    row-parallel FP8 GEMM with N = hidden, K = intermediate / TP (down_proj of the
    --model's shapes; 32B: N = 5120, K = 25600 / TP) pushing its output rows to their
    owners and then reducing / adding / normalising / quantising them
    (ms_fp8_gemm_rowpar_ar_rmsnorm: one kernel for decode-sized M, the GEMM + the op
    for larger M), against this rank's GEMM writing locally + NCCL all-reduce + the
    RMSNorm/FP8 kernel. bf16/fp16 activations
    N(0, 1). Device time per call (CUDA graph of 20 calls, max over ranks); NVLink
    bytes each rank sends per call: its partial rows to their owners and its codes to
    every peer."""
    import datetime
    from microserve_b200 import _lib, kernels
    from microserve_b200.utils import dist as tp
    from microserve_b200.utils.tp_fused import TpFused
    rank, world, local = (int(os.environ.get(k, d)) for k, d in (("RANK", "0"), ("WORLD_SIZE", "1"),
                                                                   ("LOCAL_RANK", "0")))
    torch.cuda.set_device(local)
    if world < 2:
        print(json.dumps({"kernel": "tp_rowpar", "unavailable": "needs torchrun with 2..8 ranks"}), flush=True)
        return
    torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                         device_id=torch.device("cuda", local))
    tp.init_tensor_parallel()
    _lib.load().ms_set_pdl(1)
    m = MODELS[args.model]
    H, K = m["hidden"], m["inter"] // world
    Ms = [int(x) for x in (args.rows or "1,8,64,256,1024,4096,8192").split(",")]
    dev = torch.device("cuda", local)
    f = TpFused(max(Ms), H, dev)
    g = torch.Generator(device=dev).manual_seed(rank)
    wq, sw = kernels.quantize_rows_fp8((torch.randn(H, K, device=dev, generator=g) * 0.02).half())
    nw = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half()
    for M in Ms:
        xq, sx = kernels.quantize_rows_fp8(torch.randn(M, K, device=dev, generator=g).half())
        res = torch.randn(M, H, device=dev, generator=g).half()
        y = torch.empty(M, H, device=dev, dtype=torch.float16)

        def fused():
            f.rowpar_gemm_norm(xq, sx, wq, sw, res, nw, 1e-6)

        def baseline():
            kernels.fp8_gemm(xq, sx, wq, sw, out=y)
            torch.distributed.all_reduce(y, group=tp.tp_group())
            kernels.rmsnorm(y, nw, 1e-6, res, want_fp16=False, want_fp8=True)
        sync_all()
        t_fused = max_over_ranks(time_kernel(fused))
        sync_all()
        t_base = max_over_ranks(time_kernel(baseline))
        sync_all()
        t_gemm = max_over_ranks(time_kernel(lambda: kernels.fp8_gemm(xq, sx, wq, sw, out=y)))
        R = (M + world - 1) // world
        sent = (world - 1) * R * (2 * H + H + 4)
        flops = 2 * M * H * K
        if rank == 0:
            print(json.dumps({"kernel": "tp_rowpar_gemm_allreduce_rmsnorm_fp8", "model": args.model, "tp": world,
                              "M": M, "N": H, "K": K, "fused_us": round(t_fused * 1e6, 2),
                              "gemm_nccl_rmsnorm_us": round(t_base * 1e6, 2), "gemm_alone_us": round(t_gemm * 1e6, 2),
                              "speedup": round(t_base / t_fused, 3),
                              "nvlink_sent_bytes": sent, "nvlink_GBps_if_comm_only": round(sent / t_fused / 1e9, 1),
                              "TFLOPs": round(flops / t_fused / 1e12, 1)}), flush=True)
    status = _lib.device_status()
    if rank == 0:
        print(json.dumps({"kernel": "tp_rowpar", "device_status": status}), flush=True)
    f.close()
    shutdown_distributed()


def run_kernel(args):
    """One kernel on synthetic inputs of a Qwen3 layer's shapes, timed with CUDA events
    (used for the kernel sweeps of BASELINE config 5 and for ncu captures). One JSON line
    per case. With --impl reference the reference's own Triton kernel runs on the same
    inputs (decode attention: fp8_decode_attention; GEMM: _fp8_mm on pre-quantised
    activations, as ms_fp8_gemm takes them), the GPU "beat this" bar."""
    from microserve_b200 import _lib, kernels
    from oracle import fp8_decoder as O
    ref = None
    if args.impl == "reference":
        ref = reference_kernels()
        if ref is None:
            print(json.dumps({"impl": "reference", "kernel": args.kernel,
                              "unavailable": "reference not installed in baseline/_ref"}), flush=True)
            return
    else:
        _lib.load().ms_set_pair_tiles(1 if args.pair_tiles else 0)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    m = MODELS[args.model]
    hbm_peak, _ = peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    if args.kernel == "decode_attention":
        Hq, Hkv = m["heads"] // args.gpus, m["kv_heads"] // args.gpus
        for ctx in [int(c) for c in args.ctx.split(",")]:
            B = args.batch
            nb = (ctx + BLOCK - 1) // BLOCK
            blocks = B * nb
            kc = torch.randint(0, 120, (blocks + 1, BLOCK, Hkv, HEAD_DIM), dtype=torch.uint8, device=dev,
                               generator=g).view(torch.float8_e4m3fn)
            vc = torch.randint(0, 120, (blocks + 1, BLOCK, Hkv, HEAD_DIM), dtype=torch.uint8, device=dev,
                               generator=g).view(torch.float8_e4m3fn)
            ks = torch.rand(blocks + 1, BLOCK, Hkv, device=dev, generator=g) * 1e-2 + 1e-3
            vs = torch.rand(blocks + 1, BLOCK, Hkv, device=dev, generator=g) * 1e-2 + 1e-3
            perm = torch.randperm(blocks, device=dev, generator=g).to(torch.int32)
            bt = perm.view(B, nb)
            lens = torch.full((B,), ctx, dtype=torch.int32, device=dev)
            q = torch.randn(B, Hq, HEAD_DIM, device=dev, dtype=torch.float16, generator=g)
            out = torch.empty_like(q)
            if ref is not None:
                t = time_kernel(lambda: ref[0](q, kc, vc, ks, vs, lens, bt, HEAD_DIM ** -0.5),
                                iters=args.steps, warm=args.warmup)
            else:
                t = time_kernel(lambda: kernels.paged_decode_fp8(q, kc, vc, ks, vs, lens, bt, HEAD_DIM ** -0.5,
                                                                 out=out), iters=args.steps, warm=args.warmup)
            byts = B * ctx * Hkv * (2 * HEAD_DIM + 8) + 2 * B * Hq * HEAD_DIM * 2 + B * (4 + 4 * nb)
            print(json.dumps({"kernel": "decode_attention", "impl": args.impl, "model": args.model, "tp": args.gpus,
                              "batch": B,
                              "ctx": ctx, "q_heads": Hq, "kv_heads": Hkv, "us": round(t * 1e6, 2),
                              "bytes": byts, "GBps": round(byts / t / 1e9, 1),
                              "frac_hbm": round(byts / t / 1e9 / hbm_peak, 4)}), flush=True)
            del kc, vc, ks, vs
    else:
        if args.shapes:
            shapes = [tuple(int(x) for x in sh.split(":")) for sh in args.shapes.split(",")]
        else:
            H, I, Hq, Hkv = m["hidden"], m["inter"], m["heads"], m["kv_heads"]
            t_ = args.gpus
            shapes = [(args.batch, (Hq + 2 * Hkv) * HEAD_DIM // t_, H), (args.batch, H, Hq * HEAD_DIM // t_),
                      (args.batch, 2 * I // t_, H), (args.batch, H, I // t_)]
        for (M, N, K) in shapes:
            xq, sx = O.quantize_rows(torch.randn(M, K).half())
            # enough weight copies that consecutive launches never find their weights in L2
            copies = max(2, -(-256 * 2 ** 20 // (N * K)))
            wqs = [torch.randint(0, 120, (N, K), dtype=torch.uint8, device=dev, generator=g).view(torch.float8_e4m3fn)
                   for _ in range(copies)]
            sw = torch.rand(N, device=dev, generator=g) * 1e-3
            xq, sx = xq.to(dev), sx.to(dev)
            y = torch.empty(M, N, device=dev, dtype=torch.float16)
            it = [0]

            def launch():
                if ref is not None:  # the reference's grid (fp8_linear.py:75-77)
                    ref[1][((M + 15) // 16, (N + 63) // 64)](xq, wqs[it[0] % copies], sx, sw, y, M, N, K)
                else:
                    kernels.fp8_gemm(xq, sx, wqs[it[0] % copies], sw, out=y)
                it[0] += 1
            t = time_kernel(launch, iters=args.steps, warm=args.warmup)
            byts = N * K + M * K + 2 * M * N + 4 * (M + N)
            flops = 2 * M * N * K
            line = {"kernel": "fp8_gemm", "impl": args.impl, "M": M, "N": N, "K": K, "us": round(t * 1e6, 2),
                    "GBps": round(byts / t / 1e9, 1), "frac_hbm": round(byts / t / 1e9 / hbm_peak, 4),
                    "TFLOPs": round(flops / t / 1e12, 1)}
            if ref is None:
                # the library bar: cuBLAS FP8 GEMM (torch._scaled_mm, one scale per tensor, so
                # less epilogue work than the per-row x per-channel dequantisation above)
                one = torch.ones((), device=dev)

                def cublas():
                    torch._scaled_mm(xq, wqs[it[0] % copies].t(), scale_a=one, scale_b=one, out_dtype=torch.float16)
                    it[0] += 1
                try:
                    line["cublas_scaled_mm_us"] = round(time_kernel(cublas, iters=args.steps, warm=args.warmup) * 1e6, 2)
                except RuntimeError as e:  # a shape cuBLAS does not take (K or N not a multiple of 16)
                    line["cublas_scaled_mm_us"] = None
                    line["cublas_error"] = str(e).splitlines()[0][:120]
            print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=sorted(MODELS), default="8b")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--prompt-min", type=int, default=128)
    ap.add_argument("--prompt-max", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=512)
    ap.add_argument("--max-batched-tokens", type=int, default=8192)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="tensor parallel: NCCL all-reduce instead of the fused peer-memory kernel")
    ap.add_argument("--pair-tiles", action="store_true",
                    help="one GPU: GEMM tiles on pairs of SMs (tcgen05 cta_group::2) where the planner finds them faster")
    ap.add_argument("--tp-one-kernel", action="store_true",
                    help="tensor parallel: row-parallel GEMM pushing its rows + reduce/norm tail, one kernel")
    ap.add_argument("--exact-act-scale", action="store_true",
                    help="tensor parallel: row-parallel activation scales from the full row (all-reduce max)")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch the library's kernels without programmatic dependent launch")
    ap.add_argument("--kv-blocks", type=int, default=0, help="KV-cache blocks (0: size from free memory)")
    ap.add_argument("--rows", type=str, default="",
                    help="--kernel tp_rowpar: token counts M, comma list (default 1..8192)")
    ap.add_argument("--kernel", choices=["decode_attention", "gemm", "tp_rowpar"], default=None,
                    help="time one kernel on synthetic inputs (sweeps / profiling) instead of the model")
    ap.add_argument("--ctx", type=str, default="832", help="--kernel decode_attention: context lengths, comma list")
    ap.add_argument("--shapes", type=str, default="",
                    help="--kernel gemm: M:N:K comma list (default: the 8B layer's four linears at M=--batch)")
    args = ap.parse_args()
    assert args.warmup >= 3, "at least 3 warm-up steps"
    if args.kernel == "tp_rowpar":
        run_tp_rowpar_sweep(args)
    elif args.kernel is not None:
        run_kernel(args)  # --impl reference: the reference's own Triton kernel on the same inputs
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
