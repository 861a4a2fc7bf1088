"""Model runner: weights, FP8 KV cache, batch preparation, decode CUDA graphs
and sampling (microserve/engine/model_runner.py:36-338), B200 version.

Same responsibilities and the same integer formulas as the reference:
  slot(p)       = block_table[p // block_size] * block_size + p % block_size  (:135-137)
  block tables  = int32 rows padded with -1 to the batch's longest table    (:208-216)
  decode graphs = one per batch size in {1,2,4,8} U {16,32,...,max_num_seqs};
                  pad rows write the garbage slot and have seqlen 0         (:257-281, :306-338)
Differences, all host-side or scheduling-neutral:
  * metadata is built with numpy and crosses to the GPU in ONE pinned copy
    per forward (the reference writes each element with its own copy);
  * all chunked-prefill sequences of a step run in one forward (the
    reference runs one forward per sequence) - per-token results are equal;
  * the decode graph also holds the LM head and the greedy argmax, so a
    greedy step reads back B token ids instead of B logit rows;
  * sampled tokens come back in one device->host copy per forward.
"""
from __future__ import annotations

import itertools

import numpy as np
import torch

from microserve_b200.Config import Config
from microserve_b200 import _lib, kernels
from microserve_b200.engine.sequence import Sequence
from microserve_b200.layers.attention import Attention
from microserve_b200.layers.fp8_linear import quantize_fp8_linears
from microserve_b200.models.qwen3 import Qwen3ForCausalLM
from microserve_b200.utils import dist as tp
from microserve_b200.utils.context import AttentionMode, Context, reset_context, set_context
from microserve_b200.utils.loader import load_dummy, load_model


def _load_hf_config(config: Config):
    if config.hf_config is not None:
        return config.hf_config
    from transformers import AutoConfig
    return AutoConfig.from_pretrained(config.model_dir, trust_remote_code=True)


class _HostBatch:
    """Packs int64 / int32 metadata arrays into one pinned buffer and moves
    them to the GPU with a single copy; returns device views."""

    def __init__(self, device):
        self.device = device
        self.host = torch.empty(0, dtype=torch.uint8).pin_memory()
        self.dev = torch.empty(0, dtype=torch.uint8, device=device)
        self.bytes_uploaded = 0

    def upload(self, arrays: list[np.ndarray]) -> list[torch.Tensor]:
        offs, total = [], 0
        for a in arrays:
            total = (total + 15) // 16 * 16
            offs.append(total)
            total += a.nbytes
        if self.host.numel() < total:
            self.host = torch.empty(max(total, 2 * self.host.numel()), dtype=torch.uint8).pin_memory()
        # the previous upload may still be in flight from this buffer
        torch.cuda.current_stream().synchronize() if self.dev.numel() else None
        hbuf = self.host.numpy()
        for a, o in zip(arrays, offs):
            hbuf[o:o + a.nbytes] = a.reshape(-1).view(np.uint8)
        dev = torch.empty(total, dtype=torch.uint8, device=self.device)
        dev.copy_(self.host[:total], non_blocking=True)
        self.dev = dev
        self.bytes_uploaded += total
        out = []
        for a, o in zip(arrays, offs):
            t = dev[o:o + a.nbytes].view(torch.int64 if a.dtype == np.int64 else torch.int32)
            out.append(t.view(a.shape))
        return out


class ModelRunner:
    def __init__(self, config: Config):
        self.config = config
        self.block_size = config.block_size
        self.num_blocks = config.num_kvcache_blocks
        self.enforce_eager = config.enforce_eager
        self.device = torch.device("cuda", torch.cuda.current_device())
        if config.tensor_parallel_size != tp.tp_size():
            raise RuntimeError(f"tensor_parallel_size={config.tensor_parallel_size} but the process group has "
                               f"{tp.tp_size()} ranks (call utils.dist.init_tensor_parallel first)")

        tp.set_exact_act_scale(config.tp_exact_act_scale)
        # GEMMs on SM pairs (thread-block clusters): opt-in, one GPU only; under tensor
        # parallelism every GEMM keeps one-SM tiles, the schedules verified with the
        # peer-memory collectives around them
        _lib.load().ms_set_pair_tiles(1 if (tp.tp_size() == 1 and config.gemm_pair_tiles) else 0)
        self.hf_config = hf = _load_hf_config(config)
        self.num_kv_heads = hf.num_key_value_heads // tp.tp_size()
        self.head_dim = getattr(hf, "head_dim", None) or hf.hidden_size // hf.num_attention_heads
        self.num_layers = hf.num_hidden_layers
        self.max_model_len = min(config.max_model_len, hf.max_position_embeddings)
        self.max_decode_blocks = (self.max_model_len + config.block_size - 1) // config.block_size
        self.vocab_size = hf.vocab_size
        if config.seed is not None:
            torch.manual_seed(config.seed)
        self.sample_gen = torch.Generator(device=self.device)
        self.sample_gen.manual_seed(config.seed or 0)

        prev = torch.get_default_dtype()
        torch.set_default_dtype(config.dtype)
        try:
            with torch.device(self.device):
                self.model = Qwen3ForCausalLM(hf, fused_rmsnorm=config.fused_rmsnorm)
        finally:
            torch.set_default_dtype(prev)
        self.model = self.model.to(self.device)
        if config.load_format == "dummy":
            load_dummy(self.model, hf, config.seed, self.device)
        else:
            load_model(self.model, config.model_dir)
        self.model.eval()
        self.model.requires_grad_(False)
        self.num_quantized_linears = 0
        if config.quantization == "fp8_dynamic":
            if config.dtype != torch.float16:
                raise ValueError("FP8 quantization requires torch.float16")
            self.num_quantized_linears = quantize_fp8_linears(self.model)
        # Tensor parallel on the FP8 path: row-parallel sums fused with the add + RMSNorm +
        # FP8 quantisation that follow them, over peer memory (utils/tp_fused.py).
        self.tp_fused = None
        if (tp.tp_size() > 1 and config.tp_fused_collective and self.num_quantized_linears > 0
                and config.kv_cache_dtype == "fp8_e4m3"):
            from microserve_b200.utils.tp_fused import TpFused
            rows = max(config.max_num_batched_tokens, (config.max_num_seqs + 15) // 16 * 16)
            self.tp_fused = TpFused(rows, hf.hidden_size, self.device, fused_gemm=config.tp_fused_gemm)
            self.model.model.tp_fused = self.tp_fused
        torch.cuda.empty_cache()

        if self.num_blocks <= 0:
            self.num_blocks = self._auto_num_blocks()
        self.garbage_slot = self.num_blocks * self.block_size
        cache_dtype = torch.float8_e4m3fn if config.kv_cache_dtype == "fp8_e4m3" else config.dtype
        self.kv_cache = torch.zeros(2, self.num_layers, self.num_blocks + 1, self.block_size, self.num_kv_heads,
                                    self.head_dim, dtype=cache_dtype, device=self.device)
        self.kv_scale_cache = None
        if config.kv_cache_dtype == "fp8_e4m3":
            self.kv_scale_cache = torch.ones(2, self.num_layers, self.num_blocks + 1, self.block_size,
                                             self.num_kv_heads, dtype=torch.float32, device=self.device)
        self._inject_kv_cache()
        self.host_batch = _HostBatch(self.device)

        self.graph_bs: list[int] = []
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_pool = None
        self.graph_vars: dict | None = None
        self.kernels_per_decode_step: dict[int, int] = {}  # library launches captured per graph
        if not self.enforce_eager:
            self._warmup()
            self._capture_decode_graphs()

    # ------------------------------------------------------------------ setup
    def _auto_num_blocks(self) -> int:
        cfg = self.config
        free, total = torch.cuda.mem_get_info()
        if cfg.kv_cache_dtype == "fp8_e4m3":
            per_block = 2 * self.num_layers * self.block_size * self.num_kv_heads * (self.head_dim + 4)
        else:
            per_block = 2 * self.num_layers * self.block_size * self.num_kv_heads * self.head_dim * 2
        available = (free + total * (cfg.gpu_memory_utilization - 1.0)) * 0.8
        return max(1, int(available // per_block))

    def _inject_kv_cache(self) -> None:
        layer_id = 0
        for module in self.model.modules():
            if isinstance(module, Attention):
                module.k_cache = self.kv_cache[0, layer_id]
                module.v_cache = self.kv_cache[1, layer_id]
                if self.kv_scale_cache is not None:
                    module.k_scale_cache = self.kv_scale_cache[0, layer_id]
                    module.v_scale_cache = self.kv_scale_cache[1, layer_id]
                module.kv_cache_dtype = self.config.kv_cache_dtype
                layer_id += 1
        assert layer_id == self.num_layers

    # ------------------------------------------------------- batch preparation
    def _slots(self, table: list[int], positions: np.ndarray) -> np.ndarray:
        bt = np.asarray(table, dtype=np.int64)
        return bt[positions // self.block_size] * self.block_size + positions % self.block_size

    def _tables(self, seqs: list[Sequence], width: int | None = None) -> np.ndarray:
        """Block tables as rows of int32, padded with -1 (one flat copy, no per-row writes)."""
        n = len(seqs)
        lens = np.fromiter((len(s.block_table) for s in seqs), dtype=np.int64, count=n)
        width = width or int(lens.max())
        flat = np.fromiter(itertools.chain.from_iterable(s.block_table for s in seqs), dtype=np.int32,
                           count=int(lens.sum()))
        bt = np.full((n, width), -1, dtype=np.int32)
        bt[np.arange(width)[None, :] < lens[:, None]] = flat
        return bt

    def prepare_decode(self, seqs: list[Sequence]):
        """Host arrays of a decode batch: ids, positions, slots (int64), seqlens, tables (int32).
        slot = block_table[p // block_size] * block_size + p % block_size (model_runner.py:135-136
        of the reference), read from the padded table of the batch. The tables always have
        the width of max_model_len (as the captured graphs' tables do): the decode
        attention's context split depends on that width, so eager and graph decodes of
        the same batch then run the same split and give the same bits."""
        n = len(seqs)
        assert all(s.gap == 1 and s.num_scheduled_tokens == 1 for s in seqs)
        pos = np.fromiter((s.num_computed_tokens for s in seqs), dtype=np.int64, count=n)
        ids = np.fromiter((s.token_ids[s.num_computed_tokens] for s in seqs), dtype=np.int64, count=n)
        bt = self._tables(seqs, width=max(self.max_decode_blocks, max(len(s.block_table) for s in seqs)))
        bs = self.block_size
        blk = bt[np.arange(n), pos // bs]
        if (blk < 0).any():
            raise RuntimeError("decode position beyond the sequence's allocated blocks")
        slots = blk.astype(np.int64) * bs + pos % bs
        return ids, pos, slots, (pos + 1).astype(np.int32), bt

    def prepare_prefill(self, seqs: list[Sequence]):
        ids, pos, slots, cu = [], [], [], [0]
        for s in seqs:
            assert s.num_computed_tokens == 0 and s.gap > 1
            n = s.num_scheduled_tokens
            p = np.arange(n, dtype=np.int64)
            ids.append(np.asarray(s.token_ids[:n], dtype=np.int64))
            pos.append(p)
            slots.append(self._slots(s.block_table, p))
            cu.append(cu[-1] + n)
        return (np.concatenate(ids), np.concatenate(pos), np.concatenate(slots), np.asarray(cu, dtype=np.int32))

    def prepare_chunk(self, seqs: list[Sequence]):
        ids, pos, slots, cu, kv = [], [], [], [0], []
        for s in seqs:
            start, n = s.num_computed_tokens, s.num_scheduled_tokens
            assert start > 0 and s.gap > 1 and n > 0
            p = np.arange(start, start + n, dtype=np.int64)
            ids.append(np.asarray(s.token_ids[start:start + n], dtype=np.int64))
            pos.append(p)
            slots.append(self._slots(s.block_table, p))
            cu.append(cu[-1] + n)
            kv.append(start + n)
        return (np.concatenate(ids), np.concatenate(pos), np.concatenate(slots), np.asarray(cu, dtype=np.int32),
                np.asarray(kv, dtype=np.int32), self._tables(seqs))

    @staticmethod
    def _partition_batch(seqs: list[Sequence]):
        decode, prefill, chunk = [], [], []
        for index, seq in enumerate(seqs):
            item = (index, seq)
            if seq.gap == 1:
                decode.append(item)
            elif seq.num_computed_tokens == 0:
                prefill.append(item)
            else:
                chunk.append(item)
        return decode, prefill, chunk

    # ---------------------------------------------------------------- execute
    @torch.inference_mode()
    def execute(self, seqs: list[Sequence]) -> list[int | None]:
        decode, prefill, chunk = self._partition_batch(seqs)
        outputs: list[int | None] = [None] * len(seqs)
        try:
            if decode:
                idx, group = map(list, zip(*decode))
                for i, t in zip(idx, self._run_decode_group(group)):
                    outputs[i] = t
            if prefill:
                idx, group = map(list, zip(*prefill))
                ids, pos, slots, cu = self.prepare_prefill(group)
                d_ids, d_pos, d_slots, d_cu = self.host_batch.upload([ids, pos, slots, cu])
                n = int(cu[-1])
                set_context(Context(mode=AttentionMode.PREFILL, cu_seqlens_q=d_cu, cu_seqlens_k=d_cu,
                                    max_seqlen_q=int(np.diff(cu).max()), max_seqlen_k=int(np.diff(cu).max()),
                                    slot_mapping=d_slots))
                hidden = self.model(d_ids, d_pos)
                last = torch.as_tensor(cu[1:] - 1, dtype=torch.int64).to(self.device, non_blocking=True)
                for i, t in zip(idx, self._sample_rows(group, hidden.index_select(0, last))):
                    outputs[i] = t
                del n
            if chunk:
                idx, group = map(list, zip(*chunk))
                ids, pos, slots, cu, kv, bt = self.prepare_chunk(group)
                d_ids, d_pos, d_slots, d_cu, d_kv, d_bt = self.host_batch.upload([ids, pos, slots, cu, kv, bt])
                set_context(Context(mode=AttentionMode.CHUNK_PREFILL, slot_mapping=d_slots, block_tables=d_bt,
                                    cache_seqlens=d_kv, cu_seqlens_q=d_cu, max_seqlen_q=int(np.diff(cu).max()),
                                    max_seqlen_k=int(kv.max()),
                                    prefix_len=int(kv[0] - (cu[1] - cu[0])), query_len=int(cu[1] - cu[0])))
                hidden = self.model(d_ids, d_pos)
                last = torch.as_tensor(cu[1:] - 1, dtype=torch.int64).to(self.device, non_blocking=True)
                for i, t in zip(idx, self._sample_rows(group, hidden.index_select(0, last))):
                    outputs[i] = t
        finally:
            reset_context()
        return outputs

    def _run_decode_group(self, group: list[Sequence]) -> list[int | None]:
        bs = len(group)
        ids, pos, slots, seqlens, bt = self.prepare_decode(group)
        if not self.enforce_eager and self.graphs and bs <= self.graph_bs[-1]:
            gv = self.graph_vars
            bsg = next(b for b in self.graph_bs if b >= bs)
            width = gv["block_tables"].shape[1]
            if bt.shape[1] > width:
                raise RuntimeError("block table wider than max_model_len allows")
            # pad rows: garbage slot, seqlen 0, table -1 (the reference's padding)
            pad_ids = np.zeros(bsg, np.int64); pad_ids[:bs] = ids
            pad_pos = np.zeros(bsg, np.int64); pad_pos[:bs] = pos
            pad_slots = np.full(bsg, self.garbage_slot, np.int64); pad_slots[:bs] = slots
            pad_len = np.zeros(bsg, np.int32); pad_len[:bs] = seqlens
            pad_bt = np.full((bsg, width), -1, np.int32); pad_bt[:bs, :bt.shape[1]] = bt
            d = self.host_batch.upload([pad_ids, pad_pos, pad_slots, pad_len, pad_bt])
            gv["input_ids"][:bsg].copy_(d[0])
            gv["positions"][:bsg].copy_(d[1])
            gv["slot_mapping"][:bsg].copy_(d[2])
            gv["cache_seqlens"][:bsg].copy_(d[3])
            gv["block_tables"][:bsg].copy_(d[4])
            self.graphs[bsg].replay()
            return self._finish_sampling(group, gv["logits"][:bs], gv["argmax"][:bs])
        d_ids, d_pos, d_slots, d_len, d_bt = self.host_batch.upload([ids, pos, slots, seqlens, bt])
        set_context(Context(mode=AttentionMode.DECODE, slot_mapping=d_slots, cache_seqlens=d_len,
                            block_tables=d_bt))
        hidden = self.model(d_ids, d_pos)
        return self._sample_rows(group, hidden)

    # --------------------------------------------------------------- sampling
    def _logits_and_argmax(self, hidden: torch.Tensor):
        logits = self.model.compute_logits(hidden)
        if tp.tp_size() == 1:
            return logits, kernels.argmax_rows(logits)
        return logits, tp.tp_argmax(logits, self.model.lm_head.vocab_start)

    def _sample_rows(self, seqs: list[Sequence], hidden: torch.Tensor) -> list[int | None]:
        logits, greedy = self._logits_and_argmax(hidden)
        return self._finish_sampling(seqs, logits, greedy)

    def _full_logits(self, logits: torch.Tensor) -> torch.Tensor:
        if tp.tp_size() == 1:
            return logits
        parts = [torch.empty_like(logits) for _ in range(tp.tp_size())]
        torch.distributed.all_gather(parts, logits.contiguous(), group=tp.tp_group())
        return torch.cat(parts, dim=-1)[:, :self.vocab_size]

    def _finish_sampling(self, seqs: list[Sequence], logits: torch.Tensor, greedy: torch.Tensor):
        """Greedy rows from the argmax; temperature rows follow the reference's
        `_sample` (temperature, top-k, top-p, multinomial; model_runner.py:15-34)."""
        hot = [i for i, s in enumerate(seqs)
               if s.needs_sample and s.sampling_params.temperature is not None and s.sampling_params.temperature > 0]
        tokens = greedy.clone()
        if hot:
            full = self._full_logits(logits)
            for i in hot:
                tokens[i] = self._sample_one(full[i], seqs[i].sampling_params)
        host = tokens.to("cpu").tolist()
        # the copy above synchronised the stream: a bounded in-kernel wait that ran out
        # during this step (a peer rank that died or fell out of step) makes it invalid
        _lib.raise_on_device_status("model step")
        return [host[i] if s.needs_sample else None for i, s in enumerate(seqs)]

    def _sample_one(self, row: torch.Tensor, p) -> torch.Tensor:
        logits = row.float() / p.temperature
        if p.top_k is not None and p.top_k > 0:
            k = min(p.top_k, logits.numel())
            kth = torch.topk(logits, k).values[-1]
            logits = logits.masked_fill(logits < kth, float("-inf"))
        probs = torch.softmax(logits, dim=-1)
        if p.top_p is not None and 0.0 < p.top_p < 1.0:
            sp, si = torch.sort(probs, descending=True)
            cut = torch.cumsum(sp, dim=-1) - sp > p.top_p
            sp = sp.masked_fill(cut, 0.0)
            probs = torch.zeros_like(probs).scatter_(-1, si, sp)
            probs = probs / probs.sum(dim=-1, keepdim=True)
        return torch.multinomial(probs, 1, generator=self.sample_gen)[0]

    # ------------------------------------------------------------ CUDA graphs
    def _reserve_workspace(self, max_bs: int, max_blocks: int) -> None:
        from microserve_b200 import _lib
        lib = _lib.load()
        hf = self.hf_config
        gemm = decode = 0
        for bs in self.graph_bs:
            for m in self.model.modules():
                if hasattr(m, "weight_fp8"):
                    gemm = max(gemm, lib.ms_fp8_gemm_workspace_size(bs, m.out_features, m.in_features))
            decode = max(decode, kernels.decode_workspace_bytes(bs, hf.num_attention_heads // tp.tp_size(),
                                                                self.num_kv_heads, max_blocks, self.block_size))
        kernels.workspace.reserve(gemm, self.device, "gemm")
        kernels.workspace.reserve(decode, self.device, "decode")
        kernels.workspace.reserve(lib.ms_argmax_workspace_size(max_bs), self.device, "argmax")

    @torch.inference_mode()
    def _warmup(self) -> None:
        ctx = Context(mode=AttentionMode.DECODE,
                      slot_mapping=torch.tensor([self.garbage_slot], dtype=torch.int64, device=self.device),
                      cache_seqlens=torch.tensor([1], dtype=torch.int32, device=self.device),
                      block_tables=torch.tensor([[self.num_blocks]], dtype=torch.int32, device=self.device))
        set_context(ctx)
        try:
            self.model(torch.tensor([0], device=self.device), torch.tensor([0], device=self.device))
        finally:
            reset_context()

    @torch.inference_mode()
    def _capture_decode_graphs(self) -> None:
        max_bs = self.config.max_num_seqs
        self.graph_bs = sorted(b for b in ({1, 2, 4, 8} | set(range(16, max_bs + 1, 16))) if b <= max(max_bs, 1))
        if self.graph_bs[-1] < max_bs:
            self.graph_bs.append(max_bs)
        max_blocks = (self.max_model_len + self.block_size - 1) // self.block_size
        dev = self.device
        V_local = self.model.lm_head.weight.shape[0]
        gv = dict(
            input_ids=torch.zeros(max_bs, dtype=torch.int64, device=dev),
            positions=torch.zeros(max_bs, dtype=torch.int64, device=dev),
            slot_mapping=torch.full((max_bs,), self.garbage_slot, dtype=torch.int64, device=dev),
            cache_seqlens=torch.zeros(max_bs, dtype=torch.int32, device=dev),
            block_tables=torch.full((max_bs, max_blocks), -1, dtype=torch.int32, device=dev),
            outputs=torch.zeros(max_bs, self.hf_config.hidden_size, dtype=self.config.dtype, device=dev),
            logits=torch.zeros(max_bs, V_local, dtype=self.config.dtype, device=dev),
            argmax=torch.zeros(max_bs, dtype=torch.int64, device=dev),
        )
        self.graph_vars = gv
        self._reserve_workspace(max_bs, max_blocks)
        from microserve_b200 import _lib
        lib = _lib.load()

        def body(bs):
            h = self.model(gv["input_ids"][:bs], gv["positions"][:bs])
            gv["outputs"][:bs] = h
            logits, am = self._logits_and_argmax(h)
            gv["logits"][:bs] = logits
            gv["argmax"][:bs] = am

        for bs in reversed(self.graph_bs):  # largest first: the pool is sized once
            set_context(Context(mode=AttentionMode.DECODE, slot_mapping=gv["slot_mapping"][:bs],
                                cache_seqlens=gv["cache_seqlens"][:bs], block_tables=gv["block_tables"][:bs]))
            body(bs)  # eager run: sets kernel attributes, tensor maps, allocator state
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            n0 = lib.ms_launch_count()
            with torch.cuda.graph(graph, pool=self.graph_pool):
                body(bs)
            self.kernels_per_decode_step[bs] = lib.ms_launch_count() - n0
            if self.graph_pool is None:
                self.graph_pool = graph.pool()
            self.graphs[bs] = graph
            reset_context()
        torch.cuda.synchronize()

    def release_graphs(self) -> None:
        """Destroy the captured graphs (needed before destroying an NCCL process group:
        a live graph that holds NCCL calls keeps the communicator busy). reset() frees
        each executable graph even if a caller still holds a reference to it."""
        torch.cuda.synchronize(self.device)
        for g in self.graphs.values():
            g.reset()
        self.graphs.clear()
        self.graph_pool = None
