"""Serving front end: one model runner (weights, KV cache, CUDA graphs) driven by
one scheduler. Public surface as the reference's LLMEngine
(microserve/engine/llm.py:6-53): LLMEngine(config), add(), step(), is_idle(),
generate(), num_running().

A step is: ask the scheduler for a batch, run it on the GPU (the runner checks
the device status word after every step, so a bounded in-kernel wait that ran
out raises there instead of returning tokens), hand the sampled tokens back to
the scheduler, report the sequences that finished.
"""
from __future__ import annotations

from microserve_b200.Config import Config
from microserve_b200.engine.model_runner import ModelRunner
from microserve_b200.engine.scheduler import Scheduler
from microserve_b200.engine.sequence import SamplingParams, Sequence


class LLMEngine:
    def __init__(self, config: Config):
        self.config = config
        self.runner = ModelRunner(config)
        self.scheduler = Scheduler(num_kvcache_blocks=self.runner.num_blocks, block_size=config.block_size,
                                   max_num_seqs=config.max_num_seqs,
                                   max_num_batched_tokens=config.max_num_batched_tokens,
                                   policy=config.scheduler_policy, eos_token_id=config.eos_token_id)

    def add(self, token_ids: list[int], sampling_params: SamplingParams | None = None,
            max_tokens: int = 128) -> Sequence:
        """Queue a request; the returned Sequence fills in as steps run."""
        seq = Sequence(token_ids, sampling_params=sampling_params, max_tokens=max_tokens)
        self.scheduler.add(seq)
        return seq

    def step(self) -> list[Sequence]:
        """Schedule and execute one batch; the sequences that finished in it."""
        batch = self.scheduler.schedule()
        if not batch:
            return []
        tokens = self.runner.execute(batch)
        self.scheduler.postprocess(batch, tokens)
        return [seq for seq in batch if seq.is_finished]

    def is_idle(self) -> bool:
        return self.scheduler.is_idle()

    def num_running(self) -> int:
        return len(self.scheduler.running)

    def generate(self, prompt_token_ids: list[int], sampling_params: SamplingParams | None = None,
                 max_tokens: int = 128) -> list[int]:
        """Run one request (and whatever else is queued) until it finishes; return its
        generated token ids. Raises RuntimeError if the engine stops making progress
        (a step that schedules nothing while the request is unfinished, e.g. a KV
        cache too small for the prompt)."""
        seq = self.add(prompt_token_ids, sampling_params, max_tokens)
        while not seq.is_finished and not self.is_idle():
            self.step()
            if self.scheduler.last_batch_stats is None and not seq.is_finished:
                raise RuntimeError(f"generate: no batch could be scheduled for request {seq.seq_id} "
                                   f"({len(prompt_token_ids)} prompt tokens, "
                                   f"{self.scheduler.block_manager.free_blocks_nums} free KV blocks)")
        return seq.completion_token_ids
