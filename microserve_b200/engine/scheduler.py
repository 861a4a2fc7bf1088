"""Token-budget scheduler with chunked prefill and preemption by recompute.

The decisions (which sequences run, how many tokens each gets, who is
preempted) must equal the reference's (microserve/engine/scheduler.py:7-183),
because the block ids they produce end up in the kernels' block tables and
slot mappings; tests/test_oracle_cpu.py replays scheduler traces recorded from
the reference and checks every round. The behaviour, as rules:

  * A step has a token budget (max_num_batched_tokens). It first continues
    running sequences: under "mixed" all of them, decodes (gap == 1) ahead of
    prefill chunks, otherwise in admission order; under "prefill_first" only
    prefill chunks. It stops at the first sequence with nothing left to do,
    when the budget is spent, or when a sequence cannot get KV blocks even
    after preempting one victim (then the budget is treated as spent).
  * Then it admits waiting prompts in arrival order while budget remains and
    fewer than max_num_seqs sequences run; it stops at the first prompt that
    gets no blocks or no tokens.
  * "prefill_first" runs decodes only in a step that scheduled nothing else,
    with a fresh budget.
  * A victim is the most recently admitted running sequence that is neither
    the requester, nor already scheduled in this step, nor already preempted
    in it; its blocks are freed, it restarts from its prompt and goes to the
    head of the waiting queue.
  * After the model ran, every scheduled sequence records the hashes of the
    blocks it filled and advances; a sequence whose scheduled tokens reached
    its end takes the sampled token (finishing on EOS, which is not appended,
    or on max_tokens).
"""
from __future__ import annotations

from collections import deque
from time import perf_counter

from microserve_b200.engine.block_manager import BlockManager
from microserve_b200.engine.sequence import Sequence, SequenceStatus


class _StepPlan:
    """The batch being assembled for one step and its bookkeeping."""

    __slots__ = ("budget", "batch", "continued", "preempted")

    def __init__(self, budget: int):
        self.budget = budget
        self.batch: list[Sequence] = []
        self.continued: set[int] = set()  # running sequences scheduled in this step
        self.preempted: set[int] = set()  # sequences preempted in this step

    def take(self, seq: Sequence, continued: bool) -> None:
        self.budget -= seq.num_scheduled_tokens
        self.batch.append(seq)
        if continued:
            self.continued.add(seq.seq_id)


class Scheduler:
    POLICIES = ("mixed", "prefill_first")

    def __init__(self, num_kvcache_blocks: int, block_size: int, max_num_seqs: int = 64,
                 max_num_batched_tokens: int = 4096, policy: str = "mixed", eos_token_id: int | None = None):
        if policy not in self.POLICIES:
            raise AssertionError(f"unknown scheduler policy {policy!r}")
        self.block_manager = BlockManager(num_kvcache_blocks, block_size)
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.eos_token_id = eos_token_id
        self.policy = policy
        self.last_batch_stats: dict | None = None
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()

    # ---------------------------------------------------------------- intake
    def add(self, seq: Sequence) -> None:
        now = perf_counter()
        seq.arrived_at = now
        seq.waiting_entered_at = now
        self.waiting.append(seq)

    def is_idle(self) -> bool:
        return len(self.waiting) == 0 and len(self.running) == 0

    # -------------------------------------------------------------- schedule
    def schedule(self) -> list[Sequence] | None:
        plan = _StepPlan(self.max_num_batched_tokens)
        if not self.is_idle():
            self._continue_running(plan, self._continuation_order())
            self._admit_waiting(plan)
            if self.policy == "prefill_first" and not plan.batch:
                fallback = _StepPlan(self.max_num_batched_tokens)
                fallback.continued, fallback.preempted = plan.continued, plan.preempted
                self._continue_running(fallback, [s for s in self.running if s.gap == 1], stop_on_failure=True)
                plan = fallback
        self.last_batch_stats = self._stats(plan.batch)
        return plan.batch or None

    def _continuation_order(self) -> list[Sequence]:
        if self.policy == "prefill_first":
            return [s for s in self.running if s.gap > 1]
        decodes = [s for s in self.running if s.gap == 1]
        chunks = [s for s in self.running if s.gap != 1]
        return decodes + chunks

    def _continue_running(self, plan: _StepPlan, order: list[Sequence], stop_on_failure: bool = False) -> None:
        """Main pass (stop_on_failure False): stops at a sequence with nothing to do and,
        when one cannot be served, spends the budget; skips sequences preempted in this
        step. Decode fallback (True): the order holds decodes only and the pass just
        stops at the first sequence it cannot serve, without the preemption skip (as the
        reference's fallback loop, microserve/engine/scheduler.py:86-96)."""
        for seq in order:
            if plan.budget <= 0 or (not stop_on_failure and seq.gap <= 0):
                return
            if not stop_on_failure and seq.seq_id in plan.preempted:
                continue
            if not self._reserve(seq, plan):
                if not stop_on_failure:
                    plan.budget = 0  # nothing else may jump ahead of a blocked sequence
                return
            plan.take(seq, continued=True)

    def _admit_waiting(self, plan: _StepPlan) -> None:
        while self.waiting and plan.budget > 0 and len(self.running) < self.max_num_seqs:
            seq = self.waiting[0]
            assert not seq.block_table and seq.num_computed_tokens == 0, "a waiting sequence holds KV blocks"
            if not self.block_manager.allocate(seq, plan.budget):
                return
            if seq.gap > 1 and seq.num_scheduled_tokens == 0:
                return
            self.waiting.popleft()
            self.running.append(seq)
            seq.status = SequenceStatus.RUNNING
            if seq.first_scheduled_at is None:
                seq.first_scheduled_at = perf_counter()
            self._set_tokens(seq)
            plan.take(seq, continued=False)

    def _reserve(self, seq: Sequence, plan: _StepPlan) -> bool:
        """KV blocks and a token count for a running sequence, preempting one victim
        if the blocks are short."""
        got = self.block_manager.allocate(seq, plan.budget)
        if not got:
            victim = self._pick_victim(seq, plan)
            if victim is None:
                return False
            self.preempt(victim)
            plan.preempted.add(victim.seq_id)
            got = self.block_manager.allocate(seq, plan.budget)
        if not got or (seq.gap != 1 and seq.num_scheduled_tokens == 0):
            return False
        self._set_tokens(seq)
        return True

    @staticmethod
    def _set_tokens(seq: Sequence) -> None:
        if seq.gap == 1:
            seq.num_scheduled_tokens = 1
        seq.needs_sample = seq.num_computed_tokens + seq.num_scheduled_tokens == seq.num_tokens_with_spec

    def _pick_victim(self, requester: Sequence, plan: _StepPlan) -> Sequence | None:
        for seq in reversed(self.running):
            if seq is requester or seq.seq_id in plan.continued or seq.seq_id in plan.preempted:
                continue
            return seq
        return None

    def preempt(self, seq: Sequence) -> None:
        self.block_manager.deallocate(seq)
        seq.reset_for_preempt()
        if seq in self.running:
            self.running.remove(seq)
        self.waiting.appendleft(seq)

    @staticmethod
    def _stats(batch: list[Sequence]) -> dict | None:
        if not batch:
            return None
        prefill_tokens = sum(s.num_scheduled_tokens for s in batch if s.gap > 1)
        decode_tokens = sum(s.num_scheduled_tokens for s in batch if s.gap == 1)
        return {"prefill": any(s.gap > 1 for s in batch), "decode": any(s.gap == 1 for s in batch),
                "prefill_tokens": prefill_tokens, "decode_tokens": decode_tokens}

    # ----------------------------------------------------------- postprocess
    def postprocess(self, seqs: list[Sequence], output_token_ids: list[int | None]) -> None:
        for seq, token in zip(seqs, output_token_ids):
            self._commit(seq, token)

    def _commit(self, seq: Sequence, token: int | None) -> None:
        self.block_manager.hash_blocks(seq)
        seq.num_computed_tokens += seq.num_scheduled_tokens
        seq.num_scheduled_tokens = 0
        reached_end = seq.num_computed_tokens >= seq.num_tokens_with_spec
        if not reached_end:
            seq.needs_sample = False
            return
        if token is None:
            return
        seq.needs_sample = False
        when = perf_counter()
        if self.eos_token_id is not None and token == self.eos_token_id:
            self._retire(seq)
            return
        seq.append_token(token)
        seq.token_timestamps.append(when)
        if seq.num_completion_tokens >= seq.max_tokens:
            self._retire(seq)

    def _retire(self, seq: Sequence) -> None:
        seq.status = SequenceStatus.FINISHED
        seq.finished_at = perf_counter()
        self.block_manager.deallocate(seq)
        self.running.remove(seq)
