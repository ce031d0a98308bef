"""Continuous batching over the stage pipeline: the reference's ``Scheduler`` policy
(``superl8serve/engine/scheduler.py:33-170``) and ``Sequence`` (``engine/sequence.py``),
driving ``engine.DecodePipeline`` (the ``PipelineEngine.step`` loop,
``superl8serve/dist/pipeline.py:620-635``).

Policy (as the reference): WAITING requests are admitted FIFO while RUNNING <
``max_num_seqs``, a slot and a KV block are free and the batch's prompt tokens fit
``max_batch_tokens``; admission is preferred, otherwise the RUNNING set decodes one step. A
mere count cap never preempts. Only when a slot is free but the block pool is dry does the
least-progressed running sequence go back to WAITING (its prompt becomes all its tokens, to
be recomputed), at most ``max_num_seqs`` times per ``schedule()``.

Execution. A KV slot is a fixed pipeline row. Admission prefills every admitted prompt
but its last token into that request's slot (one varlen prefill over those rows) and
parks the last token as the row's next decode input, so every output token, the first
included, comes from a decode step (greedy or the sampler). A decode step runs every row;
rows without a sequence point at a reserved scratch block, so they write and read nothing
that belongs to a request. Each row computes independently of the others, so a request's
tokens do not depend on what else is in the batch.
"""

from __future__ import annotations

import enum
from collections import deque
from dataclasses import dataclass, field

from .dist.pipeline import SamplingParams


class Status(enum.Enum):
    WAITING = enum.auto()
    RUNNING = enum.auto()
    FINISHED = enum.auto()


@dataclass
class Sequence:
    seq_id: int
    prompt_ids: list[int]
    params: SamplingParams
    status: Status = Status.WAITING
    slot: int = -1
    output_ids: list[int] = field(default_factory=list)
    length: int = 0  # KV positions committed
    max_len: int | None = None

    @property
    def num_prompt(self) -> int:
        return len(self.prompt_ids)

    @property
    def all_token_ids(self) -> list[int]:
        return self.prompt_ids + self.output_ids

    def is_finished(self, eos_id: int | None) -> bool:
        if len(self.output_ids) >= self.params.max_tokens:
            return True
        if self.max_len is not None and self.num_prompt + len(self.output_ids) >= self.max_len:
            return True
        return (eos_id is not None and not getattr(self.params, "ignore_eos", False)
                and bool(self.output_ids) and self.output_ids[-1] == eos_id)


class Scheduler:
    """Admission / preemption policy over a cache with ``alloc``, ``free``,
    ``has_free_slot``, ``has_free_block``, ``lookup_prefix`` and ``share_blocks``."""

    def __init__(self, cache, *, max_num_seqs: int, max_batch_tokens: int, eos_id: int | None):
        self.cache = cache
        self.max_num_seqs = max_num_seqs
        self.max_batch_tokens = max_batch_tokens
        self.eos_id = eos_id
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []

    def add(self, seq: Sequence):
        self.waiting.append(seq)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def cancel(self, seq_id: int) -> bool:
        """Drop a request: a WAITING one holds nothing; a RUNNING one frees its slot."""
        for seq in self.waiting:
            if seq.seq_id == seq_id:
                self.waiting.remove(seq)
                seq.status = Status.FINISHED
                return True
        for seq in self.running:
            if seq.seq_id == seq_id:
                self.running.remove(seq)
                seq.status = Status.FINISHED
                self.cache.free(seq.slot)
                seq.slot = -1
                return True
        return False

    def _preempt_one(self):
        victim = min(self.running, key=lambda s: len(s.output_ids))
        self.running.remove(victim)
        self.cache.free(victim.slot)
        if victim.is_finished(self.eos_id):
            victim.status = Status.FINISHED
            return
        victim.prompt_ids = victim.all_token_ids  # recomputed through its whole context
        victim.length = 0
        victim.slot = -1
        victim.status = Status.WAITING
        self.waiting.append(victim)

    def _has_free_block(self) -> bool:
        probe = getattr(self.cache, "has_free_block", None)
        return probe() if probe is not None else True

    def schedule(self) -> tuple[list[Sequence], bool]:
        """Returns (batch, is_prefill)."""
        batch, tokens, preempted = [], 0, 0
        while True:
            while (self.waiting and len(self.running) + len(batch) < self.max_num_seqs
                   and self.cache.has_free_slot() and self._has_free_block()):
                seq = self.waiting[0]
                if batch and tokens + seq.num_prompt > self.max_batch_tokens:
                    break
                self.waiting.popleft()
                seq.slot = self.cache.alloc()
                matched, shared = self.cache.lookup_prefix(seq.prompt_ids)
                if matched > 0 and shared:
                    self.cache.share_blocks(seq.slot, shared)
                seq.status = Status.RUNNING
                tokens += seq.num_prompt
                batch.append(seq)
            if batch:
                return batch, True
            block_pressure = (self.waiting and self.running and self.cache.has_free_slot()
                              and not self._has_free_block())
            if block_pressure and preempted < self.max_num_seqs:
                self._preempt_one()
                preempted += 1
                continue
            return list(self.running), False

    def postprocess(self, batch: list[Sequence], is_prefill: bool):
        if is_prefill:
            self.running.extend(batch)
        still = []
        for seq in self.running:
            if seq.is_finished(self.eos_id):
                seq.status = Status.FINISHED
                self.cache.free(seq.slot)
            else:
                still.append(seq)
        self.running = still


class _SlotCache:
    """The pipeline's block allocator seen through the scheduler's cache contract."""

    def __init__(self, alloc):
        self.a = alloc

    def alloc(self) -> int:
        return self.a.alloc()

    def free(self, slot: int):
        self.a.free(slot)

    def has_free_slot(self) -> bool:
        return bool(self.a._free_slots)

    def has_free_block(self) -> bool:
        return bool(self.a._free_blocks)

    def lookup_prefix(self, token_ids):  # prefix sharing is not built
        return 0, []

    def share_blocks(self, slot, blocks):
        pass


class ContinuousEngine:
    """Requests join and leave a running decode batch (``LLMEngine``-style ``add_request`` /
    ``step`` / ``generate``) over the stages of ``models``; one decode row per slot."""

    def __init__(self, models, *, max_num_seqs: int = 8, max_len: int = 2048,
                 max_batch_tokens: int = 8192, eos_id: int | None = None,
                 wire_scheme: str = "int8-had", pipeline=None):
        """``pipeline``: an already built pipeline with ``max_num_seqs`` rows and one spare
        block (default: a ``DecodePipeline`` over ``models``)."""
        if pipeline is None:
            from .engine import DecodePipeline

            pipeline = DecodePipeline(models, batch=max_num_seqs, n_micro=1, max_len=max_len,
                                      wire_scheme=wire_scheme,
                                      num_blocks=max_num_seqs * -(-max_len // 16) + 1)
        self.pipe = pipeline
        self.pipe.reserve_scratch_block()
        self.max_len = max_len
        self.sched = Scheduler(_SlotCache(self.pipe.alloc), max_num_seqs=max_num_seqs,
                               max_batch_tokens=max_batch_tokens, eos_id=eos_id)
        self.pipe.set_rows(list(range(max_num_seqs)), [0] * max_num_seqs, [0] * max_num_seqs,
                           [None] * max_num_seqs)
        self._next_id = 0
        self.seqs: dict[int, Sequence] = {}
        self._sampling = False

    def add_request(self, prompt_ids: list[int], params: SamplingParams | None = None) -> int:
        if not prompt_ids:
            raise ValueError("empty prompt")
        sid = self._next_id
        self._next_id += 1
        seq = Sequence(sid, list(prompt_ids), params or SamplingParams(), max_len=self.max_len)
        self.seqs[sid] = seq
        self.sched.add(seq)
        return sid

    def cancel(self, seq_id: int) -> bool:
        seq = self.seqs.get(seq_id)
        slot = seq.slot if seq is not None else -1
        ok = self.sched.cancel(seq_id)
        if ok and slot >= 0:
            self.pipe.set_rows([slot], [0], [0], [None])
        return ok

    def _admit(self, batch: list[Sequence]):
        pipe = self.pipe
        for seq in batch:
            need = min(seq.num_prompt + seq.params.max_tokens, self.max_len)
            pipe.alloc.ensure_capacity([seq.slot], [need])
        head = [s for s in batch if s.num_prompt >= 2]
        if head:
            pipe.prefill([s.prompt_ids[:-1] for s in head], slots=[s.slot for s in head],
                         reserve=1)
        for seq in batch:
            seq.length = seq.num_prompt - 1
        pipe.set_rows([s.slot for s in batch], [s.num_prompt - 1 for s in batch],
                      [s.prompt_ids[-1] for s in batch], [s.slot for s in batch])
        samp = [s for s in batch if s.params.temperature != 0.0 or
                s.params.repetition_penalty != 1.0]
        if samp or self._sampling:
            pipe.set_sampling_rows(
                [s.slot for s in batch],
                [{"temperature": s.params.temperature, "top_k": s.params.top_k,
                  "top_p": s.params.top_p, "repetition_penalty": s.params.repetition_penalty,
                  "seed": s.seq_id if s.params.seed is None else s.params.seed} for s in batch],
                [s.prompt_ids for s in batch])
            self._sampling = True

    def step(self) -> list[tuple[int, int]]:
        """One scheduler step: admit (prefill) or decode. Returns (seq_id, token) pairs
        produced by a decode step."""
        batch, is_prefill = self.sched.schedule()
        if not batch:
            return []
        if is_prefill:
            self._admit(batch)
            self.sched.postprocess(batch, True)
            return []
        # every row without a running sequence restarts at position 0 on the scratch block, so
        # its position never walks past its block-table row
        busy = {q.slot for q in self.sched.running}
        idle = [r for r in range(self.pipe.batch) if r not in busy]
        if idle:
            self.pipe.set_rows(idle, [0] * len(idle), [0] * len(idle), [None] * len(idle))
        self.pipe._enqueue()
        self.pipe.synchronize()
        toks = self.pipe.tokens().cpu().tolist()
        out = []
        for seq in batch:
            t = int(toks[seq.slot])
            seq.output_ids.append(t)
            seq.length += 1
            out.append((seq.seq_id, t))
        self.sched.postprocess(batch, False)
        for s in batch:
            if s.status is Status.FINISHED:
                s.slot = -1
        # a running row's next input is the token it just produced (the pipeline leaves it in
        # stage 0's ids); freed rows are parked before the next decode step
        return out

    def run(self) -> dict[int, list[int]]:
        while self.sched.has_work():
            self.step()
        return {sid: s.output_ids for sid, s in self.seqs.items()}

    def generate(self, prompts: list[list[int]], params: SamplingParams | list | None = None):
        plist = params if isinstance(params, list) else [params] * len(prompts)
        ids = [self.add_request(p, sp) for p, sp in zip(prompts, plist)]
        self.run()
        return [self.seqs[i].output_ids for i in ids]
