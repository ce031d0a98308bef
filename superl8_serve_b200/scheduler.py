"""Continuous batching over the stage pipeline: the reference's admission policy
(``superl8serve/engine/scheduler.py:33-170``, ``engine/sequence.py``; see ``Scheduler``)
driving ``engine.DecodePipeline`` (the ``PipelineEngine.step`` loop,
``superl8serve/dist/pipeline.py:620-635``).

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
    """Life cycle of a request: queued, holding a KV slot, done (slot returned)."""

    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"


@dataclass
class Sequence:
    """One request. ``prompt_ids`` is what admission prefills; after an eviction it grows to
    every token the request has so far, since its KV is gone and is recomputed."""

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
        """Stop conditions: the token budget, the context limit, or (unless ignored) EOS as
        the last generated token."""
        n_out = len(self.output_ids)
        out_of_budget = n_out >= self.params.max_tokens
        out_of_context = self.max_len is not None and self.num_prompt + n_out >= self.max_len
        hit_eos = (n_out > 0 and eos_id is not None and self.output_ids[-1] == eos_id
                   and not getattr(self.params, "ignore_eos", False))
        return out_of_budget or out_of_context or hit_eos


class Scheduler:
    """Admission and eviction over a KV cache with ``alloc() -> slot``, ``free(slot)``,
    ``has_free_slot()`` and ``has_free_block()`` (the reference's ``Scheduler`` policy,
    ``superl8serve/engine/scheduler.py:33-170``, re-stated below).

    Each ``schedule()`` call returns either a prefill batch (newly admitted requests) or the
    decode batch (every running request), never both:

    1. Admission, FIFO: the head of the queue is admitted while the running count plus the
       batch stays under ``max_num_seqs``, a slot and a block are free, and (after the first
       request of the batch) its prompt fits in what is left of ``max_batch_tokens``.
       Admission takes precedence over decoding.
    2. Eviction, only under genuine block starvation (requests wait, requests run, a slot is
       free but the block pool is empty): the running request with the fewest generated
       tokens gives its slot back and re-queues at the tail with its whole history as its
       prompt; admission is then retried. At most ``max_num_seqs`` evictions per call, so a
       call always ends. Caps on counts or tokens never evict.
    """

    def __init__(self, cache, *, max_num_seqs: int, max_batch_tokens: int, eos_id: int | None):
        self.cache = cache
        self.max_num_seqs = max_num_seqs
        self.max_batch_tokens = max_batch_tokens
        self.eos_id = eos_id
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []

    # ------------------------------------------------------------------ queue edits ----
    def add(self, seq: Sequence):
        self.waiting.append(seq)

    def has_work(self) -> bool:
        return len(self.waiting) + len(self.running) > 0

    def _release(self, seq: Sequence, status: Status):
        """Give a running request's slot back to the cache."""
        self.running.remove(seq)
        self.cache.free(seq.slot)
        seq.status = status

    def cancel(self, seq_id: int) -> bool:
        """Drop a request wherever it is; a running one returns its slot. False if unknown."""
        queued = {s.seq_id: s for s in self.waiting}
        if seq_id in queued:
            self.waiting.remove(queued[seq_id])
            queued[seq_id].status = Status.FINISHED
            return True
        live = {s.seq_id: s for s in self.running}
        if seq_id in live:
            self._release(live[seq_id], Status.FINISHED)
            live[seq_id].slot = -1
            return True
        return False

    # ------------------------------------------------------------------- the policy ----
    def _can_admit(self, batch_size: int, batch_tokens: int) -> bool:
        if not self.waiting:
            return False
        if len(self.running) + batch_size >= self.max_num_seqs:
            return False
        if not (self.cache.has_free_slot() and self.cache.has_free_block()):
            return False
        head = self.waiting[0]
        return batch_size == 0 or batch_tokens + head.num_prompt <= self.max_batch_tokens

    def _admit(self) -> list[Sequence]:
        batch: list[Sequence] = []
        tokens = 0
        while self._can_admit(len(batch), tokens):
            seq = self.waiting.popleft()
            seq.slot = self.cache.alloc()
            seq.status = Status.RUNNING
            tokens += seq.num_prompt
            batch.append(seq)
        return batch

    def _block_starved(self) -> bool:
        return bool(self.waiting and self.running and self.cache.has_free_slot()
                    and not self.cache.has_free_block())

    def evict_least_progressed(self):
        """Evict the running request with the fewest generated tokens (the first such in
        running order). A request that has already met a stop condition just finishes."""
        victim = self.running[0]
        for seq in self.running[1:]:
            if len(seq.output_ids) < len(victim.output_ids):
                victim = seq
        if victim.is_finished(self.eos_id):
            self._release(victim, Status.FINISHED)
            return
        self._release(victim, Status.WAITING)
        victim.prompt_ids = victim.all_token_ids
        victim.length = 0
        victim.slot = -1
        self.waiting.append(victim)

    def schedule(self) -> tuple[list[Sequence], bool]:
        """Returns (batch, is_prefill)."""
        for evictions in range(self.max_num_seqs + 1):
            batch = self._admit()
            if batch:
                return batch, True
            if evictions == self.max_num_seqs or not self._block_starved():
                break
            self.evict_least_progressed()
        return list(self.running), False

    def postprocess(self, batch: list[Sequence], is_prefill: bool):
        """After a step: a prefill batch joins the running set; every running request that
        met a stop condition finishes and returns its slot."""
        if is_prefill:
            self.running.extend(batch)
        for seq in [s for s in self.running if s.is_finished(self.eos_id)]:
            self._release(seq, Status.FINISHED)


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
