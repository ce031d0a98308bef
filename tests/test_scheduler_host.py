"""CPU: the continuous-batching policy (``Scheduler``) against the reference's own policy
tests (``tests/test_scheduler.py`` in superl8-serve), driven with an in-memory cache and no
model: count caps never preempt, FIFO completion with bounded work, preemption only under
genuine block-pool exhaustion, cancellation."""

from superl8_serve_b200.dist.pipeline import SamplingParams
from superl8_serve_b200.scheduler import Scheduler, Sequence, Status


class FakeCache:
    def __init__(self, num_slots, *, block_size=16, max_len=256, num_blocks=None):
        self.block_size = block_size
        self.max_blocks_per_seq = (max_len + block_size - 1) // block_size
        self.num_blocks = num_blocks if num_blocks is not None else num_slots * self.max_blocks_per_seq
        self._free_slots = list(range(num_slots))
        self._free_blocks = list(range(self.num_blocks))
        self._slot_blocks = {s: [] for s in range(num_slots)}

    def alloc(self):
        return self._free_slots.pop()

    def free(self, slot):
        self._free_blocks.extend(self._slot_blocks[slot])
        self._slot_blocks[slot] = []
        self._free_slots.append(slot)

    def has_free_slot(self):
        return bool(self._free_slots)

    def has_free_block(self):
        return bool(self._free_blocks)

    def ensure_capacity(self, slots, lengths):
        for slot, n in zip(slots, lengths):
            need = (n + self.block_size - 1) // self.block_size
            while len(self._slot_blocks[slot]) < need:
                self._slot_blocks[slot].append(self._free_blocks.pop())


def _run(sched, seqs, max_tokens):
    for s in seqs:
        sched.add(s)
    count = {"preempt": 0}
    orig = sched.evict_least_progressed

    def counting():
        count["preempt"] += 1
        orig()

    sched.evict_least_progressed = counting
    work, calls, steps = 0, {}, 0
    while sched.has_work():
        assert steps < 100_000
        batch, is_prefill = sched.schedule()
        if not batch:
            break
        steps += 1
        for seq in batch:
            if is_prefill:
                sched.cache.ensure_capacity([seq.slot], [seq.num_prompt])
                seq.length = seq.num_prompt
                work += seq.num_prompt
                calls[seq.seq_id] = calls.get(seq.seq_id, 0) + 1
            else:
                seq.length += 1
                sched.cache.ensure_capacity([seq.slot], [seq.length + 1])
            seq.output_ids.append(7)
        sched.postprocess(batch, is_prefill)
    return count["preempt"], work, calls, steps


def _mk(prompts, max_tokens):
    return [Sequence(i, list(p), SamplingParams(max_tokens=max_tokens)) for i, p in enumerate(prompts)]


def test_no_preemption_under_count_cap():
    sched = Scheduler(FakeCache(4), max_num_seqs=4, max_batch_tokens=8192, eos_id=None)
    prompts = [[1, 2, 3], [4, 5, 6, 7], [8], [9, 10], [11, 12, 13, 14, 15], [16], [17, 18], [19]]
    seqs = _mk(prompts, 6)
    pre, work, calls, _ = _run(sched, seqs, 6)
    assert pre == 0 and all(c == 1 for c in calls.values())
    assert work == sum(len(p) for p in prompts)
    assert all(len(s.output_ids) == 6 and s.status is Status.FINISHED for s in seqs)


def test_all_requests_complete_with_bounded_work():
    sched = Scheduler(FakeCache(4), max_num_seqs=4, max_batch_tokens=8192, eos_id=None)
    seqs = _mk([[i + 1, i + 2, i + 3] for i in range(24)], 5)
    pre, _, _, steps = _run(sched, seqs, 5)
    assert pre == 0 and all(len(s.output_ids) == 5 for s in seqs)
    assert steps <= 6 * (24 // 4 + 5)


def _admit(sched, seq):
    sched.add(seq)
    batch, is_prefill = sched.schedule()
    assert is_prefill and seq in batch
    sched.cache.ensure_capacity([seq.slot], [seq.num_prompt])
    seq.length = seq.num_prompt
    seq.output_ids.append(7)
    sched.postprocess(batch, is_prefill)


def test_count_cap_never_preempts():
    cache = FakeCache(3)
    sched = Scheduler(cache, max_num_seqs=3, max_batch_tokens=8192, eos_id=None)
    for i, p in enumerate([[1, 2], [3, 4], [5, 6]]):
        _admit(sched, Sequence(i, p, SamplingParams(max_tokens=50)))
    sched.add(Sequence(99, [7, 8], SamplingParams(max_tokens=50)))
    batch, is_prefill = sched.schedule()
    assert not is_prefill and len(batch) == 3 and len(sched.waiting) == 1


def test_preemption_only_on_block_exhaustion():
    cache = FakeCache(4)
    sched = Scheduler(cache, max_num_seqs=4, max_batch_tokens=8192, eos_id=None)
    _admit(sched, Sequence(0, [1, 2, 3], SamplingParams(max_tokens=50)))
    _admit(sched, Sequence(1, [4, 5, 6], SamplingParams(max_tokens=50)))
    sched.running[1].output_ids.append(7)
    cache._free_blocks.clear()
    sched.add(Sequence(2, [8, 9], SamplingParams(max_tokens=50)))
    batch, is_prefill = sched.schedule()
    assert is_prefill and batch
    assert 0 not in {s.seq_id for s in sched.running}
    victim = next(s for s in list(sched.waiting) + batch if s.seq_id == 0)
    assert victim.prompt_ids == [1, 2, 3, 7]  # recomputed through its generated token


def test_batch_token_budget_splits_admission():
    sched = Scheduler(FakeCache(8), max_num_seqs=8, max_batch_tokens=10, eos_id=None)
    for i in range(4):
        sched.add(Sequence(i, [1] * 6, SamplingParams(max_tokens=3)))
    batch, is_prefill = sched.schedule()
    assert is_prefill and [s.seq_id for s in batch] == [0]  # 6 + 6 > 10


def test_eos_finishes_and_frees_the_slot():
    cache = FakeCache(2)
    sched = Scheduler(cache, max_num_seqs=2, max_batch_tokens=8192, eos_id=5)
    _admit(sched, Sequence(0, [1, 2], SamplingParams(max_tokens=50)))
    sched.running[0].output_ids.append(5)
    sched.postprocess([], False)
    assert not sched.running and cache.has_free_slot() and len(cache._free_slots) == 2


def test_cancel_waiting_and_running():
    cache = FakeCache(2)
    sched = Scheduler(cache, max_num_seqs=2, max_batch_tokens=8192, eos_id=None)
    _admit(sched, Sequence(0, [1, 2], SamplingParams(max_tokens=50)))
    sched.add(Sequence(1, [3], SamplingParams(max_tokens=50)))
    free_before = len(cache._free_slots)
    assert sched.cancel(1) and len(cache._free_slots) == free_before
    assert sched.cancel(0) and len(cache._free_slots) == free_before + 1
    assert not sched.cancel(0) and not sched.has_work()


# ---- ContinuousEngine bookkeeping on a model-free pipeline -----------------------------

class FakePipe:
    """Rows with the DecodePipeline state calls the engine uses; a row's next token is a
    fixed function of its input id and position (what a per-row model step computes)."""

    def __init__(self, batch, max_len, V=97):
        from superl8_serve_b200.engine import BlockAllocator

        self.batch, self.max_len, self.V = batch, max_len, V
        self.max_blocks = -(-max_len // 16)
        self.alloc = BlockAllocator(batch * self.max_blocks + 1, batch, 16, self.max_blocks)
        self.scratch_block = None
        self.pos = [0] * batch
        self.ids = [0] * batch
        self.slot_of = [None] * batch
        self.out = [0] * batch
        self.kv = {}  # (slot, position) -> token written there
        self.max_seen_pos = 0

    def reserve_scratch_block(self):
        self.scratch_block = self.alloc._free_blocks.pop(0)
        return self.scratch_block

    def set_rows(self, rows, positions, ids, slots):
        for r, p, i, s in zip(rows, positions, ids, slots):
            self.pos[r], self.ids[r], self.slot_of[r] = p, i, s

    def prefill(self, prompts, *, slots, reserve=1):
        for p, s in zip(prompts, slots):
            for t, tok in enumerate(p):
                self.kv[(s, t)] = tok

    def set_sampling_rows(self, rows, params, prompts):
        raise AssertionError("greedy only here")

    @staticmethod
    def model(tok, pos, V):
        return (tok * 31 + pos * 7 + 3) % V

    def _enqueue(self):
        for r in range(self.batch):
            assert self.pos[r] < self.max_len
            self.max_seen_pos = max(self.max_seen_pos, self.pos[r])
            s = self.slot_of[r]
            if s is not None:
                # causal history must be present: every position before this one
                assert all((s, t) in self.kv for t in range(self.pos[r])), (r, s, self.pos[r])
                self.kv[(s, self.pos[r])] = self.ids[r]
            self.out[r] = self.model(self.ids[r], self.pos[r], self.V)
            self.ids[r] = self.out[r]
            self.pos[r] += 1

    def synchronize(self):
        pass

    def tokens(self):
        import torch

        return torch.tensor(self.out)


def _solo(prompt, n, V=97):
    toks, pos, tok, out = list(prompt), len(prompt) - 1, prompt[-1], []
    for _ in range(n):
        tok = FakePipe.model(tok, pos, V)
        out.append(tok)
        pos += 1
    return out


def test_continuous_engine_bookkeeping_on_a_fake_pipeline():
    from superl8_serve_b200.dist.pipeline import SamplingParams
    from superl8_serve_b200.scheduler import ContinuousEngine

    pipe = FakePipe(batch=3, max_len=48)
    eng = ContinuousEngine(None, max_num_seqs=3, max_len=48, max_batch_tokens=10, pipeline=pipe)
    prompts = [[5, 6, 7], [1], [9, 9, 9, 9, 9, 9], [2, 3], [4, 4, 4, 4], [8], [11, 12, 13]]
    maxt = [5, 9, 3, 7, 4, 12, 6]
    outs = eng.generate(prompts, [SamplingParams(max_tokens=m) for m in maxt])
    for p, m, o in zip(prompts, maxt, outs):
        assert o == _solo(p, m)
    assert not eng.sched.has_work()
    assert len(pipe.alloc._free_slots) == 3  # every slot back
    assert pipe.max_seen_pos < 48


def test_continuous_engine_stops_at_eos_and_cancels():
    from superl8_serve_b200.dist.pipeline import SamplingParams
    from superl8_serve_b200.scheduler import ContinuousEngine

    pipe = FakePipe(batch=2, max_len=64)
    first = _solo([5, 6, 7], 1)[0]
    eng = ContinuousEngine(None, max_num_seqs=2, max_len=64, eos_id=first, pipeline=pipe)
    a = eng.add_request([5, 6, 7], SamplingParams(max_tokens=20))
    b = eng.add_request([1, 2], SamplingParams(max_tokens=20))
    c = eng.add_request([3], SamplingParams(max_tokens=20))
    while eng.seqs[a].status.name != "FINISHED":
        eng.step()
    assert eng.seqs[a].output_ids == [first]
    assert eng.cancel(b) and eng.cancel(c)
    eng.run()
    assert len(pipe.alloc._free_slots) == 2


def test_pipeline_engine_step_api_on_a_fake_pipeline():
    """The reference's PipelineEngine request API (add_request / step / sequence / forget)
    over the continuous engine: requests added between steps join the running batch."""
    import types

    from superl8_serve_b200.dist.pipeline import PipelineEngine, SamplingParams
    from superl8_serve_b200.scheduler import ContinuousEngine

    st = types.SimpleNamespace(model=None, kv_cache=None)
    eng = PipelineEngine.from_stages([st, st], None, max_num_seqs=2, max_len=48)
    pipe = FakePipe(batch=2, max_len=48)
    eng._cont = ContinuousEngine(None, max_num_seqs=2, max_len=48, pipeline=pipe)
    a = eng.add_request([5, 6, 7], SamplingParams(max_tokens=4))
    eng.step()
    b = eng.add_request([2, 3], SamplingParams(max_tokens=6))  # joins while a runs
    c = eng.add_request([9], SamplingParams(max_tokens=3))     # waits for a free slot
    while eng.has_work():
        eng.step()
    assert eng.sequence(a).output_ids == _solo([5, 6, 7], 4)
    assert eng.sequence(b).output_ids == _solo([2, 3], 6)
    assert eng.sequence(c).output_ids == _solo([9], 3)
    assert eng.sequence(a).status.name == "FINISHED"
    eng.forget(a)
    assert a not in eng._cont_ids


def test_prefill_chunk_row_blocks_cover_rows_within_sequences_and_chunks():
    """Prefill row blocks: every packed row in exactly one block, no block crossing a
    sequence or a chunk, at most block_rows rows each, in row order."""
    import random

    from superl8_serve_b200.engine import chunk_row_blocks

    rnd = random.Random(5)
    for _ in range(50):
        lens = [rnd.randint(1, 700) for _ in range(rnd.randint(1, 6))]
        seq = [i for i, n in enumerate(lens) for _ in range(n)]
        chunk, R = rnd.choice([1, 7, 64, 256]), rnd.choice([1, 2, 3, 4, 8, 16])
        blocks, off = chunk_row_blocks(seq, chunk, R)
        assert len(off) == (len(seq) + chunk - 1) // chunk + 1 and off[-1] == len(blocks)
        covered = []
        for c in range(len(off) - 1):
            c0 = c * chunk
            for first, count in blocks[off[c]:off[c + 1]]:
                assert 1 <= count <= R and first + count <= chunk
                rows = list(range(c0 + first, c0 + first + count))
                assert len({seq[r] for r in rows}) == 1
                covered += rows
        assert covered == list(range(len(seq)))
