"""In-process pipeline decode: S stages (one device each, or several on one device), a batch
split into micro-batches, the codec at every stage boundary.

Scheduling. Stage s of micro-batch k waits only for stage s-1 of micro-batch k (a CUDA event,
no host synchronisation), so while stage s works on micro-batch k, stage s-1 already runs
k+1: the 1F pipeline the reference's docstring describes
(``superl8serve/dist/pipeline.py:11-13``) but its loop serialises
(``_decode_microbatched``, ``:986-1040``). The codec encoder of stage s writes straight into
stage s+1's receive buffer for that micro-batch; the argmax of the last stage writes the next
token ids that stage 0 reads on the following step.

Sequence state (positions, context lengths, block tables) lives on the device and is advanced
by a kernel, so one step needs no host round trip and, on a single device, the whole step is
captured into one CUDA graph.
"""

from __future__ import annotations

import math

import torch

from . import ops
from ._lib import call, ptr, stream
from .runtime import KVPool, MicroBatch, StageModel, StageRunner


class BlockAllocator:
    """Host-side block bookkeeping (``PagedKVCache.alloc/ensure_capacity/free``,
    ``superl8serve/engine/kv_cache.py:703-749``): free-list of physical blocks, one block
    list per slot."""

    def __init__(self, num_blocks: int, num_slots: int, block_size: int, max_blocks_per_seq: int):
        self.block_size = block_size
        self.max_blocks_per_seq = max_blocks_per_seq
        self.num_blocks = num_blocks
        self._free_blocks = list(range(num_blocks))
        self._free_slots = list(range(num_slots))
        self._slot_blocks: list[list[int]] = [[] for _ in range(num_slots)]

    def alloc(self) -> int:
        if not self._free_slots:
            raise RuntimeError("PagedKVCache: no free slots")
        return self._free_slots.pop()

    def free(self, slot: int):
        self._free_blocks.extend(self._slot_blocks[slot])
        self._slot_blocks[slot] = []
        self._free_slots.append(slot)

    def ensure_capacity(self, slots, lengths):
        for slot, n in zip(slots, lengths):
            blocks = self._slot_blocks[slot]
            need = (n + self.block_size - 1) // self.block_size
            if need > self.max_blocks_per_seq:
                raise RuntimeError("sequence longer than max_len")
            while len(blocks) < need:
                if not self._free_blocks:
                    raise RuntimeError("PagedKVCache: no free blocks")
                blocks.append(self._free_blocks.pop())

    def block_table(self, slots) -> torch.Tensor:
        bt = torch.zeros(len(slots), self.max_blocks_per_seq, dtype=torch.int32)
        for i, s in enumerate(slots):
            b = self._slot_blocks[s]
            if b:
                bt[i, : len(b)] = torch.tensor(b, dtype=torch.int32)
        return bt


def chunk_row_blocks(seq_of_row: list[int], chunk: int, block_rows: int):
    """Row blocks of packed prefill rows: chunks of ``chunk`` rows are cut into runs of at most
    ``block_rows`` consecutive rows of one sequence (``seq_of_row[i]``: row i's sequence).
    Returns (blocks, chunk_off): blocks[chunk_off[c] : chunk_off[c + 1]] are chunk c's blocks
    as (first row relative to the chunk, row count)."""
    T = len(seq_of_row)
    blocks, chunk_off = [], [0]
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        r = c0
        while r < c1:
            e = r + 1
            while e < c1 and e - r < block_rows and seq_of_row[e] == seq_of_row[r]:
                e += 1
            blocks.append((r - c0, e - r))
            r = e
        chunk_off.append(len(blocks))
    return blocks, chunk_off


class DecodePipeline:
    """Greedy W8A8 decode through ``len(models)`` stages.

    models[s] holds stage s's layers on its device. ``batch`` rows are split into
    ``n_micro`` micro-batches of ``m = ceil(batch / n_micro)`` rows.
    """

    # prompt tokens per prefill launch sequence (the tensor-core GEMM's token tile limit)
    PREFILL_CHUNK = 256

    def __init__(self, models: list[StageModel], *, batch: int, n_micro: int = 1,
                 max_len: int = 2048, block_size: int = 16, wire_scheme: str = "int8-had",
                 num_blocks: int | None = None, dtype=torch.bfloat16):
        self.models = models
        self.cfg = models[0].cfg
        self.S = len(models)
        self.batch, self.n_micro = batch, n_micro
        self.m = math.ceil(batch / n_micro)
        self.max_len = max_len
        self.block_size = block_size
        self.wire_scheme = wire_scheme
        self.max_blocks = (max_len + block_size - 1) // block_size
        nb = num_blocks or batch * self.max_blocks
        cfg = self.cfg
        self.alloc = BlockAllocator(nb, batch, block_size, self.max_blocks)
        self.pools = [KVPool(len(mdl.layers), nb, cfg.num_key_value_heads, cfg.resolved_head_dim(),
                             block_size, mdl.device) for mdl in models]
        self.runners = [StageRunner(mdl, pool, self.m, max_len, dtype)
                        for mdl, pool in zip(models, self.pools)]
        self.mbs: list[list[MicroBatch]] = []
        for mdl in models:
            dev = mdl.device
            row = []
            for k in range(n_micro):
                row.append(MicroBatch(
                    ids=torch.zeros(self.m, dtype=torch.int32, device=dev),
                    positions=torch.zeros(self.m, dtype=torch.int32, device=dev),
                    context_lens=torch.ones(self.m, dtype=torch.int32, device=dev),
                    block_table=torch.zeros(self.m, self.max_blocks, dtype=torch.int32, device=dev)))
            self.mbs.append(row)
        from .ops import codec_sizes

        H = cfg.hidden_size
        nbytes, nsc = codec_sizes(self.m, 2 * H, wire_scheme)
        # boundary s -> s+1 buffers live on stage s+1's device, one per micro-batch
        self.bufs = [[(torch.empty(nbytes, dtype=torch.uint8, device=models[s + 1].device),
                       torch.empty(max(nsc, 1), dtype=torch.float32, device=models[s + 1].device),
                       wire_scheme) for _ in range(n_micro)] for s in range(self.S - 1)]
        self.single_device = len({str(mdl.device) for mdl in models}) == 1
        if not self.single_device:
            for a, b in zip(models[:-1], models[1:]):
                call("s8b_enable_peer_access", a.device.index, b.device.index)
        self.streams = [torch.cuda.Stream(device=mdl.device) for mdl in models]
        self.events = [[torch.cuda.Event() for _ in range(n_micro)] for _ in models]
        self.slots: list[int] = []
        self.graph = self.graph_io = None
        self.rows = [min(self.m, batch - k * self.m) for k in range(n_micro)]
        self.dtype = dtype
        self.prefill_chunk = self.PREFILL_CHUNK
        self._pf = None
        self._sampling = None
        self.scratch_block = None
        self.native = False

    def set_native(self, on: bool = True):
        """Run every stage step (decode and prefill) as one ``s8b_stage_step`` call."""
        self.native = on
        for r in self.runners + (self._pf[0] if self._pf is not None else []):
            r.native = on

    # ----------------------------------------------------------------- sequence state ----
    def add_sequences(self, n: int | None = None):
        n = self.batch if n is None else n
        self.slots = [self.alloc.alloc() for _ in range(n)]
        return self.slots

    def set_state(self, positions: list[int], ids: list[int] | None = None, reserve: int = 1):
        """Host -> device: block tables covering positions + reserve tokens, positions,
        context lengths and (optionally) the input ids of every row."""
        lengths = [p + reserve for p in positions]
        self.alloc.ensure_capacity(self.slots, lengths)
        bt = self.alloc.block_table(self.slots)
        pos = torch.tensor(positions, dtype=torch.int32)
        ids_t = None if ids is None else torch.tensor(ids, dtype=torch.int32)
        for s in range(self.S):
            for k in range(self.n_micro):
                lo, r = k * self.m, self.rows[k]
                mb = self.mbs[s][k]
                mb.block_table[:r].copy_(bt[lo:lo + r])
                mb.positions[:r].copy_(pos[lo:lo + r])
                mb.context_lens[:r].copy_(pos[lo:lo + r] + 1)
                if ids_t is not None and s == 0:
                    mb.ids[:r].copy_(ids_t[lo:lo + r])

    def set_rows(self, rows: list[int], positions: list[int], ids: list[int],
                 slots: list[int | None]):
        """Host -> device state of some rows only (continuous batching): row r decodes
        ``ids[i]`` at ``positions[i]`` with the block table of KV slot ``slots[i]``; a slot of
        None parks the row on the reserved scratch block (``scratch_block``), so an idle row
        writes and reads nothing that belongs to a sequence."""
        bt = torch.zeros(len(rows), self.max_blocks, dtype=torch.int32)
        for j, sl in enumerate(slots):
            if sl is None:
                bt[j].fill_(self.scratch_block)
            else:
                b = self.alloc._slot_blocks[sl]
                bt[j, : len(b)] = torch.tensor(b, dtype=torch.int32)
                bt[j, len(b):] = self.scratch_block
        pos = torch.tensor(positions, dtype=torch.int32)
        ids_t = torch.tensor(ids, dtype=torch.int32)
        for j, row in enumerate(rows):
            k, r = divmod(row, self.m)
            for s in range(self.S):
                mb = self.mbs[s][k]
                mb.block_table[r].copy_(bt[j])
                mb.positions[r:r + 1].copy_(pos[j:j + 1])
                mb.context_lens[r:r + 1].copy_(pos[j:j + 1] + 1)
                if s == 0:
                    mb.ids[r:r + 1].copy_(ids_t[j:j + 1])

    def reserve_scratch_block(self) -> int:
        """Take one physical block out of the allocator for idle rows (``set_rows``)."""
        if self.scratch_block is None:
            self.scratch_block = self.alloc._free_blocks.pop(0)
        return self.scratch_block

    def set_sampling_rows(self, rows: list[int], params: list[dict], prompts: list[list[int]]):
        """Sampling parameters and token history of some rows only, leaving the other rows'
        state (and their histories) as they are; the first call switches every row to the
        sampler (greedy rows stay greedy)."""
        if self._sampling is None:
            self.set_sampling([{} for _ in range(self.batch)], force=True)
        for row, pr, prompt in zip(rows, params, prompts):
            k, r = divmod(row, self.m)
            smp = self.mbs[-1][k].extra["sampling"]
            smp["temperature"][r] = float(pr.get("temperature", 0.0))
            smp["top_k"][r] = int(pr.get("top_k", 0))
            smp["top_p"][r] = float(pr.get("top_p", 1.0))
            smp["penalty"][r] = float(pr.get("repetition_penalty", 1.0))
            smp["seeds"][r] = int(pr.get("seed", row)) & ((1 << 63) - 1)
            h = torch.zeros(smp["history"].shape[1], dtype=torch.int32)
            h[: min(len(prompt), h.numel())] = torch.tensor(prompt[: h.numel()], dtype=torch.int32)
            smp["history"][r].copy_(h)

    def set_ids(self, ids: list[int]):
        ids_t = torch.tensor(ids, dtype=torch.int32)
        for k in range(self.n_micro):
            lo, r = k * self.m, self.rows[k]
            self.mbs[0][k].ids[:r].copy_(ids_t[lo:lo + r])

    def tokens(self) -> torch.Tensor:
        """Next-token ids of the last step, all rows (on the last stage's device)."""
        return torch.cat([self.mbs[-1][k].ids[: self.rows[k]] for k in range(self.n_micro)])

    def logits(self, k: int = 0) -> torch.Tensor:
        return self.runners[-1].logits[: self.rows[k]]

    # ----------------------------------------------------------------------- stepping ----
    def _enqueue(self, host_io: torch.Tensor | None = None):
        """Enqueue one decode step (all micro-batches, all stages) and advance positions.

        ``host_io`` (pinned int32, one slot per row) routes every micro-batch's input ids
        through host memory on the way into stage 0: the ids left by the previous step are
        copied device -> host into ``host_io`` and back host -> device, stream-ordered, so the
        host holds each step's tokens without draining the pipeline."""
        for k in range(self.n_micro):
            r = self.rows[k]
            if host_io is not None:
                with torch.cuda.device(self.models[0].device):
                    st0 = (torch.cuda.current_stream(self.models[0].device) if self.single_device
                           else self.streams[0])
                    with torch.cuda.stream(st0):
                        dst = host_io.data_ptr() + 4 * k * self.m
                        ids = self.mbs[0][k].ids
                        call("s8b_memcpy_async", dst, ptr(ids), 4 * r, stream())
                        call("s8b_memcpy_async", ptr(ids), dst, 4 * r, stream())
            for s in range(self.S):
                dev = self.models[s].device
                st = torch.cuda.current_stream(dev) if self.single_device else self.streams[s]
                with torch.cuda.device(dev), torch.cuda.stream(st):
                    if s > 0 and not self.single_device:
                        st.wait_event(self.events[s - 1][k])
                    if s < self.S - 1 and not self.single_device:
                        # do not overwrite stage s+1's receive buffer before it was decoded
                        st.wait_event(self.events[s + 1][k])
                    self.runners[s].run(self.mbs[s][k], r,
                                        boundary_in=self.bufs[s - 1][k] if s > 0 else None,
                                        boundary_out=self.bufs[s][k] if s < self.S - 1 else None)
                    call("s8b_advance", ptr(self.mbs[s][k].positions),
                         ptr(self.mbs[s][k].context_lens), r, 1, stream())
                    if not self.single_device:
                        self.events[s][k].record(st)
            if self.S > 1:
                # next step's input ids of micro-batch k: last stage -> stage 0
                last, first = self.mbs[-1][k], self.mbs[0][k]
                if self.single_device:
                    first.ids.copy_(last.ids)
                else:
                    with torch.cuda.device(self.models[0].device), torch.cuda.stream(self.streams[0]):
                        self.streams[0].wait_event(self.events[-1][k])
                        first.ids.copy_(last.ids, non_blocking=True)

    def step(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self._enqueue()

    def step_host_io(self):
        """One step of the host-I/O graph (see capture(host_io=...))."""
        self.graph_io.replay()

    def capture(self, host_io: torch.Tensor | None = None):
        """Capture one whole step into a CUDA graph (single-device pipelines); with
        ``host_io`` the graph carries the per-micro-batch host round trip of the input ids
        and is replayed by step_host_io()."""
        if not self.single_device:
            raise RuntimeError("graph capture of a multi-device in-process pipeline is not used")
        dev = self.models[0].device
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.device(dev), torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._enqueue(host_io)
        torch.cuda.current_stream(dev).wait_stream(s)
        if host_io is None:
            self.graph = g
        else:
            self.graph_io = g
        return g

    def synchronize(self):
        for mdl in self.models:
            torch.cuda.synchronize(mdl.device)

    # --------------------------------------------------------------------- sampling ----
    def set_sampling(self, params: list[dict] | None, prompts: list[list[int]] | None = None,
                     *, force: bool = False):
        """Per-row sampling on the last stage (``s8b_sample``; the reference's
        ``Sampler.forward``, ``superl8serve/layers/sampler.py:22-86``). params[i]: temperature,
        top_k, top_p, repetition_penalty, seed. ``None`` (or all temperatures 0 with no
        penalty) keeps the greedy argmax unless ``force``. The token history used by the
        repetition penalty starts as the prompts; each step adds its input ids on the device."""
        last = self.models[-1].device
        if params is None or (not force and all(
                float(p.get("temperature", 0.0)) == 0.0 and
                float(p.get("repetition_penalty", 1.0)) == 1.0 for p in params)):
            for mb in self.mbs[-1]:
                mb.extra.pop("sampling", None)
            self._sampling = None
            return
        if len(params) != self.batch:
            raise ValueError("set_sampling() expects one parameter set per row")
        from ._lib import load

        cap = self.max_len
        hist = torch.zeros(self.batch, cap, dtype=torch.int32)
        for i, pr in enumerate(prompts or []):
            hist[i, : min(len(pr), cap)] = torch.tensor(pr[:cap], dtype=torch.int32)
        col = lambda key, dflt, dt: torch.tensor([p.get(key, dflt) for p in params], dtype=dt)  # noqa: E731
        full = {"temperature": col("temperature", 0.0, torch.float32),
                "top_k": col("top_k", 0, torch.int32), "top_p": col("top_p", 1.0, torch.float32),
                "penalty": col("repetition_penalty", 1.0, torch.float32),
                "seeds": torch.tensor([int(p.get("seed", i)) & ((1 << 63) - 1)
                                       for i, p in enumerate(params)], dtype=torch.int64),
                "history": hist}
        ws_bytes = int(load().s8b_sample_workspace_size(self.m, self.cfg.vocab_size))
        for k in range(self.n_micro):
            lo, r = k * self.m, self.rows[k]
            smp = {name: t[lo:lo + r].contiguous().to(last) for name, t in full.items()}
            smp["workspace"] = torch.empty(ws_bytes, dtype=torch.uint8, device=last)
            smp["input_ids"] = self.mbs[0][k].ids
            self.mbs[-1][k].extra["sampling"] = smp
        self._sampling = params

    # ---------------------------------------------------------------------- prefill ----
    def _prefill_state(self):
        """Prefill runners (``prefill_chunk`` rows, packed weights shared with the decode
        runners) and one boundary buffer per stage boundary."""
        if self._pf is not None and self._pf[0][0].m == self.prefill_chunk:
            return self._pf
        mp = self.prefill_chunk
        runners = [StageRunner(mdl, pool, mp, self.max_len, self.dtype, share=r)
                   for mdl, pool, r in zip(self.models, self.pools, self.runners)]
        for r in runners:
            r.native = self.native
            r.decode_step = False  # a chunk's rows write many positions of a sequence
        from .ops import codec_sizes

        nbytes, nsc = codec_sizes(mp, 2 * self.cfg.hidden_size, self.wire_scheme)
        bufs = [(torch.empty(nbytes, dtype=torch.uint8, device=self.models[s + 1].device),
                 torch.empty(max(nsc, 1), dtype=torch.float32, device=self.models[s + 1].device),
                 self.wire_scheme) for s in range(self.S - 1)]
        self._pf = (runners, bufs)
        return self._pf

    def prefill(self, prompts: list[list[int]], *, reserve: int = 1, keep_logits: bool = False,
                slots: list[int] | None = None):
        """Varlen batched prefill (``PipelineEngine._prefill``,
        ``superl8serve/dist/pipeline.py:908-984``): every prompt token of every sequence is
        one row; rows are packed sequence after sequence (the reference's ``cu_seqlens``
        order) into chunks of ``prefill_chunk`` rows, and each chunk runs through every
        stage with the codec at each boundary.

        Row (sequence i, position t) writes its K/V at t and attends over positions [0, t]
        of the paged cache (context length t + 1), after the same layer's KV write of the
        whole chunk, so it computes exactly what a decode step of that token computes: the
        result is bit-identical to feeding the prompt one token per step. The final norm,
        LM head and argmax run only in chunks where some sequence ends; the argmax of each
        sequence's last row is its first generated token (returned, one per sequence; with
        ``keep_logits`` also that row's logits). Block capacity is reserved for
        ``len(prompt) + reserve`` tokens. ``slots`` prefills only those KV slots (one prompt
        each; continuous batching admits requests this way), default every row's.

        The row state of all chunks (ids, positions, context lengths, block-table rows) goes
        to each stage's device in one pinned copy and every chunk reads a view of it, so the
        chunks are enqueued back to back with one host synchronisation at the end.
        """
        n = len(prompts)
        if slots is None and n != self.batch:
            raise ValueError("prefill() expects exactly `batch` prompts")
        if slots is not None and len(slots) != n:
            raise ValueError("prefill() needs one slot per prompt")
        if any(len(p) == 0 for p in prompts):
            raise ValueError("prefill() needs a non-empty prompt for every sequence")
        if slots is None:
            if not self.slots:
                self.add_sequences(n)
            slots = self.slots
        self.alloc.ensure_capacity(slots, [len(p) + reserve for p in prompts])
        bt = self.alloc.block_table(slots)
        runners, bufs = self._prefill_state()
        seq = torch.tensor([i for i, p in enumerate(prompts) for _ in p], dtype=torch.long)
        pos = torch.cat([torch.arange(len(p), dtype=torch.int32) for p in prompts])
        ids = torch.tensor([t for p in prompts for t in p], dtype=torch.int32)
        T = len(seq)
        # row blocks of each chunk (rows of one sequence, at most R per block), relative to
        # the chunk's first row: the prefill attention stages each block's partitions once
        R = ops.prefill_block_rows(self.cfg.num_attention_heads, self.cfg.num_key_value_heads)
        blocks, chunk_off = chunk_row_blocks(seq.tolist(), self.prefill_chunk, R)
        rbs = torch.tensor(blocks, dtype=torch.int32).reshape(-1, 2)
        host = [x.pin_memory() for x in (ids, pos, pos + 1, bt[seq], rbs)]
        state = []  # per stage: (ids, positions, context_lens, block_table, row blocks)
        for s, mdl in enumerate(self.models):
            st = torch.cuda.current_stream(mdl.device) if self.single_device else self.streams[s]
            with torch.cuda.device(mdl.device), torch.cuda.stream(st):
                state.append([x.to(mdl.device, non_blocking=True) for x in host])
        # a single stage reads and writes ids in place (argmax after embed, per chunk); a
        # last stage after others writes its own array
        out_ids = state[-1][0] if self.S == 1 else torch.empty_like(state[-1][0])
        ends = torch.cumsum(torch.tensor([len(p) for p in prompts]), 0) - 1
        lg_rows = None
        if keep_logits:
            lg_rows = torch.empty(n, self.cfg.vocab_size, dtype=self.dtype,
                                  device=self.models[-1].device)
        ev = [self.events[s][0] for s in range(self.S)]
        end_list = ends.tolist()
        for c0 in range(0, T, self.prefill_chunk):
            r = min(self.prefill_chunk, T - c0)
            chunk_ends = [(i, e - c0) for i, e in enumerate(end_list) if c0 <= e < c0 + r]
            for s in range(self.S):
                dev = self.models[s].device
                st = torch.cuda.current_stream(dev) if self.single_device else self.streams[s]
                with torch.cuda.device(dev), torch.cuda.stream(st):
                    if s > 0 and not self.single_device:
                        st.wait_event(ev[s - 1])
                    if s < self.S - 1 and not self.single_device:
                        st.wait_event(ev[s + 1])  # stage s+1 has decoded the previous chunk
                    a_ids, a_pos, a_ctx, a_bt, a_rb = state[s]
                    ci = c0 // self.prefill_chunk
                    mb = MicroBatch(ids=(out_ids if s == self.S - 1 else a_ids)[c0:c0 + r],
                                    positions=a_pos[c0:c0 + r], context_lens=a_ctx[c0:c0 + r],
                                    block_table=a_bt[c0:c0 + r],
                                    extra={"row_blocks": a_rb[chunk_off[ci]:chunk_off[ci + 1]]})
                    runners[s].run(mb, r, boundary_in=bufs[s - 1] if s > 0 else None,
                                   boundary_out=bufs[s] if s < self.S - 1 else None,
                                   head=bool(chunk_ends))
                    if s == self.S - 1 and keep_logits:
                        row_bytes = self.cfg.vocab_size * lg_rows.element_size()
                        for i, k in chunk_ends:
                            call("s8b_memcpy_async", ptr(lg_rows[i]), ptr(runners[s].logits[k]),
                                 row_bytes, stream())
                    if not self.single_device:
                        ev[s].record(st)
        self.synchronize()
        first = out_ids[ends.to(out_ids.device)].cpu().tolist()
        if keep_logits:
            return first, list(lg_rows.float().cpu())
        return first

    # ------------------------------------------------------------------- generation ----
    def generate(self, prompts: list[list[int]], max_new_tokens: int, *, keep_logits=False,
                 prefill: bool = False):
        """Greedy generation. Without ``prefill`` every row advances one token per step and
        prompt tokens are fed teacher-forced, exactly as ``oracle.model.OraclePipeline
        .generate``; with ``prefill`` the prompts go through ``prefill()`` first and every
        row then decodes from its own prompt length. Both give identical tokens and logits."""
        n = len(prompts)
        if n != self.batch:
            raise ValueError("generate() expects exactly `batch` prompts")
        if prefill:
            return self._generate_prefilled(prompts, max_new_tokens, keep_logits)
        if not self.slots:
            self.add_sequences(n)
        seqs = [list(p) for p in prompts]
        outs = [[] for _ in prompts]
        logit_log = [[] for _ in prompts]
        step = 0
        total = max(len(p) for p in prompts) + max_new_tokens
        self.set_state([0] * n, [sq[0] for sq in seqs], reserve=total)
        while any(len(o) < max_new_tokens for o in outs):
            self.set_ids([sq[step] for sq in seqs])
            self._enqueue()
            self.synchronize()
            toks = self.tokens().cpu().tolist()
            if keep_logits:
                lg = torch.cat([self.runners[-1].logits[: self.rows[k]].float().cpu()
                                for k in range(self.n_micro)]) if self.n_micro == 1 else None
            for i, sq in enumerate(seqs):
                if step >= len(prompts[i]) - 1 and len(outs[i]) < max_new_tokens:
                    outs[i].append(int(toks[i]))
                    if keep_logits and lg is not None:
                        logit_log[i].append(lg[i])
                if step + 1 >= len(sq):
                    sq.append(int(toks[i]))
            step += 1
        return (outs, logit_log) if keep_logits else outs

    def _generate_prefilled(self, prompts, max_new_tokens: int, keep_logits: bool):
        if self._sampling is not None:
            return self._generate_prefilled_sampled(prompts, max_new_tokens)
        res = self.prefill(prompts, reserve=max_new_tokens, keep_logits=keep_logits)
        first, first_logits = res if keep_logits else (res, None)
        outs = [[t] for t in first]
        logit_log = [[lg] for lg in first_logits] if keep_logits else None
        if max_new_tokens <= 0:
            outs = [[] for _ in prompts]
            return (outs, [[] for _ in prompts]) if keep_logits else outs
        # every row decodes its first generated token at its prompt length; the argmax of
        # each step feeds the next (positions advance on the device)
        self.set_state([len(p) for p in prompts], first, reserve=max_new_tokens)
        for _ in range(max_new_tokens - 1):
            self._enqueue()
            self.synchronize()
            toks = self.tokens().cpu().tolist()
            lg = None
            if keep_logits:
                lg = torch.cat([self.runners[-1].logits[: self.rows[k]].float().cpu()
                                for k in range(self.n_micro)]) if self.n_micro == 1 else None
            for i in range(len(prompts)):
                outs[i].append(int(toks[i]))
                if keep_logits and lg is not None:
                    logit_log[i].append(lg[i])
        return (outs, logit_log) if keep_logits else outs

    def _generate_prefilled_sampled(self, prompts, max_new_tokens: int):
        """Sampling after a prefill: the prompts but their last token go through prefill (its
        argmax is not used), the last prompt token through a sampled decode step, so every
        generated token comes from the sampler."""
        if any(len(p) < 2 for p in prompts):
            return self.generate(prompts, max_new_tokens)
        self.prefill([p[:-1] for p in prompts], reserve=max_new_tokens + 1)
        self.set_state([len(p) - 1 for p in prompts], [p[-1] for p in prompts],
                       reserve=max_new_tokens + 1)
        outs = [[] for _ in prompts]
        for _ in range(max_new_tokens):
            self._enqueue()
            self.synchronize()
            toks = self.tokens().cpu().tolist()
            for i in range(len(prompts)):
                outs[i].append(int(toks[i]))
        return outs
