"""Pipeline-parallel decode with the reference's stage API
(``superl8serve/dist/pipeline.py``: ``make_pipeline``, ``PipelineStage``, ``PipelineEngine``).

``make_pipeline`` splits the layer stack at ``i*L//S`` (``:452``), places each slice's
int8 weights on its GPU and gives each stage a paged KV pool sized to its own layers
(``:486-494``). ``PipelineEngine.generate`` runs greedy decode through
``engine.DecodePipeline``: micro-batches flow stage to stage with the codec fused at every
boundary and no host synchronisation inside a step.

Prompts go through the varlen prefill first (``DecodePipeline.prefill``, the reference's
``_prefill`` at ``:908-984``), then every sequence decodes from its own length.

Sampling (temperature, top-k, top-p, repetition penalty) runs on the last stage's GPU
(``s8b_sample``); its draw is counter-seeded (``SamplingParams.seed``, default the request
id) instead of the reference's torch-RNG Gumbel noise, so a run is reproducible. Host-side
``logit_processors`` are not supported.

Differences from the reference, all on purpose: the boundary scheme is fixed per engine
(``wire_scheme``, default "int8") instead of re-running the int4 gate every step, which
would need a host read-back inside the step.
"""

from __future__ import annotations

import dataclasses
import itertools
from dataclasses import dataclass, field

import torch

from ..engine import DecodePipeline
from ..runtime import StageModel


@dataclass
class SamplingParams:
    temperature: float = 0.0
    max_tokens: int = 16
    top_p: float = 1.0
    top_k: int = 0
    repetition_penalty: float = 1.0
    logit_processors: list = field(default_factory=list)
    seed: int | None = None  # draw seed (this build's; the reference draws from torch's RNG)


class PipelineStage:
    """One contiguous slice of layers on one GPU (``superl8serve/dist/pipeline.py:361-427``)."""

    def __init__(self, stage_id: int, *, model: StageModel, layer_offset: int, num_stages: int):
        self.stage_id = stage_id
        self.model = model
        self.layer_offset = layer_offset
        self.num_stages = num_stages
        self.kv_cache = None  # set by the engine's DecodePipeline (its KVPool of this stage)

    @property
    def layers(self):
        return self.model.layers

    @property
    def is_first(self) -> bool:
        return self.stage_id == 0

    @property
    def is_last(self) -> bool:
        return self.stage_id == self.num_stages - 1

    @property
    def _device(self):
        return self.model.device


def stage_bounds(n_layers: int, n_stages: int) -> list[int]:
    return [i * n_layers // n_stages for i in range(n_stages + 1)]


def balanced_stage_bounds(n_layers: int, n_stages: int, last_extra: float = 0.0,
                          first_extra: float = 0.0) -> list[int]:
    """Contiguous layer ranges minimising the largest stage cost, where a stage costs its
    layer count plus ``first_extra`` (stage 0: embedding) or ``last_extra`` (last stage: final
    norm, LM head, sampler) in layer units. The reference splits evenly (stage_bounds); in a
    decode pipeline the step time is the slowest stage's, so the head's cost is worth moving
    layers off the last stage. Exact dynamic programme over split points (ties: earlier
    boundaries)."""
    if n_stages > n_layers:
        raise ValueError("pipeline stage count cannot exceed the model layer count")
    INF = float("inf")
    # best[s][i]: minimal max cost of splitting layers [0, i) into s stages; arg: last split
    best = [[INF] * (n_layers + 1) for _ in range(n_stages + 1)]
    arg = [[0] * (n_layers + 1) for _ in range(n_stages + 1)]
    best[0][0] = 0.0
    for s_ in range(1, n_stages + 1):
        for i in range(s_, n_layers + 1):
            for j in range(s_ - 1, i):
                if best[s_ - 1][j] == INF:
                    continue
                cost = i - j + (first_extra if s_ == 1 else 0.0) + (
                    last_extra if (s_ == n_stages and i == n_layers) else 0.0)
                c = max(best[s_ - 1][j], cost)
                if c < best[s_][i] - 1e-12:
                    best[s_][i], arg[s_][i] = c, j
    bounds = [n_layers]
    i = n_layers
    for s_ in range(n_stages, 0, -1):
        i = arg[s_][i]
        bounds.append(i)
    return bounds[::-1]


def make_pipeline(cfg, weights, *, devices: tuple[int, ...] = (0, 1), max_num_seqs: int = 16,
                  max_len: int = 2048, block_size: int = 16, seed: int = 0,
                  allow_single_stage: bool = False) -> tuple[PipelineStage, ...]:
    """weights: an HF-style state dict (numpy or torch, bf16-valued floats; quantized per row
    here) or the string "synthetic" (random int8 weights generated on each GPU)."""
    n_layers = cfg.num_hidden_layers
    n_stages = len(devices)
    if n_stages < 2 and not allow_single_stage:
        raise ValueError("pipeline parallelism needs at least two devices")
    if n_stages > n_layers:
        raise ValueError("pipeline stage count cannot exceed the model layer count")
    bounds = stage_bounds(n_layers, n_stages)
    stages = []
    for sid, dev in enumerate(devices):
        start, end = bounds[sid], bounds[sid + 1]
        first, last = sid == 0, sid == n_stages - 1
        device = torch.device("cuda", dev) if isinstance(dev, int) else torch.device(dev)
        if isinstance(weights, str) and weights == "synthetic":
            model = StageModel.synthetic(cfg, start, end, device, first=first, last=last, seed=seed)
        else:
            model = StageModel.from_state_dict(cfg, weights, start, end, device, first=first,
                                               last=last)
        stages.append(PipelineStage(sid, model=model, layer_offset=start, num_stages=n_stages))
    return tuple(stages)


class PipelineEngine:
    """Greedy pipeline-parallel generation over stages from ``make_pipeline``."""

    def __init__(self, stage0: PipelineStage, stage1: PipelineStage, cfg, *, max_num_seqs: int = 16,
                 max_len: int = 2048, max_batch_tokens: int = 8192, eos_id: int | None = None,
                 wire_scheme: str | None = None, n_micro: int | None = None,
                 prefill: bool = True):
        self.stages = (stage0, stage1)
        self.cfg = cfg
        self.max_num_seqs, self.max_len = max_num_seqs, max_len
        self.eos_id = eos_id
        self.wire_scheme = wire_scheme or "int8"
        self.n_micro = n_micro
        self.prefill = prefill  # False: prompts teacher-forced through decode steps
        self._ids = itertools.count()
        self.max_batch_tokens = max_batch_tokens
        self._pending: dict[int, tuple[list[int], SamplingParams]] = {}
        self._out: dict[int, list[int]] = {}
        self._pipe: DecodePipeline | None = None
        self._cont = None  # ContinuousEngine behind step()
        self._cont_ids: dict[int, int] = {}

    @classmethod
    def from_stages(cls, stages, cfg, **kwargs):
        if len(stages) < 1:
            raise ValueError("PipelineEngine needs at least one stage")
        eng = cls(stages[0], stages[-1], cfg, **kwargs)
        eng.stages = tuple(stages)
        return eng

    @property
    def devices(self):
        return tuple(s._device.index or 0 for s in self.stages)

    def add_request(self, prompt_ids: list[int], params: SamplingParams | None = None) -> int:
        sid = next(self._ids)
        self._pending[sid] = (list(prompt_ids), params or SamplingParams())
        return sid

    def _pipeline(self, batch: int) -> DecodePipeline:
        n_micro = self.n_micro or min(len(self.stages), batch)
        if self._pipe is None or self._pipe.batch != batch or self._pipe.n_micro != n_micro:
            self._pipe = DecodePipeline([s.model for s in self.stages], batch=batch,
                                        n_micro=n_micro, max_len=self.max_len,
                                        wire_scheme=self.wire_scheme)
            for s, pool in zip(self.stages, self._pipe.pools):
                s.kv_cache = pool
        else:
            self._pipe.alloc = type(self._pipe.alloc)(self._pipe.alloc.num_blocks, batch,
                                                      self._pipe.block_size, self._pipe.max_blocks)
            self._pipe.slots = []
        return self._pipe

    def run_pending(self):
        if not self._pending:
            return
        ids = list(self._pending)
        prompts = [self._pending[i][0] for i in ids]
        params = [self._pending[i][1] for i in ids]
        if any(p.logit_processors for p in params):
            raise NotImplementedError("host logit processors are not on the s8b decode path")
        max_new = max(p.max_tokens for p in params)
        pipe = self._pipeline(len(prompts))
        pipe.set_sampling([{"temperature": p.temperature, "top_k": p.top_k, "top_p": p.top_p,
                            "repetition_penalty": p.repetition_penalty,
                            "seed": sid if p.seed is None else p.seed}
                           for sid, p in zip(ids, params)], prompts)
        outs = pipe.generate(prompts, max_new, prefill=self.prefill)
        for sid, out, p in zip(ids, outs, params):
            out = out[: p.max_tokens]
            if self.eos_id is not None and self.eos_id in out:
                out = out[: out.index(self.eos_id) + 1]
            self._out[sid] = out
        self._pending.clear()

    def generate(self, prompts: list[list[int]], params: SamplingParams | None = None):
        """All requests as one batch through the stages (prefill, then decode)."""
        sids = [self.add_request(p, params) for p in prompts]
        self.run_pending()
        return [self._out[s] for s in sids]

    # --------------------------------------------------------- continuous batching ----
    def _continuous(self):
        if self._cont is None:
            from ..scheduler import ContinuousEngine

            self._cont = ContinuousEngine([s.model for s in self.stages],
                                          max_num_seqs=self.max_num_seqs, max_len=self.max_len,
                                          max_batch_tokens=self.max_batch_tokens,
                                          eos_id=self.eos_id, wire_scheme=self.wire_scheme)
            for s, pool in zip(self.stages, self._cont.pipe.pools):
                s.kv_cache = pool
        return self._cont

    def step(self):
        """One scheduler step (``PipelineEngine.step``, ``superl8serve/dist/pipeline.py:620-635``):
        requests added since the last step join the running batch, then the scheduler
        either admits (prefills) waiting requests or decodes every running one."""
        eng = self._continuous()
        for sid in list(self._pending):
            prompt, params = self._pending.pop(sid)
            if params.seed is None:
                params = dataclasses.replace(params, seed=sid)
            self._cont_ids[sid] = eng.add_request(prompt, params)
        eng.step()

    def has_work(self) -> bool:
        return bool(self._pending) or (self._cont is not None and self._cont.sched.has_work())

    def sequence(self, seq_id: int):
        """The request's ``Sequence`` (status, prompt, output ids) of a step()-driven run."""
        return self._cont.seqs[self._cont_ids[seq_id]]

    def forget(self, seq_id: int) -> None:
        self._out.pop(seq_id, None)
        cid = self._cont_ids.pop(seq_id, None)
        if cid is not None:
            self._cont.seqs.pop(cid, None)
