"""Stage runtime: device-resident weights, paged KV pools and the per-micro-batch kernel
sequence of one pipeline stage.

One decode step of a stage, for one micro-batch of m rows (the reference's per-stage loop
in ``PipelineEngine._decode_microbatched``, ``superl8serve/dist/pipeline.py:997-1040``, over
``Qwen3DecoderLayer.forward``, ``superl8serve/models/qwen3.py:70-80``):

    [stage 0] embed(ids)                       or  [stage > 0] decode boundary -> (h, res)
    per layer:  rmsnorm_quant -> W8A8 qkv -> qkv_post (norms, RoPE, paged KV write, q quant)
                -> paged decode attention (+ fused o_proj input quant) -> W8A8 o
                -> rmsnorm_quant -> W8A8 gate_up -> SwiGLU + quant -> W8A8 down
                (sparse-MoE layer: rmsnorm_quant -> route + group -> grouped W8A8 gate_up
                 -> SwiGLU + quant -> grouped W8A8 down -> combine)
    [last]      rmsnorm_quant(final norm) -> W8A8 lm_head -> argmax
    [not last]  encode (h, res) straight into the next stage's receive buffer

Every buffer is allocated once here; ``StageRunner.run`` only launches kernels, so a whole
step can be captured into one CUDA graph per stage.

HBM layout (per stage, all device-resident): int8 weights row-major [out, in] with an fp32
scale per row (qkv and gate_up merged on the out axis), bf16 norm gains, bf16 embedding
table (stage 0), int8 LM head (last stage); KV pools [layers, blocks, Hkv, 16, 128] int8 with
[layers, blocks, Hkv, 16] fp32 scales; per-micro-batch activations of a few MB.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import ops
from ._lib import CODEC, call, load, ptr, stream
from .weights import quantize_rowwise_np


@dataclass
class ExpertShard:
    """Experts [e_lo, e_hi) of a MoE layer held on another GPU of the same stage."""

    device: torch.device
    e_lo: int
    e_hi: int
    gu_w: torch.Tensor
    gu_s: torch.Tensor
    d_w: torch.Tensor
    d_s: torch.Tensor


@dataclass
class RemoteExperts:
    """Experts [e_lo, e_hi) of a MoE layer held by another process (another GPU of the same
    stage): device addresses of that process's input buffers and flag (mapped with CUDA
    IPC), and of this process's own completion flag, call counter and status word. The
    counter advances once per MoE call on both sides, so the flags compare against it."""

    e_lo: int
    e_hi: int
    xq: int
    xs: int
    offsets: int
    sorted_token: int
    in_flag: int
    out_flag: int
    epoch: int
    status: int
    timeout_ns: int


@dataclass
class MoEWeights:
    """Sparse-MoE FFN of one layer (``SparseMoE``, ``superl8serve/models/moe.py:46-86``):
    fp32 router [E, H]; every expert's merged gate_up int8 [E, 2F, H] with row scales [E, 2F]
    and down int8 [E, H, F] with row scales [E, H] (experts stacked for the grouped GEMM).

    With expert parallelism (``StageModel.shard_experts``) the stage's own GPU keeps experts
    [0, gu_w.shape[0]) and ``shards`` hold the following contiguous ranges on other GPUs."""

    router: torch.Tensor
    gu_w: torch.Tensor
    gu_s: torch.Tensor
    d_w: torch.Tensor
    d_s: torch.Tensor
    top_k: int
    norm_topk_prob: bool = True
    scaling: float = 1.0
    shards: list = field(default_factory=list)
    remote: list = field(default_factory=list)  # RemoteExperts: ranges in other processes

    @property
    def num_experts(self) -> int:
        return self.router.shape[0]

    @property
    def local_experts(self) -> int:
        return self.gu_w.shape[0]

    @property
    def ffn(self) -> int:
        return self.d_w.shape[2]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size()
                   for t in (self.router, self.gu_w, self.gu_s, self.d_w, self.d_s))


@dataclass
class LayerWeights:
    qkv_w: torch.Tensor
    qkv_s: torch.Tensor
    o_w: torch.Tensor
    o_s: torch.Tensor
    gu_w: torch.Tensor | None  # dense FFN (None in a sparse-MoE layer)
    gu_s: torch.Tensor | None
    d_w: torch.Tensor | None
    d_s: torch.Tensor | None
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    moe: MoEWeights | None = None

    def nbytes(self) -> int:
        n = sum(t.numel() * t.element_size() for t in vars(self).values()
                if isinstance(t, torch.Tensor))
        return n + (self.moe.nbytes() if self.moe is not None else 0)

    def matrices(self) -> list[torch.Tensor]:
        """The dense int8 weight matrices of the layer (tensor-core packing, split counts)."""
        return [w for w in (self.qkv_w, self.o_w, self.gu_w, self.d_w) if w is not None]


@dataclass
class StageModel:
    """Weights of layers [start, end) of a Qwen3 model on one device."""

    cfg: object
    start: int
    end: int
    device: torch.device
    layers: list[LayerWeights]
    embed: torch.Tensor | None = None
    norm: torch.Tensor | None = None
    head_w: torch.Tensor | None = None
    head_s: torch.Tensor | None = None

    @property
    def is_first(self) -> bool:
        return self.embed is not None

    @property
    def is_last(self) -> bool:
        return self.head_w is not None

    def shard_experts(self, devices) -> "StageModel":
        """Expert parallelism inside the stage (the reference's ``TransportMoELayer``,
        ``superl8serve/models/moe_transport.py:161-345``): every MoE layer's experts are split
        into 1 + len(devices) contiguous ranges, the first staying on this stage's GPU, the
        others moved to ``devices``. The stage's GPU still routes every token and combines
        every contribution in ascending expert order, so results do not change."""
        devs = [torch.device(d) for d in devices]
        for L in self.layers:
            mw = L.moe
            if mw is None:
                continue
            E = mw.num_experts
            n = 1 + len(devs)
            cuts = [i * E // n for i in range(n + 1)]
            for i, d in enumerate(devs, start=1):
                lo, hi = cuts[i], cuts[i + 1]
                mw.shards.append(ExpertShard(d, lo, hi, mw.gu_w[lo:hi].to(d), mw.gu_s[lo:hi].to(d),
                                             mw.d_w[lo:hi].to(d), mw.d_s[lo:hi].to(d)))
            h = cuts[1]
            mw.gu_w, mw.gu_s = mw.gu_w[:h].clone(), mw.gu_s[:h].clone()
            mw.d_w, mw.d_s = mw.d_w[:h].clone(), mw.d_s[:h].clone()
        return self

    def weight_bytes(self) -> int:
        n = sum(L.nbytes() for L in self.layers)
        for t in (self.head_w, self.head_s, self.norm):
            if t is not None:
                n += t.numel() * t.element_size()
        return n

    @classmethod
    def from_state_dict(cls, cfg, sd: dict, start: int, end: int, device, *, first: bool,
                        last: bool, dtype=torch.bfloat16) -> "StageModel":
        """Quantize an HF-style float state dict (numpy or torch, bf16-valued) on the host with
        the per-row recipe and upload layers [start, end)."""
        dev = torch.device(device)

        def f(name):
            v = sd[name]
            return v.float().cpu().numpy() if isinstance(v, torch.Tensor) else np.asarray(v, np.float32)

        def q(w):
            qq, ss = quantize_rowwise_np(w)
            return torch.from_numpy(qq).to(dev), torch.from_numpy(ss).to(dev)

        def g(name):
            return torch.from_numpy(f(name)).to(dtype).to(dev)

        layers = []
        for i in range(start, end):
            p = f"model.layers.{i}"
            qkv = np.concatenate([f(f"{p}.self_attn.{n}_proj.weight") for n in "qkv"], 0)
            moe = None
            if cfg.layer_is_moe(i):
                ffn = (None, None, None, None)
                gus, dns = [], []
                for e in range(cfg.num_experts):
                    x = f"{p}.mlp.experts.{e}"
                    gus.append(quantize_rowwise_np(np.concatenate(
                        [f(f"{x}.gate_proj.weight"), f(f"{x}.up_proj.weight")], 0)))
                    dns.append(quantize_rowwise_np(f(f"{x}.down_proj.weight")))
                stack = lambda lst, j: torch.from_numpy(np.stack([t[j] for t in lst])).to(dev)  # noqa: E731
                moe = MoEWeights(torch.from_numpy(f(f"{p}.mlp.gate.weight")).to(dev),
                                 stack(gus, 0), stack(gus, 1), stack(dns, 0), stack(dns, 1),
                                 cfg.num_experts_per_tok, cfg.norm_topk_prob)
            else:
                gu = np.concatenate([f(f"{p}.mlp.gate_proj.weight"),
                                     f(f"{p}.mlp.up_proj.weight")], 0)
                ffn = (*q(gu), *q(f(f"{p}.mlp.down_proj.weight")))
            layers.append(LayerWeights(*q(qkv), *q(f(f"{p}.self_attn.o_proj.weight")), *ffn,
                                       g(f"{p}.input_layernorm.weight"),
                                       g(f"{p}.post_attention_layernorm.weight"),
                                       g(f"{p}.self_attn.q_norm.weight"),
                                       g(f"{p}.self_attn.k_norm.weight"), moe))
        m = cls(cfg, start, end, dev, layers)
        if first:
            m.embed = g("model.embed_tokens.weight")
        if last:
            m.norm = g("model.norm.weight")
            head = "model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"
            m.head_w, m.head_s = q(f(head))
        return m

    @classmethod
    def synthetic(cls, cfg, start: int, end: int, device, *, first: bool, last: bool,
                  seed: int = 0, dtype=torch.bfloat16) -> "StageModel":
        """Random int8 weights generated on the device (benchmarks of large shapes): uniform
        codes in [-127, 127] with row scales giving an effective N(0, 0.02)-sized weight."""
        dev = torch.device(device)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed * 1000 + start)
        H, D = cfg.hidden_size, cfg.resolved_head_dim()
        nh, nkv, F = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
        sw = 0.02 / 73.3

        def w(n, k):
            codes = torch.randint(-127, 128, (n, k), generator=gen, device=dev, dtype=torch.int8)
            return codes, torch.full((n,), sw, dtype=torch.float32, device=dev)

        def gain(n):
            return (1.0 + 0.1 * torch.randn(n, generator=gen, device=dev)).to(dtype)

        def moe_w():
            E, Fe = cfg.num_experts, cfg.moe_intermediate_size
            gu, gus = w(E * 2 * Fe, H)
            dn, dns = w(E * H, Fe)
            router = (0.02 * torch.randn(E, H, generator=gen, device=dev)).to(dtype).float()
            return MoEWeights(router, gu.view(E, 2 * Fe, H), gus.view(E, 2 * Fe),
                              dn.view(E, H, Fe), dns.view(E, H), cfg.num_experts_per_tok,
                              cfg.norm_topk_prob)

        layers = []
        for i in range(start, end):
            if cfg.layer_is_moe(i):
                ffn, moe = (None, None, None, None), moe_w()
            else:
                ffn, moe = (*w(2 * F, H), *w(H, F)), None
            layers.append(LayerWeights(*w((nh + 2 * nkv) * D, H), *w(H, nh * D), *ffn, gain(H),
                                       gain(H), gain(D), gain(D), moe))
        m = cls(cfg, start, end, dev, layers)
        if first:
            m.embed = (0.02 * torch.randn(cfg.vocab_size, H, generator=gen, device=dev)).to(dtype)
        if last:
            m.norm = gain(H)
            m.head_w, m.head_s = w(cfg.vocab_size, H)
        return m


class KVPool:
    """Paged int8 KV storage of one stage (``PagedKVCache`` layout,
    ``superl8serve/engine/kv_cache.py:484-512``)."""

    def __init__(self, n_layers, num_blocks, nkv, head_dim, block_size, device):
        shp = (n_layers, num_blocks, nkv, block_size, head_dim)
        self.kc = torch.zeros(shp, dtype=torch.int8, device=device)
        self.vc = torch.zeros(shp, dtype=torch.int8, device=device)
        self.ks = torch.ones(shp[:-1], dtype=torch.float32, device=device)
        self.vs = torch.ones(shp[:-1], dtype=torch.float32, device=device)
        self.block_size = block_size
        self.num_blocks = num_blocks

    def layer(self, i):
        return self.kc[i], self.ks[i], self.vc[i], self.vs[i]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.kc, self.vc, self.ks, self.vs))

    def fill_random(self, seed: int = 0):
        """Synthetic pre-filled context (benchmarks): random codes and scales."""
        g = torch.Generator(device=self.kc.device)
        g.manual_seed(seed)
        for t in (self.kc, self.vc):
            t.view(torch.uint8).random_(0, 255, generator=g)
            t.clamp_(-127, 127)
        for t in (self.ks, self.vs):
            t.uniform_(0.01, 0.05, generator=g)


@dataclass
class MicroBatch:
    """Device-side per-micro-batch decode state (stable addresses: graph-capturable)."""

    ids: torch.Tensor            # [m] int32 (stage 0 input; last stage writes next tokens)
    positions: torch.Tensor      # [m] int32, write position of the token being decoded
    context_lens: torch.Tensor   # [m] int32, positions + 1
    block_table: torch.Tensor    # [m, max_blocks] int32
    extra: dict = field(default_factory=dict)


def moe_experts(buf, off, ne, gu_w, gu_s, d_w, d_s, contrib, M, k, Fe, H, st, *, xq=None,
                xs=None, tc=True):
    """Experts [off .. off + ne) of a sparse-MoE layer on one GPU: gate_up, SwiGLU + quant,
    down into ``contrib`` (rows in assignment order; may be another GPU's buffer). ``buf``
    holds this GPU's buffers (xq / xs copies unless given, sorted_token, xg / xgs, gu, aq / as,
    status); ``off`` is the device address of the range's first offset."""
    A = M * k
    xq = buf["xq"] if xq is None else xq
    xs = buf["xs"] if xs is None else xs
    tc = tc and H % 128 == 0 and Fe % 128 == 0 and ne <= 512
    if tc:
        call("s8b_moe_gather_rows", ptr(xq), ptr(xs), ptr(buf["sorted_token"]), A, H,
             ptr(buf["xg"]), ptr(buf["xgs"]), st)
        call("s8b_moe_gemm_grouped_tc", ptr(buf["xg"]), ptr(buf["xgs"]), ptr(gu_w), ptr(gu_s),
             off, ptr(buf["gu"]), A, 2 * Fe, H, ne, M, ptr(buf["status"]), 0, st)
    else:
        call("s8b_moe_gemm_grouped", ptr(xq), ptr(xs), ptr(buf["sorted_token"]), ptr(gu_w),
             ptr(gu_s), off, ptr(buf["gu"]), A, 2 * Fe, H, ne, 0, st)
    call("s8b_silu_mul_quant", ptr(buf["gu"]), A, Fe, None, ptr(buf["aq"]), ptr(buf["as"]), 0, st)
    if tc:
        call("s8b_moe_gemm_grouped_tc", ptr(buf["aq"]), ptr(buf["as"]), ptr(d_w), ptr(d_s), off,
             contrib, A, H, Fe, ne, M, ptr(buf["status"]), 0, st)
    else:
        call("s8b_moe_gemm_grouped", ptr(buf["aq"]), ptr(buf["as"]), None, ptr(d_w), ptr(d_s),
             off, contrib, A, H, Fe, ne, 0, st)


def moe_expert_buffers(M: int, k: int, H: int, Fe: int, E: int, device, dtype=torch.bfloat16):
    """The per-GPU buffers ``moe_experts`` uses, for micro-batches of up to M tokens."""
    A = M * k
    z = lambda *n, dt=dtype: torch.zeros(n, dtype=dt, device=device)  # noqa: E731
    return {"xq": z(M, H, dt=torch.int8), "xs": z(M, dt=torch.float32),
            "offsets": z(E + 1, dt=torch.int32), "sorted_token": z(A, dt=torch.int32),
            "gu": z(A, 2 * Fe), "aq": z(A, Fe, dt=torch.int8), "as": z(A, dt=torch.float32),
            "xg": z(A, H, dt=torch.int8), "xgs": z(A, dt=torch.float32),
            "status": z(4, dt=torch.int32)}


class StageRunner:
    """Launches one stage's decode kernels for a micro-batch of up to ``m`` rows."""

    # token count from which the W8A8 GEMMs run on the tensor cores (tcgen05) instead of dp4a:
    # the dp4a GEMV streams weights at HBM speed for one token only (each further token adds
    # 16 dp4a operations per weight byte; at 4 tokens it runs at 4.2 TB/s against 5.7 for the
    # tensor cores on a 34816 x 5120 weight, at 2 tokens they tie)
    TC_MIN_TOKENS = 2

    def __init__(self, model: StageModel, pool: KVPool, m: int, max_ctx: int,
                 dtype=torch.bfloat16, tc_min_tokens: int | None = None,
                 share: "StageRunner | None" = None):
        """``share``: another runner of the same model whose packed tensor-core weight images
        this one reuses (a prefill runner beside the decode runner holds no second copy)."""
        cfg = model.cfg
        self.model, self.pool, self.m, self.max_ctx, self.dtype = model, pool, m, max_ctx, dtype
        # True: run() is one s8b_stage_step call (native replay of the same launches)
        self.native = False
        # True: every row writes only its newest position per launch (a decode step), so the
        # attention may stream older partitions early (s8b_paged_decode_q8_step); prefill
        # runners set False
        self.decode_step = True
        # True: MoE layers run their own experts only (no handshake with partner processes):
        # the stage-time measurement of a multi-process pipeline
        self.skip_remote = False
        self.H = cfg.hidden_size
        self.D = cfg.resolved_head_dim()
        self.Hq, self.Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.F = cfg.intermediate_size
        self.V = cfg.vocab_size
        self.eps = cfg.rms_norm_eps
        self.scale = self.D ** -0.5
        dev = model.device
        from .layers import rope_tables

        cos, sin = rope_tables(self.D, cfg.max_position_embeddings, cfg.rope_theta)
        self.cos, self.sin = cos.to(dev), sin.to(dev)
        e = lambda *s, dt=dtype: torch.empty(s, dtype=dt, device=dev)  # noqa: E731
        kmax = max(self.H, self.Hq * self.D, self.F)
        self.h = e(m, self.H)
        self.res = e(m, self.H)
        self.xq = e(m, kmax, dt=torch.int8)
        self.xs = e(m, dt=torch.float32)
        self.qkv = e(m, (self.Hq + 2 * self.Hkv) * self.D)
        self.q_i8 = e(m, self.Hq, self.D, dt=torch.int8)
        self.q_s = e(m, self.Hq, dt=torch.float32)
        self.attn = e(m, self.Hq * self.D)
        self.gu = e(m, 2 * self.F)
        self.ws = torch.zeros(ops.decode_workspace_bytes(m, self.Hq, self.D, max_ctx),
                              dtype=torch.uint8, device=dev)
        if model.is_last:
            self.logits = e(m, self.V)
        self.dev = dev
        self.tc_min = self.TC_MIN_TOKENS if tc_min_tokens is None else tc_min_tokens
        n_max = max([w.shape[0] for L in model.layers for w in L.matrices()]
                    + ([model.head_w.shape[0]] if model.is_last else []) + [self.H])
        self.tc_ws = ops.gemm_tc_workspace(m, n_max, dev) if m >= self.tc_min else None
        # tensor-core path: every weight also kept as contiguous unit images (packed once)
        self.packed: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        if self.tc_ws is not None and share is not None and share.model is model and share.packed:
            self.packed = share.packed
        elif self.tc_ws is not None:
            mats = [w for L in model.layers for w in L.matrices()]
            if model.is_last:
                mats.append(model.head_w)
            with torch.cuda.device(dev):
                for w in mats:
                    self.packed[id(w)] = (w, ops.pack_weights_tc(w))
        # split-K partial outputs (GEMM out_kind 2) consumed by the following row kernel
        self.splits: dict[tuple[int, int], int] = {}
        self.part = None
        if self.tc_ws is not None:
            lib = load()
            need = 0
            for L in model.layers:
                for w in L.matrices():
                    N, K = w.shape
                    c = int(lib.s8b_gemm_tc_split_count(m, N, K))
                    self.splits[(N, K)] = c
                    need = max(need, c * m * N)
            self.part = torch.empty(need, dtype=torch.int32, device=dev)
        # sparse-MoE layers: router input, routing / grouping state and per-assignment rows
        moes = [L.moe for L in model.layers if L.moe is not None]
        self.moe_buf = None
        if moes:
            k = max(mw.top_k for mw in moes)
            E = max(mw.num_experts for mw in moes)
            Fe = max(mw.ffn for mw in moes)
            A = m * k
            i32 = lambda *n: torch.empty(n, dtype=torch.int32, device=dev)  # noqa: E731
            self.moe_buf = {
                "y": e(m, self.H), "topi": i32(m, k), "topw": e(m, k), "offsets": i32(E + 1),
                "sorted_assign": i32(A), "sorted_token": i32(A), "assign_pos": i32(A),
                "gu": e(A, 2 * Fe), "aq": e(A, Fe, dt=torch.int8),
                "as": e(A, dt=torch.float32), "contrib": e(A, self.H),
                # tensor-core grouped GEMM: expert input rows gathered into assignment order
                "xg": e(A, self.H, dt=torch.int8), "xgs": e(A, dt=torch.float32),
                "status": torch.zeros(4, dtype=torch.int32, device=dev)}
            # expert-parallel partners: inputs copied in, gate_up / SwiGLU rows of their own
            self.moe_peer: dict[str, dict] = {}
            for d in sorted({str(sh.device) for mw in moes for sh in mw.shards}):
                pd = torch.device(d)
                call("s8b_enable_peer_access", dev.index, pd.index)
                call("s8b_enable_peer_access", pd.index, dev.index)
                z = lambda *n, dt=dtype: torch.zeros(n, dtype=dt, device=pd)  # noqa: E731
                self.moe_peer[d] = {
                    "xq": z(m, self.H, dt=torch.int8), "xs": z(m, dt=torch.float32),
                    "offsets": z(E + 1, dt=torch.int32), "sorted_token": z(A, dt=torch.int32),
                    "gu": z(A, 2 * Fe), "aq": z(A, Fe, dt=torch.int8),
                    "as": z(A, dt=torch.float32), "xg": z(A, self.H, dt=torch.int8),
                    "xgs": z(A, dt=torch.float32), "status": z(4, dt=torch.int32),
                    "stream": torch.cuda.Stream(device=pd),
                    "ev_in": torch.cuda.Event(), "ev_out": torch.cuda.Event()}

    # ---------------------------------------------------------------------- pieces ----
    def _gemm(self, xq, xs, w, s, out, M):
        if self.tc_ws is not None and M >= self.tc_min:
            pk = self.packed.get(id(w))
            if pk is not None and pk[0] is w:
                call("s8b_gemm_w8a8_tc_packed", ptr(xq), ptr(xs), ptr(pk[1]), ptr(s), ptr(out), 0,
                     M, w.shape[0], w.shape[1], 0, ptr(self.tc_ws), self.tc_ws.numel(), stream())
                return
            call("s8b_gemm_w8a8_tc", ptr(xq), ptr(xs), ptr(w), ptr(s), ptr(out), 0, M, w.shape[0],
                 w.shape[1], 0, ptr(self.tc_ws), self.tc_ws.numel(), stream())
        else:
            call("s8b_gemm_w8a8", ptr(xq), ptr(xs), ptr(w), ptr(s), ptr(out), 0, M, w.shape[0],
                 w.shape[1], 0, stream())

    def _gemm_split(self, w, M):
        """Tensor-core GEMM with its split-K partials left in self.part (out_kind 2); returns
        the split count. The following row kernel sums and dequantizes them."""
        pk = self.packed[id(w)][1]
        N, K = w.shape
        call("s8b_gemm_w8a8_tc_packed", ptr(self.xq), ptr(self.xs), ptr(pk), None, ptr(self.part),
             2, M, N, K, 0, ptr(self.tc_ws), self.tc_ws.numel(), stream())
        return self.splits[(N, K)]

    def _rms_quant(self, h, res_in, res_out, w, M, K, src=None, y_out=None):
        """RMSNorm + activation quant; ``src`` = (C, weight scales) reads h from the split-K
        partials of the preceding GEMM instead of ``h``, ``src`` = ("codec", payload, scales,
        scheme) reads h and the residual from the previous stage's codec payload; ``y_out``
        also keeps the normalized dtype row."""
        if src is None:
            call("s8b_rmsnorm_quant", ptr(h), ptr(res_in), ptr(res_out), ptr(w), self.eps,
                 ptr(self.xq), ptr(self.xs), ptr(y_out), M, K, 0, stream())
        elif src[0] == "codec":  # the stage prologue: the received payload decoded on load
            _, pay, sc, scheme = src
            call("s8b_rmsnorm_quant_codec", pay.data_ptr(), sc.data_ptr(), CODEC[scheme],
                 ptr(res_out), ptr(w), self.eps, ptr(self.xq), ptr(self.xs), M, K, 0, stream())
        else:
            C, ws = src
            call("s8b_rmsnorm_quant_split", ptr(self.part), C, ptr(self.xs), ptr(ws), ptr(res_in),
                 ptr(res_out), ptr(w), self.eps, ptr(self.xq), ptr(self.xs), ptr(y_out), M, K,
                 0, stream())

    MOE_TC = True  # expert GEMMs on the tensor cores where the shape allows (K % 128 == 0)

    def _moe_experts(self, buf, off, ne, gu_w, gu_s, d_w, d_s, contrib, M, k, Fe, st, *,
                     xq=None, xs=None):
        moe_experts(buf, off, ne, gu_w, gu_s, d_w, d_s, contrib, M, k, Fe, self.H, st,
                    xq=xq, xs=xs, tc=self.MOE_TC)

    def _moe_ffn(self, mw: MoEWeights, M: int):
        """Sparse-MoE FFN (``SparseMoE.forward``, ``superl8serve/models/moe.py:88-141``) on
        the post-attention RMSNorm output: its dtype rows (router) in moe_buf["y"], its int8
        rows in self.xq / self.xs (expert input). Result: self.h [M, H]."""
        b, st, k = self.moe_buf, stream(), mw.top_k
        E, Fe, A, H = mw.num_experts, mw.ffn, M * mw.top_k, self.H
        call("s8b_moe_route", ptr(b["y"]), 0, ptr(mw.router), M, H, E, k,
             int(mw.norm_topk_prob), mw.scaling, ptr(b["topi"]), ptr(b["topw"]),
             ptr(b["offsets"]), ptr(b["sorted_assign"]), ptr(b["sorted_token"]),
             ptr(b["assign_pos"]), st)
        # experts on partner GPUs: token rows and routing go over NVLink, the partner runs its
        # expert range (offsets from e_lo on: the same global row numbering) and its down
        # projection stores the contribution rows straight into this GPU's buffer
        home = torch.cuda.current_stream()
        for sh in mw.shards:
            pb = self.moe_peer[str(sh.device)]
            for dst, src, n in ((pb["xq"], self.xq, M * H), (pb["xs"], self.xs, 4 * M),
                                (pb["offsets"], b["offsets"], 4 * (E + 1)),
                                (pb["sorted_token"], b["sorted_token"], 4 * A)):
                call("s8b_memcpy_async", ptr(dst), ptr(src), n, st)
            pb["ev_in"].record(home)
            with torch.cuda.device(sh.device), torch.cuda.stream(pb["stream"]):
                ps, ne = pb["stream"], sh.e_hi - sh.e_lo
                ps.wait_event(pb["ev_in"])
                off = ptr(pb["offsets"]) + 4 * sh.e_lo
                self._moe_experts(pb, off, ne, sh.gu_w, sh.gu_s, sh.d_w, sh.d_s,
                                  ptr(b["contrib"]), M, k, Fe, stream())
                pb["ev_out"].record(ps)
        # experts in other processes (one process per GPU): inputs go into the partner's
        # buffers by peer copies, a release flag starts it, its down projection stores into
        # this GPU's contribution buffer and raises this GPU's flag (RemoteExperts)
        remote = [] if self.skip_remote else mw.remote
        for rx in remote:  # one launch: the four copies, then the partner's flag
            put = ((rx.xq, self.xq, M * H), (rx.xs, self.xs, 4 * M),
                   (rx.offsets, b["offsets"], 4 * (E + 1)),
                   (rx.sorted_token, b["sorted_token"], 4 * A))
            dsts = (ctypes.c_void_p * 4)(*[d for d, _, _ in put])
            srcs = (ctypes.c_void_p * 4)(*[ptr(x) for _, x, _ in put])
            nbytes = (ctypes.c_size_t * 4)(*[n for _, _, n in put])
            call("s8b_peer_put_flag", dsts, srcs, nbytes, 4, rx.in_flag, rx.epoch, 1, st)
        self._moe_experts(b, ptr(b["offsets"]), mw.local_experts, mw.gu_w, mw.gu_s, mw.d_w,
                          mw.d_s, ptr(b["contrib"]), M, k, Fe, st, xq=self.xq, xs=self.xs)
        for rx in remote:
            call("s8b_flag_wait", rx.out_flag, rx.epoch, 1, rx.timeout_ns, rx.status, st)
        if remote:  # one MoE call done on every side
            call("s8b_counter_add", remote[0].epoch, 1, st)
        for sh in mw.shards:
            home.wait_event(self.moe_peer[str(sh.device)]["ev_out"])
        call("s8b_moe_combine", ptr(b["contrib"]), ptr(b["topw"]), ptr(b["topi"]),
             ptr(b["assign_pos"]), ptr(self.h), M, k, H, 0, st)

    def layer(self, li: int, mb: MicroBatch, M: int, first_layer_of_model: bool, h_src=None,
              keep_split: bool = False):
        """One decoder layer. ``h_src`` says where the layer input comes from (None: self.h;
        (C, ws): split-K partials of the previous down projection). Returns the same for the
        layer output: partials when the tensor-core path runs and ``keep_split`` is set."""
        L = self.model.layers[li]
        kc, ks, vc, vs = self.pool.layer(li)
        H, st = self.H, stream()
        split = self.part is not None and M >= self.tc_min
        # input_layernorm (fused residual add, except on the model's first layer)
        self._rms_quant(self.h, None if first_layer_of_model else self.res, self.res, L.in_norm,
                        M, H, src=h_src)
        post = (ptr(mb.positions), ptr(self.cos), ptr(self.sin), self.cos.shape[0], ptr(L.q_norm),
                ptr(L.k_norm), self.eps, M, self.Hq, self.Hkv, self.D, ptr(self.q_i8),
                ptr(self.q_s), None, ptr(kc), ptr(ks), ptr(vc), ptr(vs), None,
                ptr(mb.block_table), mb.block_table.shape[1], self.pool.block_size, 0, st)
        if split:
            C = self._gemm_split(L.qkv_w, M)
            call("s8b_qkv_post_split", ptr(self.part), C, ptr(self.xs), ptr(L.qkv_s), *post)
        else:
            self._gemm(self.xq, self.xs, L.qkv_w, L.qkv_s, self.qkv, M)
            call("s8b_qkv_post", ptr(self.qkv), *post)
        rb = mb.extra.get("row_blocks")
        if rb is not None:  # prefill rows: each row block's partitions staged once
            call("s8b_paged_prefill_q8", ptr(self.q_i8), ptr(self.q_s), ptr(kc), ptr(ks),
                 ptr(vc), ptr(vs), ptr(mb.block_table), ptr(mb.context_lens), ptr(rb),
                 rb.shape[0], ptr(self.attn), ptr(self.xq), ptr(self.xs), M, self.Hq, self.Hkv,
                 self.D, self.pool.block_size, mb.block_table.shape[1], self.max_ctx,
                 self.scale, ptr(self.ws), self.ws.numel(), 0, st)
        else:
            call("s8b_paged_decode_q8_step" if self.decode_step else "s8b_paged_decode_q8",
                 ptr(self.q_i8), ptr(self.q_s), ptr(kc), ptr(ks), ptr(vc),
                 ptr(vs), ptr(mb.block_table), ptr(mb.context_lens), ptr(self.attn),
                 ptr(self.xq), ptr(self.xs), M, self.Hq, self.Hkv, self.D,
                 self.pool.block_size, mb.block_table.shape[1], self.max_ctx, self.scale,
                 ptr(self.ws), self.ws.numel(), 0, st)
        if L.moe is not None:
            if split:
                C = self._gemm_split(L.o_w, M)
                self._rms_quant(None, self.res, self.res, L.post_norm, M, H, src=(C, L.o_s),
                                y_out=self.moe_buf["y"])
            else:
                self._gemm(self.xq, self.xs, L.o_w, L.o_s, self.h, M)
                self._rms_quant(self.h, self.res, self.res, L.post_norm, M, H,
                                y_out=self.moe_buf["y"])
            self._moe_ffn(L.moe, M)
            return None
        if split:
            C = self._gemm_split(L.o_w, M)
            self._rms_quant(None, self.res, self.res, L.post_norm, M, H, src=(C, L.o_s))
            C = self._gemm_split(L.gu_w, M)
            call("s8b_silu_mul_quant_split", ptr(self.part), C, ptr(self.xs), ptr(L.gu_s), M,
                 self.F, None, ptr(self.xq), ptr(self.xs), 0, st)
            if keep_split:
                return (self._gemm_split(L.d_w, M), L.d_s)
            self._gemm(self.xq, self.xs, L.d_w, L.d_s, self.h, M)
            return None
        self._gemm(self.xq, self.xs, L.o_w, L.o_s, self.h, M)
        self._rms_quant(self.h, self.res, self.res, L.post_norm, M, H)
        self._gemm(self.xq, self.xs, L.gu_w, L.gu_s, self.gu, M)
        call("s8b_silu_mul_quant", ptr(self.gu), M, self.F, None, ptr(self.xq), ptr(self.xs), 0, st)
        self._gemm(self.xq, self.xs, L.d_w, L.d_s, self.h, M)
        return None

    def run(self, mb: MicroBatch, M: int | None = None, *, boundary_in=None, boundary_out=None,
            head: bool = True):
        """Enqueue the stage's work for one micro-batch on the current stream.

        boundary_in: (payload, scales, scheme) received from the previous stage.
        boundary_out: (payload, scales, scheme) in the next stage's memory (may be a peer's).
        head: on the last stage, run the final norm, LM head and argmax (a prefill chunk in
        which no sequence ends needs only the layers, which fill the KV cache).
        """
        M = self.m if M is None else M
        st = stream()
        if self.native:
            from .native import stage_desc

            d = stage_desc(self, mb, M, boundary_in, boundary_out, head)
            call("s8b_stage_step", ctypes.addressof(d), st)
            return
        first_model_layer = self.model.start == 0
        h_src = None
        if self.model.is_first:
            call("s8b_embed", ptr(mb.ids), ptr(self.model.embed), M, self.H, ptr(self.h), 0, st)
        else:  # stage prologue: the first RMSNorm decodes the received [hidden | residual]
            pay, sc, scheme = boundary_in
            h_src = ("codec", pay, sc, scheme)
        n = len(self.model.layers)
        for li in range(n):
            h_src = self.layer(li, mb, M, first_model_layer and li == 0, h_src=h_src,
                               keep_split=True)
        if self.model.is_last:
            if not head:
                return
            self._rms_quant(self.h, self.res, self.res, self.model.norm, M, self.H, src=h_src)
            self._gemm(self.xq, self.xs, self.model.head_w, self.model.head_s, self.logits, M)
            smp = mb.extra.get("sampling")
            if smp is None:
                call("s8b_argmax", ptr(self.logits), M, self.V, ptr(mb.ids), 0, st)
            else:
                # temperature / top-k / top-p / repetition penalty (s8b_sample); the step's
                # input ids come from stage 0's buffer of this micro-batch
                call("s8b_sample", ptr(self.logits), 0, M, self.V, ptr(smp["temperature"]),
                     ptr(smp["top_k"]), ptr(smp["top_p"]), ptr(smp["penalty"]),
                     ptr(smp["input_ids"]), ptr(mb.positions), ptr(smp["history"]),
                     smp["history"].shape[1], ptr(smp["seeds"]), ptr(smp["workspace"]),
                     smp["workspace"].numel(), ptr(mb.ids), st)
        else:  # stage epilogue: the encoder reduces the last down projection's partials
            pay, sc, scheme = boundary_out
            if h_src is not None:
                C, ws = h_src
                call("s8b_codec_encode_split", ptr(self.part), C, ptr(self.xs), ptr(ws),
                     ptr(self.res), M, self.H, self.H, CODEC[scheme], pay.data_ptr(),
                     sc.data_ptr(), 0, st)
            else:
                call("s8b_codec_encode", ptr(self.h), ptr(self.res), M, self.H, self.H,
                     CODEC[scheme], pay.data_ptr(), sc.data_ptr(), 0, st)

