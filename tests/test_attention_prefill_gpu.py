"""GPU: the varlen prefill attention (``s8b_paged_prefill_q8``) against the decode attention
and the oracle, bit for bit.

Prefill rows are packed sequence after sequence; row (sequence i, position t) attends over
positions [0, t] of its sequence's paged cache (context t + 1), the layout the reference's
varlen prefill gives ``attn_int8_varlen`` (``superl8serve/dist/pipeline.py:908-984``). The
persistent attention kernel then takes a work unit per (row block, kv head, partition): it
stages the partition once and serves the block's rows as columns of its tensor-core tiles
(up to 16 / G rows); every row must still equal its own decode unit, and the oracle's
``paged_decode``. Cases: ragged prompt lengths (1 token, partition
edges 255/256/257, several partitions), every GQA group size the kernels instantiate, block
sizes 1 to 256, row blocks cut at every size from 1 to the maximum, rows of one sequence
split over several blocks, and the counters reused by a second launch."""

import numpy as np
import pytest
import torch

from oracle import kernels as ok
from oracle import numerics as on

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture
def rng():
    return np.random.default_rng(2024)


def _to_dev(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in arrays]


def _case(rng, seq_lens, Hq, Hkv, bs):
    """Paged cache with random codes; block tables a random permutation; one row per prompt
    token with context position + 1."""
    maxb = (max(seq_lens) + bs - 1) // bs
    S = len(seq_lens)
    nb = S * maxb + 3
    kc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    vc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    ks = rng.uniform(0.01, 0.05, (nb, Hkv, bs)).astype(np.float32)
    vs = rng.uniform(0.01, 0.05, (nb, Hkv, bs)).astype(np.float32)
    perm = rng.permutation(nb)
    seq_bt = np.zeros((S, maxb + 1), dtype=np.int32)
    for i in range(S):
        seq_bt[i, :maxb] = perm[i * maxb:(i + 1) * maxb]
    seq = np.concatenate([np.full(n, i) for i, n in enumerate(seq_lens)])
    cl = np.concatenate([np.arange(1, n + 1) for n in seq_lens]).astype(np.int32)
    bt = seq_bt[seq]
    B = len(cl)
    qq = rng.integers(-127, 128, (B, Hq, 128), dtype=np.int8)
    qs = rng.uniform(0.002, 0.02, (B, Hq)).astype(np.float32)
    return kc, ks, vc, vs, bt, cl, qq, qs


def _run(case, seq_lens, block_rows, bs, Hq, launches=1):
    from superl8_serve_b200 import ops

    kc, ks, vc, vs, bt, cl, qq, qs = case
    B = len(cl)
    blocks = np.array(ops.prefill_row_blocks(seq_lens, block_rows), dtype=np.int32).reshape(-1, 2)
    qqd, qsd, kcd, ksd, vcd, vsd, btd, cld, rbd = _to_dev(qq, qs, kc, ks, vc, vs, bt, cl, blocks)
    max_ctx = int(cl.max())
    ws = torch.zeros(ops.decode_workspace_bytes(B, Hq, 128, max_ctx), dtype=torch.uint8,
                     device=DEV)
    oq = torch.empty((B, Hq * 128), dtype=torch.int8, device=DEV)
    osc = torch.empty(B, dtype=torch.float32, device=DEV)
    for _ in range(launches):
        out = ops.paged_prefill_q8(qqd, qsd, kcd, ksd, vcd, vsd, btd, cld, rbd, max_ctx,
                                   128 ** -0.5, out_q=oq, out_s=osc, workspace=ws)
    torch.cuda.synchronize()
    assert ops.decode_status(ws, B, Hq) == 0
    dec_q = torch.empty_like(oq)
    dec_s = torch.empty_like(osc)
    dec = ops.paged_decode_q8(qqd, qsd, kcd, ksd, vcd, vsd, btd, cld, max_ctx, 128 ** -0.5,
                              out_q=dec_q, out_s=dec_s)
    return out, oq, osc, dec, dec_q, dec_s


@pytest.mark.parametrize("seq_lens,Hq,Hkv,bs", [
    ([300, 1, 257, 40], 32, 8, 16),    # Qwen3-8B heads (G = 4, 4 rows per block)
    ([513], 40, 8, 16),                # 27B heads (G = 5, 3 rows)
    ([256, 255], 32, 4, 16),           # 30B-A3B heads (G = 8, 2 rows)
    ([70, 129], 8, 8, 32),             # G = 1, 16 rows per block
    ([100, 3], 16, 8, 64),             # G = 2, 8 rows
    ([60, 200], 24, 8, 256),           # G = 3, 5 rows, one block per partition
    ([33, 90], 12, 2, 8),              # G = 6, 2 rows
    ([77], 21, 3, 8),                  # G = 7, 2 rows
])
def test_prefill_attention_equals_decode_and_oracle(rng, seq_lens, Hq, Hkv, bs):
    from superl8_serve_b200 import ops

    case = _case(rng, seq_lens, Hq, Hkv, bs)
    R = ops.prefill_block_rows(Hq, Hkv)
    assert R == 16 // (Hq // Hkv)
    out, oq, osc, dec, dec_q, dec_s = _run(case, seq_lens, R, bs, Hq, launches=2)
    assert torch.equal(out, dec) and torch.equal(oq, dec_q) and torch.equal(osc, dec_s)
    kc, ks, vc, vs, bt, cl, qq, qs = case
    B = len(cl)
    sel = np.unique(np.r_[0, B - 1, np.linspace(0, B - 1, 24).astype(int)])
    ref = ok.paged_decode(qq[sel], qs[sel], kc, ks, vc, vs, bt[sel], cl[sel], bs,
                          128 ** -0.5).reshape(len(sel), -1)
    assert np.array_equal(out.float().cpu().numpy()[sel], ref)
    rq, rs = on.quant_rows_i8(ref)
    assert np.array_equal(oq.cpu().numpy()[sel], rq) and np.array_equal(osc.cpu().numpy()[sel], rs)


@pytest.mark.parametrize("block_rows", [1, 2, 3, 4])
def test_prefill_attention_any_block_size(rng, block_rows):
    """Blocks smaller than the maximum (and rows of one sequence over many blocks) give the
    same rows."""
    seq_lens = [290, 17]
    case = _case(rng, seq_lens, 32, 8, 16)
    out, oq, osc, dec, dec_q, dec_s = _run(case, seq_lens, block_rows, 16, 32)
    assert torch.equal(out, dec) and torch.equal(oq, dec_q) and torch.equal(osc, dec_s)
