"""CPU: the oracle against the golden fixtures produced by the reference's own module graph
(tests/golden/make_golden.py) and against the reference's tolerance bars."""

import json

import numpy as np
import pytest

from oracle import codec as oc
from oracle import kernels as ok
from oracle import numerics as on
from oracle.model import OraclePipeline, quantize_state_dict
from superl8_serve_b200.config import tiny
from superl8_serve_b200.weights import random_state_dict

PROMPTS = [[3, 1, 4, 1, 5], [9, 2, 6], [5, 3, 5, 8, 9, 7, 9]]


@pytest.fixture(scope="module")
def tiny_qw():
    cfg = tiny()
    return cfg, quantize_state_dict(random_state_dict(cfg, 11, w_std=0.1), cfg)


@pytest.mark.parametrize("tag,stages,scheme", [
    ("s1", 1, "int8"), ("s2_int8", 2, "int8"), ("s2_int8had", 2, "int8-had"),
    ("s3_int4had", 3, "int4-had")])
def test_oracle_pipeline_matches_reference_module_graph(golden_dir, tiny_qw, tag, stages, scheme):
    """Greedy tokens and bf16 logits of the oracle's own driver == the reference's
    Qwen3ForCausalLM / make_pipeline graph run with the same kernels (bit for bit)."""
    d = np.load(golden_dir / "tiny_qwen3_decode.npz")
    cfg, qw = tiny_qw
    p = OraclePipeline(cfg, qw, n_stages=stages, wire_scheme=scheme, num_slots=4, max_len=64)
    assert p.bounds == list(d[f"{tag}_bounds"])
    outs, logits = p.generate(PROMPTS, 8)
    assert np.array_equal(np.array(outs), d[f"{tag}_tokens"])
    assert np.array_equal(np.array(logits, dtype=np.float32), d[f"{tag}_logits"])


@pytest.mark.parametrize("tag,stages,scheme", [("s1", 1, "int8"), ("s3_int4had", 3, "int4-had")])
def test_oracle_prefill_equals_teacher_forced_decode(golden_dir, tiny_qw, tag, stages, scheme):
    """The varlen prefill (all prompt rows in one batch, each attending over its own prefix)
    followed by per-sequence decode gives the reference graph's tokens and logits bit for
    bit: a prompt row computes exactly what the decode step of that token computes."""
    d = np.load(golden_dir / "tiny_qwen3_decode.npz")
    cfg, qw = tiny_qw
    p = OraclePipeline(cfg, qw, n_stages=stages, wire_scheme=scheme, num_slots=4, max_len=64)
    outs, logits = p.generate_prefilled(PROMPTS, 8)
    assert np.array_equal(np.array(outs), d[f"{tag}_tokens"])
    assert np.array_equal(np.array(logits, dtype=np.float32), d[f"{tag}_logits"])


def test_eager_rmsnorm_close_to_reference(golden_dir):
    e = np.load(golden_dir / "eager_numerics.npz")
    res = ok.add_residual(e["norm_x"], e["norm_r"])
    assert np.array_equal(res, e["norm_res"])
    y = ok.rmsnorm(res, e["norm_w"], 1e-6)
    # reference eager path: torch rsqrt + fp32 mean; ours: fp64 sum + 1/sqrt -> <= 1 bf16 ulp
    rel = np.abs(y - e["norm_y"]) / np.maximum(np.abs(e["norm_y"]), 1e-3)
    assert rel.max() <= 2 ** -7


def test_rope_tables_and_rotation_close_to_reference(golden_dir):
    e = np.load(golden_dir / "eager_numerics.npz")
    cos, sin = ok.rope_tables(128, 4096, 1e6)
    assert np.array_equal(cos, e["rope_cos"]) and np.array_equal(sin, e["rope_sin"])
    pos = e["rope_pos"].reshape(-1)
    c, s = cos[pos][:, None, None, :], sin[pos][:, None, None, :]
    for x, ref in ((e["rope_q"], e["rope_qr"]), (e["rope_k"], e["rope_kr"])):
        y = ok.rope(x, c, s)
        # reference eager casts cos/sin to bf16 first; ours keeps them binary32
        assert np.abs(y - ref).max() <= 0.05 * max(1.0, np.abs(ref).max())
        assert np.corrcoef(y.ravel(), ref.ravel())[0, 1] > 0.9999


def test_silu_mul_close_to_reference(golden_dir):
    e = np.load(golden_dir / "eager_numerics.npz")
    y = ok.silu_mul(e["silu_in"])
    ref = e["silu_out"]
    assert np.abs(y - ref).max() <= 2 ** -7 * max(1.0, np.abs(ref).max())


def test_greedy_argmax_matches_reference_sampler(golden_dir):
    e = np.load(golden_dir / "eager_numerics.npz")
    assert np.array_equal(ok.argmax_rows(e["samp_logits"]), e["samp_tok"])


def test_exp_accuracy():
    x = np.linspace(-80, 0, 20001, dtype=np.float32)
    y = on.exp_s8b(x)
    ref = np.exp(x.astype(np.float64))
    # binary32 rounding of t = x*log2(e) dominates: relative error ~ |x| * 6e-8
    assert np.max(np.abs(y - ref) / ref / np.maximum(1.0, np.abs(x))) < 1e-7
    assert on.exp_s8b(np.float32(0.0)) == 1.0
    assert on.exp_s8b(np.float32(-200.0)) == 0.0
    assert np.isinf(on.exp_s8b(np.float32(100.0)))


def test_hadamard_is_orthonormal_involution():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((16, 128)).astype(np.float32)
    y = on.hadamard128(on.hadamard128(x))
    assert np.abs(y - x).max() < 1e-5
    i = np.arange(128)
    pc = np.vectorize(lambda v: bin(v).count("1"))(i[:, None] & i[None, :])
    H = (1 - 2 * (pc % 2)) / np.sqrt(128)
    assert np.abs(on.hadamard128(x) - x @ H).max() < 1e-5


def test_weight_quant_recipe_matches_reference_helper():
    """tests/test_layers.py:29-33 recipe: s = absmax.clamp_min(1e-6)/127, q=round(w/s)."""
    rng = np.random.default_rng(1)
    w = rng.standard_normal((64, 256)).astype(np.float32)
    w[3] = 0
    q, s = on.quantize_weight_rowwise(w)
    assert q.dtype == np.int8 and np.abs(q).max() <= 127
    assert np.allclose(s[3], np.float32(1e-6) / 127)
    assert np.array_equal(np.abs(q).max(axis=1)[np.arange(64) != 3], np.full(63, 127))


def _activation(shape, seed, outlier=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32)
    if outlier:
        x[..., :: max(1, shape[-1] // 8)] += 12.0
    return on.round_bf16(x)


@pytest.mark.parametrize("scheme,bar", [("int8", (35.0, 0.999)), ("int8-had", (35.0, 0.999)),
                                        ("int4", (14.0, 0.98)), ("int4-had", (14.0, 0.98)),
                                        ("nf4", (16.0, 0.985))])
def test_codec_meets_reference_bars(scheme, bar):
    """Acceptance bars of superl8serve/dist/__init__.py:46-52 on Gaussian activations."""
    x = _activation((4 * 64, 256), 2)
    pay, sc = oc.encode(x, scheme)
    xr = oc.decode(pay, sc, scheme, 256)
    sqnr, cos = oc.accuracy(x, xr)
    assert sqnr >= bar[0] and cos >= bar[1]


def test_codec_fp16_lossless_and_hadamard_helps_outliers():
    x = _activation((64, 128), 3, outlier=True)
    pay, sc = oc.encode(x, "fp16")
    assert np.array_equal(oc.decode(pay, sc, "fp16", 128), x)
    r4 = oc.accuracy(x, oc.decode(*oc.encode(x, "int4"), "int4", 128))[0]
    rh = oc.accuracy(x, oc.decode(*oc.encode(x, "int4-had"), "int4-had", 128))[0]
    assert rh > r4


def test_nf4_codebook_is_the_published_construction():
    """The pinned binary32 table equals the NF4 construction (normal quantiles, normalised)."""
    cb = oc.nf4_codebook()
    assert cb.dtype == np.float32 and cb.shape == (16,)
    np.testing.assert_allclose(cb, oc.NF4, rtol=0, atol=2e-7)
    assert oc.NF4[0] == -1.0 and oc.NF4[7] == 0.0 and oc.NF4[15] == 1.0
    assert np.all(np.diff(oc.NF4) > 0)


def test_nf4_codes_nearest_entry_lowest_on_ties():
    """nf4 codes: each value's code is the nearest table entry to x / absmax; a value exactly
    halfway between two entries takes the lower index; an all-zero group encodes to the
    0.0 entry with scale 0 and decodes to +0."""
    x = np.zeros((2, 128), np.float32)
    mids = ((oc.NF4[:-1] + oc.NF4[1:]) / 2).astype(np.float32)
    x[0, : mids.size] = mids
    x[0, 127] = 1.0  # absmax 1: y == x
    pay, sc = oc.encode(x, "nf4")
    assert sc.shape == (2, 1) and sc[0, 0] == 1.0 and sc[1, 0] == 0.0
    codes = np.stack([pay & 0xF, pay >> 4], -1).reshape(2, 128)
    for i, m in enumerate(mids):
        d = np.abs(m - oc.NF4).astype(np.float32)
        assert codes[0, i] == int(np.argmin(d))
        assert codes[0, i] in (i, i + 1)
    assert np.all(codes[1] == 7)
    out = oc.decode(pay, sc, "nf4", 128)
    assert np.array_equal(out[1], np.zeros(128, np.float32)) and not np.signbit(out[1]).any()
    assert np.array_equal(out[0, 127:], [1.0])


def test_nf4_wire_bytes_equal_int4():
    """nf4 is a 4-bit code with one fp32 scale per 128 values
    (superl8serve/dist/transfer_model.py:31,40), so it weighs what int4 weighs."""
    assert oc.wire_bytes(4, 8192, "nf4") == oc.wire_bytes(4, 8192, "int4")
    pay, sc = oc.encode(_activation((4, 8192), 9), "nf4")
    assert pay.nbytes + sc.nbytes == oc.wire_bytes(4, 8192, "nf4")


def test_codec_wire_bytes_match_reference_handle(golden_dir):
    """TransferHandle.on_wire_bytes of the reference (payload + fp32 scales)."""
    host = json.loads((golden_dir / "host_logic.json").read_text())
    got = {s: b for s, b, _ in host["on_wire_bytes"]}
    assert oc.wire_bytes(4, 8192, "int8") == got["int8"]
    assert oc.wire_bytes(4, 8192, "int4") == got["int4"]
    assert oc.wire_bytes(4, 8192, "fp16") == got["fp16"]


def test_codec_config2_outliers_int8_and_int4():
    """BASELINE config 2 input: N(0,1) with 0.1% of channels x20."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((64, 4096)).astype(np.float32)
    x[:, rng.choice(4096, 4, replace=False)] *= 20
    x = on.round_bf16(x)
    for scheme, bar in (("int8-had", 35.0), ("int4-had", 14.0)):
        pay, sc = oc.encode(x, scheme)
        assert oc.accuracy(x, oc.decode(pay, sc, scheme, 4096))[0] >= bar


def test_paged_decode_matches_dense_softmax():
    """Partitioned, order-fixed attention == plain softmax attention on the same int8 data."""
    rng = np.random.default_rng(7)
    B, Hq, Hkv, bs, nb = 2, 4, 2, 16, 64
    kc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    vc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    ks = rng.uniform(0.01, 0.03, (nb, Hkv, bs)).astype(np.float32)
    vs = rng.uniform(0.01, 0.03, (nb, Hkv, bs)).astype(np.float32)
    qq = rng.integers(-127, 128, (B, Hq, 128), dtype=np.int8)
    qs = rng.uniform(0.005, 0.02, (B, Hq)).astype(np.float32)
    bt = np.stack([rng.permutation(nb)[:40], rng.permutation(nb)[:40]]).astype(np.int32)
    cl = np.array([600, 17], dtype=np.int32)
    out = ok.paged_decode(qq, qs, kc, ks, vc, vs, bt, cl, bs, 128 ** -0.5)
    for b in range(B):
        n = cl[b]
        j = np.arange(n)
        rows = bt[b][j // bs] * Hkv * bs + j % bs
        for h in range(Hq):
            g = h // (Hq // Hkv)
            r = (bt[b][j // bs] * Hkv + g) * bs + j % bs
            k = kc.reshape(-1, 128)[r] * ks.reshape(-1)[r][:, None]
            v = vc.reshape(-1, 128)[r] * vs.reshape(-1)[r][:, None]
            q = qq[b, h] * qs[b, h]
            s = (k.astype(np.float64) @ q) * 128 ** -0.5
            p = np.exp(s - s.max())
            ref = (p / p.sum()) @ v
            assert np.abs(out[b, h] - ref).max() < 1e-2 * max(1.0, np.abs(ref).max())
        del rows


def test_k_side_int8_meets_reference_bar():
    """The reference's K-cache bar (superl8-serve tests/test_k8v3_cache.py:113-120): Hadamard
    rotation, per-row int8, dequantize and rotate back -> cos >= 0.999 and SQNR >= 35 dB."""
    rng = np.random.default_rng(11)
    T, Hkv, D, bs = 40, 2, 128, 16
    k = on.round_bf16(rng.standard_normal((T, Hkv, D)).astype(np.float32))
    k[:, :, rng.choice(D, 2, replace=False)] *= 10  # outlier channels
    nb = -(-T // bs)
    kc = np.zeros((nb, Hkv, bs, D), np.int8)
    vc = np.zeros_like(kc)
    ks = np.zeros((nb, Hkv, bs), np.float32)
    vs = np.zeros_like(ks)
    ok.kv_write_paged(k, k, kc, ks, vc, vs, np.arange(T, dtype=np.int32), bs)
    rows = ok.flat_rows(np.arange(T, dtype=np.int32), Hkv, bs).reshape(-1)
    deq = kc.reshape(-1, D)[rows].astype(np.float32) * ks.reshape(-1)[rows][:, None]
    back = on.hadamard128(deq).reshape(T, Hkv, D)
    x, y = k.astype(np.float64).ravel(), back.astype(np.float64).ravel()
    sqnr = 10 * np.log10((x ** 2).sum() / ((x - y) ** 2).sum())
    cos = x @ y / np.linalg.norm(x) / np.linalg.norm(y)
    assert sqnr >= 35.0 and cos >= 0.999


def test_paged_int8_decode_meets_reference_bar_against_unquantized_attention():
    """The reference's paged-decode bar (superl8-serve tests/test_paged_engine.py:98-101):
    int8 KV (rotated K), int8 query, partitioned softmax with 15-bit p.v against plain fp32
    attention on the unquantized q, k, v -> cos > 0.995."""
    rng = np.random.default_rng(12)
    B, Hq, Hkv, D, bs, ctx = 2, 8, 2, 128, 16, 700
    q = on.round_bf16(rng.standard_normal((B, Hq, D)).astype(np.float32))
    k = on.round_bf16(rng.standard_normal((B * ctx, Hkv, D)).astype(np.float32))
    v = on.round_bf16(rng.standard_normal((B * ctx, Hkv, D)).astype(np.float32))
    nb = B * -(-ctx // bs)
    kc = np.zeros((nb, Hkv, bs, D), np.int8)
    vc = np.zeros_like(kc)
    ks = np.zeros((nb, Hkv, bs), np.float32)
    vs = np.zeros_like(ks)
    per = -(-ctx // bs)
    bt = np.arange(nb, dtype=np.int32).reshape(B, per)
    slots = np.concatenate([bt[b][np.arange(ctx) // bs] * bs + np.arange(ctx) % bs
                            for b in range(B)]).astype(np.int32)
    ok.kv_write_paged(k, v, kc, ks, vc, vs, slots, bs)
    qq, qs = ok.quant_q_for_attn(q)
    out = ok.paged_decode(qq, qs, kc, ks, vc, vs, bt, np.full(B, ctx, np.int32), bs, D ** -0.5)
    for b in range(B):
        kb, vb = k[b * ctx:(b + 1) * ctx], v[b * ctx:(b + 1) * ctx]
        for h in range(Hq):
            g = h // (Hq // Hkv)
            s = (kb[:, g].astype(np.float64) @ q[b, h]) * D ** -0.5
            p = np.exp(s - s.max())
            ref = (p / p.sum()) @ vb[:, g]
            got = out[b, h].astype(np.float64)
            assert got @ ref / np.linalg.norm(got) / np.linalg.norm(ref) > 0.995
