"""CPU: the C-ABI library loads and exports every entry point include/s8b.h declares; the
host-side logic (block allocator, stage split, peer-route policy, wire accounting) matches the
reference's own behaviour recorded in tests/golden/host_logic.json."""

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from superl8_serve_b200 import _lib
from superl8_serve_b200.dist import peer_routes as pr
from superl8_serve_b200.dist.pipeline import stage_bounds
from superl8_serve_b200.engine import BlockAllocator

REPO = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    names = []
    for h in (REPO / "include").glob("*.h"):
        txt = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(s8b_[a-z0-9_]+)\s*\(", txt)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_strerror_and_version(lib):
    assert _lib.strerror(0) == "ok"
    assert "timed out" in _lib.strerror(-6)
    assert lib.s8b_version() >= 1
    assert lib.s8b_ipc_handle_size() == 64


@pytest.mark.parametrize("call", [
    lambda L: L.s8b_quant_rows(None, 0, None, None, 4, 16, None),
    lambda L: L.s8b_gemm_w8a8(None, None, None, None, None, 0, 1, 1, 16, 0, None),
    lambda L: L.s8b_paged_decode_q8(*([None] * 11), 1, 4, 2, 128, 16, 4, 64, 0.1, None, 0, 0, None),
    lambda L: L.s8b_codec_encode(None, None, 1, 128, 0, 1, None, None, 0, None),
    lambda L: L.s8b_flag_wait(None, None, 0, 1000, None, None),
    lambda L: L.s8b_exp_f32(None, None, 5, None),
])
def test_null_arguments_are_rejected_without_touching_the_gpu(lib, call):
    assert call(lib) == -8


def test_shape_and_scheme_validation(lib):
    buf = 1  # any non-null pointer: validation happens before dereference
    assert lib.s8b_gemm_w8a8(buf, buf, buf, buf, buf, 0, 1, 1, 17, 0, None) == -1  # K % 16
    assert lib.s8b_codec_encode(buf, None, 1, 100, 0, 2, buf, buf, 0, None) == -1  # -had needs 128
    assert lib.s8b_codec_encode(buf, None, 1, 128, 0, 9, buf, buf, 0, None) == -2  # scheme
    assert lib.s8b_quant_rows(256, 7, 256, 256, 1, 16, None) == -2  # dtype
    assert lib.s8b_quant_rows(buf, 0, buf, buf, 1, 16, None) == -3  # misaligned row pointer
    # workspace too small
    assert lib.s8b_paged_decode_q8(*([16] * 11), 1, 4, 2, 128, 16, 4, 64, 0.1, 16, 1, 0, None) == -7


def test_workspace_and_codec_sizes(lib):
    P = (2049 + 255) // 256
    # status word (256-byte region) first, then the (row, head) and row counters
    counters = 256 + (64 * 32 * 4 + 64 * 4 + 255) // 256 * 256
    assert lib.s8b_paged_decode_status_offset(64, 32) == 0
    assert lib.s8b_paged_decode_status_offset(3, 16) == 0
    assert lib.s8b_set_attention_impl(3) == -8
    assert lib.s8b_paged_decode_workspace_size(64, 32, 128, 2049) == counters + 64 * 32 * P * 130 * 4
    assert lib.s8b_codec_payload_bytes(4, 8192, 2, 0) == 4 * 8192
    assert lib.s8b_codec_scale_count(4, 8192, 2) == 4
    assert lib.s8b_codec_payload_bytes(4, 8192, 4, 0) == 4 * 4096
    assert lib.s8b_codec_scale_count(4, 8192, 4) == 4 * 64
    assert lib.s8b_codec_payload_bytes(4, 8192, 0, 0) == 4 * 8192 * 2


def test_product_fails_loudly_on_cpu_tensors():
    from superl8_serve_b200 import ops

    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quant_rows(torch.zeros(2, 16, dtype=torch.bfloat16))


def test_stage_bounds_match_reference(host_golden):
    for key, bounds in host_golden["stage_bounds"].items():
        L, S = map(int, key.split("_"))
        assert stage_bounds(L, S) == bounds


def test_block_allocator_matches_reference_paged_cache(host_golden):
    g = host_golden["kv_alloc"]
    a = BlockAllocator(num_blocks=4 * 4, num_slots=4, block_size=16, max_blocks_per_seq=4)
    s0, s1 = a.alloc(), a.alloc()
    a.ensure_capacity([s0, s1], [20, 33])
    s2 = a.alloc()
    a.free(s0)
    a.ensure_capacity([s2, s1], [5, 50])
    assert [s0, s1, s2] == g["slots"]
    assert a._slot_blocks == g["slot_blocks"]
    assert a.block_table([s1, s2]).tolist() == g["block_table_bc"]
    bs = 16
    sm = [a._slot_blocks[s][p // bs] * bs + p % bs for s, p in zip([s1, s2, s1], [0, 3, 49])]
    assert sm == g["slot_mapping"]
    from oracle.kernels import flat_rows

    assert flat_rows(np.array([0, 17, 49]), 2, 16).reshape(-1).tolist() == g["flat_rows"]
    assert a.num_blocks - len(a._free_blocks) == g["used_blocks"]


def test_parse_validated_pairs_matches_reference(host_golden):
    for spec, want in host_golden["parse_validated_pairs"].items():
        if isinstance(want, str):
            with pytest.raises(ValueError):
                pr.parse_validated_pairs(spec)
        else:
            assert sorted(map(list, pr.parse_validated_pairs(spec))) == want


def test_select_route_matches_reference(host_golden):
    for spec, src, dst, cap, want in host_golden["select_route"]:
        val = pr.parse_validated_pairs(spec)
        assert list(pr.select_route(src, dst, validated=val, capability=cap)) == want


def test_validated_pairs_env_names(monkeypatch):
    monkeypatch.delenv(pr.VALIDATED_PAIRS_ENV, raising=False)
    monkeypatch.setenv(pr.LEGACY_VALIDATED_PAIRS_ENV, "0,1")
    assert pr.validated_pairs() == frozenset({(0, 1)})
    monkeypatch.setenv(pr.VALIDATED_PAIRS_ENV, "2,3")
    assert pr.validated_pairs() == frozenset({(2, 3)})
    assert pr.peer_route_allowed(2, 3, capability=True) == (True, "validated-p2p")
    assert pr.peer_route_allowed(0, 1, capability=True) == (False, "not-validated")
    assert pr.all_pairs_spec([0, 1, 2]) == "0,1;0,2;1,2"


def test_accuracy_report_matches_reference(golden_dir, host_golden):
    from superl8_serve_b200.dist import accuracy_report

    d = np.load(golden_dir / "acc_inputs.npz")
    rep = accuracy_report(torch.from_numpy(d["x"]), torch.from_numpy(d["xr"]), "int8")
    want = host_golden["accuracy_report"]
    assert rep["sqnr_db"] == pytest.approx(want["sqnr_db"], rel=1e-6)
    assert rep["cos"] == pytest.approx(want["cos"], rel=1e-6)
    assert rep["sqnr_pass"] == want["sqnr_pass"] and rep["cos_pass"] == want["cos_pass"]
    x = torch.from_numpy(d["x"])
    assert accuracy_report(x, x.clone(), "fp16")["sqnr_db"] == float("inf")


def test_transfer_handle_wire_bytes_match_reference(host_golden):
    from superl8_serve_b200.dist import TransferHandle

    pays = {"int8": ((4, 8192), torch.int8, (4,)), "int4": ((4, 4096), torch.int8, (4, 64)),
            "fp16": ((4, 8192), torch.bfloat16, (0,))}
    for scheme, want, want_ms in host_golden["on_wire_bytes"]:
        shp, dt, sc = pays[scheme]
        h = TransferHandle(0, 1, scheme, torch.Size((4, 1, 8192)), torch.bfloat16, None,
                           torch.empty(shp, dtype=dt), torch.empty(sc), 0.0, 0.0)
        assert h.on_wire_bytes == want
        assert h.theoretical_wire_ms == pytest.approx(want_ms)


def test_stage_descriptor_layout_matches_the_library(lib):
    """The ctypes mirrors of S8bStageDesc / S8bLayerDesc have the C sizes, and a missing
    descriptor is rejected before any CUDA call."""
    import ctypes

    from superl8_serve_b200.native import LayerDesc, StageDesc

    assert ctypes.sizeof(StageDesc) == lib.s8b_stage_desc_size()
    assert ctypes.sizeof(LayerDesc) == lib.s8b_layer_desc_size()
    assert lib.s8b_stage_step(None, None) == -8


def test_ctypes_signatures_match_header_prototypes():
    """Every prototype in include/s8b.h has the same parameter count and C types in the
    ctypes table the package binds with (a float passed where the C side expects a pointer,
    or a missing argument, would otherwise go unnoticed until a kernel misbehaves)."""
    import ctypes as C
    import re

    text = (REPO / "include" / "s8b.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"typedef struct .*?\} \w+;", "", text, flags=re.S)

    def ctype(param: str):
        p = " ".join(param.split())
        if "*" in p:
            return "ptr"
        base = p.rsplit(" ", 1)[0] if " " in p else p
        base = base.replace("const ", "")
        return {"float": C.c_float, "double": C.c_double, "size_t": C.c_size_t,
                "int": C.c_int, "int32_t": C.c_int32, "uint32_t": C.c_uint32,
                "uint64_t": C.c_uint64, "long long": C.c_longlong}[base]

    checked = 0
    for name, params in re.findall(r"\b(s8b_\w+)\s*\(([^;{]*?)\)\s*;", text):
        params = params.strip()
        want = [] if params in ("", "void") else [ctype(q) for q in params.split(",")]
        got = _lib.SIGNATURES[name][1]
        assert len(got) == len(want), name
        for g, w in zip(got, want):
            if w == "ptr":
                assert g in (C.c_void_p, C.c_char_p), name
            else:
                assert C.sizeof(g) == C.sizeof(w) and (g is C.c_float) == (w is C.c_float) \
                    and (g is C.c_double) == (w is C.c_double), (name, g, w)
        checked += 1
    assert checked >= 55


@pytest.mark.parametrize("kind", ["gauss", "outliers", "laplace", "const"])
def test_wire_scheme_gate_logic_matches_reference(host_golden, monkeypatch, kind):
    """``select_wire_scheme`` / ``verify_boundary_fidelity`` against the reference's own gate
    on the same seeded inputs, with the oracle codec standing in for the GPU codec (the GPU
    run of the same check is in test_transport_gpu)."""
    from oracle import codec as oc
    from superl8_serve_b200.dist import Compressed, codec_quality as cq

    def compress(x, scheme="int8", group_size=None):
        pay, sc = oc.encode(x.float().numpy(), scheme)
        return Compressed(scheme, tuple(x.shape), x.dtype, group_size, pay, sc, x.shape[-1])

    def decompress(c):
        return torch.from_numpy(oc.decode(c.payload, c.scales, c.scheme, c.d)).to(c.dtype)

    monkeypatch.setattr(cq, "compress_activation", compress)
    monkeypatch.setattr(cq, "decompress_activation", decompress)
    g = host_golden["codec_gate"][kind]
    x = torch.from_numpy(oc.gate_activation(kind, seed=g["seed"])).to(torch.bfloat16)
    assert cq.select_wire_scheme(x) == g["scheme"]
    for scheme in ("int4", "int8"):
        sq, cos = cq.verify_boundary_fidelity(x, scheme)
        want_sq, want_cos = g[scheme]
        assert sq == (float("inf") if want_sq == "inf" else pytest.approx(want_sq, rel=1e-6))
        assert cos == pytest.approx(want_cos, rel=1e-6)


def test_nf4_sizes_and_prefill_block_rows(lib):
    """Host-side answers of the library: nf4 weighs what int4 weighs (4-bit codes, one fp32
    scale per 128 values); prefill row blocks hold 16 / G rows (the tile's 16 columns)."""
    assert lib.s8b_codec_payload_bytes(4, 8192, 5, 0) == 4 * 4096
    assert lib.s8b_codec_scale_count(4, 8192, 5) == 4 * 64
    for Hq, Hkv in ((32, 8), (40, 8), (32, 4), (8, 8), (16, 8), (24, 8), (12, 2), (21, 3)):
        assert lib.s8b_paged_prefill_block_rows(Hq, Hkv) == 16 // (Hq // Hkv)
    assert lib.s8b_paged_prefill_block_rows(36, 4) == -1   # G = 9: more heads than a tile row
    assert lib.s8b_paged_prefill_block_rows(30, 8) == -1   # Hq not a multiple of Hkv
    buf = 1
    assert lib.s8b_codec_encode(buf, None, 1, 128, 0, 6, buf, buf, 0, None) == -2  # past nf4
