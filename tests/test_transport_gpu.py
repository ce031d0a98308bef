"""GPU: the transport seam (``send`` / ``recv`` / ``TransferHandle`` / the wire-scheme gate)
against the CPU oracle codec, bit for bit.

``send`` (``superl8serve/dist/__init__.py:163-265``) compresses on the source GPU and
delivers the codes to ``dst`` either by peer stores straight from the encoder (route allowed
by the validated-pairs policy and the driver) or through pinned host memory (route denied,
or the same device). ``recv`` (``:268-302``) decodes on the destination. Both branches must
deliver the oracle's codes and reconstruct the oracle's output. The two-GPU cases skip on a
one-GPU box; the same-device case takes the pinned-staging branch on any box.

The gate (``superl8serve/dist/codec_quality.py:16-93``) is checked against the reference's
own ``select_wire_scheme`` / ``verify_boundary_fidelity`` run on the same seeded inputs
(``tests/golden/host_logic.json``, ``codec_gate``).
"""

import numpy as np
import pytest
import torch

from oracle import codec as oc
from oracle.numerics import round_bf16

pytestmark = pytest.mark.gpu
SCHEMES = ["int8", "int8-had", "int4", "int4-had", "nf4", "fp16"]
two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


def _x(seed, T=6, D=4096, dev="cuda:0"):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, D)).astype(np.float32)
    x[:, rng.choice(D, 4, replace=False)] *= 20
    x = round_bf16(x)
    return x, torch.from_numpy(x).to(torch.bfloat16).to(dev)


def _check(h, xh, scheme, dst, used_p2p):
    from superl8_serve_b200.dist import recv

    assert h.src_device == 0 and h.dst_device == dst and h.used_p2p == used_p2p
    assert h.d_payload.device == torch.device("cuda", dst)
    assert h.compress_elapsed_ms > 0 and h.p2p_elapsed_ms >= 0
    T, D = xh.shape
    if scheme == "fp16":
        got = h.d_payload.cpu()[: T * D * 2].view(torch.bfloat16).float().numpy().reshape(T, D)
        assert np.array_equal(got, xh)
        assert h.on_wire_bytes == T * D * 2
    else:
        po, so = oc.encode(xh, scheme)
        got = h.d_payload.cpu().numpy()[: po.nbytes].view(po.dtype).reshape(po.shape)
        assert np.array_equal(got, po)
        assert np.array_equal(h.d_scales.cpu().numpy().reshape(so.shape), so)
        assert h.on_wire_bytes == po.nbytes + so.nbytes
    out = recv(h)
    assert out.device == torch.device("cuda", dst) and h.decompress_elapsed_ms is not None
    want = xh if scheme == "fp16" else oc.decode(po, so, scheme, D)
    assert np.array_equal(out.float().cpu().numpy(), want)


@pytest.mark.parametrize("scheme", SCHEMES)
def test_send_recv_same_device_takes_pinned_staging(scheme):
    from superl8_serve_b200.dist import send

    xh, x = _x(1)
    _check(send(x, 0, scheme=scheme), xh, scheme, 0, False)


@two_gpus
@pytest.mark.parametrize("scheme", SCHEMES)
def test_send_recv_peer_route_allowed(monkeypatch, scheme):
    """Validated pair 0,1 and peer capability: the encoder stores into GPU 1's buffers."""
    from superl8_serve_b200.dist import peer_routes, send

    monkeypatch.setenv(peer_routes.VALIDATED_PAIRS_ENV, "0,1")
    if not peer_routes.peer_capability(0, 1):
        pytest.skip("the driver reports no peer access between GPU 0 and GPU 1")
    xh, x = _x(2)
    _check(send(x, 1, scheme=scheme), xh, scheme, 1, True)


@two_gpus
@pytest.mark.parametrize("scheme", ["int8-had", "int4-had"])
def test_send_recv_peer_route_denied(monkeypatch, scheme):
    """No validated pair: the codes go through pinned host memory to GPU 1."""
    from superl8_serve_b200.dist import peer_routes, send

    monkeypatch.setenv(peer_routes.VALIDATED_PAIRS_ENV, "")
    assert peer_routes.peer_route_allowed(0, 1)[1] == "not-validated"
    xh, x = _x(3)
    _check(send(x, 1, scheme=scheme), xh, scheme, 1, False)


@pytest.mark.parametrize("kind", oc.GATE_INPUTS)
def test_wire_scheme_gate_matches_reference(host_golden, kind):
    from superl8_serve_b200.dist.codec_quality import select_wire_scheme, verify_boundary_fidelity

    g = host_golden["codec_gate"][kind]
    x = torch.from_numpy(oc.gate_activation(kind, seed=g["seed"])).to(torch.bfloat16).cuda()
    assert select_wire_scheme(x) == g["scheme"]
    for scheme in ("int4", "int8"):
        sq, cos = verify_boundary_fidelity(x, scheme)
        want_sq, want_cos = g[scheme]
        if want_sq == "inf":
            assert sq == float("inf")
        else:
            assert sq == pytest.approx(want_sq, rel=1e-5)
        # (the codes are bit-exact; torch reduces the cosine on the device in another order)
        assert cos == pytest.approx(want_cos, rel=1e-5)


@pytest.mark.parametrize("scheme,bars", [("nf4", (16.0, 0.985)), ("int4", (14.0, 0.98)),
                                         ("int8", (35.0, 0.999))])
def test_codec_meets_reference_bars_fp16_input(scheme, bars):
    """The reference's acceptance checks (tests/test_transport.py:78-86,
    tests/test_codec_quality.py:57-61): a [4, 64, 256] fp16 N(0, 1) activation round-trips
    above the scheme's SQNR / cosine bars, through ``verify_boundary_fidelity`` and
    ``accuracy_report``."""
    from superl8_serve_b200.dist import accuracy_report, compress_activation, decompress_activation
    from superl8_serve_b200.dist.codec_quality import verify_boundary_fidelity

    g = torch.Generator().manual_seed(0)
    x = torch.randn((4, 64, 256), generator=g).half().cuda()
    sq, cos = verify_boundary_fidelity(x, scheme)
    assert sq > bars[0] and cos > bars[1]
    c = compress_activation(x, scheme=scheme, group_size=128 if scheme != "int8" else None)
    xr = decompress_activation(c)
    assert xr.dtype == torch.float16 and xr.shape == x.shape
    rep = accuracy_report(x, xr, scheme)
    assert rep["sqnr_pass"] and rep["cos_pass"]
    assert (rep["sqnr_bar"], rep["cos_bar"]) == bars
