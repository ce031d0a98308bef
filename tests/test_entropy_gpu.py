"""GPU: the rANS kernels through the C ABI against the reference's own streams (golden) and
the oracle; the entropy stage of send / recv."""

import numpy as np
import pytest
import torch

from oracle import entropy as oe
from superl8_serve_b200.dist import entropy as ent

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
CASES = ["int8_codes", "int4_codes", "constant42", "uniform", "skewed", "one_byte", "empty"]


@pytest.fixture(scope="module")
def g(golden_dir):
    return np.load(golden_dir / "rans.npz")


@pytest.mark.parametrize("case", CASES)
def test_single_stream_is_the_reference_byte_stream(g, case):
    data = g[f"{case}_data"]
    enc, freqs, _ = ent.encode(torch.from_numpy(data).to(DEV))
    assert np.array_equal(freqs, g[f"{case}_freqs"])
    assert np.array_equal(enc.cpu().numpy(), g[f"{case}_enc"])
    dec = ent.decode(torch.from_numpy(g[f"{case}_enc"]).to(DEV), g[f"{case}_freqs"], data.size)
    assert np.array_equal(dec.cpu().numpy(), data)


@pytest.mark.parametrize("S", [7, 256])
def test_multi_stream_matches_oracle_and_round_trips(g, S):
    rng = np.random.default_rng(S)
    data = np.concatenate([g["int8_codes_data"],
                           np.minimum(rng.geometric(0.2, 60000), 255).astype(np.uint8)])
    buf, freqs, lens = ent.encode(torch.from_numpy(data).to(DEV), n_streams=S)
    streams, ofreqs = oe.encode(data, n_streams=S)
    assert np.array_equal(freqs, ofreqs)
    lens_h = lens.cpu().numpy()
    b = buf.cpu().numpy()
    n = data.size
    for i in range(S):
        off = 2 * (n * i // S) + 4 * i
        assert b[off:off + lens_h[i]].tobytes() == streams[i]
    dec = ent.decode(buf, freqs, n, lengths=lens)
    assert np.array_equal(dec.cpu().numpy(), data)


def test_decode_reports_a_stream_that_ends_early(g):
    data = g["uniform_data"]
    enc = torch.from_numpy(g["uniform_enc"][-4:].copy()).to(DEV)  # the final state alone
    with pytest.raises(RuntimeError):
        ent.decode(enc, g["uniform_freqs"], data.size)


@pytest.mark.parametrize("scheme", ["int8", "int8-had", "int4-had"])
def test_send_recv_entropy_stage_is_lossless(scheme):
    from superl8_serve_b200.dist import recv, send

    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal((8, 2048)).astype(np.float32)).to(torch.bfloat16)
    x = x.to(DEV)
    plain = recv(send(x, 0, scheme=scheme))
    h = send(x, 0, scheme=scheme, entropy=True)
    assert h.entropy_freqs is not None and h.entropy_n > 0
    assert h.on_wire_bytes == h.d_payload.numel() + h.d_scales.numel() * 4 + 512
    assert torch.equal(recv(h), plain)
