"""The weight file, the seeded random init and the fingerprint (CPU only)."""
import os

import numpy as np
import pytest
import torch

from mayfly_chess_b200 import weights as W


@pytest.mark.parametrize("tag,arch", [("small", W.SMALL), ("full", W.FULL)])
def test_state_spec_is_chessnets(meta, tag, arch):
    """The parameter list the random init walks is ChessNet's own state dict order (recorded from the reference
    model by the fixture generator)."""
    assert [k for k, _ in W.state_spec(arch)] == meta[f"state_keys_{tag}"]


def test_fingerprints(meta):
    assert W.fingerprint(W.random_state(W.SMALL, 0)) == meta["fingerprint_small_seed0"]
    assert W.fingerprint(W.random_state(W.FULL, 1)) == meta["fingerprint_full_seed1"]


def test_random_state_rule():
    st = W.random_state(W.SMALL, 0)
    assert torch.equal(st["enc.layers.0.norm1.weight"], torch.ones(256))
    assert torch.equal(st["ln.bias"], torch.zeros(256))
    w = st["enc.layers.0.linear1.weight"]
    assert abs(float(w.std()) - 0.02) < 0.001 and abs(float(w.mean())) < 0.001
    # same seed, same weights; another seed, other weights
    assert torch.equal(W.random_state(W.SMALL, 0)["piece.weight"], st["piece.weight"])
    assert not torch.equal(W.random_state(W.SMALL, 1)["piece.weight"], st["piece.weight"])


@pytest.mark.parametrize("precision", ["f16", "bf16", "e4m3"])
def test_cnw_roundtrip(tmp_path, precision):
    st = W.random_state(W.SMALL, 0)
    path = os.path.join(tmp_path, "n.cnw")
    amax = np.tile(np.array([4.0, 2.5, 5.0, 3.0], np.float32), (W.SMALL.layers, 1))
    hdr = W.write_cnw(path, st, W.SMALL, precision, act_amax=amax if precision == "e4m3" else None)
    h2, t = W.read_cnw(path)
    assert h2 == hdr
    assert h2["version"] == (1 if precision == "f16" else 2)
    assert h2["fingerprint"] == W.fingerprint(st)
    for e in h2["tensors"]:
        assert e["offset"] % 256 == 0
    np.testing.assert_array_equal(t["piece"], st["piece.weight"].numpy())
    q = t["L1.ff2_w"]
    ref = st["enc.layers.1.linear2.weight"]
    if precision == "f16":
        np.testing.assert_array_equal(q, ref.half().numpy())
    elif precision == "bf16":
        np.testing.assert_array_equal(W.bf16_bits_to_f32(q).numpy(), ref.bfloat16().float().numpy())
    else:
        deq = W.e4m3_to_f32(q, t["L1.ff2_w_scale"])
        rel = (deq - ref).abs().max() / ref.abs().max()
        assert rel < 2 ** -3      # e4m3 keeps 3 mantissa bits
        # the static input scales: ACT_HEADROOM x max |x| maps to 448
        np.testing.assert_allclose(t["L2.act_scale"], amax[2] * W.ACT_HEADROOM / 448.0, rtol=1e-6)
    # the heads stay 16-bit in every precision
    assert t["heads_w"].dtype == (np.float16 if precision == "f16" else np.uint16)


def test_cnw_rejects_bad_magic(tmp_path):
    path = os.path.join(tmp_path, "bad.cnw")
    with open(path, "wb") as f:
        f.write(b"NOTCNW01" + b"\0" * 64)
    with pytest.raises(ValueError):
        W.read_cnw(path)


def test_bf16_rounding_is_nearest_even():
    x = torch.tensor([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5e-3], dtype=torch.float32)
    bits = W.to_bf16_bits(x)
    assert torch.equal(W.bf16_bits_to_f32(bits), x.bfloat16().float())


def test_e4m3_needs_calibration(tmp_path):
    st = W.random_state(W.SMALL, 0)
    with pytest.raises(ValueError):
        W.write_cnw(os.path.join(tmp_path, "n.cnw"), st, W.SMALL, "e4m3")
    with pytest.raises(ValueError):
        W.act_scales(np.ones((W.SMALL.layers, 3)), W.SMALL)
    s = W.act_scales(np.zeros((W.SMALL.layers, 4)), W.SMALL)
    assert np.all(s == 1.0)       # a product input that is all zeros keeps scale 1


def test_v1_writer_matches_the_reference_exporter(tmp_path):
    """A version-1 (f16) file from this writer is byte-for-byte the reference exporter's
    (mayfly/chess/cudanet/export_cudanet.py) for the same weights: the same header fields, fingerprint
    (mcts_cpp.fingerprint) included, and every tensor's name, dtype, shape, offset, size and SHA-256, summarised
    in tests/golden/cnw_v1_seed1.json by tests/golden/make_golden.py. So the evaluator's reader of its own f16
    files is the reader of the reference's."""
    import hashlib
    import json
    import os
    from conftest import GOLDEN
    from mayfly_chess_b200 import weights as W
    with open(os.path.join(GOLDEN, "cnw_v1_seed1.json")) as f:
        ref = json.load(f)
    path = str(tmp_path / "seed1_f16.cnw")
    W.write_cnw(path, W.random_state(W.FULL, 1), W.FULL, "f16")
    hdr, arrays = W.read_cnw(path)
    assert os.path.getsize(path) == ref["file_bytes"]
    assert {k: v for k, v in hdr.items() if k not in ("tensors", "source")} == ref["header"]
    assert len(hdr["tensors"]) == len(ref["tensors"])
    for mine, theirs in zip(hdr["tensors"], ref["tensors"]):
        sha = hashlib.sha256(np.ascontiguousarray(arrays[mine["name"]]).tobytes()).hexdigest()
        assert dict(mine, sha256=sha) == theirs, mine["name"]
