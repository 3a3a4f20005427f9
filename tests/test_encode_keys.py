"""The batch encoder from transposition keys (mayfly/chess/encode.py:73-100 encode_keys).

tests/golden/keys_seed1.npz holds encode.py's own outputs (run by tests/golden/make_golden.py) for 2,048 seed-1
positions, the fixed edge-case positions and 4,096 synthetic keys. The CPU tests pin the numpy restatement
(oracle/encode_oracle.py) to it; the GPU tests hold the CUDA encoder (cudanet_encode_keys) and the key-fed
evaluator (cudanet_evaluate_keys, cudanet_begin_keys) to it, bit for bit.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

KEYS = os.path.join(GOLDEN, "keys_seed1.npz")


@pytest.fixture(scope="module")
def golden():
    z = np.load(KEYS)
    return {k: z[k] for k in z.files}


def test_oracle_matches_reference_encode_keys(golden):
    from oracle import encode_oracle as E
    ids, cast, hm, ep = E.encode_keys(golden["keys"], golden["ep_sq"], golden["clock"])
    np.testing.assert_array_equal(ids, golden["ids"])
    np.testing.assert_array_equal(cast, golden["cast"])
    np.testing.assert_array_equal(hm, golden["hm"])
    np.testing.assert_array_equal(ep, golden["ep"])


def test_fixture_covers_the_edge_cases(golden):
    keys, cast = golden["keys"], golden["cast"]
    assert (keys[:, 8] == 0).sum() > 1000                   # black to move: mirrored frames
    assert (golden["ep"] > 0).sum() > 100                    # en passant squares
    assert (golden["clock"] > 100).sum() > 100               # clocks past the cap
    assert cast.sum(0).min() > 100                           # every castling column set somewhere
    h8 = np.uint64(1) << np.uint64(63)
    assert ((keys[:, 5] & keys[:, 7] & h8) != 0).sum() > 10  # a black king on h8 (the 2K wrap-around)


def test_real_positions_match_the_position_fixture(golden):
    """The first 2,048 keys are positions_seed1.npz rows 0..2047, whose inputs came from chess_core encode."""
    from mayfly_chess_b200.inputs import PositionSet
    b = PositionSet(os.path.join(GOLDEN, "positions_seed1.npz")).batch(0, 2048)
    for k in ("ids", "cast", "hm", "ep"):
        np.testing.assert_array_equal(golden[k][:2048], b[k])


def test_keys_from_tuples():
    from mayfly_chess_b200.cudanet_py import keys_from_tuples
    t = [(1, 2, 3, 4, 5, 6, 7, 8, True, 9, None), (2**64 - 1, 0, 0, 0, 0, 0, 0, 0, False, 0, 21)]
    K, ep = keys_from_tuples(t)
    assert K.dtype == np.uint64 and K.shape == (2, 10)
    assert K[0].tolist() == [1, 2, 3, 4, 5, 6, 7, 8, 1, 9] and K[1, 0] == np.uint64(2**64 - 1)
    assert ep.tolist() == [-1, 21]


# ---------------------------------------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _dev(torch, golden, lo, hi):
    return [torch.from_numpy(np.ascontiguousarray(golden[k][lo:hi]).view(np.int64)).cuda()
            for k in ("keys", "ep_sq", "clock")]


@pytest.mark.gpu
@pytest.mark.parametrize("lo,hi", [(0, 6582), (0, 1), (5, 8), (2048, 2486), (2486, 6582), (100, 101)])
def test_gpu_encoder_matches_reference(torch_cuda, golden, lo, hi):
    from mayfly_chess_b200.cudanet_py import encode_keys_device
    hi = min(hi, golden["keys"].shape[0])
    ids, cast, hm, ep = encode_keys_device(*_dev(torch_cuda, golden, lo, hi))
    torch_cuda.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), golden["ids"][lo:hi])
    np.testing.assert_array_equal(cast.cpu().numpy(), golden["cast"][lo:hi])
    np.testing.assert_array_equal(hm.cpu().numpy(), golden["hm"][lo:hi])
    np.testing.assert_array_equal(ep.cpu().numpy(), golden["ep"][lo:hi])


@pytest.mark.gpu
def test_gpu_encoder_empty_batch_and_errors(torch_cuda):
    import ctypes
    from mayfly_chess_b200 import cudanet_py as cp
    lib = cp.load()
    err = ctypes.create_string_buffer(256)
    assert lib.cudanet_encode_keys(None, None, None, 0, None, None, None, None, None, err, 256) == 0
    assert lib.cudanet_encode_keys(None, None, None, 3, None, None, None, None, None, err, 256) == -1
    assert b"null pointer" in err.value
    assert lib.cudanet_encode_keys(None, None, None, -1, None, None, None, None, None, err, 256) == -1


@pytest.mark.gpu
def test_reference_signature(torch_cuda, golden):
    """encode_keys(keys, hms) as encode.py takes it: python-chess key tuples and clocks."""
    from mayfly_chess_b200.cudanet_py import encode_keys
    n = 300
    tuples = [tuple(bool(k[8]) if j == 8 else int(k[j]) for j in range(10)) + (None if e < 0 else int(e),)
              for k, e in zip(golden["keys"][:n], golden["ep_sq"][:n])]
    ids, cast, hm, ep = encode_keys(tuples, golden["clock"][:n].tolist())
    np.testing.assert_array_equal(ids, golden["ids"][:n])
    np.testing.assert_array_equal(cast, golden["cast"][:n])
    np.testing.assert_array_equal(hm, golden["hm"][:n])
    np.testing.assert_array_equal(ep, golden["ep"][:n])


@pytest.fixture(scope="module")
def net16(tmp_path_factory):
    """The small (config 1) net in bf16: the key path changes only how the inputs arrive."""
    from mayfly_chess_b200 import weights as W
    from mayfly_chess_b200.cudanet_py import CudaNet
    path = str(tmp_path_factory.mktemp("keys") / "small.cnw")
    W.write_cnw(path, W.random_state(W.SMALL, 0), W.SMALL, "bf16")
    net = CudaNet(path)
    yield net
    net.close()


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 7, 64, 256])
def test_evaluate_keys_equals_evaluate(torch_cuda, golden, net16, B):
    from mayfly_chess_b200.inputs import PositionSet
    b = PositionSet(os.path.join(GOLDEN, "positions_seed1.npz")).batch(0, B)
    ref = net16.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    got = net16.evaluate_keys(golden["keys"][:B], golden["ep_sq"][:B], golden["clock"][:B], b["I"], b["M"])
    for r, g in zip(ref, got):
        np.testing.assert_array_equal(r, g)


@pytest.mark.gpu
def test_begin_keys_pipeline(torch_cuda, golden, net16):
    """begin_keys and begin queued together; end returns them in order, each equal to its own evaluate."""
    from mayfly_chess_b200.inputs import PositionSet
    ps = PositionSet(os.path.join(GOLDEN, "positions_seed1.npz"))
    a, c = ps.batch(0, 96), ps.batch(96, 40)
    ra = net16.evaluate(a["ids"], a["cast"], a["hm"], a["ep"], a["I"], a["M"])
    rc = net16.evaluate(c["ids"], c["cast"], c["hm"], c["ep"], c["I"], c["M"])
    net16.begin_keys(golden["keys"][:96], golden["ep_sq"][:96], golden["clock"][:96], a["I"], a["M"])
    net16.begin(c["ids"], c["cast"], c["hm"], c["ep"], c["I"], c["M"])
    ga, gc = net16.end(), net16.end()
    for r, g in zip(ra + rc, ga + gc):
        np.testing.assert_array_equal(r, g)


@pytest.mark.gpu
def test_evaluate_keys_checks(torch_cuda, golden, net16):
    with pytest.raises(ValueError):
        net16.evaluate_keys(golden["keys"][:4], golden["ep_sq"][:3], golden["clock"][:4], np.zeros((4, 2), np.int64),
                            np.ones((4, 2), bool))
    with pytest.raises(ValueError):
        B = net16.max_batch + 1
        net16.evaluate_keys(np.zeros((B, 10), np.uint64), np.zeros(B, np.int64), np.zeros(B, np.int64),
                            np.zeros((B, 1), np.int64), np.ones((B, 1), bool))
