"""The CPU oracle (oracle/chessnet_oracle.py) against golden vectors the reference's own ChessNet produced
(tests/golden/make_golden.py), and the fixtures' inputs against the reference's chess core."""
import numpy as np
import pytest

from conftest import golden_case
from mayfly_chess_b200 import weights as W
from oracle import chessnet_oracle as O

# the oracle restates the same fp32 arithmetic in a different order (SDPA vs explicit softmax, etc.)
TOL_LOGIT = 2e-5
TOL_PROB = 2e-6


@pytest.mark.parametrize("case,arch,seed", [("small_seed0_b256", W.SMALL, 0), ("small_seed0_fixed", W.SMALL, 0),
                                            ("full_seed1_b64", W.FULL, 1)])
def test_oracle_matches_reference(case, arch, seed):
    b, ref = golden_case(case)
    st = W.random_state(arch, seed)
    pol, val, qv, P, Q = O.evaluate(st, arch, b)
    assert np.abs(pol - ref["pol"]).max() < TOL_LOGIT
    assert np.abs(val - ref["val"]).max() < TOL_PROB
    assert np.abs(qv - ref["qv"]).max() < TOL_PROB
    assert np.abs(P[:4] - ref["policy_rows"]).max() < TOL_LOGIT
    assert np.abs(Q[:4] - ref["qvalue_rows"]).max() < TOL_LOGIT
    # the reference's padding convention
    for i, w in enumerate(b["widths"]):
        assert (pol[i, w:] == 0).all() and (qv[i, w:] == 0).all()


def test_b1024_fixture_agrees_with_b64():
    """The config-2 fixture (1,024 rows, reference forward in chunks of 256) gives its first 64 rows what the
    64-row fixture gives them (the reference's float32 CPU arithmetic, batched differently), and the oracle gives
    a slice of it within the oracle's bars."""
    from conftest import golden_b1024
    b, ref = golden_b1024()
    b64, r64 = golden_case("full_seed1_b64")
    w = b64["I"].shape[1]
    for k in ("pol", "qv", "pol_bf16w", "qv_bf16w", "pol_e4m3w", "qv_e4m3w"):
        assert np.abs(ref[k][:64, :w] - r64[k]).max() < TOL_LOGIT, k
    for k in ("val", "val_bf16w", "val_e4m3w"):
        assert np.abs(ref[k][:64] - r64[k]).max() < TOL_PROB, k
    st = W.random_state(W.FULL, 1)
    sl = {k: v[960:976] for k, v in b.items()}
    sl["I"], sl["M"] = sl["I"][:, :int(sl["widths"].max())], sl["M"][:, :int(sl["widths"].max())]
    pol, val, qv, _, _ = O.evaluate(st, W.FULL, sl)
    w = sl["I"].shape[1]
    assert np.abs(pol - ref["pol"][960:976, :w]).max() < TOL_LOGIT
    assert np.abs(val - ref["val"][960:976]).max() < TOL_PROB
    assert np.abs(qv - ref["qv"][960:976, :w]).max() < TOL_PROB


def test_post_no_legal_move_gives_minus_one():
    pol = np.zeros((1, 4162), np.float32)
    import torch
    p, v, q = O.post(torch.from_numpy(pol), torch.from_numpy(pol), np.zeros((1, 3), np.int64),
                     np.zeros((1, 3), bool))
    assert v[0] == -1.0 and (p == 0).all() and (q == 0).all()


def test_fixed_positions_cover_edge_cases():
    b, _ = golden_case("small_seed0_fixed")
    w = b["widths"]
    assert w.max() == 218            # the most legal moves known
    assert (w == 1).sum() >= 2       # positions with a single legal move
    assert (b["hm"] == 100).any()    # clocks past 100 are capped
    assert (b["ep"] > 0).any()       # a legal en passant capture
    promo = b["I"][b["M"]]
    assert (promo >= 4096).any()     # underpromotions


def test_fixture_inputs_match_chess_core(chesscore):
    """The committed seed-1 position set is what the reference's chess core gives for the seeded playouts."""
    from mayfly_chess_b200.inputs import PositionSet
    import os
    from conftest import GOLDEN
    ps = PositionSet(os.path.join(GOLDEN, "positions_seed1.npz"))
    got = chesscore.encode_batch(chesscore.random_playouts(48, seed=1, max_plies=120))
    want = ps.batch(0, 48)
    for k in ("ids", "cast", "hm", "ep", "widths"):
        np.testing.assert_array_equal(got[k], want[k])
    np.testing.assert_array_equal(got["I"][got["M"]], want["I"][want["M"]])


def test_chess_core_known_answers(chesscore):
    """Known facts of standard chess through the reference's chess core: 20 moves from the start, the
    218-move position, a pinned en passant that must not be encoded."""
    P = chesscore
    start = P.Position()
    codes, idx = start.legal()
    assert len(codes) == 20
    ids, cast, hm, ep = start.encode()
    assert list(ids[:8]) == [4, 2, 3, 5, 6, 3, 2, 4] and list(ids[56:64]) == [10, 8, 9, 11, 12, 9, 8, 10]
    assert list(cast) == [1, 1, 1, 1] and hm == 0 and ep == 0
    assert len(P.Position("R6R/3Q4/1Q4Q1/4Q3/2Q4Q/Q4Q2/pp1Q4/kBNN1KB1 w - - 0 1").legal()[0]) == 218
    assert P.Position("8/8/8/K2pP2r/8/8/8/7k w - d6 0 1").encode()[3] == 0
    # a legal en passant capture, square d6 + 1 in white's frame
    assert P.Position("rnbqkbnr/ppp1p1pp/8/3pPp2/8/8/PPPP1PPP/RNBQKBNR w KQkq f6 0 3").encode()[3] == 45 + 1
