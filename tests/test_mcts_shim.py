"""The Python search's _dispatch/_collect on this evaluator (mayfly_chess_b200.mcts_shim, mcts.py:1074-1421).

mcts.py itself needs python-chess, which is not installed, so the tree here is a stand-in with the attributes
the two methods read (stats, value_from_q, timing_fixes, _ml) and the batches are _prepare-shaped dicts built
from the position fixtures. The CPU tests cover the host logic with a fake evaluator; the GPU tests run the real
one against the oracle and against CudaNet.evaluate, with two batches in flight as the search's pipeline keeps
them.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN


class Cut:
    """mcts.py:375-382 _Cut: a policy row already cut to one node's legal moves."""
    __slots__ = ("row",)

    def __init__(self, row):
        self.row = row


class Tree:
    def __init__(self, **kw):
        self.stats = {"evals": 0, "batches": 0}
        self.value_from_q = True
        self.timing_fixes = True
        self.mlh = False
        self._ml = "unset"
        self.__dict__.update(kw)


def prep_of(b):
    widths = b["M"].sum(1).astype(np.int64)
    return {"nodes": list(range(len(widths))), "ids": b["ids"], "cast": b["cast"], "hm": b["hm"], "ep": b["ep"],
            "I": b["I"], "Ip": b["I"], "M": b["M"], "widths": widths}


class FakeNet:
    def __init__(self):
        self.fly = []

    def begin(self, ids, cast, hm, ep, I, M):
        B, W = np.asarray(I).shape
        self.fly.append((B, W))

    def end(self):
        B, W = self.fly.pop(0)
        pol = np.arange(B * W, dtype=np.float32).reshape(B, W)
        return pol, np.full(B, 0.25, np.float32), -pol


def test_shim_host_logic():
    from mayfly_chess_b200 import mcts_shim
    from mayfly_chess_b200.inputs import PositionSet
    b = PositionSet(os.path.join(GOLDEN, "small_seed0_b256.npz")).batch(0, 5)
    t = mcts_shim.install(Tree(), FakeNet(), cut=Cut)
    p = prep_of(b)
    h1, h2 = t._dispatch(p), t._dispatch(p)
    pol, val, qv = t._collect(h1)
    t._collect(h2)
    W = b["I"].shape[1]
    assert len(pol) == 5 and all(isinstance(c, Cut) and c.row.dtype == np.float32 for c in pol)
    for i, w in enumerate(p["widths"]):
        np.testing.assert_array_equal(pol[i].row, np.arange(i * W, i * W + w, dtype=np.float32))
        np.testing.assert_array_equal(qv[i], -pol[i].row)
    assert val.dtype == np.float32 and (val == 0.25).all()
    assert t.stats["evals"] == 10 and t.stats["batches"] == 2 and t._ml is None
    assert t.stats["pass_s"] >= 0 and t.stats["wait_s"] >= 0


def test_shim_refuses_what_the_evaluator_does_not_compute():
    from mayfly_chess_b200 import mcts_shim
    from mayfly_chess_b200.inputs import PositionSet
    b = PositionSet(os.path.join(GOLDEN, "small_seed0_b256.npz")).batch(0, 2)
    with pytest.raises(ValueError):
        mcts_shim.install(Tree(value_from_q=False), FakeNet(), cut=Cut)
    t = mcts_shim.install(Tree(), FakeNet(), cut=Cut)
    p = prep_of(b)
    with pytest.raises(ValueError):
        t._dispatch(dict(p, theirs=[0.0, 1.0]))
    with pytest.raises(ValueError):
        t._dispatch(dict(p, Ip=np.zeros_like(p["I"])))
    with pytest.raises(ValueError):
        mcts_shim.install(Tree(mlh=True), FakeNet(), cut=Cut)._dispatch(p)
    with pytest.raises(ValueError):
        mcts_shim.install(Tree(), FakeNet())        # no _Cut in this module


@pytest.mark.gpu
def test_shim_on_the_evaluator(tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mayfly_chess_b200 import mcts_shim
    from mayfly_chess_b200 import weights as W
    from mayfly_chess_b200.cudanet_py import CudaNet
    from mayfly_chess_b200.inputs import PositionSet
    from oracle import chessnet_oracle as O
    st = W.random_state(W.SMALL, 0)
    path = str(tmp_path / "small_bf16.cnw")
    W.write_cnw(path, st, W.SMALL, "bf16")
    ps = PositionSet(os.path.join(GOLDEN, "small_seed0_b256.npz"))
    a, c = ps.batch(0, 48), ps.batch(48, 17)
    with CudaNet(path) as net:
        direct = [net.evaluate(x["ids"], x["cast"], x["hm"], x["ep"], x["I"], x["M"]) for x in (a, c)]
        t = mcts_shim.install(Tree(), net, cut=Cut)
        ha, hc = t._dispatch(prep_of(a)), t._dispatch(prep_of(c))       # two in flight, as the pipeline keeps
        got = [t._collect(ha), t._collect(hc)]
    for x, (pol, val, qv), (dp, dv, dq) in zip((a, c), got, direct):
        widths = x["M"].sum(1)
        np.testing.assert_array_equal(val, dv)
        rp, rv, rq, _, _ = O.evaluate(st, W.SMALL, x)
        for i, w in enumerate(widths):
            np.testing.assert_array_equal(pol[i].row, dp[i, :w])
            np.testing.assert_array_equal(qv[i], dq[i, :w])
            assert np.abs(pol[i].row - rp[i, :w]).max() <= 2e-2
            assert np.abs(qv[i] - rq[i, :w]).max() / 2 <= 5e-3
        assert np.abs(val - rv).max() / 2 <= 5e-3
    assert t.stats["evals"] == 65 and t.stats["batches"] == 2
