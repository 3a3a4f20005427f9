"""MCTS._dispatch / MCTS._collect (mayfly/chess/mcts.py:1074-1421) on the B200 evaluator.

The Python search sends each leaf batch through _dispatch (queue the forward pass without waiting) and reads it
back with _collect (wait, then hand the search the policy at each node's legal moves, the leaf values and every
child's q). install(tree, net) replaces those two methods on one MCTS instance with calls to this evaluator:

    _dispatch(prep)  net.begin(ids, cast, hm, ep, I, M) from _prepare's batch (mcts.py:1004-1058): the inputs are
                     copied into pinned staging and the pass is queued; nothing waits. Two batches may be in
                     flight (the search's pipeline, mcts.py:2883-2886).
    _collect(h)      net.end(): the oldest batch's (pol, val, qv), returned in the shape the sw25_one_copy path
                     returns them (mcts.py:1388-1404): one _Cut per node holding its legal-move logits, val as a
                     float32 array, one float32 q array per node, and the same counters.

The evaluator computes what _dispatch's value_from_q tail computes (softmax of the policy at the legal moves,
weights on sigmoid(q), val = 2 sum - 1, qv = 2 q - 1), so it covers the search's default configuration:
value_from_q on, castle_prior "king" (the policy gathered at I), no opponent adapter and no moves-left head.
Anything else raises ValueError at dispatch rather than silently computing something else.
"""
import sys
import time

import numpy as np


def install(tree, net, cut=None):
    """Route `tree`'s network calls to `net` (a mayfly_chess_b200.cudanet_py.CudaNet). `cut` is mcts.py's _Cut
    class, found in the tree's own module when not given."""
    if cut is None:
        cut = getattr(sys.modules.get(type(tree).__module__), "_Cut", None)
        if cut is None:
            raise ValueError("the tree's module has no _Cut class; pass cut=")
    if not getattr(tree, "value_from_q", True):
        raise ValueError("the evaluator computes the value from q (value_from_q); this tree reads a value head")

    def _dispatch(prep):
        if "theirs" in prep:
            raise ValueError("the opponent adapter needs the hidden state, which this evaluator does not return")
        if prep.get("Ip") is not None and prep.get("Ip") is not prep["I"]:
            raise ValueError("castle_prior other than 'king' gathers the policy at other indices than q")
        if getattr(tree, "mlh", False):
            raise ValueError("the moves-left head is not part of this evaluator")
        t0 = time.perf_counter() if getattr(tree, "timing_fixes", False) else None
        net.begin(prep["ids"], prep["cast"], prep["hm"], prep["ep"], prep["I"], prep["M"])
        if t0 is not None:
            tree.stats["pass_s"] = tree.stats.get("pass_s", 0.0) + (time.perf_counter() - t0)
        return {"nodes": prep["nodes"], "b200": True, "widths": list(prep["widths"]), "ml": None}

    def _collect(h):
        nodes, widths = h["nodes"], h["widths"]
        t0 = time.perf_counter() if getattr(tree, "timing_fixes", False) else None
        pol, val, qv = net.end()
        if t0 is not None:
            tree.stats["wait_s"] = tree.stats.get("wait_s", 0.0) + (time.perf_counter() - t0)
        n = len(nodes)
        cuts = [cut(np.array(pol[i, :widths[i]], dtype=np.float32)) for i in range(n)]
        qs = [np.array(qv[i, :widths[i]], dtype=np.float32) for i in range(n)]
        tree._ml = None
        tree.stats["evals"] = tree.stats.get("evals", 0) + n
        tree.stats["batches"] = tree.stats.get("batches", 0) + 1
        return cuts, np.array(val, dtype=np.float32), qs

    tree._dispatch = _dispatch
    tree._collect = _collect
    return tree
