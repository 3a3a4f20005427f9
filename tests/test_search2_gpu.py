"""The reference's own C++ search (mayfly/chess/cpp/search2.cpp, built from its sources into
oracle/_ref/libsearch2_b200.so by oracle/Makefile) running on this evaluator through the product adapter
mayfly_chess_b200/adapters/cudanet_backend_b200.h (mayfly2::Net over the C ABI, search2.h:55-88).

What is checked:
  * the searches run to their visit targets and pick a legal root move;
  * every batch the reference's search encoded, evaluated through the adapter, matches the CPU oracle on the same
    inputs within the bf16 bars (the search's own encoding, I/M layout and the Out layout are what the adapter
    hands over);
  * repeatability: the same search twice gives the same tree, bit for bit;
  * the pipeline (Settings::pipeline 1, two batches in flight through cudanet_begin/cudanet_end) gives the same
    tree as mayfly2::Net's default submit/collect, which search2.h:72-75 defines as evaluating on collect.
"""
import ctypes
import os

import numpy as np
import pytest

from conftest import REPO

LIB = os.path.join(REPO, "oracle", "_ref", "libsearch2_b200.so")
FENS = [
    "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1",
    "r1bqkb1r/pppp1ppp/2n2n2/4p3/2B1P3/5N2/PPPP1PPP/RNBQK2R w KQkq - 4 4",
    "rnbqkbnr/ppp1p1pp/8/3pPp2/8/8/PPPP1PPP/RNBQKBNR w KQkq f6 0 3",
    "8/8/3k4/8/3K4/8/4P3/8 b - - 31 70",
]


@pytest.fixture(scope="module")
def s2():
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libsearch2_b200.so not built (needs the reference checkout: make -C oracle)")
    L = ctypes.CDLL(LIB)
    vp, i32, cp = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
    L.s2_open.argtypes = [cp, i32, i32, cp, i32]
    L.s2_open.restype = vp
    L.s2_close.argtypes = [vp]
    L.s2_record.argtypes = [vp, i32]
    L.s2_recorded.argtypes = [vp]
    L.s2_recorded.restype = i32
    L.s2_get.argtypes = [vp, i32, ctypes.POINTER(i32), ctypes.POINTER(i32)] + [vp] * 9
    L.s2_get.restype = i32
    L.s2_search.argtypes = [vp, cp, i32, i32, ctypes.c_double, vp, vp, i32, ctypes.POINTER(i32), vp, cp, i32]
    L.s2_search.restype = i32
    L.s2_backend.argtypes = [vp, i32, i32] + [vp] * 10 + [cp, i32]
    L.s2_backend.restype = i32
    return L


@pytest.fixture(scope="module")
def small_net(tmp_path_factory):
    from mayfly_chess_b200 import weights as W
    st = W.random_state(W.SMALL, 0)
    path = str(tmp_path_factory.mktemp("s2") / "small_bf16.cnw")
    W.write_cnw(path, st, W.SMALL, "bf16")
    return path, st


class Search:
    def __init__(self, L, path, mode):
        self.L = L
        err = ctypes.create_string_buffer(1024)
        self.h = L.s2_open(path.encode(), 0, mode, err, 1024)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def run(self, fen, batch=48, pipeline=0, target=400):
        moves = np.zeros(256, np.int32)
        N = np.zeros(256, np.float32)
        chosen = ctypes.c_int(-2)
        stats = np.zeros(8, np.int64)
        err = ctypes.create_string_buffer(1024)
        n = self.L.s2_search(self.h, fen.encode(), batch, pipeline, float(target), moves.ctypes.data,
                             N.ctypes.data, 256, ctypes.byref(chosen), stats.ctypes.data, err, 1024)
        if n < 0:
            raise RuntimeError(err.value.decode())
        return moves[:n].copy(), N[:n].copy(), chosen.value, stats

    def batches(self):
        out = []
        for i in range(self.L.s2_recorded(self.h)):
            B, w = ctypes.c_int(0), ctypes.c_int(0)
            self.L.s2_get(self.h, i, ctypes.byref(B), ctypes.byref(w), *([None] * 9))
            B, w = B.value, w.value
            a = dict(ids=np.zeros((B, 64), np.int64), cast=np.zeros((B, 4), np.float32), hm=np.zeros(B, np.int64),
                     ep=np.zeros(B, np.int64), I=np.zeros((B, w), np.int64), M=np.zeros((B, w), np.uint8),
                     pol=np.zeros((B, w), np.float32), val=np.zeros(B, np.float32), qv=np.zeros((B, w), np.float32))
            assert self.L.s2_get(self.h, i, ctypes.byref(ctypes.c_int()), ctypes.byref(ctypes.c_int()),
                                 *[a[k].ctypes.data for k in ("ids", "cast", "hm", "ep", "I", "M", "pol", "val",
                                                              "qv")]) == 0
            out.append(a)
        return out

    def close(self):
        self.L.s2_close(self.h)


@pytest.mark.gpu
def test_search_runs_on_the_evaluator(s2, small_net):
    path, _ = small_net
    s = Search(s2, path, 0)
    try:
        for fen in FENS:
            moves, N, chosen, stats = s.run(fen, target=300)
            assert len(moves) > 0 and 0 <= chosen < len(moves)
            assert N.sum() > 0 and stats[4] > 1               # visits below the root, a tree grown
            assert stats[0] > 0 and stats[1] > 0          # evaluations went through the adapter
    finally:
        s.close()


@pytest.mark.gpu
def test_search_batches_match_the_oracle(s2, small_net):
    from oracle import chessnet_oracle as O
    path, st = small_net
    from mayfly_chess_b200 import weights as W
    s = Search(s2, path, 0)
    try:
        s2.s2_record(s.h, 1)
        s.run(FENS[1], batch=64, target=500)
        recs = s.batches()
    finally:
        s.close()
    assert len(recs) >= 3
    worst = 0.0
    for r in recs[:6]:
        b = {k: r[k] for k in ("ids", "cast", "hm", "ep", "I")}
        b["M"] = r["M"].astype(bool)
        rp, rv, rq, _, _ = O.evaluate(st, W.SMALL, b)
        m = b["M"]
        worst = max(worst, float(np.abs(r["pol"] - rp)[m].max()))
        assert float(np.abs(r["qv"] - rq)[m].max()) / 2 <= 5e-3
        assert float(np.abs(r["val"] - rv).max()) / 2 <= 5e-3
        assert (r["pol"][~m] == 0).all() and (r["qv"][~m] == 0).all()
    assert worst <= 2e-2, worst


@pytest.mark.gpu
@pytest.mark.parametrize("pipeline", [0, 1])
def test_search_is_repeatable(s2, small_net, pipeline):
    path, _ = small_net
    s = Search(s2, path, 0)
    try:
        a = s.run(FENS[0], pipeline=pipeline, target=600)
        b = s.run(FENS[0], pipeline=pipeline, target=600)
    finally:
        s.close()
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert a[2] == b[2]


@pytest.mark.gpu
def test_pipeline_through_begin_end_equals_default_pipeline(s2, small_net):
    path, _ = small_net
    mine, dflt = Search(s2, path, 0), Search(s2, path, 1)
    try:
        for fen in FENS[:3]:
            a = mine.run(fen, pipeline=1, target=500)
            b = dflt.run(fen, pipeline=1, target=500)
            np.testing.assert_array_equal(a[0], b[0])
            np.testing.assert_array_equal(a[1], b[1])
            assert a[2] == b[2]
            np.testing.assert_array_equal(a[3][:5], b[3][:5])   # the counters (the rest are timings)
    finally:
        mine.close()
        dflt.close()


@pytest.mark.gpu
@pytest.mark.parametrize("batch,pipeline", [(48, 0), (256, 1)])
def test_search_throughput_146m(s2, tmp_path_factory, batch, pipeline):
    """The reference's search on the 146M bf16 net: evaluations a second and the network's share of the steps
    (Settings::prof), printed for the record."""
    from mayfly_chess_b200 import weights as W
    path = str(tmp_path_factory.mktemp("s2full") / "full_bf16.cnw")
    W.write_cnw(path, W.random_state(W.FULL, 1), W.FULL, "bf16")
    s = Search(s2, path, 0)
    try:
        s.run(FENS[1], batch=batch, pipeline=pipeline, target=2000)       # warm-up: graphs for the batch sizes
        moves, N, chosen, st = s.run(FENS[1], batch=batch, pipeline=pipeline, target=20000)
    finally:
        s.close()
    step_s, net_s, enc_s = st[5] / 1e6, st[6] / 1e6, st[7] / 1e6
    print(f"\nsearch2 on the 146M bf16 net, batch {batch}, pipeline {pipeline}: {st[0]} evaluations in {st[1]} "
          f"batches, {st[0] / step_s:.0f} evaluations/s over {step_s:.2f} s of steps; network {100 * net_s / step_s:.0f}%"
          f", encoding {100 * enc_s / step_s:.0f}% of it; {N.sum():.0f} root visits, {st[4]} tree nodes")
    assert 0 <= chosen < len(moves) and st[0] > 1000


@pytest.mark.gpu
def test_netbackend_full_rows(s2, small_net):
    """mayfly::NetBackend (make_cuda_backend): the cut policy scattered into full 4,162-wide rows, 0 elsewhere,
    val and qv as mayfly2::Net gives them."""
    from mayfly_chess_b200.cudanet_py import CudaNet
    from mayfly_chess_b200.inputs import PositionSet
    from conftest import GOLDEN
    path, _ = small_net
    b = PositionSet(os.path.join(GOLDEN, "small_seed0_b256.npz")).batch(0, 40)
    B, wide = b["I"].shape
    widths = b["M"].sum(1).astype(np.int32)
    policy = np.full((B, 4162), np.nan, np.float32)
    val = np.zeros(B, np.float32)
    qv = np.zeros((B, wide), np.float32)
    M = b["M"].astype(np.uint8)
    s = Search(s2, path, 0)
    try:
        err = ctypes.create_string_buffer(1024)
        rc = s2.s2_backend(s.h, B, wide, *[np.ascontiguousarray(a).ctypes.data for a in
                                           (b["ids"], b["cast"], b["hm"], b["ep"], b["I"], M, widths, policy, val,
                                            qv)], err, 1024)
        assert rc == 0, err.value
    finally:
        s.close()
    with CudaNet(path) as net:
        pol, v, q = net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    np.testing.assert_array_equal(val, v)
    np.testing.assert_array_equal(qv, q)
    expect = np.zeros((B, 4162), np.float32)
    for r in range(B):
        expect[r, b["I"][r, :widths[r]]] = pol[r, :widths[r]]
    np.testing.assert_array_equal(policy, expect)


@pytest.mark.gpu
def test_adapter_reports_errors(s2, tmp_path):
    err = ctypes.create_string_buffer(1024)
    h = s2.s2_open(str(tmp_path / "missing.cnw").encode(), 0, 0, err, 1024)
    assert not h
    assert b"cudanet_create" in err.value
