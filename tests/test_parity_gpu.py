"""The evaluator end to end through the C ABI (CudaNet, the reference's Python interface) against golden
outputs of the reference's own ChessNet (tests/golden, made by make_golden.py), on a B200.

Tolerances (at the legal moves), against the float32 reference model: policy logits max |diff| <= 2e-2 with
bf16 products, win probabilities sigmoid(q) and (val+1)/2 within 5e-3, and the top move agreeing on every row
without a near tie (best move ahead by more than 0.2 logits). The fp16 path (the reference backend's own
precision) is held to 5e-3 on the logits and >= 99.5% top-move agreement on all rows.

bf16 top-move agreement. Rounding the weights to bf16, which the bf16 configuration prescribes, on its own already
moves the top move of near-tie rows: the reference model itself, evaluated in float32 with its weights rounded as
the bf16 weight file stores them (golden pol_bf16w, ...), agrees with the float32 model on only 98.6% of the 146M
net's rows, and bf16 activations move rows whose two best logits are closer than the 2e-2 logit tolerance either
way. So in bf16 every "decided" row (the reference's best move ahead by more than twice the logit tolerance) must
agree, against the float32 model and against the rounded reference model (which isolates the evaluator's own
arithmetic), and the overall agreement must stay >= 98% and >= 99% against them; the overall figure is printed.
The f16 path meets the 99.5% bar outright.

Every case also checks: no non-finite value, padding exactly 0, and a second run over the same batches
bit-identical (replays of captured graphs)."""
import os

import numpy as np
import pytest

from conftest import golden_b1024, golden_case
from parity import metrics, verdict
from mayfly_chess_b200 import weights as W

pytestmark = pytest.mark.gpu

TOL = {"bf16": {"pol_max": 2e-2, "q_max": 5e-3, "val_max": 5e-3},
       "f16": {"pol_max": 5e-3, "q_max": 1e-3, "val_max": 1e-3}}
TOP1_MIN = 0.995                                   # the north star's bar (f16 path)
TOP1_BF16 = {"fp32": 0.98, "bf16w": 0.99}          # bf16 path floors (see the module docstring)


@pytest.fixture(scope="session")
def nets(tmp_path_factory):
    import torch
    from mayfly_chess_b200 import build, cudanet_py
    build.build()
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = tmp_path_factory.mktemp("cnw")
    out = {}
    states = {"small": (W.SMALL, W.random_state(W.SMALL, 0)), "full": (W.FULL, W.random_state(W.FULL, 1))}
    for tag, (arch, st) in states.items():
        for prec in ("bf16", "f16"):
            path = os.path.join(d, f"{tag}_{prec}.cnw")
            W.write_cnw(path, st, arch, prec)
            out[(tag, prec)] = cudanet_py.CudaNet(path)
    yield out
    for n in out.values():
        n.close()


def run(net, b):
    return net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])


CASES = {"small": ["small_seed0_b256", "small_seed0_fixed"], "full": ["full_seed1_b64", "full_seed1_fixed"]}


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("tag", ["small", "full"])
def test_parity_against_reference(nets, tag, prec):
    net = nets[(tag, prec)]
    assert net.precision() == prec
    hits = hits_w = hits_model = rows = 0
    for case in CASES[tag]:
        b, ref = golden_case(case)
        got = run(net, b)
        m = metrics((ref["pol"], ref["val"], ref["qv"]), got, b["widths"])
        print(case, prec, "vs fp32 model", m)
        for key, lim in TOL[prec].items():
            assert m[key] <= lim, (case, key, m[key])
        assert m["nonfinite"] == 0 and m["pad_nonzero"] == 0
        assert m["top1_clear"] == 1.0 and m["top1_decided"] == 1.0, m
        hits += m["top1_hits"]
        rows += m["rows"]
        if prec == "bf16":
            mw = metrics((ref["pol_bf16w"], ref["val_bf16w"], ref["qv_bf16w"]), got, b["widths"])
            print(case, prec, "vs bf16-weight model", mw)
            for key, lim in TOL[prec].items():
                assert mw[key] <= lim, (case, key, mw[key])
            assert mw["top1_decided"] == 1.0, mw
            hits_w += mw["top1_hits"]
            model = metrics((ref["pol"], ref["val"], ref["qv"]), (ref["pol_bf16w"], ref["val_bf16w"],
                                                                  ref["qv_bf16w"]), b["widths"])
            hits_model += model["top1_hits"]
        again = run(net, b)
        for x, y in zip(got, again):
            assert np.array_equal(x, y), "two runs of the same batch differ"
    print(f"top-1 vs fp32 model {hits}/{rows}", f"vs bf16-weight model {hits_w}/{rows}; the bf16-weight "
          f"model itself vs fp32 {hits_model}/{rows}" if prec == "bf16" else "")
    if prec == "bf16":
        assert hits / rows >= TOP1_BF16["fp32"], (hits, hits_model, rows)
        assert hits_w / rows >= TOP1_BF16["bf16w"], (hits_w, rows)
    else:
        assert hits / rows >= TOP1_MIN, (hits, rows)


def _show(name, m):
    r = m["ref_form"]
    print(f"  {name}: pol max {r['pol']['max']:.4f} mean {r['pol']['mean']:.5f} | prior max {r['prior']['max']:.5f} "
          f"mean {r['prior']['mean']:.2e} | val max {r['val']['max']:.5f} mean {r['val']['mean']:.5f} | qv max "
          f"{r['qv']['max']:.5f} mean {r['qv']['mean']:.5f} | top1 {m['top1_hits']}/{m['rows']} (clear "
          f"{m['top1_clear']:.4f} of {m['clear_rows']}, decided {m['top1_decided']:.4f} of {m['decided_rows']}) "
          f"top3 {m['top3']:.4f}")


@pytest.mark.parametrize("prec", ["bf16", "f16"])
def test_parity_config2_b1024(nets, prec):
    """BASELINE config 2 at its own batch: the bench's 1,024 positions (positions_seed1.npz rows 0..1023) in one
    call of CudaNet.evaluate, so the product shapes (66,560 rows), tile choices and the captured B = 1,024 graph are
    the ones the bench times, against the reference ChessNet's float32 outputs (full_seed1_b1024.npz). The
    reference's full metric set (mayfly/chess/cudanet/test_cudanet.py:288-340): logits, softmax prior, value, per
    move q, top move and top 3, and, as its yardstick, no worse on any max or mean than the bf16 autocast pass the
    Python search plays (the oracle restatement run that way on this GPU, mcts.py:1296-1318).

    bf16: the north star's logit / win-probability bars, every row without a near tie, every decided row, top 3
    >= 0.97 and the reference's prior bars; the overall top move >= 98% against the float32 model (the bf16-weight
    model itself only reaches about 98.6%, module docstring). f16: the reference's verdict in full (its top-move bar
    0.99) and the north star's 99.5%. Top-1 is also reported over these 1,024 rows and the 502 of the other
    146M fixtures together."""
    from oracle import chessnet_oracle as O
    net = nets[("full", prec)]
    b, ref = golden_b1024()
    assert b["I"].shape[0] == 1024
    got = run(net, b)
    m = metrics((ref["pol"], ref["val"], ref["qv"]), got, b["widths"])
    print(f"\nconfig 2, B=1024, {prec}:")
    _show("evaluator vs fp32 model", m)
    st = W.random_state(W.FULL, 1)
    ac = O.evaluate(st, W.FULL, b, device="cuda", autocast_bf16=True)
    mbf = metrics((ref["pol"], ref["val"], ref["qv"]), ac[:3], b["widths"])
    _show("bf16 autocast pass vs fp32 model", mbf)
    for key, lim in TOL[prec].items():
        assert m[key] <= lim, (key, m[key])
    # every fixture row of the 146M net: these 1,024 and the 502 of the 64-row and fixed-position cases
    hits, clear_ok, clear, rows = m["top1_hits"], m["top1_clear"] * m["clear_rows"], m["clear_rows"], m["rows"]
    for case in CASES["full"]:
        bc, rc = golden_case(case)
        mc = metrics((rc["pol"], rc["val"], rc["qv"]), run(net, bc), bc["widths"])
        hits, rows = hits + mc["top1_hits"], rows + mc["rows"]
        clear_ok, clear = clear_ok + mc["top1_clear"] * mc["clear_rows"], clear + mc["clear_rows"]
    print(f"  top-1 over all {rows} rows of the 146M fixtures: {hits}/{rows} = {hits / rows:.4f}; without near "
          f"ties {round(clear_ok)}/{clear}")
    if prec == "bf16":
        mw = metrics((ref["pol_bf16w"], ref["val_bf16w"], ref["qv_bf16w"]), got, b["widths"])
        _show("evaluator vs the bf16-weight model", mw)
        model = metrics((ref["pol"], ref["val"], ref["qv"]), (ref["pol_bf16w"], ref["val_bf16w"], ref["qv_bf16w"]),
                        b["widths"])
        _show("the bf16-weight model itself vs fp32", model)
        assert mw["top1_decided"] == 1.0 and mw["top1"] >= TOP1_BF16["bf16w"], mw
        bad = verdict(m, mbf, top1_min=TOP1_BF16["fp32"])
    else:
        bad = verdict(m, None)
        assert hits / rows >= TOP1_MIN, (hits, rows)
    assert m["top1_decided"] == 1.0, m
    assert not bad, bad
    again = run(net, b)
    for x, y in zip(got, again):
        assert np.array_equal(x, y), "two runs of the same batch differ"


def test_full_logits(nets):
    """The raw heads of the first rows against the reference's full policy and qvalue logits."""
    net = nets[("full", "bf16")]
    b, ref = golden_case("full_seed1_b64")
    pol, val, qv, logits = net.evaluate_logits(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    n = ref["policy_rows"].shape[0]
    assert np.abs(logits[:n, :4162] - ref["policy_rows"]).max() <= 2e-2
    q = 1 / (1 + np.exp(-logits[:n, 4162:].astype(np.float64)))
    qr = 1 / (1 + np.exp(-ref["qvalue_rows"].astype(np.float64)))
    assert np.abs(q - qr).max() <= 5e-3
    p2, v2, q2 = run(net, b)
    assert np.array_equal(pol, p2) and np.array_equal(val, v2) and np.array_equal(qv, q2)


@pytest.mark.parametrize("B", [1, 3, 47, 64, 129])
def test_batch_sizes_and_slices(nets, B):
    """Odd batch sizes (M tails, one board) give each row the same numbers as the row had in a bigger batch
    (rows are independent), within the rounding of the pass."""
    net = nets[("full", "bf16")]
    from mayfly_chess_b200.inputs import PositionSet
    from conftest import GOLDEN
    ps = PositionSet(os.path.join(GOLDEN, "positions_seed1.npz"))
    big = ps.batch(0, 256)
    pb, vb, qb = run(net, big)
    small = ps.batch(0, B)
    ps_, vs, qs = run(net, small)
    w = small["I"].shape[1]
    assert np.abs(ps_ - pb[:B, :w]).max() < 1e-4
    assert np.abs(vs - vb[:B]).max() < 1e-4


def test_row_order_does_not_change_outputs(nets, tmp_path, monkeypatch):
    """Every other kernel of a layer's chain walks its rows (LayerNorm rows, the products' M blocks, the attention's
    boards) in descending order, to start on what the kernel before it left in L2. A handle made with
    MAYFLY_CUDANET_ORDER=fwd walks them all forward; both give the same bits (438 boards: 28,470 rows, many M
    blocks of every product)."""
    from mayfly_chess_b200 import cudanet_py
    b, _ = golden_case("full_seed1_fixed")
    want = run(nets[("full", "bf16")], b)
    path = str(tmp_path / "full_bf16.cnw")
    W.write_cnw(path, W.random_state(W.FULL, 1), W.FULL, "bf16")
    monkeypatch.setenv("MAYFLY_CUDANET_ORDER", "fwd")
    fwd = cudanet_py.CudaNet(path)
    try:
        got = run(fwd, b)
    finally:
        fwd.close()
    for x, y in zip(want, got):
        assert np.array_equal(x, y)


def test_begin_end_pipeline(nets):
    net = nets[("full", "bf16")]
    b1, _ = golden_case("full_seed1_b64")
    b2, _ = golden_case("full_seed1_fixed")
    want1, want2 = run(net, b1), run(net, b2)
    net.begin(b1["ids"], b1["cast"], b1["hm"], b1["ep"], b1["I"], b1["M"])
    net.begin(b2["ids"], b2["cast"], b2["hm"], b2["ep"], b2["I"], b2["M"])
    with pytest.raises(RuntimeError):
        net.begin(b1["ids"], b1["cast"], b1["hm"], b1["ep"], b1["I"], b1["M"])   # a third is refused
    got1 = net.end()
    got2 = net.end()
    for x, y in zip(want1 + want2, got1 + got2):
        assert np.array_equal(x, y)
    with pytest.raises(RuntimeError):
        net.end()


def test_evaluate_device_matches_host(nets):
    import torch
    net = nets[("full", "bf16")]
    b, _ = golden_case("full_seed1_b64")
    want = run(net, b)
    t = {k: torch.from_numpy(np.ascontiguousarray(b[k])).cuda() for k in ("ids", "cast", "hm", "ep", "I")}
    M = torch.from_numpy(b["M"].astype(np.uint8)).cuda()
    B, wide = b["I"].shape
    pol = torch.empty(B, wide, device="cuda")
    val = torch.empty(B, device="cuda")
    qv = torch.empty(B, wide, device="cuda")
    net.evaluate_device(t["ids"], t["cast"], t["hm"], t["ep"], t["I"], M, pol, val, qv)
    net.check(torch.cuda.current_stream())
    for x, y in zip(want, (pol.cpu().numpy(), val.cpu().numpy(), qv.cpu().numpy())):
        assert np.array_equal(x, y)


def test_errors_come_back_as_exceptions(nets):
    net = nets[("small", "bf16")]
    b, _ = golden_case("small_seed0_b256")
    with pytest.raises(ValueError):
        net.evaluate(b["ids"][:, :63], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    with pytest.raises(ValueError):
        net.evaluate(b["ids"][:0], b["cast"][:0], b["hm"][:0], b["ep"][:0], b["I"][:0], b["M"][:0])
    wide = np.zeros((1, 257), np.int64)
    with pytest.raises(RuntimeError, match="wide"):
        net.evaluate(b["ids"][:1], b["cast"][:1], b["hm"][:1], b["ep"][:1], wide, wide.astype(bool))
    # the handle still works afterwards
    run(net, b)


def test_bad_indices_are_clamped(nets):
    """Out-of-range piece ids, clocks and policy indices read inside their tables (kernels clamp them)."""
    net = nets[("small", "bf16")]
    b, _ = golden_case("small_seed0_b256")
    ids = b["ids"][:4].copy()
    ids[:, 0] = 99
    hm = np.array([-5, 500, 101, 0], np.int64)
    I = b["I"][:4].copy()
    I[:, 0] = 100000
    pol, val, qv = net.evaluate(ids, b["cast"][:4], hm, b["ep"][:4], I, b["M"][:4])
    assert np.isfinite(pol).all() and np.isfinite(val).all() and np.isfinite(qv).all()


def test_fingerprint_and_profile(nets, meta):
    net = nets[("full", "bf16")]
    assert net.fingerprint() == meta["fingerprint_full_seed1"]
    prof = net.profile(64, reps=2)
    assert list(prof)[-1] == "graph_pass" and all(v >= 0 for v in prof.values())
    assert prof["graph_pass"] > 0


def test_bad_weight_file(tmp_path):
    from mayfly_chess_b200 import cudanet_py
    p = tmp_path / "bad.cnw"
    p.write_bytes(b"MFCNW001" + b"\x02\x00\x00\x00{}")
    with pytest.raises(RuntimeError, match="cudanet_create"):
        cudanet_py.CudaNet(str(p))
