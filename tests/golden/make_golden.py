"""Generates the committed golden fixtures from the REFERENCE itself, in a container that has the reference
checkout (it is not needed, and not present, where the tests and the bench run).

    python tests/golden/make_golden.py --ref <reference checkout>     (or MAYFLY_REFERENCE=<checkout> in the env)

What it does:
  1. Builds the reference's own C++ chess core (make -C oracle) and uses it, through oracle/positions.py, for
     every position: seeded random playouts (numpy PCG64; seed 0 with 0..80 plies for the CPU correctness
     config, seed 1 with 0..120 plies for the 146M configs) and the reference's fixed edge-case positions, read
     as text from mayfly/chess/cudanet/test_cudanet.py (FIXED, :68-103) and mayfly/chess/cpp/positions.json.
     python-chess is not installed, so the SAN lines of test_cudanet.py (:106-118) are not used.
  2. Imports the reference's ChessNet (mayfly/chess/chess_net.py) and export_ts (Export, post) with a stub
     `chess` module of constants (the forward never calls python-chess), loads the seeded random-init state
     (mayfly_chess_b200.weights.random_state) with load_state_dict(strict=True), which pins the state dict's
     names and shapes, and runs the reference in float32 on the CPU with the MHA fast path off, as
     cudanet/test_cudanet.py:177-194 reference() does.
  3. Writes, per case, the inputs and the reference outputs at the legal moves (pol with 0 on padding, val, qv
     with 0 on padding) plus the full logits of a few rows, and the 8,192-position seed-1 set the bench uses.
     Each case also holds the outputs of the same reference model with its weight matrices rounded as a bf16
     or an e4m3 weight file stores them (pol_bf16w, pol_e4m3w, ...), which separates what the prescribed weight
     rounding costs from what the evaluator's own arithmetic costs.

Fixtures (all small .npz):
  positions_seed1.npz         8,192 seed-1 positions, compact (mayfly_chess_b200/inputs.py PositionSet)
  small_seed0_b256.npz        config 1: d 256, 4 layers, 8 heads, FFN 1024, seed-0 weights, 256 seed-0 positions
  small_seed0_fixed.npz       the same net on the reference's fixed edge-case positions
  full_seed1_b64.npz          the 146M net (d 1024, 16 layers, 16 heads, FFN 2048), seed-1 weights, the first 64
                              seed-1 positions
  full_seed1_fixed.npz        the 146M net on the fixed edge-case positions
  keys_seed1.npz              the batch encoder from transposition keys (encode.py:73-100 encode_keys, run
                              itself): the first 2,048 seed-1 positions, the fixed positions and 4,096 seeded
                              synthetic keys (random bitboards, kings on the corners, castling bits, black to
                              move, clocks past 100), with encode_keys' ids, cast, hm and ep for each; the real
                              positions are also checked against chess_core.cpp:582-612 encode
  cnw_v1_seed1.json           what the reference's own exporter (mayfly/chess/cudanet/export_cudanet.py, run on a
                              checkpoint of the seed-1 146M random-init state) writes: its header fields (the
                              fingerprint mcts_cpp.fingerprint computes) and every tensor's name, dtype, shape,
                              offset, size and SHA-256; the file itself (290 MB) is not kept
  meta.json                   fingerprints, state dict names and shapes, how each case was made

  full_seed1_b1024.npz        the 146M net on the first 1,024 seed-1 positions (positions_seed1.npz rows
                              0..1023, the bench's own batch): the reference outputs at the legal moves only,
                              flattened row after row (pol, qv; val per row), with the bf16w and e4m3w controls

    python tests/golden/make_golden.py --only keys     regenerates keys_seed1.npz alone (seconds)
    python tests/golden/make_golden.py --only cnw      regenerates cnw_v1_seed1.json alone (a minute)
    python tests/golden/make_golden.py --only b1024    regenerates full_seed1_b1024.npz alone (a few minutes)
"""
import argparse
import ast
import json
import os
import subprocess
import sys
import time
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from mayfly_chess_b200 import weights as W   # noqa: E402
from mayfly_chess_b200.inputs import pack    # noqa: E402


def chess_stub():
    """The constants chess_net.py, moves.py and encode.py read at import (python-chess values)."""
    m = types.ModuleType("chess")
    m.PAWN, m.KNIGHT, m.BISHOP, m.ROOK, m.QUEEN, m.KING = 1, 2, 3, 4, 5, 6
    m.WHITE, m.BLACK = True, False
    m.square_mirror = lambda sq: sq ^ 0x38
    m.square_rank = lambda sq: sq >> 3
    m.STARTING_FEN = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"
    return m


def import_reference(ref):
    chess_dir = os.path.join(ref, "mayfly", "chess")
    sys.modules.setdefault("chess", chess_stub())
    for d in (chess_dir, os.path.join(chess_dir, "cpp")):
        if d not in sys.path:
            sys.path.insert(0, d)
    import chess_net   # noqa: E402
    import export_ts   # noqa: E402
    return chess_net, export_ts


def fixed_fens(ref):
    """FIXED from test_cudanet.py (parsed, not executed) and every FEN of cpp/positions.json with its history."""
    from oracle import positions as P
    src = open(os.path.join(ref, "mayfly", "chess", "cudanet", "test_cudanet.py"), encoding="utf-8").read()
    fens = []
    for node in ast.walk(ast.parse(src)):
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "FIXED" for t in node.targets):
            for e in node.value.elts:
                fens.append(P.START_FEN if isinstance(e, ast.Attribute) else e.value)
    out = []
    for f in fens:
        p = P.Position(f)
        if p.legal()[0]:
            out.append(("test_cudanet.FIXED", f, p))
    for e in json.load(open(os.path.join(ref, "mayfly", "chess", "cpp", "positions.json"))):
        p = P.Position(e["fen"])
        for u in e["hist"]:
            codes, _ = p.legal()
            match = [c for c in codes if uci(c) == u]
            if len(match) != 1:
                raise RuntimeError(f"{e['name']}: history move {u} not legal")
            p.push(match[0])
        if p.legal()[0]:
            out.append(("positions.json:" + e["name"], e["fen"], p))
    return out


def uci(code):
    f, t, promo = (code >> 6) & 63, code & 63, code >> 12
    s = "abcdefgh"[f & 7] + "12345678"[f >> 3] + "abcdefgh"[t & 7] + "12345678"[t >> 3]
    return s + (" pnbrqk"[promo] if promo else "")


def reference_outputs(chess_net, export_ts, arch, state, batch):
    """ChessNet float32 on the CPU through export_ts.Export and export_ts.post (test_cudanet.py:177-194), with
    pol cut to the legal moves (test_cudanet.py:167-173 cut) and qv set to 0 on padding."""
    m = chess_net.ChessNet(d=arch.d, nhead=arch.heads, layers=arch.layers, dim_ff=arch.ff, qhead=True)
    m.load_state_dict({**state, "posidx": torch.arange(64)}, strict=True)
    m = m.float().eval()
    mha = torch.backends.mha
    fast = mha.get_fastpath_enabled()
    mha.set_fastpath_enabled(False)
    try:
        with torch.no_grad():
            exp = export_ts.Export(m).eval()
            pol, qval = exp(*export_ts.inputs(batch, "cpu"))
            r = export_ts.post(pol, qval, batch, "cpu")
    finally:
        mha.set_fastpath_enabled(fast)
    B, wide = batch["I"].shape
    P = np.zeros((B, wide), np.float32)
    Q = np.array(r["qv"], np.float32)
    for i, k in enumerate(batch["widths"]):
        P[i, :k] = r["policy"][i, batch["I"][i, :k]]
        Q[i, k:] = 0.0
    return P, r["val"].astype(np.float32), Q, pol.numpy(), qval.numpy()


def synthetic_keys(n, seed):
    """n seeded transposition keys that stress encode_keys' bit arithmetic: random piece bitboards split between
    the colours, kings on a1/h1/a8/h8 or anywhere, random castling-rights bits on both back ranks, either side
    to move, en passant squares or None, clocks 0..300. Not all are legal chess positions; the encoder's
    arithmetic is defined on any key."""
    rng = np.random.Generator(np.random.PCG64(seed))
    keys = np.zeros((n, 10), np.uint64)
    ep = np.full(n, -1, np.int64)
    corners = np.array([0, 7, 56, 63], np.uint64)
    for i in range(n):
        occ = rng.integers(0, 2**63, dtype=np.uint64) & rng.integers(0, 2**63, dtype=np.uint64)
        types = rng.integers(0, 6, 64)
        bb = [np.uint64(0)] * 6
        for sq in range(64):
            if (int(occ) >> sq) & 1:
                bb[types[sq]] |= np.uint64(1) << np.uint64(sq)
        kings = np.uint64(0)
        for c in range(2):
            sq = corners[rng.integers(0, 4)] if rng.random() < 0.5 else np.uint64(rng.integers(0, 64))
            kings |= np.uint64(1) << sq
        for t in range(5):
            bb[t] &= ~kings
        bb[5] = kings
        allp = np.uint64(0)
        for t in range(6):
            allp |= bb[t]
        white_mask = rng.integers(0, 2**63, dtype=np.uint64) | (np.uint64(rng.integers(0, 2)) << np.uint64(63))
        keys[i, :6] = bb
        keys[i, 6] = allp & white_mask
        keys[i, 7] = allp & ~white_mask
        keys[i, 8] = rng.integers(0, 2)
        cr = np.uint64(0)
        for sq in (0, 7, 56, 63, int(rng.integers(0, 8)), 56 + int(rng.integers(0, 8))):
            if rng.random() < 0.5:
                cr |= np.uint64(1) << np.uint64(sq)
        keys[i, 9] = cr
        if rng.random() < 0.3:
            ep[i] = int(rng.integers(16, 24)) if keys[i, 8] == 0 else int(rng.integers(40, 48))
    clock = rng.integers(0, 301, n).astype(np.int64)
    return keys, ep, clock


def keys_case(ref, meta):
    """keys_seed1.npz: encode.py's own encode_keys on keys from chess_core positions and on synthetic keys."""
    from oracle import positions as P
    import encode   # noqa: E402  (mayfly/chess/encode.py, with the constants stub as `chess`)
    pos = P.random_playouts(2048, seed=1, max_plies=120) + [p for _, _, p in fixed_fens(ref)]
    k_pos, ep_pos, clock_pos = P.key_batch(pos)
    k_syn, ep_syn, clock_syn = synthetic_keys(4096, seed=7)
    keys = np.concatenate([k_pos, k_syn])
    ep_sq = np.concatenate([ep_pos, ep_syn])
    clock = np.concatenate([clock_pos, clock_syn])
    tuples = [tuple(bool(k[8]) if j == 8 else int(k[j]) for j in range(10)) + (None if e < 0 else int(e),)
              for k, e in zip(keys, ep_sq)]
    ids, cast, hm, ep = encode.encode_keys(tuples, [int(c) for c in clock])
    for i, p in enumerate(pos):   # the reference's two encoders agree on real positions
        e_ids, e_cast, e_hm, e_ep = p.encode()
        if not (np.array_equal(e_ids, ids[i]) and np.array_equal(e_cast, cast[i]) and e_hm == hm[i]
                and e_ep == ep[i]):
            raise SystemExit(f"encode_keys and chess_core encode differ at position {i}")
    np.savez_compressed(os.path.join(HERE, "keys_seed1.npz"), keys=keys, ep_sq=ep_sq, clock=clock,
                        ids=ids.astype(np.int64), cast=cast.astype(np.float32), hm=hm.astype(np.int64),
                        ep=ep.astype(np.int64), n_positions=np.int64(len(pos)))
    meta["cases"]["keys_seed1"] = {
        "B": int(keys.shape[0]), "positions": len(pos),
        "note": "encode.py encode_keys outputs: 2,048 seed-1 positions (positions_seed1 rows 0..2047), the fixed "
                "positions, then 4,096 synthetic keys (seed 7); real positions checked against chess_core encode"}
    print(f"keys_seed1: {keys.shape[0]} keys ({len(pos)} positions)")


def cnw_case(ref):
    """cnw_v1_seed1.json: the reference exporter's file for the seed-1 146M state, summarised."""
    import hashlib
    import tempfile
    sys.path.insert(0, os.path.join(ref, "mayfly", "chess", "cudanet"))
    import export_cudanet   # noqa: E402
    st = W.random_state(W.FULL, 1)
    with tempfile.TemporaryDirectory() as d:
        ck = os.path.join(d, "seed1.pt")
        torch.save({"model": {**st, "posidx": torch.arange(64)},
                    "cfg": {"d": W.FULL.d, "layers": W.FULL.layers, "nhead": W.FULL.heads, "ff_mult": 2.0}}, ck)
        out = os.path.join(d, "seed1.cnw")
        argv = sys.argv
        sys.argv = ["export_cudanet.py", ck, out]
        try:
            export_cudanet.main()
        finally:
            sys.argv = argv
        hdr, arrays = export_cudanet.read_cnw(out)
        size = os.path.getsize(out)
    fix = {"generator": "tests/golden/make_golden.py --only cnw (mayfly/chess/cudanet/export_cudanet.py main)",
           "file_bytes": size,
           "header": {k: v for k, v in hdr.items() if k not in ("tensors", "source")},
           "tensors": [dict(e, sha256=hashlib.sha256(np.ascontiguousarray(arrays[e["name"]]).tobytes()).hexdigest())
                       for e in hdr["tensors"]]}
    with open(os.path.join(HERE, "cnw_v1_seed1.json"), "w") as f:
        json.dump(fix, f, indent=0)
    print(f"cnw_v1_seed1: {len(fix['tensors'])} tensors, {size / 1e6:.1f} MB, fingerprint {hdr['fingerprint']}")


def check_state_spec(chess_net, arch):
    m = chess_net.ChessNet(d=arch.d, nhead=arch.heads, layers=arch.layers, dim_ff=arch.ff, qhead=True)
    ref = [(k, tuple(v.shape)) for k, v in m.state_dict().items() if v.is_floating_point()]
    mine = [(k, tuple(s)) for k, s in W.state_spec(arch)]
    if ref != mine:
        raise SystemExit(f"state_spec differs from ChessNet's state dict for {arch}")
    return [k for k, _ in ref]


def save_case(name, arch, seed, batch, outs, note, meta, full_rows=4, rounded=None):
    """rounded: {tag: outputs} of the same reference model with its weights rounded the way a weight file of
    that precision stores them (mayfly_chess_b200.weights.dequantised_state), saved as pol_<tag> etc."""
    P, V, Q, pol_full, q_full = outs
    extra = {}
    for tag, (p2, v2, q2, _, _) in (rounded or {}).items():
        extra.update({f"pol_{tag}": p2, f"val_{tag}": v2, f"qv_{tag}": q2})
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **pack(batch), pol=P, val=V, qv=Q,
                        policy_rows=pol_full[:full_rows].astype(np.float32),
                        qvalue_rows=q_full[:full_rows].astype(np.float32), **extra)
    meta["cases"][name] = {"arch": [arch.d, arch.layers, arch.heads, arch.ff], "seed": seed,
                           "B": int(batch["ids"].shape[0]), "wide": int(batch["I"].shape[1]), "note": note}


def b1024_case(chess_net, export_ts, meta):
    """full_seed1_b1024.npz: config 2 at its own batch. The reference forward runs in chunks of 256 rows (each
    row's arithmetic does not depend on the others in the batch); the outputs are kept at the legal moves only,
    concatenated row after row in positions_seed1.npz order, which the test re-pads from the position set."""
    from mayfly_chess_b200.inputs import PositionSet
    ps = PositionSet(os.path.join(HERE, "positions_seed1.npz"))
    B, chunk = 1024, 256
    st = W.random_state(W.FULL, 1)
    states = {"": st, "_bf16w": W.dequantised_state(st, W.FULL, "bf16"),
              "_e4m3w": W.dequantised_state(st, W.FULL, "e4m3")}
    out = {}
    t = time.time()
    for tag, s in states.items():
        pols, qvs, vals = [], [], []
        for c in range(0, B, chunk):
            b = ps.batch(c, chunk)
            P_, V_, Q_, _, _ = reference_outputs(chess_net, export_ts, W.FULL, s, b)
            for i, k in enumerate(b["widths"]):
                pols.append(P_[i, :k])
                qvs.append(Q_[i, :k])
            vals.append(V_)
        out["pol" + tag] = np.concatenate(pols).astype(np.float32)
        out["qv" + tag] = np.concatenate(qvs).astype(np.float32)
        out["val" + tag] = np.concatenate(vals).astype(np.float32)
        print(f"full_seed1_b1024{tag}: {time.time() - t:.1f} s", flush=True)
    widths = ps.widths[:B].astype(np.uint16)
    np.savez_compressed(os.path.join(HERE, "full_seed1_b1024.npz"), widths=widths, first_row=np.int64(0), **out)
    meta["cases"]["full_seed1_b1024"] = {
        "arch": [W.FULL.d, W.FULL.layers, W.FULL.heads, W.FULL.ff], "seed": 1, "B": B,
        "note": "positions_seed1.npz rows 0..1023 (the bench's batch); outputs at the legal moves only, "
                "flattened; reference forward in chunks of 256 rows; bf16w / e4m3w controls"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MAYFLY_REFERENCE"),
                    help="the reference checkout (default: $MAYFLY_REFERENCE)")
    ap.add_argument("--only", choices=["keys", "cnw", "b1024"], help="regenerate one fixture alone")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or MAYFLY_REFERENCE")
    subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), f"REF={args.ref}"], check=True)
    from oracle import positions as P

    chess_net, export_ts = import_reference(args.ref)
    if args.only == "cnw":
        cnw_case(args.ref)
        return
    if args.only == "b1024":
        with open(os.path.join(HERE, "meta.json")) as f:
            meta = json.load(f)
        b1024_case(chess_net, export_ts, meta)
        with open(os.path.join(HERE, "meta.json"), "w") as f:
            json.dump(meta, f, indent=1)
        return
    if args.only == "keys":
        with open(os.path.join(HERE, "meta.json")) as f:
            meta = json.load(f)
        keys_case(args.ref, meta)
        with open(os.path.join(HERE, "meta.json"), "w") as f:
            json.dump(meta, f, indent=1)
        return
    meta = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__, "cases": {}}
    for tag, arch in (("small", W.SMALL), ("full", W.FULL)):
        meta[f"state_keys_{tag}"] = check_state_spec(chess_net, arch)

    fixed = fixed_fens(args.ref)
    fixed_batch = P.encode_batch([p for _, _, p in fixed])
    meta["fixed_sources"] = [s for s, _, _ in fixed]
    print(f"{len(fixed)} fixed positions, widths {fixed_batch['widths'].min()}..{fixed_batch['widths'].max()}")

    # the bench's position set: 8,192 seed-1 playouts of 0..120 plies
    t = time.time()
    seed1_pos = P.random_playouts(8192, seed=1, max_plies=120)
    seed1 = P.encode_batch(seed1_pos)
    np.savez_compressed(os.path.join(HERE, "positions_seed1.npz"), **pack(seed1))
    print(f"positions_seed1: 8192 positions in {time.time() - t:.1f} s, widths "
          f"{seed1['widths'].min()}..{seed1['widths'].max()}")

    # config 1: the small net, seed 0
    small0 = P.encode_batch(P.random_playouts(256, seed=0, max_plies=80))
    st = W.random_state(W.SMALL, 0)
    meta["fingerprint_small_seed0"] = W.fingerprint(st)
    def run(arch, st, batch):
        outs = reference_outputs(chess_net, export_ts, arch, st, batch)
        rounded = {tag: reference_outputs(chess_net, export_ts, arch, W.dequantised_state(st, arch, prec), batch)
                   for tag, prec in (("bf16w", "bf16"), ("e4m3w", "e4m3"))}
        return outs, rounded

    o, rd = run(W.SMALL, st, small0)
    save_case("small_seed0_b256", W.SMALL, 0, small0, o, "256 seed-0 playouts of 0..80 plies", meta, rounded=rd)
    o, rd = run(W.SMALL, st, fixed_batch)
    save_case("small_seed0_fixed", W.SMALL, 0, fixed_batch, o, "fixed edge cases", meta, rounded=rd)

    # config 2 subsets: the 146M net, seed 1
    st = W.random_state(W.FULL, 1)
    meta["fingerprint_full_seed1"] = W.fingerprint(st)
    b64 = P.encode_batch(seed1_pos[:64])
    t = time.time()
    o, rd = run(W.FULL, st, b64)
    save_case("full_seed1_b64", W.FULL, 1, b64, o, "the first 64 seed-1 positions (positions_seed1.npz rows 0..63)",
              meta, rounded=rd)
    o, rd = run(W.FULL, st, fixed_batch)
    save_case("full_seed1_fixed", W.FULL, 1, fixed_batch, o, "fixed edge cases", meta, rounded=rd)
    print(f"146M reference forward: {time.time() - t:.1f} s")
    b1024_case(chess_net, export_ts, meta)
    keys_case(args.ref, meta)
    cnw_case(args.ref)
    with open(os.path.join(HERE, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("done")


if __name__ == "__main__":
    main()
