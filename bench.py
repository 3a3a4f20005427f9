"""Throughput of MayFly's batched network evaluation on B200s: positions evaluated per second.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch 1024] [--precision bf16|f16|e4m3]
                    [--impl reference] [--no-fp8] [--no-strong] [--no-sweep] [--no-cpu]

Workload (the metric's configuration): the 146M trunk (d 1024, 16 layers, 16 heads, FFN
2048, 65 tokens, policy + qvalue heads and the search's reduction) with seed-1 random-init weights in bf16,
evaluating 1,024 seed-1 random-playout positions per GPU per step (tests/golden/positions_seed1.npz; rank r
takes positions r*1024 .. r*1024+1023, so 8 ranks cover the whole 8,192-position set of config 5). One
independent evaluator per GPU, no collective on the data path (weak scaling: 1,024 positions per GPU).

  value      positions/s with inputs resident in HBM: K passes through cudanet_evaluate_device, timed with
             CUDA events on the launching stream between a barrier + synchronize on both sides, max over ranks.
             The working set (285 MB of weights, ~1.2 GB of activations) is far larger than L2.
  e2e        the same metric through the reference-facing API, CudaNet.evaluate on host numpy arrays: each step
             copies the inputs into pinned staging and up, and the outputs down and out (wall clock).
  parity     rank 0's e2e outputs at B = 1,024 (positions 0..1023) against the reference ChessNet's float32
             outputs for the same positions (tests/golden/full_seed1_b1024.npz).
  roofline   the dominant product, qkv (the CTA-pair tcgen05 GEMM, one launch per layer): its algorithmic FLOPs per
             launch / its mean launch time, from CUDA events around each step of an eager pass on the evaluator's
             stream (cudanet_profile), against the measured BURST bf16 peak (each launch is timed alone, for well
             under a second). `traffic` is its DRAM bytes per launch from the ncu capture
             (profiles/gemm_qkv_pair_*), scaled by B / 1,024. The whole trunk-GEMM family and the whole pass are
             reported beside it against the same peak.
  fp8        BASELINE config 4 (N = 1 only): the e4m3 evaluator and the bf16 evaluator on the same 4,096 positions
             on this GPU, positions/s of each and their ratio, the e4m3 pass's parity against the float32
             reference (and the reference model with e4m3-rounded weights, the control), and its dominant
             product's roofline against twice the measured burst bf16 peak (no FP8 peak is measured).
  strong     BASELINE config 5: 8,192 positions a step split evenly over the N ranks (device time, max over
             ranks); at N > 1 rank 0 also times all 8,192 alone, and efficiency = value / (N x that).
  latency_sweep  BASELINE config 3: p50 / p99 per call through CudaNet.evaluate at B = 1, 16, 64, 128, 256 and
             the weight stream's GB/s (bytes of the weights / p50).
  ranks      at N > 1: every rank's device time of the timed region and median SM clock, and the straggler (the
             rank with the longest time, which sets `value`).
  cpu_baseline  the CPU fp32 restatement of the reference forward (oracle/, test infrastructure) on this host's
             cores: the median of 5 calls on 64 positions after 2 warm-up calls.

--total 8192 runs the whole line as strong scaling (8,192 positions per step split over the ranks). The
default keeps 1,024 positions per GPU (weak scaling), the metric's configuration.

--precision e4m3 --batch 4096 runs the whole line on the e4m3 evaluator (config 4 alone).

--impl reference times the reference's CPU path (the same fp32 restatement, all host threads) on the same
metric and configuration (1,024 positions a step), rank 0 only.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "NN positions evaluated/sec (146M trunk, bs1024, 1/2/4/8 B200); p50 latency at bs64"
# DRAM bytes (read + write) of one qkv launch per position, from the ncu captures in profiles/
# (the qkv product's ncu captures at B = 1,024: 142.9 + 355.6 MB in bf16, 71.5 + 355.7 MB with e4m3 operands)
QKV_TRAFFIC_PER_POS = {"bf16": (142905088 + 355564544) / 1024, "e4m3": (71474944 + 355708928) / 1024}
CALIB_ROWS = (7936, 8192)   # positions_seed1.npz rows the e4m3 input scales are calibrated on
POSITIONS = os.path.join(REPO, "tests", "golden", "positions_seed1.npz")
PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def keys_of_inputs(b):
    """White-to-move transposition keys whose encoding is exactly this batch's inputs (the position files keep
    the encoded inputs, not the keys): piece boards from ids, castling-rights bits on the rook corners for each
    right cast sets (the king sits on its back rank whenever one is set), the en passant square from ep, the
    clock from hm. Checked against the GPU encoder before use."""
    ids = b["ids"]
    B = ids.shape[0]
    sq = np.uint64(1) << np.arange(64, dtype=np.uint64)
    keys = np.zeros((B, 10), np.uint64)
    for t in range(6):
        keys[:, t] = ((ids == t + 1) | (ids == t + 7)) @ sq
    keys[:, 6] = ((ids >= 1) & (ids <= 6)) @ sq
    keys[:, 7] = (ids >= 7) @ sq
    keys[:, 8] = 1
    corner = np.array([1 << 7, 1 << 0, 1 << 63, 1 << 56], np.uint64)
    keys[:, 9] = (b["cast"] > 0) @ corner
    ep_sq = np.where(b["ep"] > 0, b["ep"] - 1, -1).astype(np.int64)
    return keys, ep_sq, b["hm"].astype(np.int64)


def flops_per_position(d=1024, layers=16, heads=16, ff=2048, tokens=65, moves=4162):
    """FLOPs of one position (multiply-add = 2): (algorithmic, executed, executed by the trunk products).
    Algorithmic: the four trunk products, attention and the heads of every token. Executed: the evaluator runs
    the last layer past its qkv product for the CLS row alone (the heads read nothing else), so that layer's
    attention, out and FFN count one query / one row."""
    dh = d // heads
    layer = 3 * d * d + d * d + 2 * d * ff
    gemm = tokens * layers * layer
    att = layers * heads * 2 * tokens * tokens * dh
    gemm_x = tokens * (layers - 1) * layer + tokens * 3 * d * d + (d * d + 2 * d * ff)
    att_x = (layers - 1) * heads * 2 * tokens * tokens * dh + heads * 2 * tokens * dh
    return 2 * (gemm + att + 2 * moves * d), 2 * (gemm_x + att_x + 2 * moves * d), 2 * gemm_x


class Clocks:
    """nvidia-smi samples of one GPU every 100 ms while running; stop(t0, t1) summarises the samples taken inside
    the timed window [t0, t1] (time.monotonic), the nearest later samples when the window is shorter than the
    sampling period."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def stop(self, t0=None, t1=None):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        lines = self.lines
        if t0 is not None:
            inside = [ln for t, ln in lines if t0 <= t <= t1]
            lines = inside or [ln for t, ln in lines if t >= t0][:2]
        else:
            lines = [ln for _, ln in lines]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 8:
                continue
            try:
                sm.append(float(p[0]))
                mx.append(float(p[1]))
            except ValueError:
                continue
            for n, v in zip(names, p[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "samples inside the timed region" if t0 is not None else "all samples"}


def load_peaks():
    try:
        with open(PEAKS) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return FALLBACK_PEAKS, "fallback"


def cpu_model():
    """The host CPU's model name (lscpu, else /proc/cpuinfo)."""
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for ln in out.splitlines():
            if ln.startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_sample(n_pos, threads, calls=5, warmup=2):
    """Positions/s of the CPU fp32 oracle (test infrastructure): the median of `calls` timed calls on n_pos
    positions of the workload each (different positions per call), after `warmup` untimed calls."""
    import torch
    from mayfly_chess_b200 import weights as W
    from mayfly_chess_b200.inputs import PositionSet
    from oracle import chessnet_oracle as O
    torch.set_num_threads(threads)
    st = W.random_state(W.FULL, 1)
    ps = PositionSet(POSITIONS)
    ts = []
    for i in range(warmup + calls):
        b = ps.batch(i * n_pos, n_pos)
        t0 = time.perf_counter()
        O.evaluate(st, W.FULL, b)
        if i >= warmup:
            ts.append(time.perf_counter() - t0)
    return n_pos / statistics.median(ts), ts


def workload_config(args, B, world, wide, precision):
    """The `config` object of both arms' lines (the same workload, so the two lines compare)."""
    return {"workload": ("config 4 (e4m3 layer products, calibrated static input scales)"
                         if precision == "e4m3" else "config 2") +
                        ": 146M trunk (d1024 L16 H16 FF2048, 65 tokens), seed-1 random-init "
                        f"weights, {B} seed-1 random-playout positions per GPU per step",
            "batch_per_gpu": B, "global_batch": B * world, "wide": wide, "precision": precision,
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "working set larger than L2 (285 MB weights + ~1.2 GB activations per pass)"}


def bench_reference(args):
    """--impl reference: the reference's CPU implementation of the path (its fp32 forward and _collect
    arithmetic, restated in oracle/chessnet_oracle.py; the reference's own code cannot travel here) timed with
    every host thread on the same configuration as the product's line: each timed step evaluates the same
    1,024 seed-1 positions (rank 0's batch) in one call. The warm-up steps run 32 positions each (they only
    bring the thread pool and the allocator up to speed)."""
    from mayfly_chess_b200 import replicas
    rank, world, _ = replicas.rank_env()
    if rank != 0:
        return
    import torch
    from mayfly_chess_b200 import weights as W
    from mayfly_chess_b200.inputs import PositionSet
    from oracle import chessnet_oracle as O
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    st = W.random_state(W.FULL, 1)
    ps = PositionSet(POSITIONS)
    start, B = replicas.shard(0, world, len(ps), total=args.total or None, per_rank=None if args.total else args.batch)
    b = ps.batch(start, B)
    for i in range(args.warmup):
        O.evaluate(st, W.FULL, ps.batch(start + 32 * i, 32))
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        O.evaluate(st, W.FULL, b)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    v = B * args.steps / total
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "positions/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "strong" if args.total else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, B, world, b["I"].shape[1], args.precision),
        "cpu_baseline": {"value": v, "unit": "positions/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
                         "sample": f"{args.steps} steps of the same {B} positions in one call each (fp32 torch "
                                   "restatement of ChessNet + post, all host threads); warm-up steps of 32"},
        "e2e": {"value": v, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def b1024_reference():
    """(batch of positions 0..1023, {pol, val, qv, pol_e4m3w, ...}) from tests/golden/full_seed1_b1024.npz: the
    reference ChessNet's float32 outputs at the legal moves, re-padded to the batch."""
    from mayfly_chess_b200.inputs import PositionSet
    z = np.load(os.path.join(REPO, "tests", "golden", "full_seed1_b1024.npz"))
    widths = z["widths"].astype(np.int64)
    b = PositionSet(POSITIONS).batch(int(z["first_row"]), len(widths))
    if not np.array_equal(b["widths"], widths):
        raise SystemExit("full_seed1_b1024.npz does not match positions_seed1.npz")
    ref = {}
    for k in z.files:
        if k.startswith(("pol", "qv")):
            ref[k] = np.zeros(b["I"].shape, np.float32)
            ref[k][b["M"]] = z[k]
        elif k.startswith("val"):
            ref[k] = z[k]
    return b, ref


def parity_summary(ref, got, widths):
    """The parity metrics of tests/parity.py (the reference's metric set), the headline figures only."""
    sys.path.insert(0, os.path.join(REPO, "tests"))
    from parity import metrics
    m = metrics(ref, got, widths)
    keys = ("pol_max", "pol_mean", "prior_max", "prior_mean", "q_max", "val_max", "top1", "top1_clear", "top3",
            "rows", "nonfinite", "pad_nonzero")
    return {k: m[k] for k in keys}


def device_pass_ms(net, b, steps, warmup):
    """Mean device milliseconds of a pass over batch b through cudanet_evaluate_device (inputs in HBM), CUDA
    events on the launching stream."""
    import torch
    B, wide = b["I"].shape
    dev = {k: torch.from_numpy(np.ascontiguousarray(b[k])).cuda() for k in ("ids", "cast", "hm", "ep", "I")}
    Md = torch.from_numpy(b["M"].astype(np.uint8)).cuda()
    pol, val, qv = torch.empty(B, wide, device="cuda"), torch.empty(B, device="cuda"), torch.empty(B, wide,
                                                                                                   device="cuda")
    for _ in range(warmup):
        net.evaluate_device(dev["ids"], dev["cast"], dev["hm"], dev["ep"], dev["I"], Md, pol, val, qv)
    s = torch.cuda.current_stream()
    net.check(s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        net.evaluate_device(dev["ids"], dev["cast"], dev["hm"], dev["ep"], dev["I"], Md, pol, val, qv)
    e1.record(s)
    torch.cuda.synchronize()
    net.check(s)
    return e0.elapsed_time(e1) / steps


def bench_latency(args):
    """--latency B: p50 / p99 of K calls of CudaNet.evaluate on B host positions after W warm-up calls, with
    the weight stream's GB/s, on cuda:0 (the command the small-batch ncu captures run)."""
    from mayfly_chess_b200 import weights as W
    from mayfly_chess_b200.cudanet_py import CudaNet
    from mayfly_chess_b200.inputs import PositionSet
    B = args.latency
    os.environ.setdefault("MAYFLY_CUDANET_MAX_BATCH", str(max(B, 1024)))
    st = W.random_state(W.FULL, 1)
    tmp = tempfile.mkdtemp(prefix="mayfly_b200_")
    path = os.path.join(tmp, f"net_{args.precision}.cnw")
    if args.precision == "e4m3":
        from mayfly_chess_b200 import quant
        amax = quant.calibrate(st, W.FULL, PositionSet(POSITIONS).batch(CALIB_ROWS[0], CALIB_ROWS[1] - CALIB_ROWS[0]))
        quant.write_e4m3(path, st, W.FULL, amax)
    else:
        W.write_cnw(path, st, W.FULL, args.precision)
    net = CudaNet(path)
    os.remove(path)
    b = PositionSet(POSITIONS).batch(0, B)
    for _ in range(args.warmup):
        net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
        ts.append(time.perf_counter() - t0)
    prof = net.profile(B, reps=3)
    net.close()
    ts.sort()
    p50, p99 = ts[len(ts) // 2], ts[min(len(ts) - 1, int(len(ts) * 0.99))]
    wbytes = (151265280 + 1302528) if args.precision == "e4m3" else (285483008 + 811008)
    print(json.dumps({"metric": f"p50 latency per call at batch {B} (config 3)", "value": 1000 * p50, "unit": "ms",
                      "p99_ms": 1000 * p99, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
                      "dtype": args.precision, "batch": B, "weight_stream_gbs": wbytes / p50 / 1e9,
                      "graph_pass_ms": prof["graph_pass"], "profile_ms": prof}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--total", type=int, default=0,
                    help="strong scaling (config 5): this many positions per step over all ranks (overrides --batch)")
    ap.add_argument("--precision", default="bf16", choices=["bf16", "f16", "e4m3"])
    ap.add_argument("--impl", default="own", choices=["own", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=64, help="positions per call of the cpu_baseline sample")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-fp8", action="store_true", help="leave out the fp8 object (config 4)")
    ap.add_argument("--no-strong", action="store_true", help="leave out the strong object (config 5)")
    ap.add_argument("--latency", type=int, default=0, metavar="B",
                    help="config 3 at one batch size alone: K timed CudaNet.evaluate calls at batch B (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        return bench_reference(args)
    if args.latency:
        return bench_latency(args)

    import torch
    import torch.distributed as dist
    from mayfly_chess_b200 import weights as W
    from mayfly_chess_b200 import cudanet_py
    from mayfly_chess_b200.cudanet_py import CudaNet
    from mayfly_chess_b200.inputs import PositionSet
    from mayfly_chess_b200 import replicas

    rank, world, local = replicas.rank_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        replicas.barrier(dist, torch.cuda.synchronize)

    def max_over_ranks(x):
        return replicas.max_over_ranks(x, dist, "cuda")

    ps = PositionSet(POSITIONS)
    try:
        start, B = replicas.shard(rank, world, len(ps), total=args.total or None,
                                  per_rank=None if args.total else args.batch)
    except ValueError as e:
        raise SystemExit(str(e))
    STRONG_TOTAL = 8192
    do_strong = not args.no_strong and not args.total and args.precision != "e4m3" and STRONG_TOTAL % world == 0
    do_fp8 = not args.no_fp8 and world == 1 and args.precision == "bf16"
    FP8_B = 4096
    # one evaluator serves every batch size this rank runs (a CUDA graph per size)
    need = [B]
    if do_strong:
        need.append(STRONG_TOTAL if rank == 0 else STRONG_TOTAL // world)
    if do_fp8:
        need.append(FP8_B)
    os.environ.setdefault("MAYFLY_CUDANET_MAX_BATCH", str(max(need + [1024])))
    arch = W.FULL
    st = W.random_state(arch, 1)
    tmp = tempfile.mkdtemp(prefix="mayfly_b200_")
    path = os.path.join(tmp, f"net_{args.precision}_{rank}.cnw")
    if args.precision == "e4m3":
        from mayfly_chess_b200 import quant
        amax = quant.calibrate(st, arch, ps.batch(CALIB_ROWS[0], CALIB_ROWS[1] - CALIB_ROWS[0]), device=local)
        quant.write_e4m3(path, st, arch, amax)
    else:
        W.write_cnw(path, st, arch, args.precision)
    net = CudaNet(path, device=local)
    os.remove(path)
    b = ps.batch(start, B)
    wide = b["I"].shape[1]

    # ---------------------------------------------------------------- value: inputs resident in HBM
    dev = {k: torch.from_numpy(np.ascontiguousarray(b[k])).cuda() for k in ("ids", "cast", "hm", "ep", "I")}
    Md = torch.from_numpy(b["M"].astype(np.uint8)).cuda()
    pol = torch.empty(B, wide, device="cuda")
    val = torch.empty(B, device="cuda")
    qv = torch.empty(B, wide, device="cuda")

    def step_dev():
        net.evaluate_device(dev["ids"], dev["cast"], dev["hm"], dev["ep"], dev["I"], Md, pol, val, qv)

    for _ in range(args.warmup):
        step_dev()
    net.check(torch.cuda.current_stream())
    vis = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    gpu_index = vis[local] if local < len(vis) else local   # nvidia-smi counts physical devices
    clocks = Clocks(gpu_index)
    clocks.start()
    time.sleep(0.3)
    barrier()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.monotonic()
    e0.record(s)
    for _ in range(args.steps):
        step_dev()
    e1.record(s)
    barrier()
    clk = clocks.stop(w0, time.monotonic())
    net.check(s)
    own_ms = e0.elapsed_time(e1)
    dev_ms = max_over_ranks(own_ms)
    value = world * B * args.steps / (dev_ms / 1000.0)
    ranks = None
    if world > 1:
        # every rank's device time and median SM clock, and the straggler (the rank whose time is the job's)
        mine = torch.tensor([own_ms, float(clk.get("sm_mhz") or 0.0)], dtype=torch.float64, device="cuda")
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        rows = [t.tolist() for t in every]
        slow = max(range(world), key=lambda r: rows[r][0])
        ranks = {"ms": [round(r[0], 3) for r in rows], "sm_mhz": [r[1] for r in rows],
                 "straggler": {"rank": slow, "ms": round(rows[slow][0], 3), "sm_mhz": rows[slow][1]}}

    # ---------------------------------------------------------------- e2e: host arrays through the C ABI
    for _ in range(2):
        net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        p_h, v_h, q_h = net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    e2e_s = time.perf_counter() - t0
    barrier()
    e2e_s = max_over_ranks(e2e_s)
    e2e = world * B * args.steps / e2e_s
    h2d = B * (64 * 8 + 8 + 8 + 16) + B * wide * 9
    d2h = 256 + 4 * B * (2 * wide + 1)
    parity = None
    if start == 0 and B == 1024:
        rb, ref = b1024_reference()
        tag = "_e4m3w" if args.precision == "e4m3" else ""
        parity = {"against": "reference ChessNet float32 outputs, positions 0..1023 (tests/golden/full_seed1_b1024.npz)",
                  **parity_summary((ref["pol"], ref["val"], ref["qv"]), (p_h, v_h, q_h), rb["widths"])}
        if tag:
            parity["vs_e4m3_weight_model"] = parity_summary((ref["pol" + tag], ref["val" + tag], ref["qv" + tag]),
                                                            (p_h, v_h, q_h), rb["widths"])

    # ---------------------------------------------------------------- the key-fed path (encode on the GPU)
    keys, ep_sq, clock = keys_of_inputs(b)
    kd = [torch.from_numpy(a.view(np.int64)).cuda() for a in (keys, ep_sq, clock)]
    enc = cudanet_py.encode_keys_device(*kd)
    for k, t in zip(("ids", "cast", "hm", "ep"), enc):
        if not np.array_equal(t.cpu().numpy(), b[k]):
            raise SystemExit(f"the GPU encoder disagrees with the batch's {k}")
    # device time per launch: 50 launches queued behind a sleep kernel, so host pacing does not count
    lib = cudanet_py.load()
    errb = cudanet_py.ctypes.create_string_buffer(256)
    cs = cudanet_py.ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outp = [t.data_ptr() for t in enc]
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda._sleep(20_000_000)
    ev[0].record()
    for _ in range(50):
        if lib.cudanet_encode_keys(kd[0].data_ptr(), kd[1].data_ptr(), kd[2].data_ptr(), B, *outp, cs, errb, 256):
            raise SystemExit(f"cudanet_encode_keys: {errb.value.decode()}")
    ev[1].record()
    torch.cuda.synchronize()
    enc_us = ev[0].elapsed_time(ev[1]) * 1000 / 50
    cpu_enc_us = None
    if rank == 0 and not args.no_cpu:
        from oracle import encode_oracle     # the numpy restatement of encode.py encode_keys, timed on the host
        t0 = time.perf_counter()
        for _ in range(20):
            encode_oracle.encode_keys(keys, ep_sq, clock)
        cpu_enc_us = (time.perf_counter() - t0) / 20 * 1e6
    for _ in range(2):
        net.evaluate_keys(keys, ep_sq, clock, b["I"], b["M"])
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        net.evaluate_keys(keys, ep_sq, clock, b["I"], b["M"])
    e2e_keys_s = max_over_ranks(time.perf_counter() - t0)
    encoder = {"kernel": "encode_keys_kernel (one launch per batch, 64 threads a board)",
               "kernel_us": enc_us, "bytes_per_launch": 644 * B,
               "achieved_gbs": 644 * B / (enc_us * 1e-6) / 1e9,
               "cpu_numpy_us": cpu_enc_us, "cpu_numpy": "encode.py encode_keys restated on arrays (oracle/), "
                                                        "one host thread, same batch",
               "e2e_keys": {"value": world * B * args.steps / e2e_keys_s, "unit": "positions/s",
                            "h2d_bytes_per_step": B * 96 + B * wide * 9, "d2h_bytes_per_step": d2h}}

    # ---------------------------------------------------------------- roofline of the dominant kernel
    peaks, peak_kind = load_peaks()
    burst = float(peaks.get("bf16_tflops"))
    sustained = float(peaks.get("bf16_tflops_sustained", burst))

    def roofline_of(prof, Bp, precision):
        qkv_flop = 2.0 * Bp * arch.tokens * 3 * arch.d * arch.d
        achieved = qkv_flop / (prof["qkv"] / arch.layers / 1000.0) / 1e12
        traffic = QKV_TRAFFIC_PER_POS.get(precision)
        peak = burst * (2.0 if precision == "e4m3" else 1.0)
        eb = 1 if precision == "e4m3" else 2
        return {"bound": "tensor", "kernel": "gemm_tc_pair_kernel, the qkv product (one per layer)",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": (f"2 x {peak_kind} bf16 burst (no measured FP8 peak)" if precision == "e4m3"
                                else f"{peak_kind} bf16 burst (each launch timed alone)"),
                "frac_of_sustained": achieved / (sustained * peak / burst),
                "traffic": traffic * Bp if traffic is not None else None, "flop_per_launch": qkv_flop,
                "algorithmic_bytes_per_launch": Bp * arch.tokens * arch.d * eb + 3 * arch.d * arch.d * eb
                                                + Bp * arch.tokens * 3 * arch.d * 2,
                "timing": "CUDA events around each step of an eager pass (cudanet_profile), mean of 3"}

    prof = net.profile(B, reps=3)
    fl_alg, fl_pos, gemm_fl_pos = flops_per_position()
    roofline = roofline_of(prof, B, args.precision)
    trunk_gemm_ms = prof["qkv"] + prof["out"] + prof["ff1"] + prof["ff2"]
    launches = 4 * arch.layers
    family = gemm_fl_pos * B / (trunk_gemm_ms / 1000.0) / 1e12
    peak = roofline["peak"]

    # ---------------------------------------------------------------- config 5: strong scaling over 8,192
    strong = None
    if do_strong:
        sb = ps.batch(rank * (STRONG_TOTAL // world), STRONG_TOTAL // world)
        barrier()
        ms = max_over_ranks(device_pass_ms(net, sb, args.steps, 3))
        strong = {"total_positions": STRONG_TOTAL, "per_rank": STRONG_TOTAL // world, "ms_per_step": ms,
                  "value": STRONG_TOTAL / (ms / 1000.0), "unit": "positions/s",
                  "timing": "device time of K passes over each rank's share, max over ranks"}
        if world > 1:
            one = None
            if rank == 0:
                one = device_pass_ms(net, ps.batch(0, STRONG_TOTAL), args.steps, 3)
            barrier()
            if rank == 0:
                strong["single_gpu_ms_per_step"] = one
                strong["single_gpu_value"] = STRONG_TOTAL / (one / 1000.0)
                strong["efficiency"] = strong["value"] / (world * strong["single_gpu_value"])
        else:
            strong["efficiency"] = 1.0

    # ---------------------------------------------------------------- config 4: e4m3 against bf16 at 4,096
    fp8 = None
    if do_fp8:
        from mayfly_chess_b200 import quant
        fb = ps.batch(0, FP8_B)
        amax = quant.calibrate(st, arch, ps.batch(CALIB_ROWS[0], CALIB_ROWS[1] - CALIB_ROWS[0]), device=local)
        p8 = os.path.join(tmp, "net_e4m3.cnw")
        quant.write_e4m3(p8, st, arch, amax)
        net8 = CudaNet(p8, device=local)
        os.remove(p8)
        device_pass_ms(net8, fb, 3, 3)
        device_pass_ms(net, fb, 3, 3)
        ck = Clocks(gpu_index)
        ck.start()
        time.sleep(0.3)
        w0 = time.monotonic()
        ms8 = device_pass_ms(net8, fb, args.steps, 3)
        ms16 = device_pass_ms(net, fb, args.steps, 3)
        ck_out = ck.stop(w0, time.monotonic())
        rb, ref = b1024_reference()
        got8 = net8.evaluate(rb["ids"], rb["cast"], rb["hm"], rb["ep"], rb["I"], rb["M"])
        prof8 = net8.profile(FP8_B, reps=3)
        net8.close()
        fp8 = {"config": "config 4: e4m3 layer matrices (per-output-channel scales), e4m3 product inputs at static "
                         "per-layer scales calibrated on 256 seed-1 positions outside the batch, bf16 residual "
                         "stream, bf16 heads; the same 4,096 seed-1 positions through both evaluators",
               "batch": FP8_B,
               "e4m3": {"value": FP8_B / (ms8 / 1000.0), "ms_per_step": ms8},
               "bf16": {"value": FP8_B / (ms16 / 1000.0), "ms_per_step": ms16},
               "ratio": ms16 / ms8, "unit": "positions/s", "clocks": ck_out,
               "parity_vs_fp32": parity_summary((ref["pol"], ref["val"], ref["qv"]), got8, rb["widths"]),
               "parity_vs_e4m3_weight_model": parity_summary((ref["pol_e4m3w"], ref["val_e4m3w"], ref["qv_e4m3w"]),
                                                             got8, rb["widths"]),
               "e4m3_weight_model_vs_fp32": parity_summary((ref["pol"], ref["val"], ref["qv"]),
                                                           (ref["pol_e4m3w"], ref["val_e4m3w"], ref["qv_e4m3w"]),
                                                           rb["widths"]),
               "roofline": roofline_of(prof8, FP8_B, "e4m3"), "profile_ms": prof8}

    # ---------------------------------------------------------------- latency (config 3) and CPU baseline
    sweep = {}
    if not args.no_sweep:
        for Bs in (1, 16, 64, 128, 256):
            bs = ps.batch(start, Bs)
            for _ in range(5):
                net.evaluate(bs["ids"], bs["cast"], bs["hm"], bs["ep"], bs["I"], bs["M"])
            ts = []
            for _ in range(200):
                t0 = time.perf_counter()
                net.evaluate(bs["ids"], bs["cast"], bs["hm"], bs["ep"], bs["I"], bs["M"])
                ts.append(time.perf_counter() - t0)
            ts.sort()
            p50, p99 = ts[len(ts) // 2], ts[int(len(ts) * 0.99)]
            # matrices (bf16, or e4m3 layer matrices + bf16 heads) + f32 vectors and scales, read once per call
            wbytes = (151265280 + 1302528) if args.precision == "e4m3" else (285483008 + 811008)
            sweep[str(Bs)] = {"p50_ms": 1000 * p50, "p99_ms": 1000 * p99, "positions_per_s": Bs / p50,
                              "weight_stream_gbs": wbytes / p50 / 1e9,
                              "hbm_frac": wbytes / p50 / 1e9 / float(peaks.get("hbm_gbs", 6650.0))}
    cpu = None
    if rank == 0 and not args.no_cpu:
        cores = os.cpu_count() or 1
        v, ts = cpu_sample(args.cpu_sample, cores)
        cpu = {"value": v, "unit": "positions/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
               "sample": f"median of 5 calls on {args.cpu_sample} seed-1 positions each (after 2 warm-up calls) "
                         "of the 146M net, fp32 torch restatement of the reference forward + post (oracle/), "
                         "all host threads",
               "call_seconds": ts}

    net.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    out = {
        "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.total else "weak",
        "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
        "config": workload_config(args, B, world, wide, args.precision),
        "e2e": {"value": e2e, "unit": "positions/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": (1 + 7 * arch.layers - 1 + 2 + 1) * args.steps,
        "roofline": roofline,
        "gemm_family": {"kernels": "qkv, out, ff1, ff2 of every layer (64 launches)", "achieved": family,
                        "unit": "TFLOP/s", "frac": family / peak, "flop_per_launch": gemm_fl_pos * B / launches},
        "pass": {"flop_per_position": fl_pos, "flop_per_position_algorithmic": fl_alg,
                 "tflops_whole_pass": fl_pos * value / world / 1e12,
                 "frac_whole_pass": fl_pos * value / world / 1e12 / peak, "profile_ms": prof},
        "p50_latency_ms_bs64": sweep.get("64", {}).get("p50_ms"),
        "clocks": clk,
        "ranks": ranks,
        "parity": parity,
        "fp8": fp8,
        "strong": strong,
        "latency_sweep": sweep,
        "encoder": encoder,
        "cpu_baseline": cpu,
    }
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
