"""The FP8 (e4m3) path on a B200, through the C ABI.

Kernels: the e4m3 products (every epilogue, single-CTA and CTA-pair tiles), the LayerNorm and attention with
e4m3 outputs, each against a float32/float64 PyTorch reference of the same op. An e4m3 output must be within
one e4m3 unit in the last place of the exact value (correct rounding is half a unit; the other half covers a
value that the kernel's different summation order moves across a rounding midpoint).

Calibration: CudaNet.calibrate's per-layer input ranges against the oracle's, measured on the same positions.

The evaluator: an e4m3 weight file (per-output-channel weight scales, static input scales calibrated on 256
seed-1 positions that no parity case uses) end to end, against
  * the oracle running the same quantisation in float32 (e4m3 weights, every product input rounded to e4m3 at
    the file's scales, the residual stream rounded to bf16 as the FP8 evaluator stores it). This cannot be a
    tight bound: a product input that the evaluator computes a few bf16
    ulps away from the oracle (q, k, v and P are bf16 in the evaluator, f32 in the oracle) rounds to the
    other e4m3 neighbour whenever the two straddle a rounding midpoint, which happens to a few percent of the
    elements, each then off by a whole e4m3 step (6-12%). Two FP8 passes that differ only in such rounding
    noise differ by about as much as the quantisation itself costs, so the bars are set at that size (the
    146M net: 0.25 max, 0.04 mean on the policy logits), at least 90% of the top moves must agree and every
    row whose best move leads by more than twice the logit bar must; the kernels' own arithmetic is held to
    one e4m3 ulp by the kernel tests above;
  * the float32 reference model, and the reference model with only its weights e4m3-rounded (golden
    pol_e4m3w, ...): what the quantisation itself costs. These are reported (printed) with loose sanity
    bars: rounding the weights alone already moves the 146M net's policy logits by up to 0.18, three times
    the 6e-2 FP8 bar, so that bar is out of reach of any e4m3-weight evaluator on these random-init weights.
"""
import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN, golden_case
from parity import metrics
from mayfly_chess_b200 import weights as W

pytestmark = pytest.mark.gpu

CALIB_ROWS = (7936, 8192)          # positions_seed1.npz rows used to calibrate (no parity case reads them)


@pytest.fixture(scope="module")
def k():
    from mayfly_chess_b200 import build, cudanet_py
    build.build()
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return cudanet_py


def e4m3_ulp(y):
    """The spacing of the e4m3 values around |y| (2^-9 below the smallest normal, 2^-6)."""
    e = torch.floor(torch.log2(y.abs().clamp(min=2.0 ** -6)))
    return 2.0 ** (e - 3)


def assert_e4m3_close(got_u8, y, slack=0.0):
    """got (e4m3 bytes) within one e4m3 ulp (+ slack) of y saturated to +-448."""
    got = got_u8.view(torch.float8_e4m3fn).float()
    assert torch.isfinite(got).all()
    ys = y.float().clamp(-448.0, 448.0)
    excess = ((got - ys).abs() - (e4m3_ulp(ys) + slack)).max().item()
    assert excess <= 0, excess


def _f8(t):
    return t.clamp(-448.0, 448.0).to(torch.float8_e4m3fn)


# ------------------------------------------------------------------------------------------------ kernels
@pytest.mark.parametrize("epi", [0, 2, 3, 4, 5])
@pytest.mark.parametrize("M,N,K,bn", [(195, 1024, 1024, 0), (4160, 3072, 1024, 256), (1300, 1024, 2048, 128),
                                      (65, 2048, 1024, 0), (300, 8336, 1024, 256), (128, 256, 128, 256),
                                      (260, 1024, 1024, 64),
                                      # CTA pairs: 256 x 256 tiles, M and N tails, K = 2048
                                      (4160, 3072, 1024, 2), (1300, 1024, 2048, 2), (300, 8336, 1024, 2),
                                      (65, 512, 128, 2)])
def test_gemm_f8(k, epi, M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(M * 5 + N + K + epi)
    A = _f8(torch.randn(M, K, device="cuda", generator=g) * 2)
    Wt = _f8(torch.randn(N, K, device="cuda", generator=g) * 16)
    colscale = (torch.rand(N, device="cuda", generator=g) + 0.5) * 1e-3
    bias = torch.randn(N, device="cuda", generator=g) * 0.02
    inv = 300.0
    acc = (A.double() @ Wt.double().t())
    v = acc * colscale.double() + bias.double()
    if epi == 0:
        Cfull = torch.full((M, N + 8), float("nan"), device="cuda", dtype=torch.bfloat16)
    elif epi == 4:
        Cfull = torch.full((M, N + 16), 0x7F, device="cuda", dtype=torch.uint8)   # 0x7F: e4m3 NaN
    else:
        Cfull = torch.full((M, N + 4), float("nan"), device="cuda")
    if epi == 5:
        Cfull = torch.full((M, N + 8), float("nan"), device="cuda", dtype=torch.bfloat16)
    C = Cfull[:, :N]
    if epi in (2, 5):
        C.copy_(torch.randn(M, N, device="cuda", generator=g))
    C0 = C.clone()
    k.k_gemm_f8(A, Wt, colscale, bias, C, epi, inv, bn)
    torch.cuda.synchronize()
    pad = Cfull[:, N:]
    assert (pad == 0x7F).all() if epi == 4 else torch.isnan(pad).all()
    if epi == 4:
        # gelu(v) * inv, some of it past 448 (saturates)
        assert_e4m3_close(C, F.gelu(v) * inv)
        return
    ref = v + C0.double() if epi in (2, 5) else v
    # products of e4m3 values are exact in f32, only the summation order differs; bf16 output adds one rounding,
    # and the bf16 residual (epi 5) a second one, of v itself, before it is added into C
    rel = 2.0 ** -8 if epi in (0, 5) else 0.0
    tol = 1e-4 + rel * ref.abs() + (rel * v.abs() if epi == 5 else 0.0)
    excess = ((C.double() - ref).abs() - tol).max().item()
    assert math.isfinite(excess) and excess <= 0, excess


def test_gemm_f8_bad_epilogue_refused(k):
    A = torch.zeros(128, 128, device="cuda", dtype=torch.float8_e4m3fn)
    Wt = torch.zeros(128, 128, device="cuda", dtype=torch.float8_e4m3fn)
    s = torch.ones(128, device="cuda")
    C = torch.zeros(128, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="epi must be"):
        k.k_gemm_f8(A, Wt, s, s, C, 1, 1.0)     # the 16-bit GELU epilogue is not an FP8 one


def test_gemm_f8_repeatable(k):
    A = _f8(torch.randn(4160, 1024, device="cuda"))
    Wt = _f8(torch.randn(2048, 1024, device="cuda") * 16)
    s = torch.full((2048,), 1e-3, device="cuda")
    b = torch.zeros(2048, device="cuda")
    C1 = torch.empty(4160, 2048, device="cuda", dtype=torch.uint8)
    C2 = torch.empty_like(C1)
    k.k_gemm_f8(A, Wt, s, b, C1, 4, 100.0)
    k.k_gemm_f8(A, Wt, s, b, C2, 4, 100.0)
    assert torch.equal(C1, C2)


@pytest.mark.parametrize("xdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [256, 1024])
@pytest.mark.parametrize("stride", [1, 65])
def test_layernorm_f8(k, xdtype, d, stride):
    n = 300
    x = (torch.randn(n * stride, d, device="cuda") * 3 + 0.5).to(xdtype)
    g = torch.randn(d, device="cuda")
    b = torch.randn(d, device="cuda")
    h = torch.full((n, d), 0x7F, device="cuda", dtype=torch.uint8)
    mul = 448.0 / 9.0
    k.k_layernorm_f8(x, g, b, h, n, d, mul, stride)
    torch.cuda.synchronize()
    y = F.layer_norm(x[::stride].float(), (d,), g, b, 1e-5) * mul
    assert_e4m3_close(h, y, slack=1e-4 * mul)


@pytest.mark.parametrize("kernel", ["default", "mma", "tc", "tc4"])
@pytest.mark.parametrize("d,heads", [(1024, 16), (256, 8)])
@pytest.mark.parametrize("B", [1, 3, 64])
def test_attention_f8(k, kernel, d, heads, B):
    if kernel != "default" and d // heads != 64:
        pytest.skip("the kernels chosen by name are the head-width-64 ones")
    rows = B * 65
    torch.manual_seed(1000 * B + d)
    qkv = torch.randn(rows, 3 * d, device="cuda").to(torch.bfloat16)
    att = torch.full((rows, d), 0x7F, device="cuda", dtype=torch.uint8)
    mul = 100.0
    if kernel == "default":
        k.k_attention_f8(qkv, att, B, d, heads, mul)
    else:
        k.k_attention_kernel(qkv, att, B, d, heads, {"mma": 0, "tc": 1, "tc4": 4}[kernel], mul)
    torch.cuda.synchronize()
    dh = d // heads
    q, kk, v = qkv.float().view(B, 65, 3, heads, dh).permute(2, 0, 3, 1, 4).unbind(0)
    p = torch.softmax(q @ kk.transpose(-1, -2) / math.sqrt(dh), -1)
    ref = (p @ v).transpose(1, 2).reshape(rows, d)
    pv_abs = (p @ v.abs()).transpose(1, 2).reshape(rows, d)
    # P is rounded to bf16 before the second product (at most 2^-8 sum_j p_j |v_j| on an output), then one e4m3
    # rounding
    assert_e4m3_close(att, ref * mul, slack=mul * (2.0 ** -8 * pv_abs + 1e-4))


# ------------------------------------------------------------------------------------------------ calibration
def _calib_batch():
    from mayfly_chess_b200.inputs import PositionSet
    ps = PositionSet(os.path.join(GOLDEN, "positions_seed1.npz"))
    return ps.batch(CALIB_ROWS[0], CALIB_ROWS[1] - CALIB_ROWS[0])


def test_calibrate_matches_oracle_ranges(k, tmp_path):
    """The bf16 pass's measured input ranges against the float32 oracle's on the same 256 positions."""
    from oracle import chessnet_oracle as O
    st = W.random_state(W.SMALL, 0)
    path = os.path.join(tmp_path, "s.cnw")
    W.write_cnw(path, st, W.SMALL, "bf16")
    b = _calib_batch()
    with k.CudaNet(path) as net:
        got = net.calibrate(b["ids"], b["cast"], b["hm"], b["ep"])
        with pytest.raises(ValueError):
            net.calibrate(b["ids"][:0], b["cast"][:0], b["hm"][:0], b["ep"][:0])
    rec = np.zeros((W.SMALL.layers, 4))
    O.forward(st, W.SMALL, b["ids"], b["cast"], b["hm"], b["ep"], record=rec)
    assert got.shape == (W.SMALL.layers, 4)
    np.testing.assert_allclose(got, rec, rtol=3e-2)


# ------------------------------------------------------------------------------------------------ the evaluator
ARCH = {"small": (W.SMALL, 0), "full": (W.FULL, 1)}
CASES = {"small": ["small_seed0_b256", "small_seed0_fixed"], "full": ["full_seed1_b64", "full_seed1_fixed"]}
ORACLE_CASE = {"small": "small_seed0_b256", "full": "full_seed1_b64"}   # also run through the FP8 oracle

# the e4m3 evaluator against the oracle's FP8 pass in float32 (rounding-noise sized: module docstring)
TOL_FQ = {"small": {"pol_max": 0.08, "pol_mean": 0.015, "q_max": 0.02, "val_max": 0.01},
          "full": {"pol_max": 0.25, "pol_mean": 0.04, "q_max": 0.05, "val_max": 0.015}}
# sanity bars against the float32 model (the quantisation's cost; see the module docstring)
TOL_FP32 = {"pol_max": 0.5, "q_max": 0.1, "val_max": 0.1}


@pytest.fixture(scope="module")
def f8nets(k, tmp_path_factory):
    from mayfly_chess_b200 import quant
    d = tmp_path_factory.mktemp("cnw8")
    b = _calib_batch()
    out = {}
    for tag, (arch, seed) in ARCH.items():
        st = W.random_state(arch, seed)
        amax = quant.calibrate(st, arch, b)
        path = os.path.join(d, f"{tag}_e4m3.cnw")
        quant.write_e4m3(path, st, arch, amax)
        _, t = W.read_cnw(path)
        act = np.stack([t[f"L{i}.act_scale"] for i in range(arch.layers)])
        out[tag] = (k.CudaNet(path), st, act)
    yield out
    for n, _, _ in out.values():
        n.close()


def run(net, b):
    return net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])


@pytest.mark.parametrize("tag", ["small", "full"])
def test_fp8_against_fp8_oracle(f8nets, tag):
    from oracle import chessnet_oracle as O
    net, st, act = f8nets[tag]
    arch = ARCH[tag][0]
    assert net.precision() == "e4m3"
    b, _ = golden_case(ORACLE_CASE[tag])
    ref = O.evaluate(W.dequantised_state(st, arch, "e4m3"), arch, b, act=act, resid_bf16=True)
    got = run(net, b)
    # a row whose best move leads by more than twice the logit bar cannot change its top move within the bar
    m = metrics(ref[:3], got, b["widths"], decided_gap=2 * TOL_FQ[tag]["pol_max"])
    print(tag, "e4m3 vs FP8 oracle", m)
    for key, lim in TOL_FQ[tag].items():
        assert m[key] <= lim, (key, m[key])
    assert m["nonfinite"] == 0 and m["pad_nonzero"] == 0
    assert m["top1_decided"] == 1.0 and m["top1"] >= 0.9, m


@pytest.mark.parametrize("tag", ["small", "full"])
def test_fp8_against_reference(f8nets, tag):
    net, _, _ = f8nets[tag]
    for case in CASES[tag]:
        b, ref = golden_case(case)
        got = run(net, b)
        m = metrics((ref["pol"], ref["val"], ref["qv"]), got, b["widths"])
        mw = metrics((ref["pol_e4m3w"], ref["val_e4m3w"], ref["qv_e4m3w"]), got, b["widths"])
        mq = metrics((ref["pol"], ref["val"], ref["qv"]),
                     (ref["pol_e4m3w"], ref["val_e4m3w"], ref["qv_e4m3w"]), b["widths"])
        print(case, "e4m3 vs fp32 model", m)
        print(case, "e4m3 vs e4m3-weight model", mw)
        print(case, "e4m3-weight model vs fp32 model (weight rounding alone)", mq)
        for key, lim in TOL_FP32.items():
            assert m[key] <= lim, (case, key, m[key])
        assert m["nonfinite"] == 0 and m["pad_nonzero"] == 0
        # replays are bit-identical
        again = run(net, b)
        for x, y in zip(got, again):
            assert np.array_equal(x, y)


def test_row_order_does_not_change_outputs_f8(k, f8nets, tmp_path, monkeypatch):
    """The FP8 pass with every kernel walking its rows forward (MAYFLY_CUDANET_ORDER=fwd) gives the same bits as
    the default, which alternates the order along each layer's chain (438 boards)."""
    from mayfly_chess_b200 import quant
    net, st, _ = f8nets["full"]
    b, _ = golden_case("full_seed1_fixed")
    want = net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    path = str(tmp_path / "full_e4m3.cnw")
    quant.write_e4m3(path, st, W.FULL, quant.calibrate(st, W.FULL, _calib_batch()))
    monkeypatch.setenv("MAYFLY_CUDANET_ORDER", "fwd")
    fwd = k.CudaNet(path)
    try:
        got = fwd.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
    finally:
        fwd.close()
    for x, y in zip(want, got):
        assert np.array_equal(x, y)
