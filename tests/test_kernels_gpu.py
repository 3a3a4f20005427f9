"""Single kernels through the C ABI against plain PyTorch fp32 references of the same op (B200 only)."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def k():
    from mayfly_chess_b200 import build, cudanet_py
    build.build()
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return cudanet_py


def _ref_gemm(A, W, bias, epi, C0=None):
    y = A.float() @ W.float().t() + bias
    if epi == 1:
        y = F.gelu(y)
    if epi == 2:
        y = C0 + y
    return y


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
@pytest.mark.parametrize("M,N,K,bn", [(195, 1024, 1024, 0), (4160, 3072, 1024, 256), (1300, 1024, 2048, 128),
                                      (65, 2048, 1024, 64), (300, 8328, 1024, 256), (300, 8324, 1024, 256),
                                      (128, 256, 64, 256),
                                      # CTA pairs (bn 2): 256 x 256 tiles, M and N tails, K = 2048
                                      (4160, 3072, 1024, 2), (300, 8328, 1024, 2), (1300, 1024, 2048, 2),
                                      (65, 512, 128, 2)])
def test_gemm(k, dtype, epi, M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K + epi)
    A = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(dtype)
    bias = torch.randn(N, device="cuda", generator=g) * 0.02
    if epi in (0, 1):
        if N % 8:
            pytest.skip("16-bit output rows must be whole 16-byte units (the heads' 8,324 columns are f32)")
        # a padded pitch: the padding must never be written
        Cfull = torch.full((M, N + 8), float("nan"), device="cuda", dtype=dtype)
        C = Cfull[:, :N]
    elif epi == 2:
        C = torch.randn(M, N, device="cuda", generator=g)
    else:
        Cfull = torch.full((M, N + 4), float("nan"), device="cuda")
        C = Cfull[:, :N]
    C0 = C.clone()
    k.k_gemm(A, W, bias, C, epi, bn)
    torch.cuda.synchronize()
    ref = _ref_gemm(A, W, bias, epi, C0.float())
    if epi != 2:
        assert torch.isnan(Cfull[:, N:]).all()
    # f32 accumulation of K products of 16-bit inputs (summation order differs from torch's: 1e-3 absolute),
    # and 16-bit outputs add one rounding of the result (half an ulp: 2^-9 relative for bf16, 2^-12 for f16)
    rel = 0.0 if epi in (2, 3) else (2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11)
    excess = ((C.float() - ref).abs() - (1e-3 + rel * ref.abs())).max().item()
    assert math.isfinite(excess) and excess <= 0, excess


def test_gelu_epilogue_is_exact_erf_gelu(k):
    """The GELU epilogue against F.gelu (exact erf) over a dense range: an identity W makes acc = A exactly, so
    every f16 value of x in [-10, 10) goes through the epilogue once; the f16 output must be the correctly
    rounded exact GELU to within one f16 unit in the last place."""
    K = 1024
    x = torch.arange(-10.0, 10.0, 20.0 / (256 * K), device="cuda").to(torch.float16).view(256, K)
    W = torch.eye(K, device="cuda", dtype=torch.float16)
    b = torch.zeros(K, device="cuda")
    C = torch.empty(256, K, device="cuda", dtype=torch.float16)
    k.k_gemm(x, W, b, C, 1)
    torch.cuda.synchronize()
    ref = exact_gelu(x).float()
    ulp = torch.clamp(ref.abs(), min=2.0 ** -14) * 2.0 ** -10
    assert ((C.float() - ref).abs() <= ulp + 1e-7).all()


def exact_gelu(x):
    """x * Phi(x) in float64 as x * erfc(-x / sqrt(2)) / 2: F.gelu's x * (1 + erf(x / sqrt(2))) / 2 cancels to
    exactly 0 in float64 once x < -8.3 (erf rounds to -1), where GELU is still about -1e-16."""
    xd = x.double()
    return 0.5 * xd * torch.special.erfc(-xd / math.sqrt(2.0))


def test_gelu_epilogue_bf16_every_value(k):
    """The bf16 GELU epilogue (the one the bf16 passes run) on every bf16 value x with 2^-60 <= |x| < 10, and 0:
    an identity W makes acc = x exactly, and the bf16 output must be within one bf16 unit in the last place of the
    exact-erf GELU (exact_gelu, float64) everywhere, the far negative tail included (|GELU| ~ 1e-22 at -10).
    Below 2^-60 GELU is x / 2 to far better than a bf16 ulp."""
    K = 1024
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float()
    keep = torch.isfinite(bits) & (bits.abs() < 10) & ((bits.abs() >= 2.0 ** -60) | (bits == 0))
    vals = bits[keep]
    n = (vals.numel() + K - 1) // K * K
    x = torch.zeros(n).index_copy_(0, torch.arange(vals.numel()), vals).view(-1, K).cuda().to(torch.bfloat16)
    W = torch.eye(K, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(K, device="cuda")
    C = torch.empty(x.shape[0], K, device="cuda", dtype=torch.bfloat16)
    k.k_gemm(x, W, b, C, 1)
    torch.cuda.synchronize()
    ref = exact_gelu(x).float()
    ulp = torch.clamp(ref.abs(), min=2.0 ** -126) * 2.0 ** -7
    err = (C.float() - ref).abs()
    assert (err <= ulp).all(), (err / ulp).max().item()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_repeatable(k, dtype):
    A = torch.randn(4160, 1024, device="cuda").to(dtype)
    W = (torch.randn(2048, 1024, device="cuda") * 0.02).to(dtype)
    b = torch.zeros(2048, device="cuda")
    C1 = torch.empty(4160, 2048, device="cuda", dtype=dtype)
    C2 = torch.empty_like(C1)
    k.k_gemm(A, W, b, C1, 1)
    k.k_gemm(A, W, b, C2, 1)
    assert torch.equal(C1, C2)


@pytest.mark.parametrize("kernel", ["default", "tc", "mma", "tc4"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d,heads", [(1024, 16), (256, 8)])
@pytest.mark.parametrize("B", [1, 3, 64, 300])
def test_attention(k, kernel, dtype, d, heads, B):
    """The evaluator's attention kernel, and each kernel for head width 64 on its own: the mma.sync kernel and
    the two- and four-group tensor-memory kernels."""
    if kernel != "default" and d // heads != 64:
        pytest.skip("the kernels chosen by name are the head-width-64 ones")
    rows = B * 65
    torch.manual_seed(1000 * B + d)
    qkv = torch.randn(rows, 3 * d, device="cuda").to(dtype)
    att = torch.full((rows, d), float("nan"), device="cuda", dtype=dtype)
    if kernel in ("mma", "tc4"):
        k.k_attention_kernel(qkv, att, B, d, heads, 0 if kernel == "mma" else 4)
    else:
        (k.k_attention_tc if kernel == "tc" else k.k_attention)(qkv, att, B, d, heads)
    torch.cuda.synchronize()
    dh = d // heads
    q, kk, v = qkv.float().view(B, 65, 3, heads, dh).permute(2, 0, 3, 1, 4).unbind(0)
    p = torch.softmax(q @ kk.transpose(-1, -2) / math.sqrt(dh), -1)
    ref = (p @ v).transpose(1, 2).reshape(rows, d)
    pv_abs = (p @ v.abs()).transpose(1, 2).reshape(rows, d)
    # P is rounded to 16 bits (unit roundoff u) before the second product, which moves an output by at most
    # u * sum_j p_j |v_j|; the output is rounded once more (u |o|); the rest (f32 sums, 2^x) is far below 1e-4
    u = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    excess = ((att.float() - ref).abs() - (u * (pv_abs + ref.abs()) + 1e-4)).max().item()
    assert math.isfinite(excess) and excess <= 0, excess


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d,heads", [(1024, 16), (256, 8)])
@pytest.mark.parametrize("B", [1, 3, 300])
def test_attention_cls(k, dtype, d, heads, B):
    """The last layer's attention for each board's CLS query only, against the full attention's row 0."""
    rows = B * 65
    qkv = torch.randn(rows, 3 * d, device="cuda").to(dtype)
    att = torch.full((B, d), float("nan"), device="cuda", dtype=dtype)
    k.k_attention_cls(qkv, att, B, d, heads)
    torch.cuda.synchronize()
    dh = d // heads
    q, kk, v = qkv.float().view(B, 65, 3, heads, dh).permute(2, 0, 3, 1, 4).unbind(0)
    o = torch.softmax(q[:, :, :1] @ kk.transpose(-1, -2) / math.sqrt(dh), -1) @ v     # (B, heads, 1, dh)
    ref = o.reshape(B, d)
    # f32 dot products and probabilities (no 16-bit rounding of P), one rounding of the output
    rel = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    excess = ((att.float() - ref).abs() - (1e-4 + rel * ref.abs())).max().item()
    assert math.isfinite(excess) and excess <= 0, excess


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [256, 1024])
@pytest.mark.parametrize("stride", [1, 65])
def test_layernorm(k, dtype, d, stride):
    n = 300
    x = torch.randn(n * stride, d, device="cuda") * 3 + 0.5
    g = torch.randn(d, device="cuda")
    b = torch.randn(d, device="cuda")
    h = torch.empty(n, d, device="cuda", dtype=dtype)
    k.k_layernorm(x, g, b, h, n, d, stride)
    torch.cuda.synchronize()
    ref = F.layer_norm(x[::stride], (d,), g, b, 1e-5)
    rel = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11      # one rounding of the output
    excess = ((h.float() - ref).abs() - (1e-4 + rel * ref.abs())).max().item()
    assert excess <= 0, excess


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(195, 1024, 1024), (4160, 1024, 2048), (1300, 512, 1024), (300, 256, 1024),
                                   (66560, 1024, 1024)])
def test_gemm_resln(k, dtype, M, N, K):
    """The residual product fused with the next LayerNorm (clusters of N / 256 CTAs exchanging row statistics)."""
    g0 = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g0).to(dtype)
    W = (torch.randn(N, K, device="cuda", generator=g0) * 0.02).to(dtype)
    bias = torch.randn(N, device="cuda", generator=g0) * 0.02
    X = torch.randn(M, N, device="cuda", generator=g0) * 3 + 0.5
    g = torch.randn(N, device="cuda", generator=g0)
    b = torch.randn(N, device="cuda", generator=g0)
    H = torch.full((M, N), float("nan"), device="cuda", dtype=dtype)
    X0 = X.clone()
    k.k_gemm_resln(A, W, bias, X, g, b, H)
    torch.cuda.synchronize()
    xr = X0 + (A.float() @ W.float().t() + bias)
    assert (X - xr).abs().max().item() < 2e-3
    hr = F.layer_norm(X, (N,), g, b, 1e-5)          # normalise the kernel's own X: isolates the LayerNorm
    rel = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    excess = ((H.float() - hr).abs() - (2e-4 + rel * hr.abs())).max().item()
    assert math.isfinite(excess) and excess <= 0, excess
