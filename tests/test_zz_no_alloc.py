"""The allocation-free product (cudanet_k_gemm_noalloc) through the C ABI on a B200.

Who needs it: a caller that cannot call cudaMalloc, such as a process whose GPU memory is reserved in full up
front, or a search thread that must not take the device-wide synchronisation an allocation costs while other
batches are in flight. Its only scratch (the kernel's error word) is a static device array shared by every call,
which each call clears in stream order before its launch. So two calls in a row must each give what the ordinary
entry point (cudanet_k_gemm) gives, bit for bit, and what a float32 torch product gives within the GEMM tests'
tolerance. This file is named to run last."""
import ctypes
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


def _ref(A, W, bias, epi, C0):
    """The product in float32: acc + bias, then GELU (epi 1) or the residual add (epi 2)."""
    y = A.float() @ W.float().t() + bias
    if epi == 1:
        y = F.gelu(y)
    if epi == 2:
        y = C0.float() + y
    return y


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_noalloc_matches_ordinary_two_calls(k, dtype, epi):
    g = torch.Generator(device="cuda").manual_seed(11 + epi)
    M, N, K = 4160, 2048, 1024
    for call in range(2):
        A = torch.randn(M, K, device="cuda", generator=g).to(dtype)
        W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(dtype)
        bias = torch.randn(N, device="cuda", generator=g) * 0.02
        out_dtype = dtype if epi in (0, 1) else torch.float32
        C0 = torch.randn(M, N, device="cuda", generator=g).to(out_dtype)
        want, got = C0.clone(), C0.clone()      # the residual epilogue adds into C
        k.k_gemm(A, W, bias, want, epi)
        k.k_gemm_noalloc(A, W, bias, got, epi)
        torch.cuda.synchronize()
        # the same kernel on the same inputs: the results agree exactly (within 0, the tightest tolerance)
        assert torch.equal(got, want), f"call {call}: max diff {(got.float() - want.float()).abs().max().item()}"
        assert torch.isfinite(got.float()).all()
        # and the float32 product within the GEMM tests' bar (test_kernels_gpu.test_gemm): 1e-3 absolute for the
        # f32 accumulation order, plus one rounding of a 16-bit output
        rel = 0.0 if epi in (2, 3) else (2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11)
        ref = _ref(A, W, bias, epi, C0)
        excess = ((got.float() - ref).abs() - (1e-3 + rel * ref.abs())).max().item()
        assert math.isfinite(excess) and excess <= 0, f"call {call}: {excess}"


def test_noalloc_rejects_what_the_ordinary_rejects(k):
    A = torch.randn(128, 100, device="cuda").to(torch.bfloat16)      # K not a multiple of 64
    W = torch.randn(256, 100, device="cuda").to(torch.bfloat16)
    b = torch.zeros(256, device="cuda")
    C = torch.empty(128, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="noalloc"):
        k.k_gemm_noalloc(A, W, b, C, 0)
    # a row pitch shorter than a row (ldc < N), through the C function itself: both entry points refuse it on
    # the host, before anything is queued
    lib = k.load()
    A = torch.randn(128, 128, device="cuda").to(torch.bfloat16)
    W = torch.randn(256, 128, device="cuda").to(torch.bfloat16)
    C = torch.zeros(128, 256, device="cuda", dtype=torch.bfloat16)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for fn in (lib.cudanet_k_gemm, lib.cudanet_k_gemm_noalloc):
        err = ctypes.create_string_buffer(256)
        rc = fn(1, 0, 0, A.data_ptr(), W.data_ptr(), b.data_ptr(), C.data_ptr(), 128, 256, 128, 128, stream, err, 256)
        assert rc == -1 and b"ldc < N" in err.value
    torch.cuda.synchronize()
    assert (C == 0).all()
    # and still works afterwards
    want, got = torch.empty_like(C), torch.empty_like(C)
    k.k_gemm(A, W, b, want, 0)
    k.k_gemm_noalloc(A, W, b, got, 0)
    assert torch.equal(got, want)
