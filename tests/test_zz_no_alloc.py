"""The allocation-free product (cudanet_k_gemm_noalloc) against the ordinary one (cudanet_k_gemm), through the
C ABI on a B200. It exists for callers that cannot call cudaMalloc: a process whose GPU memory is reserved up
front, or a search thread that must not stall in-flight batches on an allocation. Its scratch (the kernel's error
word) is a static device array, so this checks that two calls in a row each give the ordinary entry point's
result, with the word from the first call not leaking into the second. This file is named to run last."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def k():
    from mayfly_chess_b200 import build, cudanet_py
    build.build()
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return cudanet_py


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


def test_noalloc_rejects_what_the_ordinary_rejects(k):
    A = torch.randn(128, 100, device="cuda").to(torch.bfloat16)      # K not a multiple of 64
    W = torch.randn(256, 100, device="cuda").to(torch.bfloat16)
    b = torch.zeros(256, device="cuda")
    C = torch.empty(128, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="noalloc"):
        k.k_gemm_noalloc(A, W, b, C, 0)
    # and still works afterwards
    A = torch.randn(128, 128, device="cuda").to(torch.bfloat16)
    W = torch.randn(256, 128, device="cuda").to(torch.bfloat16)
    want, got = torch.empty_like(C), torch.empty_like(C)
    k.k_gemm(A, W, b, want, 0)
    k.k_gemm_noalloc(A, W, b, got, 0)
    assert torch.equal(got, want)
