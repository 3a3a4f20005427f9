"""The C ABI library: it loads without a GPU, exports every entry point include/cudanet_b200.h declares, and
fails loudly (NULL / -1 with a reason) where it cannot work. No compute call is made here."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "cudanet_b200.h")
REFERENCE_ABI = ["cudanet_create", "cudanet_evaluate", "cudanet_fingerprint", "cudanet_max_batch",
                 "cudanet_profile", "cudanet_profile_names", "cudanet_destroy"]


def declared():
    text = open(HEADER).read()
    return re.findall(r"CUDANET_API\s+[\w\s\*]+?\b(cudanet_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    from mayfly_chess_b200 import build, cudanet_py
    build.build()
    return cudanet_py.load()


def test_header_declares_reference_abi():
    names = declared()
    for n in REFERENCE_ABI:
        assert n in names
    assert len(names) == len(set(names))


def test_every_declared_symbol_is_exported(lib):
    for n in declared():
        assert hasattr(lib, n), n


def test_profile_names(lib):
    buf = ctypes.create_string_buffer(512)
    n = lib.cudanet_profile_names(buf, len(buf))
    names = buf.value.decode().split(",")
    assert n == len(buf.value)
    assert names == ["embed", "ln1", "qkv", "attention", "out", "ln2", "ff1", "gelu", "ff2", "cls_ln", "heads",
                     "graph_pass"]


def test_null_handles(lib):
    buf = ctypes.create_string_buffer(64)
    assert lib.cudanet_max_batch(None) == -1
    assert lib.cudanet_fingerprint(None, buf, len(buf)) == -1
    lib.cudanet_destroy(None)      # never fails
    err = ctypes.create_string_buffer(256)
    assert lib.cudanet_evaluate(None, 1, 1, None, None, None, None, None, None, None, None, None, err, 256) == -1
    assert b"null handle" in err.value


def test_create_fails_with_a_reason(lib, tmp_path):
    err = ctypes.create_string_buffer(512)
    assert not lib.cudanet_create(None, 0, err, 512)
    assert err.value
    err = ctypes.create_string_buffer(512)
    assert not lib.cudanet_create(str(tmp_path / "missing.cnw").encode(), 0, err, 512)
    assert err.value          # no device here, or no such file: either way a reason comes back


def test_error_text_is_cut_to_err_len(lib):
    err = ctypes.create_string_buffer(8)
    lib.cudanet_evaluate(None, 1, 1, None, None, None, None, None, None, None, None, None, err, 8)
    assert len(err.value) == 7


def test_python_wrapper_fails_loudly_without_library(tmp_path):
    from mayfly_chess_b200 import cudanet_py
    with pytest.raises(FileNotFoundError):
        cudanet_py.CudaNet(str(tmp_path / "x.cnw"), dll=str(tmp_path / "nolib.so"))


def test_python_wrapper_checks_inputs_as_the_reference_does():
    """CudaNet's argument checks (mayfly/chess/cudanet/cudanet_py.py:105-133): the same exceptions and messages,
    run on a handle object that never reaches the library."""
    import numpy as np
    from mayfly_chess_b200 import cudanet_py
    net = object.__new__(cudanet_py.CudaNet)
    net._h, net.max_batch = None, 4
    ok = dict(ids=np.zeros((2, 64), np.int64), cast=np.zeros((2, 4), np.float32), hm=np.zeros(2, np.int64),
              ep=np.zeros(2, np.int64), I=np.zeros((2, 3), np.int64), M=np.ones((2, 3), bool))
    with pytest.raises(RuntimeError, match="CudaNet is closed"):
        net._inputs(**ok)
    net._h = ctypes.c_void_p(1)
    B, wide, ids, cast, hm, ep, I, M = net._inputs(**ok)
    assert (B, wide) == (2, 3) and M.dtype == np.uint8 and ids.flags.c_contiguous
    assert M.base is not None or M.ctypes.data == ok["M"].ctypes.data     # a bool mask is viewed, not copied
    with pytest.raises(ValueError, match=r"I: shape \(6,\), expected \(B, wide\)"):
        net._inputs(**{**ok, "I": np.zeros(6, np.int64)})
    with pytest.raises(ValueError, match=r"batch 5: cudanet takes 1 to 4 \(env MAYFLY_CUDANET_MAX_BATCH\)"):
        net._inputs(**{**ok, "I": np.zeros((5, 3), np.int64)})
    with pytest.raises(ValueError, match="wide must be at least 1"):
        net._inputs(**{**ok, "I": np.zeros((2, 0), np.int64)})
    with pytest.raises(ValueError, match=r"cast: shape \(2, 3\), expected \(2, 4\)"):
        net._inputs(**{**ok, "cast": np.zeros((2, 3), np.float32)})
    # Fortran-ordered or other-typed inputs are converted, not refused
    _, _, ids2, *_ = net._inputs(**{**ok, "ids": np.asfortranarray(np.ones((2, 64), np.int32))})
    assert ids2.dtype == np.int64 and ids2.flags.c_contiguous and (ids2 == 1).all()
