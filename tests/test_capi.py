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
