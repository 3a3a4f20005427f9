"""Shared fixtures. GPU tests are marked `gpu` and need a B200; everything else runs on the CPU."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def meta():
    with open(os.path.join(GOLDEN, "meta.json")) as f:
        return json.load(f)


def golden_case(name):
    """(batch dict, reference outputs dict) of a committed fixture."""
    from mayfly_chess_b200.inputs import PositionSet
    path = os.path.join(GOLDEN, name + ".npz")
    ps = PositionSet(path)
    z = np.load(path)
    packed = {"ids", "cast", "hm", "ep", "widths", "moves"}
    ref = {k: z[k] for k in z.files if k not in packed}
    return ps.batch(0, len(ps)), ref


@pytest.fixture(scope="session")
def chesscore():
    """The reference's chess core (oracle/_ref), built by oracle/Makefile from the reference checkout when it is
    missing (where there is no checkout the build fails and the tests that need it are skipped)."""
    lib = os.path.join(REPO, "oracle", "_ref", "libchesscore.so")
    if not os.path.exists(lib):
        ref = os.environ.get("MAYFLY_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference")
        subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), f"REF={ref}"], capture_output=True)
    if not os.path.exists(lib):
        pytest.skip("oracle/_ref/libchesscore.so not built and no reference checkout to build it from")
    from oracle import positions
    return positions


@pytest.fixture(autouse=True)
def _seeded(request):
    """Every test draws its random inputs from a seed fixed by its own name, so a run is repeatable."""
    import zlib
    seed = zlib.crc32(request.node.nodeid.encode()) & 0x7FFFFFFF
    np.random.seed(seed)
    try:
        import torch
        torch.manual_seed(seed)
    except ImportError:
        pass
    yield


def golden_b1024():
    """(batch dict, reference outputs dict) of full_seed1_b1024.npz: positions_seed1.npz rows 0..1023 as one
    padded batch, and the fixture's flattened legal-move outputs re-padded to it (0 on padding)."""
    from mayfly_chess_b200.inputs import PositionSet
    z = np.load(os.path.join(GOLDEN, "full_seed1_b1024.npz"))
    ps = PositionSet(os.path.join(GOLDEN, "positions_seed1.npz"))
    widths = z["widths"].astype(np.int64)
    b = ps.batch(int(z["first_row"]), len(widths))
    assert np.array_equal(b["widths"], widths), "the fixture's rows are not the position set's"
    ref = {}
    for k in z.files:
        if k.startswith(("pol", "qv")):
            ref[k] = np.zeros(b["I"].shape, np.float32)
            ref[k][b["M"]] = z[k]
        elif k.startswith("val"):
            ref[k] = z[k]
    return b, ref
