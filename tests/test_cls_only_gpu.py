"""The last layer run for the CLS rows only (the heads read nothing else, chess_net.py:194) against the whole last
layer (MAYFLY_CUDANET_CLS_ONLY=0), in both precisions and at batch sizes that give the B-row products their
smallest and their pair tiles. The switch is read once per process, so each setting runs in its own child
process on the same weight file and inputs; the outputs must agree to rounding (the CLS-query attention kernel
sums in another order than the full attention kernel)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import GOLDEN, REPO

CHILD = r"""
import sys, numpy as np
sys.path.insert(0, sys.argv[1])
from mayfly_chess_b200.cudanet_py import CudaNet
from mayfly_chess_b200.inputs import PositionSet
b = PositionSet(sys.argv[3]).batch(0, int(sys.argv[4]))
with CudaNet(sys.argv[2]) as net:
    pol, val, qv = net.evaluate(b["ids"], b["cast"], b["hm"], b["ep"], b["I"], b["M"])
np.savez(sys.argv[5], pol=pol, val=val, qv=qv)
"""


def run(path, B, cls_only, out):
    env = dict(os.environ, MAYFLY_CUDANET_CLS_ONLY="1" if cls_only else "0")
    subprocess.run([sys.executable, "-c", CHILD, REPO, path, os.path.join(GOLDEN, "positions_seed1.npz"), str(B),
                    out], env=env, check=True, timeout=600)
    z = np.load(out)
    return z["pol"], z["val"], z["qv"]


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mayfly_chess_b200 import weights as W
    d = tmp_path_factory.mktemp("clsonly")
    st = W.random_state(W.FULL, 1)
    p16 = str(d / "full_bf16.cnw")
    W.write_cnw(p16, st, W.FULL, "bf16")
    return d, p16


@pytest.mark.gpu
@pytest.mark.parametrize("B", [3, 300])
def test_cls_only_last_layer_matches_the_whole_layer(files, B):
    d, path = files
    a = run(path, B, True, str(d / f"a{B}.npz"))
    b = run(path, B, False, str(d / f"b{B}.npz"))
    np.testing.assert_allclose(a[0], b[0], atol=5e-3, rtol=0)     # policy logits at the legal moves
    np.testing.assert_allclose(a[1], b[1], atol=2e-3, rtol=0)     # value
    np.testing.assert_allclose(a[2], b[2], atol=2e-3, rtol=0)     # per-move q
    print(f"\nB={B}: CLS-only vs whole last layer, policy max |d| {np.abs(a[0] - b[0]).max():.2e}, "
          f"val {np.abs(a[1] - b[1]).max():.2e}, q {np.abs(a[2] - b[2]).max():.2e}")
