"""The FP8 (e4m3) weight file: per-output-channel weight scales and static per-layer input scales.

The weight scales come from the weights alone (absmax / 448 per output channel, weights.to_e4m3). The input
scales of the four layer products (qkv, out, ff1, ff2) are static: they come from the ranges the 16-bit
evaluator measures on calibration positions (CudaNet.calibrate, one pass on the GPU), so the e4m3 pass
quantises each product's input in its producer's epilogue with no extra pass over the activations.

    amax = calibrate(state, arch, positions, device=0)       # float32 [layers, 4]
    write_e4m3(path, state, arch, amax)
"""
import os
import tempfile

from . import weights as W
from .cudanet_py import CudaNet


def calibrate(state, arch, batch, device=0, dll=None):
    """max |x| of each layer's four product inputs over the positions of `batch` (a dict with ids, cast, hm,
    ep as CudaNet.evaluate takes them), measured by the bf16 evaluator on `device`."""
    fd, path = tempfile.mkstemp(suffix=".cnw")
    os.close(fd)
    try:
        W.write_cnw(path, state, arch, "bf16")
        with CudaNet(path, device, dll) as net:
            return net.calibrate(batch["ids"], batch["cast"], batch["hm"], batch["ep"])
    finally:
        os.remove(path)


def write_e4m3(path, state, arch, act_amax, source="random-init"):
    """The e4m3 weight file of `state` with input scales from `act_amax` (calibrate's result)."""
    return W.write_cnw(path, state, arch, "e4m3", source=source, act_amax=act_amax)
