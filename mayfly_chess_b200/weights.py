"""The network's architecture numbers, its seeded random-init weights, and the weight file the evaluator loads.

Weight file (".cnw"), after mayfly/chess/cudanet/cudanet_spec.h:35-55 and cudanet/export_cudanet.py:149-196:
    bytes 0..7   magic b"MFCNW001"
    bytes 8..11  uint32 little endian, length of the JSON header that follows
    JSON header  {"version", "d", "layers", "heads", "ff", "tokens", "moves", "fingerprint", "source",
                  "tensors": [{"name", "dtype", "shape", "offset", "nbytes"}, ...]}
    zero padding to a multiple of 256 (the data start), then every tensor at a 256-aligned offset from it.
Version 1 is the reference's file: the five big matrices of a layer and heads_w in "f16", the rest "f32".
Version 2 is this evaluator's: the same names and layout, with the matrices in "bf16" (raw bits, round to
nearest even from fp32), or in "e4m3" (float8 e4m3fn) each with a "<name>_scale" f32 [out] tensor holding the
per-output-channel scale (absmax / 448), so that W[o, :] ~= scale[o] * e4m3[o, :]. Version 2 also records
"precision" ("bf16" or "e4m3"). An e4m3 file also holds, per layer, "L<i>.act_scale" f32 [4]: the static
scales of the inputs of the layer's four products (qkv, out, ff1, ff2), x ~= act_scale * e4m3, set from
ranges measured on calibration positions (ACT_HEADROOM x max |x| / 448). The heads stay bf16 in an e4m3 file.
The evaluator accepts both versions and runs its products in the file's type: a version 1 file in f16 (as the
reference backend does), a bf16 file in bf16, an e4m3 file's layer products on e4m3 operands.

Random init (the seeded weights every parity test and the bench use): a ChessNet(d, nhead, layers, dim_ff,
qhead=True) state dict (mayfly/chess/chess_net.py:89-119) in its own order. Every LayerNorm weight is 1 and bias
0 (no draws); every other floating-point tensor, in state dict order, is drawn N(0, 0.02) from one
torch.Generator seeded with `seed` (torch.randn * 0.02). The heads the search does not read (value and the
auxiliary heads) are drawn too, so the stream matches the reference model's parameter list exactly.
"""
import hashlib
import json
import os
import struct
from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch

MAGIC = b"MFCNW001"
ALIGN = 256
N_MOVES = 4162          # mayfly/chess/moves.py:32 (4,096 from-to + 66 underpromotions)
TOKENS = 65             # CLS + 64 squares (chess_net.py:190-192)
HM_BUCKETS = 102        # chess_net.py:115
PIECES = 13             # chess_net.py:93
MATRICES = ("qkv_w", "out_w", "ff1_w", "ff2_w")
E4M3_MAX = 448.0
# An activation scale maps ACT_HEADROOM x the calibrated max |x| to 448, so that positions a little outside the
# calibration set's range are not clipped. e4m3's relative precision is the same across its normal range (3
# mantissa bits), so the headroom costs only the bottom binade.
ACT_HEADROOM = 2.0


@dataclass(frozen=True)
class Arch:
    d: int
    layers: int
    heads: int
    ff: int
    tokens: int = TOKENS
    moves: int = N_MOVES

    @property
    def dh(self):
        return self.d // self.heads


# the search's network (cudanet/cudanet_spec.h:22-31, train_av.py:60-61) and the CPU correctness config
FULL = Arch(d=1024, layers=16, heads=16, ff=2048)
SMALL = Arch(d=256, layers=4, heads=8, ff=1024)


def state_spec(arch):
    """[(name, shape)] of ChessNet(d, nhead, layers, dim_ff, qhead=True)'s floating-point state dict, in order.

    Module.state_dict saves a module's own parameters, then its buffers, then its children in registration
    order (chess_net.py:93-119; nn.TransformerEncoderLayer registers self_attn, linear1, linear2, norm1, norm2).
    The int64 buffer posidx is not floating point and is left out."""
    d, ff, m = arch.d, arch.ff, arch.moves
    spec = [("cls", (1, 1, d)), ("ep_mark", (d,)),
            ("piece.weight", (PIECES, d)), ("pos.weight", (64, d)),
            ("cast.weight", (d, 4)), ("cast.bias", (d,))]
    for i in range(arch.layers):
        p = f"enc.layers.{i}."
        spec += [(p + "self_attn.in_proj_weight", (3 * d, d)), (p + "self_attn.in_proj_bias", (3 * d,)),
                 (p + "self_attn.out_proj.weight", (d, d)), (p + "self_attn.out_proj.bias", (d,)),
                 (p + "linear1.weight", (ff, d)), (p + "linear1.bias", (ff,)),
                 (p + "linear2.weight", (d, ff)), (p + "linear2.bias", (d,)),
                 (p + "norm1.weight", (d,)), (p + "norm1.bias", (d,)),
                 (p + "norm2.weight", (d,)), (p + "norm2.bias", (d,))]
    spec += [("ln.weight", (d,)), ("ln.bias", (d,)),
             ("policy.weight", (m, d)), ("policy.bias", (m,)),
             ("value.weight", (1, d)), ("value.bias", (1,)),
             ("qvalue.weight", (m, d)), ("qvalue.bias", (m,)),
             ("h_material.weight", (2, d)), ("h_material.bias", (2,)),
             ("h_king.weight", (2, d)), ("h_king.bias", (2,)),
             ("h_pawns.weight", (6, d)), ("h_pawns.bias", (6,)),
             ("h_mob.weight", (1, d)), ("h_mob.bias", (1,)),
             ("h_bishop.weight", (2, d)), ("h_bishop.bias", (2,)),
             ("hm.weight", (HM_BUCKETS, d))]
    return spec


def _is_norm(name):
    return ".norm1." in name or ".norm2." in name or name.startswith("ln.")


def random_state(arch, seed):
    """The seeded N(0, 0.02) state dict (module docstring), fp32 CPU tensors by ChessNet name."""
    g = torch.Generator().manual_seed(int(seed))
    out = OrderedDict()
    for name, shape in state_spec(arch):
        if _is_norm(name):
            out[name] = torch.ones(shape) if name.endswith("weight") else torch.zeros(shape)
        else:
            out[name] = torch.randn(shape, generator=g, dtype=torch.float32) * 0.02
    return out


def fingerprint(state):
    """mayfly/chess/mcts_cpp.py:121-132: SHA-1 over the names and first 32 float32 values of the first and last
    four floating-point tensors of the state dict."""
    keys = [k for k, v in state.items() if torch.is_tensor(v) and v.is_floating_point()]
    h = hashlib.sha1()
    for k in keys[:4] + keys[-4:]:
        h.update(k.replace("_orig_mod.", "").encode())
        h.update(state[k].detach().flatten()[:32].float().cpu().numpy().tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------------------------------- quantisers
def to_bf16_bits(t):
    """fp32 tensor -> numpy uint16 of its bf16 bits (round to nearest even)."""
    return t.detach().float().contiguous().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def bf16_bits_to_f32(a):
    return torch.from_numpy(np.array(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).float()


def to_e4m3(t):
    """fp32 [out, in] -> (uint8 e4m3fn bits [out, in], f32 scale [out]), per-output-channel absmax / 448.
    A row of zeros gets scale 1."""
    w = t.detach().float()
    amax = w.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (w / scale[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).numpy(), scale.numpy().astype("<f4")


def act_scales(act_amax, arch):
    """The per-layer input scales [layers, 4] an e4m3 file stores, from calibrated max |x| [layers, 4]."""
    a = np.asarray(act_amax, np.float32)
    if a.shape != (arch.layers, 4) or not np.all(np.isfinite(a)) or np.any(a < 0):
        raise ValueError(f"act_amax: needs finite non-negative [{arch.layers}, 4], got {a.shape}")
    return np.where(a > 0, a * ACT_HEADROOM / E4M3_MAX, 1.0).astype("<f4")


def e4m3_to_f32(bits, scale):
    q = torch.from_numpy(np.array(bits, dtype=np.uint8)).view(torch.float8_e4m3fn).float()
    return q * torch.from_numpy(np.asarray(scale, np.float32))[:, None]


# ---------------------------------------------------------------------------------------------------- the file
def cnw_tensors(state, arch, precision="bf16", act_amax=None):
    """[(name, dtype, numpy array)] in cudanet_spec.h's order (export_cudanet.py:95-129 tensors), the matrices
    in `precision`: "f16" (the reference's version 1), "bf16" or "e4m3" (version 2, with *_scale tensors and,
    from act_amax [layers, 4], each layer's act_scale)."""
    if precision == "e4m3":
        if act_amax is None:
            raise ValueError("an e4m3 file needs act_amax: the calibrated input ranges (mayfly_chess_b200.quant)")
        acts = act_scales(act_amax, arch)
    def f32(t):
        return np.ascontiguousarray(t.detach().float().cpu().numpy(), dtype="<f4")

    def mat(name, t):
        if precision == "f16":
            return [(name, "f16", np.ascontiguousarray(t.detach().float().half().numpy(), dtype="<f2"))]
        if precision == "bf16":
            return [(name, "bf16", to_bf16_bits(t))]
        if precision == "e4m3":
            q, s = to_e4m3(t)
            return [(name, "e4m3", q), (name + "_scale", "f32", s)]
        raise ValueError(f"precision {precision!r}")

    d = arch.d
    out = [("piece", "f32", f32(state["piece.weight"])), ("pos", "f32", f32(state["pos.weight"])),
           ("cls", "f32", f32(state["cls"].reshape(d))), ("cast_w", "f32", f32(state["cast.weight"])),
           ("cast_b", "f32", f32(state["cast.bias"])), ("hm", "f32", f32(state["hm.weight"])),
           ("ep_mark", "f32", f32(state["ep_mark"]))]
    for i in range(arch.layers):
        p = f"enc.layers.{i}."
        out += [(f"L{i}.n1_g", "f32", f32(state[p + "norm1.weight"])),
                (f"L{i}.n1_b", "f32", f32(state[p + "norm1.bias"]))]
        out += mat(f"L{i}.qkv_w", state[p + "self_attn.in_proj_weight"])
        out += [(f"L{i}.qkv_b", "f32", f32(state[p + "self_attn.in_proj_bias"]))]
        out += mat(f"L{i}.out_w", state[p + "self_attn.out_proj.weight"])
        out += [(f"L{i}.out_b", "f32", f32(state[p + "self_attn.out_proj.bias"])),
                (f"L{i}.n2_g", "f32", f32(state[p + "norm2.weight"])),
                (f"L{i}.n2_b", "f32", f32(state[p + "norm2.bias"]))]
        out += mat(f"L{i}.ff1_w", state[p + "linear1.weight"])
        out += [(f"L{i}.ff1_b", "f32", f32(state[p + "linear1.bias"]))]
        out += mat(f"L{i}.ff2_w", state[p + "linear2.weight"])
        out += [(f"L{i}.ff2_b", "f32", f32(state[p + "linear2.bias"]))]
        if precision == "e4m3":
            out += [(f"L{i}.act_scale", "f32", np.ascontiguousarray(acts[i]))]
    out += [("ln_g", "f32", f32(state["ln.weight"])), ("ln_b", "f32", f32(state["ln.bias"]))]
    # the heads stay 16-bit in every precision: they are 0.1% of the work and set the policy's accuracy
    heads = torch.cat([state["policy.weight"], state["qvalue.weight"]], 0)
    out += mat("heads_w", heads) if precision != "e4m3" else [("heads_w", "bf16", to_bf16_bits(heads))]
    out += [("heads_b", "f32", f32(torch.cat([state["policy.bias"], state["qvalue.bias"]], 0)))]
    return out


def _align(n):
    return (n + ALIGN - 1) // ALIGN * ALIGN


def write_cnw(path, state, arch, precision="bf16", source="random-init", act_amax=None):
    """Write the weight file for `state` (export_cudanet.py:149-173 write_cnw), returning its header."""
    arrays = cnw_tensors(state, arch, precision, act_amax)
    entries, off = [], 0
    for name, dt, a in arrays:
        off = _align(off)
        entries.append({"name": name, "dtype": dt, "shape": list(a.shape), "offset": off, "nbytes": int(a.nbytes)})
        off += a.nbytes
    hdr = {"version": 1 if precision == "f16" else 2, "d": arch.d, "layers": arch.layers, "heads": arch.heads,
           "ff": arch.ff, "tokens": arch.tokens, "moves": arch.moves, "fingerprint": fingerprint(state),
           "source": source}
    if precision != "f16":
        hdr["precision"] = precision
    hdr["tensors"] = entries
    js = json.dumps(hdr, separators=(",", ":")).encode("ascii")
    start = _align(8 + 4 + len(js))
    part = path + ".part"
    with open(part, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<I", len(js)))
        f.write(js)
        f.write(b"\0" * (start - f.tell()))
        for e, (_, _, a) in zip(entries, arrays):
            f.write(b"\0" * (start + e["offset"] - f.tell()))
            f.write(np.ascontiguousarray(a).tobytes())
        f.write(b"\0" * (_align(f.tell()) - f.tell()))
    os.replace(part, path)
    return hdr


_NP = {"f16": "<f2", "f32": "<f4", "bf16": "<u2", "e4m3": "u1"}


def read_cnw(path):
    """(header, {name: numpy array}) of a weight file (export_cudanet.py:176-196 read_cnw); bf16 comes back as
    uint16 bits and e4m3 as uint8 bits."""
    with open(path, "rb") as f:
        raw = f.read()
    if raw[:8] != MAGIC:
        raise ValueError(f"{path}: bad magic {raw[:8]!r}")
    (n,) = struct.unpack("<I", raw[8:12])
    if 12 + n > len(raw):
        raise ValueError(f"{path}: header runs past the end")
    hdr = json.loads(raw[12:12 + n].decode("ascii"))
    start = _align(12 + n)
    out = {}
    for e in hdr["tensors"]:
        dt = np.dtype(_NP[e["dtype"]])
        count = int(np.prod(e["shape"])) if e["shape"] else 1
        if e["offset"] % ALIGN or e["nbytes"] != count * dt.itemsize:
            raise ValueError(f"{path}: tensor {e['name']} misaligned or wrong size")
        if start + e["offset"] + e["nbytes"] > len(raw):
            raise ValueError(f"{path}: tensor {e['name']} runs past the end")
        out[e["name"]] = np.frombuffer(raw, dtype=dt, count=count, offset=start + e["offset"]).reshape(e["shape"])
    return hdr, out


def dequantised_state(state, arch, precision):
    """The fp32 state the evaluator effectively holds at `precision`: every matrix the weight file stores in
    16 or 8 bits replaced by its rounded value (used to separate rounding error from kernel error)."""
    out = OrderedDict((k, v.clone()) for k, v in state.items())
    names = {"qkv_w": "self_attn.in_proj_weight", "out_w": "self_attn.out_proj.weight",
             "ff1_w": "linear1.weight", "ff2_w": "linear2.weight"}
    for i in range(arch.layers):
        for short, long in names.items():
            k = f"enc.layers.{i}.{long}"
            if precision == "bf16":
                out[k] = bf16_bits_to_f32(to_bf16_bits(state[k]))
            elif precision == "e4m3":
                out[k] = e4m3_to_f32(*to_e4m3(state[k]))
            elif precision == "f16":
                out[k] = state[k].half().float()
    for k in ("policy.weight", "qvalue.weight"):
        out[k] = state[k].half().float() if precision == "f16" else bf16_bits_to_f32(to_bf16_bits(state[k]))
    return out
