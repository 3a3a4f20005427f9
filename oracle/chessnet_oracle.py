"""TEST INFRASTRUCTURE ONLY: the CPU fp32 oracle of MayFly's batched network evaluation.

A plain-torch restatement, on the CPU in float32, of the forward the search calls per leaf batch and of the
search's reduction of the two heads. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
it, as the checker; the product never imports it. It is pinned against the reference's own ChessNet (imported
from the reference checkout) through the committed fixtures under tests/golden/ (make_golden.py).

  forward(state, arch, ids, cast, hm, ep) -> (policy [B, 4162], qvalue [B, 4162])
      mayfly/chess/chess_net.py:176-204 ChessNet.forward, with the encoder layer written out as
      chess_net.py:148-165 _encode_sdpa writes it (pre-norm nn.TransformerEncoderLayer, exact erf GELU, LN eps
      1e-5, no final encoder norm), then the final LayerNorm on the CLS row (chess_net.py:194) and the policy
      and qvalue heads (chess_net.py:199-204). cpp/export_ts.py:63-70 Export returns the same pair.
  post(policy, qvalue, I, M) -> (pol [B, wide], val [B], qv [B, wide])
      cpp/export_ts.py:147-156 post (= mcts.py:1152-1164 _collect) with the evaluator's padding convention
      (cudanet/kernels_heads.cu:88-143): pol and qv are 0 on padding, a row with no legal move gets val = -1.

The FP8 evaluator has no counterpart in the reference (its FP8 study was a simulation,
mayfly/docs/cuda_backend.md:150-152). For it, forward takes two options: `act` [layers, 4] rounds the input
of each layer's four products (qkv, out, ff1, ff2) to e4m3 at that static scale, as the evaluator's producers
do (with the weight matrices already e4m3-rounded by weights.dequantised_state, this is the FP8 pass in fp32
arithmetic); `resid_bf16` keeps the residual stream in bf16 as the FP8 evaluator stores it: the embedding is
rounded to bf16, and each residual add rounds the product's output v to bf16 and then the sum (the evaluator adds
bf16(v) into the stream with a bf16 reduction in memory); `record` [layers, 4] receives max |.| of those inputs
(what the evaluator's calibration measures).

The reference's Python search plays a bf16 autocast pass of the same module on the GPU (mayfly/chess/mcts.py:
1296-1318, torch.autocast("cuda", torch.bfloat16) around ChessNet.forward), which its own parity check uses as the
yardstick a backend must be no worse than (cudanet/test_cudanet.py:323-340). forward(..., device="cuda",
autocast_bf16=True) runs this restatement that way: under autocast, with attention through
F.scaled_dot_product_attention as nn.MultiheadAttention and chess_net.py:160 compute it.
"""
import contextlib
import math

import torch
import torch.nn.functional as F

LN_EPS = 1e-5


def embed(state, arch, ids, cast, hm, ep):
    """chess_net.py:182-192: piece + square embeddings, the en passant mark, and the CLS token."""
    d = arch.d
    B = ids.shape[0]
    x = state["piece.weight"][ids] + state["pos.weight"][None]                 # (B, 64, d)
    has = (ep > 0).to(x.dtype)[:, None]
    rows = torch.arange(B, device=x.device)
    sq = (ep - 1).clamp(min=0)
    x[rows, sq] = x[rows, sq] + state["ep_mark"] * has
    cls = (state["cls"].reshape(1, 1, d) + F.linear(cast, state["cast.weight"], state["cast.bias"])[:, None, :]
           + state["hm.weight"][hm][:, None, :])
    return torch.cat([cls, x], dim=1)                                            # (B, 65, d)


def fq_e4m3(x, scale):
    """x rounded to the e4m3 grid at `scale`: scale * e4m3(x / scale), round to nearest even, saturating at
    +-448 (the evaluator's cvt.rn.satfinite)."""
    return (x / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float() * scale


def _same(t):
    return t


def _bf16(t):
    return t.bfloat16().float()


def layer(state, arch, i, x, act=None, record=None, resid=_same, sdpa=False):
    """One pre-norm encoder layer (chess_net.py:154-164); act / record as in the module docstring, resid rounds
    the residual stream after each add, sdpa computes attention with F.scaled_dot_product_attention."""
    B, L, d = x.shape
    H, dh = arch.heads, arch.dh
    p = f"enc.layers.{i}."

    def product_input(t, j):
        if record is not None:
            record[i, j] = max(float(record[i, j]), float(t.abs().max()))
        return fq_e4m3(t, float(act[i][j])) if act is not None else t

    h = F.layer_norm(x, (d,), state[p + "norm1.weight"], state[p + "norm1.bias"], LN_EPS)
    qkv = F.linear(product_input(h, 0), state[p + "self_attn.in_proj_weight"], state[p + "self_attn.in_proj_bias"])
    q, k, v = qkv.view(B, L, 3, H, dh).permute(2, 0, 3, 1, 4).unbind(0)         # each (B, H, L, dh)
    if sdpa:
        o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, L, d)
    else:
        s = torch.matmul(q, k.transpose(-1, -2)) * (1.0 / math.sqrt(dh))
        o = torch.matmul(torch.softmax(s, dim=-1), v).transpose(1, 2).reshape(B, L, d)
    x = resid(x + resid(F.linear(product_input(o, 1), state[p + "self_attn.out_proj.weight"],
                                 state[p + "self_attn.out_proj.bias"])))
    h = F.layer_norm(x, (d,), state[p + "norm2.weight"], state[p + "norm2.bias"], LN_EPS)
    f = F.gelu(F.linear(product_input(h, 2), state[p + "linear1.weight"], state[p + "linear1.bias"]))
    return resid(x + resid(F.linear(product_input(f, 3), state[p + "linear2.weight"], state[p + "linear2.bias"])))


@torch.no_grad()
def forward(state, arch, ids, cast, hm, ep, act=None, record=None, resid_bf16=False, device=None,
            autocast_bf16=False):
    """device: where to run (the state's tensors are moved there); autocast_bf16: the Python search's bf16
    autocast pass (module docstring), CUDA only."""
    dev = torch.device(device or "cpu")
    state = {k: v.to(dev) for k, v in state.items()}
    ids = torch.as_tensor(ids, dtype=torch.long, device=dev)
    cast = torch.as_tensor(cast, dtype=torch.float32, device=dev)
    hm = torch.as_tensor(hm, dtype=torch.long, device=dev)
    ep = torch.as_tensor(ep, dtype=torch.long, device=dev)
    resid = _bf16 if resid_bf16 else _same
    ctx = torch.autocast("cuda", torch.bfloat16) if autocast_bf16 else contextlib.nullcontext()
    with ctx:
        x = resid(embed(state, arch, ids, cast, hm, ep))
        for i in range(arch.layers):
            x = layer(state, arch, i, x, act, record, resid, sdpa=autocast_bf16)
        hc = F.layer_norm(x[:, 0], (arch.d,), state["ln.weight"], state["ln.bias"], LN_EPS)
        return (F.linear(hc, state["policy.weight"], state["policy.bias"]),
                F.linear(hc, state["qvalue.weight"], state["qvalue.bias"]))


@torch.no_grad()
def post(policy, qvalue, I, M):
    """_collect's arithmetic at the legal moves (module docstring)."""
    It = torch.as_tensor(I, dtype=torch.long, device=policy.device)
    Mt = torch.as_tensor(M, device=policy.device).to(torch.bool)
    q = torch.sigmoid(qvalue.float())
    lg = torch.gather(policy.float(), 1, It)
    w = torch.softmax(lg.masked_fill(~Mt, float("-inf")), -1)
    qg = torch.gather(q, 1, It)
    val = (w * qg).sum(1) * 2.0 - 1.0
    val = torch.where(Mt.any(1), val, torch.full_like(val, -1.0))
    pol = lg.masked_fill(~Mt, 0.0)
    qv = (qg * 2.0 - 1.0).masked_fill(~Mt, 0.0)
    return pol.cpu().numpy(), val.cpu().numpy(), qv.cpu().numpy()


def evaluate(state, arch, b, act=None, resid_bf16=False, device=None, autocast_bf16=False):
    """The oracle's answer for one batch dict (ids, cast, hm, ep, I, M): (pol, val, qv) as the evaluator
    returns them, plus the full (policy, qvalue) logits (float32)."""
    policy, qvalue = forward(state, arch, b["ids"], b["cast"], b["hm"], b["ep"], act, resid_bf16=resid_bf16,
                             device=device, autocast_bf16=autocast_bf16)
    pol, val, qv = post(policy, qvalue, b["I"], b["M"])
    return pol, val, qv, policy.float().cpu().numpy(), qvalue.float().cpu().numpy()
