"""Parity metrics of the evaluator against the reference outputs, at the legal moves only, after
mayfly/chess/cudanet/test_cudanet.py:288-320 (metrics): max and mean |diff| of the policy logits, of the
win probabilities sigmoid(q) = (qv + 1) / 2 and (val + 1) / 2, how often the top move agrees (also over rows
whose best move leads the second by more than TIE_GAP logits, and over "decided" rows whose lead exceeds twice the
logit tolerance), non-finite values and nonzero padding."""
import numpy as np

TIE_GAP = 0.20       # cudanet/test_cudanet.py:62


def metrics(ref, got, widths, decided_gap=0.04):
    """decided_gap: rows whose reference best move leads the second by more than this are "decided"; a logit
    error within the tolerance (2e-2) cannot reorder them, so they must all agree."""
    rp, rv, rq = (np.asarray(a, np.float64) for a in ref)
    gp, gv, gq = (np.asarray(a, np.float64) for a in got)
    pol, q, top1, clear, clear_ok, dec, dec_ok = [], [], 0, 0, 0, 0, 0
    nonfinite = int((~np.isfinite(gp)).sum() + (~np.isfinite(gv)).sum() + (~np.isfinite(gq)).sum())
    pad = 0
    for i, k in enumerate(widths):
        k = int(k)
        a, g = rp[i, :k], gp[i, :k]
        pol.append(np.abs(a - g))
        q.append(np.abs(rq[i, :k] - gq[i, :k]) / 2)
        pad += int((gp[i, k:] != 0).sum() + (gq[i, k:] != 0).sum())
        ra, ga = np.argsort(-a, kind="stable"), np.argsort(-g, kind="stable")
        top1 += int(ra[0] == ga[0])
        gap = a[ra[0]] - a[ra[1]] if k > 1 else np.inf
        if gap > TIE_GAP:
            clear += 1
            clear_ok += int(ra[0] == ga[0])
        if gap > decided_gap:
            dec += 1
            dec_ok += int(ra[0] == ga[0])
    pol, q = np.concatenate(pol), np.concatenate(q)
    wdl = np.abs(rv - gv) / 2
    n = len(widths)
    return {"pol_max": float(pol.max()), "pol_mean": float(pol.mean()), "q_max": float(q.max()),
            "q_mean": float(q.mean()), "val_max": float(wdl.max()), "val_mean": float(wdl.mean()),
            "top1": top1 / n, "top1_hits": top1, "rows": n, "top1_clear": clear_ok / max(clear, 1),
            "clear_rows": clear, "top1_decided": dec_ok / max(dec, 1), "decided_rows": dec,
            "nonfinite": nonfinite, "pad_nonzero": pad}
