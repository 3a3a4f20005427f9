"""Parity metrics of the evaluator against the reference outputs, at the legal moves only, after
mayfly/chess/cudanet/test_cudanet.py:288-320 (metrics) and :323-340 (verdict).

metrics() gives, in this repository's units: max and mean |diff| of the policy logits, of the win probabilities
sigmoid(q) = (qv + 1) / 2 and (val + 1) / 2, of the softmax prior over each row's legal moves (temperature 1,
test_cudanet.py:59), how often the top move agrees (also over rows whose best move leads the second by more than
TIE_GAP logits, and over "decided" rows whose lead exceeds twice the logit tolerance), how often the top 3 moves
agree as a set (test_cudanet.py:311-312), non-finite values and nonzero padding. It also carries the same
differences in the reference's own units (`ref_form`: val and qv in [-1, 1], not halved), which verdict() holds to
the reference's pass lines (TOL, TOP1_MIN, TOP1_CLEAR_MIN, TOP3_MIN, test_cudanet.py:58-65), and, given the
metrics of the bf16 autocast pass the Python search plays, to "no worse than it on every max and mean"."""
import numpy as np

TIE_GAP = 0.20       # cudanet/test_cudanet.py:62
# cudanet/test_cudanet.py:58-61, 63-65: the reference's pass lines against the float32 model
REF_TOL = {"pol": {"max": 0.10, "mean": 0.010}, "prior": {"max": 0.010, "mean": 2e-4},
           "val": {"max": 0.010, "mean": 0.002}, "qv": {"max": 0.020, "mean": 0.002}}
REF_TOP1_MIN, REF_TOP1_CLEAR_MIN, REF_TOP3_MIN = 0.99, 1.0, 0.97


def _softmax(x):
    e = np.exp(x - x.max())
    return e / e.sum()


def metrics(ref, got, widths, decided_gap=0.04):
    """decided_gap: rows whose reference best move leads the second by more than this are "decided"; a logit
    error within the tolerance (2e-2) cannot reorder them, so they must all agree."""
    rp, rv, rq = (np.asarray(a, np.float64) for a in ref)
    gp, gv, gq = (np.asarray(a, np.float64) for a in got)
    pol, prior, q, top1, top3, clear, clear_ok, dec, dec_ok = [], [], [], 0, 0, 0, 0, 0, 0
    nonfinite = int((~np.isfinite(gp)).sum() + (~np.isfinite(gv)).sum() + (~np.isfinite(gq)).sum())
    pad = 0
    for i, k in enumerate(widths):
        k = int(k)
        a, g = rp[i, :k], gp[i, :k]
        pol.append(np.abs(a - g))
        prior.append(np.abs(_softmax(a) - _softmax(g)))
        q.append(np.abs(rq[i, :k] - gq[i, :k]) / 2)
        pad += int((gp[i, k:] != 0).sum() + (gq[i, k:] != 0).sum())
        ra, ga = np.argsort(-a, kind="stable"), np.argsort(-g, kind="stable")
        top1 += int(ra[0] == ga[0])
        k3 = min(3, k)
        top3 += int(set(ra[:k3].tolist()) == set(ga[:k3].tolist()))
        gap = a[ra[0]] - a[ra[1]] if k > 1 else np.inf
        if gap > TIE_GAP:
            clear += 1
            clear_ok += int(ra[0] == ga[0])
        if gap > decided_gap:
            dec += 1
            dec_ok += int(ra[0] == ga[0])
    pol, prior, q = np.concatenate(pol), np.concatenate(prior), np.concatenate(q)
    wdl = np.abs(rv - gv) / 2
    n = len(widths)
    ref_form = {"pol": {"max": float(pol.max()), "mean": float(pol.mean())},
                "prior": {"max": float(prior.max()), "mean": float(prior.mean())},
                "val": {"max": float(2 * wdl.max()), "mean": float(2 * wdl.mean())},
                "qv": {"max": float(2 * q.max()), "mean": float(2 * q.mean())}}
    return {"pol_max": float(pol.max()), "pol_mean": float(pol.mean()), "q_max": float(q.max()),
            "q_mean": float(q.mean()), "val_max": float(wdl.max()), "val_mean": float(wdl.mean()),
            "prior_max": float(prior.max()), "prior_mean": float(prior.mean()),
            "top1": top1 / n, "top1_hits": top1, "top3": top3 / n, "top3_hits": top3, "rows": n,
            "top1_clear": clear_ok / clear if clear else 1.0, "clear_rows": clear,
            "top1_decided": dec_ok / dec if dec else 1.0,
            "decided_rows": dec, "nonfinite": nonfinite, "pad_nonzero": pad, "ref_form": ref_form}


def verdict(m, bf=None, top1_min=REF_TOP1_MIN):
    """The reference's pass lines (test_cudanet.py:323-340) this result fails, as sentences (empty: it passes).
    bf: metrics of the bf16 autocast pass on the same rows; every max and mean must then be no worse than it."""
    bad = []
    if m["nonfinite"]:
        bad.append(f"{m['nonfinite']} values are NaN or infinite")
    if m["pad_nonzero"]:
        bad.append(f"{m['pad_nonzero']} padding values are not 0")
    for key, lim in REF_TOL.items():
        for stat, x in lim.items():
            v = m["ref_form"][key][stat]
            if v > x:
                bad.append(f"{key} {stat} abs {v:.3g} > {x:g}")
            if bf is not None and v > bf["ref_form"][key][stat]:
                bad.append(f"{key} {stat} abs {v:.3g} worse than bf16 autocast's {bf['ref_form'][key][stat]:.3g}")
    if m["top1"] < top1_min:
        bad.append(f"top move agrees on {m['top1']:.4f} < {top1_min}")
    if m["top1_clear"] < REF_TOP1_CLEAR_MIN:
        bad.append(f"top move without a near tie agrees on {m['top1_clear']:.4f} < {REF_TOP1_CLEAR_MIN}")
    if m["top3"] < REF_TOP3_MIN:
        bad.append(f"top 3 agrees on {m['top3']:.4f} < {REF_TOP3_MIN}")
    return bad
