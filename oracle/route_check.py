"""Tie-aware routing agreement: the reference's rule restated in numpy (the checker of
cpg_route_check).

TEST INFRASTRUCTURE ONLY: imported by tests/ as the oracle, never by the package.

Restates tools/check_qwen3_baseline.py:39-72 (the rule models/qwen3-30b-a3b/MODEL.md section 6
calls the definition of routing agreement), for one layer's tokens:
  p = softmax(logits) per token (here in float64);
  thr = the K-th largest p;
  a recorded selection (taken as a set) is valid when every chosen expert has p >= thr - 1e-12,
  every expert with p > thr + 1e-12 is chosen, and the number of chosen experts above
  thr + 1e-12 equals the number of experts above it;
  a valid selection is "resolved by a tie" when fewer experts lie above thr + 1e-12 than were
  chosen;
  weights: |sum(w) - 1| and |w - p[chosen] / sum(p[chosen])| (maxima).
The reference stops a layer at its first invalid token; this returns every token's verdict.
"""
from __future__ import annotations

import numpy as np

EPS = 1e-12


def route_check(logits: np.ndarray, topk: np.ndarray, wt: np.ndarray) -> dict:
    lg = np.asarray(logits, np.float64)
    T, E = lg.shape
    K = topk.shape[1]
    p = np.exp(lg - lg.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    kth = np.sort(p, axis=-1)[:, -K]
    bad, ties, first_bad = 0, 0, -1
    valid_tok = np.zeros(T, bool)
    tie_tok = np.zeros(T, bool)
    for t in range(T):
        ids = topk[t].tolist()
        if any(j < 0 or j >= E for j in ids):
            ok = False
            rec = set()
        else:
            rec = set(ids)
            thr = kth[t]
            chosen_ok = all(p[t, j] >= thr - EPS for j in rec)
            above = {j for j in range(E) if p[t, j] > thr + EPS}
            n_above_sel = sum(1 for j in rec if p[t, j] > thr + EPS)
            ok = chosen_ok and above <= rec and n_above_sel == len(above)
        valid_tok[t] = ok
        if not ok:
            bad += 1
            if first_bad < 0:
                first_bad = t
        elif len(above) < len(rec):
            ties += 1
            tie_tok[t] = True
    valid = np.all((topk >= 0) & (topk < E), axis=1)
    safe = np.where(valid[:, None], topk, 0)
    got = np.take_along_axis(p, safe, -1)
    want = got / got.sum(-1, keepdims=True)
    w = np.asarray(wt, np.float64)
    w_err = float(np.abs(want - w)[valid].max()) if valid.any() else 0.0
    sum_err = float(np.abs(w.sum(-1) - 1.0).max()) if T else 0.0
    return {"bad": bad, "ties": ties, "first_bad": first_bad, "sum_err": sum_err, "w_err": w_err,
            "valid": valid_tok, "tie": tie_tok}
