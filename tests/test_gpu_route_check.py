"""Routing agreement under ties on the device (cpg_route_check) against the oracle's restatement
of tools/check_qwen3_baseline.py:39-72 and against that script's own verdicts on the same trace
(tests/golden/route_check.npz, made by tests/golden/make_route_golden.py)."""
import numpy as np
import pytest

import route_check as RC

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_route_check_matches_oracle_and_reference(golden):
    from cachepotato_b200.qwen3 import route_check
    g = golden("route_check.npz")
    mismatch, ties = [], 0
    for i in range(int(g["n_layers"])):
        lg, top, w = g[f"logits{i}"], g[f"topk{i}"].astype(np.int32), g[f"wt{i}"]
        want = RC.route_check(lg, top, w)
        got = route_check(torch.from_numpy(lg).cuda(), torch.from_numpy(top).cuda(), torch.from_numpy(w).cuda())
        assert (got["bad"], got["ties"], got["first_bad"]) == (want["bad"], want["ties"], want["first_bad"]), i
        assert abs(got["sum_err"] - want["sum_err"]) <= 1e-12 and abs(got["w_err"] - want["w_err"]) <= 1e-12
        if got["bad"]:
            mismatch.append(i)
            ties += int(want["tie"][:got["first_bad"]].sum())
        else:
            ties += got["ties"]
    assert mismatch == g["ref_mismatch"].tolist() and ties == int(g["ref_ties"])


def test_route_check_out_of_range_ids():
    from cachepotato_b200.qwen3 import route_check
    rng = np.random.default_rng(3)
    lg = rng.normal(0, 1, (5, 128)).astype(np.float32)
    top = np.argsort(-lg, axis=1)[:, :8].astype(np.int32)
    p = np.exp(lg.astype(np.float64) - lg.max(1, keepdims=True))
    w = np.take_along_axis(p, top, 1)
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    top[2, 5] = 128                                        # planted on the host: an id past E
    want = RC.route_check(lg, top, w)
    got = route_check(torch.from_numpy(lg).cuda(), torch.from_numpy(top).cuda(), torch.from_numpy(w).cuda())
    assert got["bad"] == want["bad"] == 1 and got["first_bad"] == want["first_bad"] == 2
    assert got["w_err"] < 1e-6
