"""Golden verdicts of the reference's tie-aware routing check (tools/check_qwen3_baseline.py), for
the routing-agreement oracle (oracle/route_check.py) and cpg_route_check.

Run where the reference tree exists (it executes the reference's own script, unmodified, on a
trace file in its input format):

    python tests/golden/make_route_golden.py [reference_tree]

Writes tests/golden/route_check.npz: per layer the inputs (router logits rounded to bf16 so that
exact ties occur, as in the recorded traces, MODEL.md section 6; selections; weights) and the
reference's verdicts (which layers mismatch, the tie count, the weight errors it prints).
"""
import json
import os
import re
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "route_check.npz")
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
import oracle as O  # noqa: E402  (only for the reference tree's location)


def bf16(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000          # round to nearest even
    return u.view(np.float32)


def softmax64(lg):
    p = np.exp(lg.astype(np.float64) - lg.max(-1, keepdims=True))
    return p / p.sum(-1, keepdims=True)


def make_layers(seed: int = 5, L: int = 6, T: int = 40, E: int = 128, K: int = 8):
    rng = np.random.default_rng(seed)
    layers = []
    for i in range(L):
        lg = bf16(rng.normal(0.0, 0.6 if i % 2 else 0.15, (T, E)))   # narrow spread: many ties
        p = softmax64(lg)
        top = np.zeros((T, K), np.int32)
        for t in range(T):
            # a valid top-K under ties: sort by p, break ties by a per-layer permutation of ids
            key = rng.permutation(E) if i % 3 else np.arange(E)
            order = np.lexsort((key, -p[t]))
            top[t] = order[:K]
        w = np.take_along_axis(p, top, -1)
        w = (w / w.sum(-1, keepdims=True)).astype(np.float32)
        if i == 3:                                           # planted: an expert below the threshold
            t = 17
            below = np.argsort(-p[t])[K + 3]
            top[t, K - 1] = below
        if i == 4:                                           # planted: the 9th in place of a strictly larger one
            for t in range(T):
                srt = np.argsort(-p[t], kind="stable")
                if p[t, srt[K - 1]] > p[t, srt[K]] + 1e-9:
                    top[t, 0] = srt[K]
                    top[t, 1:] = [j for j in srt[:K] if j != srt[0]][:K - 1]
                    break
        layers.append((lg, top, w))
    return layers


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else O.REF_TREE
    layers = make_layers()
    arrays = {"meta": json.dumps({"layers": len(layers), "dtype": "bf16"})}
    for i, (lg, top, w) in enumerate(layers):
        arrays[f"L{i}.mlp.gate"] = lg
        arrays[f"L{i}.top8"] = top.astype(np.int64)
        arrays[f"L{i}.top8_w"] = w
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "trace.npz")
        np.savez(path, **arrays)
        out = subprocess.run([sys.executable, os.path.join(ref, "tools", "check_qwen3_baseline.py"), path],
                             capture_output=True, text=True).stdout
    m = re.search(r"trace vs recorded router logits: (AGREE \(all layers\)|MISMATCH in \[([0-9, ]*)\])", out)
    mismatch = [int(v) for v in m.group(2).split(",")] if m and m.group(2) else []
    ties = int(re.search(r"\[(\d+) selections resolved by a tie\]", out).group(1)) if "resolved by a tie" in out else 0
    sum_err = float(re.search(r"routing weights sum to 1 \(max \|err\|\): ([0-9.e+-]+)", out).group(1))
    w_err = float(re.search(r"weights vs softmax\+renormalise \(max \|err\|\): ([0-9.e+-]+)", out).group(1))
    save = {f"logits{i}": lg for i, (lg, _, _) in enumerate(layers)}
    save.update({f"topk{i}": top for i, (_, top, _) in enumerate(layers)})
    save.update({f"wt{i}": w for i, (_, _, w) in enumerate(layers)})
    save.update(n_layers=len(layers), ref_mismatch=np.array(mismatch, np.int32), ref_ties=ties,
                ref_sum_err=sum_err, ref_w_err=w_err)
    np.savez_compressed(OUT, **save)
    print(out)
    print("wrote", OUT, "mismatch", mismatch, "ties", ties)


if __name__ == "__main__":
    main()
