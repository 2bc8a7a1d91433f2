"""Seeded synthetic workloads for the benchmark configurations (no dataset exists for this path:
the reference's own measurements run on synthetic inputs too).

Router calibration for the batched-decode configuration: the router rows are scaled per expert,
W[e] *= s_e, by a deterministic multiplicative iteration so that the realised top-k load
histogram approaches a Zipf(s) law. The target is the expected per-rank load of Gumbel-top-k
sampling from p_r ∝ r^-s (K distinct experts per token), ranks assigned to experts by a seeded
permutation. Scaling cannot make one expert win for every token (a logit is negative for about
half the tokens whatever its scale), so the realised histogram is reported, not assumed.
"""
from __future__ import annotations

import numpy as np


def zipf_target_counts(E: int, K: int, T: int, s: float, seed: int, trials: int = 400) -> np.ndarray:
    """Expected tokens per expert rank (descending) for Gumbel-top-K draws from p_r ∝ r^-s."""
    rng = np.random.default_rng(seed)
    logp = -s * np.log(np.arange(1, E + 1, dtype=np.float64))
    counts = np.zeros(E)
    for _ in range(trials):
        g = logp[None, :] + rng.gumbel(size=(T, E))
        top = np.argpartition(-g, K - 1, axis=1)[:, :K]
        counts += np.bincount(top.ravel(), minlength=E)
    return counts / trials


def topk_counts(z: np.ndarray, scale: np.ndarray, K: int) -> np.ndarray:
    """Per-expert selection counts of top-K over rows of z * scale (softmax is monotone)."""
    v = z * scale[None, :]
    top = np.argpartition(-v, K - 1, axis=1)[:, :K]
    return np.bincount(top.ravel(), minlength=z.shape[1])


def calibrate_router_scales(z: np.ndarray, K: int, s: float, seed: int, iters: int = 300) -> np.ndarray:
    """Per-expert router row scales so top-K loads over the rows of z (T, E) follow Zipf(s)."""
    T, E = z.shape
    target_rank = zipf_target_counts(E, K, T, s, seed)
    perm = np.random.default_rng(seed + 1).permutation(E)
    target = np.empty(E)
    target[perm] = target_rank                     # expert perm[r] gets rank r
    scale = np.ones(E)
    best, best_err = scale.copy(), np.inf
    for _ in range(iters):
        c = topk_counts(z, scale, K)
        err = float(np.abs(c - target).sum())
        if err < best_err:
            best, best_err = scale.copy(), err
        scale = scale * np.exp(0.25 * (np.log(target + 0.5) - np.log(c + 0.5)))
        scale = np.clip(scale, 1e-3, 1e3)
    return best.astype(np.float32)


def zipf_assignment(T: int, E: int, K: int, s: float, q: float, seed: int):
    """Prefill routing drawn directly (no router): K distinct experts per token by Gumbel-top-k
    over Zipf-Mandelbrot popularities p_r ∝ (r + q)^-s with the ranks shuffled over expert ids;
    weights = softmax of the drawn scores renormalised over the chosen K. With T=4096, E=128,
    K=8, s=1.2, q=20 the expert groups hold roughly 90-900 tokens."""
    rng = np.random.default_rng(seed)
    logp = -s * np.log(np.arange(1, E + 1) + q)
    perm = rng.permutation(E)
    g = logp[None, :] + rng.gumbel(size=(T, E))
    top = np.argsort(-g, axis=1)[:, :K]
    sc = np.take_along_axis(g, top, 1)
    w = np.exp(sc - sc.max(1, keepdims=True))
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    return perm[top].astype(np.int32), w


def load_stats(topk: np.ndarray, E: int) -> dict:
    """Realised per-expert load of topk ids (any shape) -> summary used in reports."""
    c = np.bincount(np.asarray(topk).ravel(), minlength=E)
    nz = c[c > 0]
    return {"distinct_experts": int((c > 0).sum()), "max_load": int(c.max()),
            "min_active_load": int(nz.min()) if nz.size else 0}


def rmsnorm_rows(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = x.astype(np.float32)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + np.float32(eps))


class _DevRange:
    """A raw device range with __cuda_array_interface__, for viewing library-owned buffers."""

    def __init__(self, ptr: int, nbytes: int, typestr: str):
        item = int(typestr[-1])
        self.__cuda_array_interface__ = {"shape": (nbytes // item,), "typestr": typestr,
                                         "data": (ptr, False), "version": 2, "strides": None}


def device_view(torch, ptr: int, nbytes: int, dtype: str = "f4"):
    """A torch view of nbytes of device memory at ptr (no copy)."""
    ts = {"f4": "<f4", "u1": "|u1", "i4": "<i4"}[dtype]
    return torch.as_tensor(_DevRange(ptr, nbytes, ts), device="cuda")
