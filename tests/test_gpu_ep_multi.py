"""cpg_moe_ep across GPUs: one process per GPU, NCCL between them. Every rank's block output for
its tokens must match the single-process expert loop (qwen3_moe.c:199-222 with the routing
given) within the block tolerance. Skipped with fewer than two GPUs."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SHAPES = {"small": (256, 256, 16, 4, 32), "qwen3": (2048, 768, 128, 8, 128)}


def _inputs(orc, O, shape, G, seed):
    D, F, E, K, T = shape
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=seed, oracle=orc)
    xn = orc.normal(G * T * D, seed + 1, 1.0).reshape(G * T, D)
    rng = np.random.default_rng(seed + 2)
    idx = np.stack([rng.permutation(E)[:K] for _ in range(G * T)]).astype(np.int32)
    wt = rng.random((G * T, K)).astype(np.float32) + 0.1
    return L, xn, idx, (wt / wt.sum(1, keepdims=True)).astype(np.float32)


def _worker(rank, G, uid, shape_name, seed, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "oracle"), here]
    import torch
    torch.cuda.set_device(rank)
    import oracle as O
    from helpers import device_layer
    from cachepotato_b200.qwen3 import ExpertParallel
    orc = O.Oracle()
    shape = SHAPES[shape_name]
    T = shape[4]
    L, xn, idx, wt = _inputs(orc, O, shape, G, seed)
    sl = slice(rank * T, (rank + 1) * T)
    ep = ExpertParallel(G, rank, uid)
    try:
        local = device_layer(L.shard(rank, G))
        got = ep.forward(local, torch.from_numpy(xn[sl]).cuda(), torch.from_numpy(idx[sl]).cuda(),
                         torch.from_numpy(wt[sl]).cuda()).cpu().numpy()
    finally:
        ep.close()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), got)


@pytest.mark.parametrize("shape_name", ["small", "qwen3"])
def test_ep_multi_gpu(tmp_path, orc, shape_name):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    import oracle as O
    import torch.multiprocessing as mp
    from cachepotato_b200.qwen3 import ExpertParallel
    G = 4 if n >= 4 and shape_name == "small" else 2
    seed = 840
    uid = ExpertParallel.unique_id()
    mp.start_processes(_worker, args=(G, uid, shape_name, seed, str(tmp_path)), nprocs=G, join=True,
                       start_method="spawn")
    got = np.concatenate([np.load(tmp_path / f"rank{r}.npy") for r in range(G)])
    L, xn, idx, wt = _inputs(orc, O, SHAPES[shape_name], G, seed)
    want = orc.moe_apply(L, xn, idx, wt)
    assert np.abs(got - want).max() / np.abs(want).max() <= 1e-3
