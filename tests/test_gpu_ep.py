"""Expert parallelism on the GPU: cpg_moe_apply_rows (the owner side) against the oracle, and
cpg_moe_ep through NCCL against the oracle's expert loop (qwen3_moe.c:199-222 with the routing
given) and the numpy model of the exchange (oracle/ep_model.py). One rank here; the 2-GPU run
of the same check is tests/test_gpu_ep_multi.py."""
import numpy as np
import pytest

import oracle as O
import ep_model
from conftest import max_rel
from helpers import BLOCK_TOL, device_layer

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _routing(T, E, K, seed):
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    wt = rng.random((T, K)).astype(np.float32) + 0.1
    return idx, (wt / wt.sum(1, keepdims=True)).astype(np.float32)


def test_apply_rows_empty_slots(orc):
    from cachepotato_b200.qwen3 import moe_apply_rows
    D, F, E, K, R = 256, 256, 16, 4, 50
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=810, oracle=orc)
    rows = orc.normal(R * D, 811, 1.0).reshape(R, D).astype(np.float16)
    idx, wt = _routing(R, E, K, 812)
    rng = np.random.default_rng(813)
    empty = rng.random((R, K)) < 0.5
    empty[7] = True                                  # a row with no slot at all
    ide = np.where(empty, -1, idx).astype(np.int32)
    got = moe_apply_rows(device_layer(L), torch.from_numpy(rows).cuda(), torch.from_numpy(ide).cuda(),
                         torch.from_numpy(wt).cuda()).cpu().numpy()
    want = ep_model.owner_compute(orc, L, rows, ide, wt)
    assert (got[7] == 0).all()
    assert max_rel(got, want) <= BLOCK_TOL


@pytest.mark.parametrize("shape", [(256, 256, 16, 4, 40), (2048, 768, 128, 8, 96)])
def test_ep_single_rank(orc, shape):
    from cachepotato_b200.qwen3 import ExpertParallel
    D, F, E, K, T = shape
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=820 + D, oracle=orc)
    xn = orc.normal(T * D, 821, 1.0).reshape(T, D)
    idx, wt = _routing(T, E, K, 822)
    ep = ExpertParallel(1, 0, ExpertParallel.unique_id())
    try:
        dl = device_layer(L)
        base = torch.ones((T, D), dtype=torch.float32, device="cuda")
        got = ep.forward(dl, torch.from_numpy(xn).cuda(), torch.from_numpy(idx).cuda(), torch.from_numpy(wt).cuda(),
                         mlp=base).cpu().numpy() - 1.0
    finally:
        ep.close()
    want = orc.moe_apply(L, xn, idx, wt)
    assert max_rel(got, want) <= BLOCK_TOL


def test_ep_rejects_bad_ids(orc):
    from cachepotato_b200 import CpgError
    from cachepotato_b200.qwen3 import ExpertParallel
    D, F, E, K, T = 256, 256, 16, 4, 8
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=830, oracle=orc)
    xn = orc.normal(T * D, 831, 1.0).reshape(T, D)
    idx, wt = _routing(T, E, K, 832)
    idx[2, 1] = E + 3                                # planted on the host
    ep = ExpertParallel(1, 0, ExpertParallel.unique_id())
    try:
        with pytest.raises(CpgError):
            ep.forward(device_layer(L), torch.from_numpy(xn).cuda(), torch.from_numpy(idx).cuda(),
                       torch.from_numpy(wt).cuda())
    finally:
        ep.close()
