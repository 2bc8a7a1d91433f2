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


# ------------------------------------------------------------------ a rank that leaves
def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _leaver(rank, G, uid, sport, mode, out_path):
    """EP steps on the GPU, each gated by the host heartbeat; rank 1 stops after step 1 with its
    stream drained (mode 'leave': announces it; 'die': exits silently). Rank 0 must raise PeerLost
    at step 2 before posting that step's collectives, abort its communicator and return."""
    import sys
    import time
    os.environ["NCCL_NVLS_ENABLE"] = "0"            # no NVLink multicast objects in this test
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "oracle"), here]
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    import oracle as O
    from helpers import device_layer
    from cachepotato_b200.qwen3 import EpHeartbeat, ExpertParallel, PeerLost
    store = dist.TCPStore("127.0.0.1", sport, G, rank == 0, timeout=__import__("datetime").timedelta(seconds=60))
    hb = EpHeartbeat(store, rank, G, timeout_s=3.0, prefix=f"g_{mode}")
    orc = O.Oracle()
    shape = SHAPES["small"]
    T = shape[4]
    L, xn, idx, wt = _inputs(orc, O, shape, G, 850)
    sl = slice(rank * T, (rank + 1) * T)
    ep = ExpertParallel(G, rank, uid, timeout_ms=10000)
    local = device_layer(L.shard(rank, G))
    x, i, w = (torch.from_numpy(a[sl]).cuda() for a in (xn, idx, wt))
    steps_done = 0
    for step in range(4):
        if rank == 1 and step == 2:
            ep.wait()                                   # nothing of this rank in flight
            if mode == "leave":
                with open(out_path + ".left", "w") as f:     # when it left (monotonic clock: one host)
                    f.write(f"{time.monotonic():.6f}")
                hb.leave()
            os._exit(0)
        t0 = time.monotonic()
        try:
            hb.step()
        except PeerLost as e:
            t_seen = time.monotonic()
            ep.abort()
            with open(out_path, "w") as f:
                f.write(f"{steps_done} {t_seen - t0:.3f} {t_seen:.6f} {e}")
            ep.close()
            os._exit(0)
        ep.forward(local, x, i, w)
        ep.wait()
        steps_done += 1
    with open(out_path, "w") as f:
        f.write(f"{steps_done} 0 0 no PeerLost")
    ep.close()
    os._exit(0)


@pytest.mark.parametrize("mode", ["leave", "die"])
def test_ep_peer_lost_between_steps_on_gpus(tmp_path, mode):
    """The heartbeat protocol of the CPU test (tests/test_ep_gloo.py) with the real NCCL
    communicator on two GPUs: the survivor reports the lost peer instead of hanging."""
    import time
    import torch.multiprocessing as mp
    from cachepotato_b200.qwen3 import ExpertParallel
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    out = str(tmp_path / f"ep_lost_{mode}.txt")
    ctx = mp.start_processes(_leaver, args=(2, ExpertParallel.unique_id(), _free_port(), mode, out), nprocs=2,
                             join=False, start_method="spawn")
    deadline = time.monotonic() + 180
    while not ctx.join(timeout=1):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.terminate()
            pytest.fail("ranks did not finish: the survivor hung")
    done, waited, seen, msg = open(out).read().split(" ", 3)
    assert int(done) == 2, msg                       # steps 0 and 1 ran on both GPUs
    if mode == "leave":
        # noticed at once: from the peer's leave() to the survivor's PeerLost (the survivor may
        # have waited longer in all, for however far the peer's host thread lagged behind)
        assert "left" in msg, msg
        assert float(seen) - float(open(out + ".left").read()) < 1.0, (seen, waited)
    else:
        assert "did not reach" in msg, msg               # noticed at the 3 s deadline
        assert float(waited) < 10.0, waited
