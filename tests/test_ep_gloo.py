"""Expert parallelism, host-level protocol across 2 ranks on the CPU (gloo): the plan / pack /
all-to-all / owner experts / all-to-all / combine layout of cpg_moe_ep, restated in numpy
(oracle/ep_model.py), must reproduce the single-process expert loop (qwen3_moe.c:199-222 with
the routing given) within the block tolerance, for uneven and empty owner shares."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

D, F, E, K, T = 256, 256, 16, 4, 24       # T tokens per rank


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _routing(G, seed, skew):
    rng = np.random.default_rng(seed)
    TT = G * T
    p = np.ones(E)
    if skew:                                   # rank 1 owns nearly nothing
        p[E // 2:] = 0.02
    p /= p.sum()
    idx = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(TT)]).astype(np.int32)
    wt = rng.random((TT, K)).astype(np.float32) + 0.1
    wt /= wt.sum(1, keepdims=True)
    return idx, wt.astype(np.float32)


def _worker(rank, G, port, seed, skew, out_path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.join(os.path.dirname(here), "oracle"), here]
    import torch.distributed as dist
    import oracle as O
    import ep_model
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=G)
    orc = O.Oracle()
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=seed, oracle=orc)
    xn_all = orc.normal(G * T * D, seed + 1, 1.0).reshape(G * T, D)
    idx_all, wt_all = _routing(G, seed + 2, skew)
    sl = slice(rank * T, (rank + 1) * T)

    def exchange(parts):
        send = torch.from_numpy(np.ascontiguousarray(np.stack(parts)))
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)
        return list(recv.numpy())

    mlp = ep_model.run_rank(orc, L.shard(rank, G), xn_all[sl], idx_all[sl], wt_all[sl], G, exchange)
    gathered = [torch.empty((T, D)) for _ in range(G)]
    dist.all_gather(gathered, torch.from_numpy(mlp))
    if rank == 0:
        np.save(out_path, torch.cat(gathered).numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("skew", [False, True])
def test_ep_protocol_two_ranks(orc, skew):
    import oracle as O
    import torch.multiprocessing as mp
    G, seed = 2, 77
    out_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")   # git-ignored
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, f"ep_gloo_mlp_{int(skew)}.npy")
    mp.start_processes(_worker, args=(G, _free_port(), seed, skew, out), nprocs=G, join=True, start_method="spawn")
    got = np.load(out)
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=seed, oracle=orc)
    xn = orc.normal(G * T * D, seed + 1, 1.0).reshape(G * T, D)
    idx, wt = _routing(G, seed + 2, skew)
    want = orc.moe_apply(L, xn, idx, wt)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= 1e-3, err


def test_ep_plan_layout():
    import ep_model
    idx = np.array([[0, 5, 6, 1], [4, 5, 6, 7], [0, 1, 2, 3]], np.int32)
    wt = np.full((3, 4), 0.25, np.float32)
    pos, ide, w = ep_model.plan(idx, wt, G=2, E_l=4)
    assert pos.tolist() == [[0, 0], [-1, 1], [1, -1]]
    assert ide[0, 0].tolist() == [0, -1, -1, 1] and ide[1, 0].tolist() == [-1, 1, 2, -1]
    assert ide[1, 1].tolist() == [0, 1, 2, 3] and ide[0, 1].tolist() == [0, 1, 2, 3]
    assert (ide[0, 2] == -1).all() and (w[0, 2] == 0).all()


# ------------------------------------------------------------------ a rank that leaves
def _leaver(rank, G, port, sport, mode, out_path):
    """Steps of the EP protocol, each gated by the host heartbeat; rank 1 stops after step 1
    (mode 'leave': announces it; mode 'die': exits silently). Rank 0 must raise PeerLost at
    step 2 without entering that step's collective."""
    import sys
    import time
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "oracle"), here]
    import torch.distributed as dist
    import oracle as O
    import ep_model
    from cachepotato_b200.qwen3 import EpHeartbeat, PeerLost
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=G)
    store = dist.TCPStore("127.0.0.1", sport, G, rank == 0)
    hb = EpHeartbeat(store, rank, G, timeout_s=3.0, prefix=f"t_{mode}")
    orc = O.Oracle()
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=5, oracle=orc)
    xn = orc.normal(T * D, 6 + rank, 1.0).reshape(T, D)
    idx, wt = _routing(G, 7, False)
    sl = slice(rank * T, (rank + 1) * T)

    def exchange(parts):
        send = torch.from_numpy(np.ascontiguousarray(np.stack(parts)))
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)
        return list(recv.numpy())

    steps_done = 0
    for step in range(4):
        if rank == 1 and step == 2:
            if mode == "leave":
                hb.leave()
            os._exit(0)                      # between steps: nothing of this rank in flight
        t0 = time.monotonic()
        try:
            hb.step()
        except PeerLost as e:
            with open(out_path, "w") as f:
                f.write(f"{steps_done} {time.monotonic() - t0:.3f} {e}")
            os._exit(0)                      # the collective of this step was never entered
        ep_model.run_rank(orc, L.shard(rank, G), xn, idx[sl], wt[sl], G, exchange)
        steps_done += 1
    with open(out_path, "w") as f:
        f.write(f"{steps_done} 0 no PeerLost")
    os._exit(0)


@pytest.mark.parametrize("mode", ["leave", "die"])
def test_ep_peer_lost_between_steps_is_reported_not_hung(mode):
    import time
    import torch.multiprocessing as mp
    out_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, f"ep_peer_lost_{mode}.txt")
    if os.path.exists(out):
        os.unlink(out)
    ctx = mp.start_processes(_leaver, args=(2, _free_port(), _free_port(), mode, out), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 120
    while not ctx.join(timeout=1):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.terminate()
            pytest.fail("ranks did not finish: the survivor hung")
    done, waited, msg = open(out).read().split(" ", 2)
    assert int(done) == 2, msg                       # steps 0 and 1 ran on both ranks
    assert "PeerLost" not in msg and ("left" in msg if mode == "leave" else "did not reach" in msg), msg
    # a rank that announced its departure is noticed at once, a silent one at the deadline
    assert float(waited) < (1.5 if mode == "leave" else 10.0), waited
