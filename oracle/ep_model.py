"""Test infrastructure (the checker, not the product): a numpy restatement of the expert-parallel
exchange that cpg_moe_ep runs on the GPUs (cachepotato_b200/csrc/ep.cu), so its host-level
protocol can be exercised across processes on the CPU (gloo) and compared with the
single-process expert loop (engine/blocks/qwen3_moe.c:199-222 with the routing given).

Layout, per source rank with T tokens, G ranks, E_l experts per rank, K slots:
  plan   pos[t, p] = position of token t in the rows sent to owner p (tokens ascending), or -1;
         send_ide[p, q, j] = local expert id of slot j of the token at q, or -1 (not on p);
         send_wt[p, q, j] its weight (0 when empty). Capacity T rows per owner.
  pack   send_rows[p, q] = fp16(xn[t]) for pos[t, p] = q
  owner  out[r] = sum over the valid slots j of row r, in slot order, of wt * expert(row r)
  return one f32 row per (token, owner); the source adds them in ascending owner rank.
"""
from __future__ import annotations

import numpy as np


def plan(idx: np.ndarray, wt: np.ndarray, G: int, E_l: int):
    T, K = idx.shape
    pos = np.full((T, G), -1, np.int32)
    send_ide = np.full((G, T, K), -1, np.int32)
    send_wt = np.zeros((G, T, K), np.float32)
    owner = idx // E_l
    for p in range(G):
        q = 0
        for t in range(T):
            mine = owner[t] == p
            if mine.any():
                pos[t, p] = q
                send_ide[p, q] = np.where(mine, idx[t] - p * E_l, -1)
                send_wt[p, q] = np.where(mine, wt[t], 0.0)
                q += 1
    return pos, send_ide, send_wt


def pack_rows(xn: np.ndarray, pos: np.ndarray) -> np.ndarray:
    T, D = xn.shape
    G = pos.shape[1]
    rows = np.zeros((G, T, D), np.float16)
    for p in range(G):
        m = pos[:, p] >= 0
        rows[p, pos[m, p]] = xn[m].astype(np.float16)
    return rows


def owner_compute(orc, local_layer, rows: np.ndarray, ide: np.ndarray, wt: np.ndarray) -> np.ndarray:
    """rows (R, D) fp16, ide/wt (R, K): the local experts over the rows with at least one slot."""
    R, D = rows.shape
    out = np.zeros((R, D), np.float32)
    live = (ide >= 0).any(1)
    if live.any():
        idx = np.where(ide[live] >= 0, ide[live], 0).astype(np.int32)
        w = np.where(ide[live] >= 0, wt[live], 0.0).astype(np.float32)
        out[live] = orc.moe_apply(local_layer, rows[live].astype(np.float32), idx, w)
    return out


def combine(pos: np.ndarray, back: np.ndarray) -> np.ndarray:
    """back (G, T, D): the owners' rows for this source; mlp = their sum, ascending owner."""
    G, T, D = back.shape
    mlp = np.zeros((T, D), np.float32)
    for p in range(G):
        m = pos[:, p] >= 0
        mlp[m] += back[p, pos[m, p]]
    return mlp


def run_rank(orc, local_layer, xn, idx, wt, G: int, exchange):
    """One rank of the protocol; exchange(list of G arrays to send) -> list of G arrays received."""
    E_l = local_layer.n_experts
    pos, send_ide, send_wt = plan(idx, wt, G, E_l)
    rows = pack_rows(xn, pos)
    recv_rows = exchange(list(rows))
    recv_ide = exchange(list(send_ide))
    recv_wt = exchange(list(send_wt))
    T, D = xn.shape
    out = owner_compute(orc, local_layer, np.concatenate(recv_rows).reshape(G * T, D),
                        np.concatenate(recv_ide).reshape(G * T, -1), np.concatenate(recv_wt).reshape(G * T, -1))
    back = exchange(list(out.reshape(G, T, D)))
    return combine(pos, np.stack(back))
