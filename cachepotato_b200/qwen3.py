"""Host-side mirror of the reference interface for the Qwen3-MoE expert path.

Names follow the reference: the kernel entry points of engine/kernels/kernels.h
(matmul_wx, matmul_wx_q8, matmul_wx_q4, q8_dequant_row, q4_dequant_row) take host numpy
arrays, overwrite `out` and raise on failure; qwen3_mm is the encoding dispatch of
engine/blocks/qwen3_moe.c:36-40; MoELayer is the MoE half of QW3Layer / qwen3_layer_kv
(engine/blocks/qwen3_moe.h:21-95). Device memory is torch CUDA tensors (plumbing only); every
computation runs in libcpg_b200.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import ENC_F32, ENC_Q4, ENC_Q8, GROUP_BYTES, MoeDesc, Qwen3Attn, Qwen3Desc, Tensor, check, lib


def row_bytes(enc: int, n_in: int) -> int:
    return 4 * n_in if enc == ENC_F32 else (n_in // 32) * GROUP_BYTES[enc]


def _np_ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ------------------------------------------------------------------ kernels.h mirror (host)
def _host_mm(fn, out: np.ndarray, x: np.ndarray, w: np.ndarray, n_in: int, n_out: int) -> None:
    assert out.dtype == np.float32 and out.flags.c_contiguous and out.size >= n_out
    x = np.ascontiguousarray(x, dtype=np.float32)
    fn(_np_ptr(out), _np_ptr(x), _np_ptr(np.ascontiguousarray(w)), n_in, n_out)
    err = _lib.last_error()          # the void drop-ins clear it on entry
    if err:
        raise _lib.CpgError(_lib.CPG_EINVAL, err)


def matmul_wx(out: np.ndarray, x: np.ndarray, w: np.ndarray, n_in: int, n_out: int) -> None:
    """out[i] = sum_k w[i*n_in+k] x[k] (engine/kernels/kernels.c:84)."""
    _host_mm(lib().cpg_matmul_wx, out, x, np.ascontiguousarray(w, dtype=np.float32), n_in, n_out)


def matmul_wx_q8(out: np.ndarray, x: np.ndarray, w: np.ndarray, n_in: int, n_out: int) -> None:
    """Q8_0 row-major W·x (engine/kernels/kernels.c:368)."""
    _host_mm(lib().cpg_matmul_wx_q8, out, x, w, n_in, n_out)


def matmul_wx_q4(out: np.ndarray, x: np.ndarray, w: np.ndarray, n_in: int, n_out: int) -> None:
    """Q4_0 row-major W·x (engine/kernels/kernels.c:514)."""
    _host_mm(lib().cpg_matmul_wx_q4, out, x, w, n_in, n_out)


def _host_dq(fn, blocks: np.ndarray, out: np.ndarray, n: int) -> None:
    assert out.dtype == np.float32 and out.size >= n
    fn(_np_ptr(np.ascontiguousarray(blocks, dtype=np.uint8)), _np_ptr(out), n)
    err = _lib.last_error()
    if err:
        raise _lib.CpgError(_lib.CPG_EINVAL, err)


def q8_dequant_row(blocks: np.ndarray, out: np.ndarray, n: int) -> None:
    """Bit-exact Q8_0 decode (engine/kernels/kernels.c:143)."""
    _host_dq(lib().cpg_q8_dequant_row, blocks, out, n)


def q4_dequant_row(blocks: np.ndarray, out: np.ndarray, n: int) -> None:
    """Bit-exact Q4_0 decode (engine/kernels/kernels.c:463)."""
    _host_dq(lib().cpg_q4_dequant_row, blocks, out, n)


# ------------------------------------------------------------------ device entry points
def _torch():
    import torch
    return torch


def _stream_ptr(stream) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def dequant(blocks, n: int, enc: int, stream=None):
    """Device decode of n values -> float32 tensor (bit-exact with the reference)."""
    torch = _torch()
    out = torch.empty(n, dtype=torch.float32, device=blocks.device)
    check(lib().cpg_dequant(out.data_ptr(), blocks.data_ptr(), enc, n, _stream_ptr(stream)))
    return out


def quantize(x, enc: int, stream=None):
    """Device encode of a float32 tensor -> uint8 blocks (bit-exact with format/q4.py, q8.py)."""
    torch = _torch()
    x = x.contiguous()
    out = torch.empty(x.numel() // 32 * GROUP_BYTES[enc], dtype=torch.uint8, device=x.device)
    check(lib().cpg_quantize(out.data_ptr(), x.data_ptr(), enc, x.numel(), _stream_ptr(stream)))
    return out


def qwen3_mm(w, enc: int, x, n_in: int, n_out: int, stream=None):
    """out (T, n_out) = W·x[t] for x (T, n_in) on the device (qwen3_moe.c:36-40)."""
    torch = _torch()
    x = x.contiguous().view(-1, n_in)
    T = x.shape[0]
    out = torch.empty((T, n_out), dtype=torch.float32, device=x.device)
    check(lib().cpg_matvec(out.data_ptr(), x.data_ptr(), Tensor(w.data_ptr(), enc), n_in, n_out, T,
                           _stream_ptr(stream)))
    return out


def route_check(logits, topk, wt, stream=None) -> dict:
    """Routing agreement under ties on the device (cpg_route_check): the rule of
    tools/check_qwen3_baseline.py:39-72 for one layer's tokens. logits (T, E), topk (T, K) and
    wt (T, K) on the device. Returns the invalid-token count, the tie count, the first invalid
    token (-1 if none) and the two weight errors."""
    torch = _torch()
    logits = logits.contiguous().float()
    topk = topk.contiguous().to(torch.int32)
    wt = wt.contiguous().float()
    T, E = logits.shape
    K = topk.shape[1]
    stats, errs = (ctypes.c_int * 3)(), (ctypes.c_double * 2)()
    check(lib().cpg_route_check(logits.data_ptr(), topk.data_ptr(), wt.data_ptr(), T, E, K, stats, errs,
                                _stream_ptr(stream)))
    return {"bad": stats[0], "ties": stats[1], "first_bad": stats[2], "sum_err": errs[0], "w_err": errs[1]}


@dataclass
class MoEOutputs:
    mlp: object
    x_out: object
    router: object
    topk_idx: object
    wt: object


class MoELayer:
    """The MoE half of one Qwen3 layer, weights resident on the device.

    ln2 (d_model) f32, wgate (n_experts, d_model) f32, and the experts either as one blob
    with a fixed region stride (Wg | Wu | Wd per expert, as CPW1 v4 lays them out) or as a
    list of 3*n_experts device pointers.
    """

    def __init__(self, ln2, wgate, enc: int, d_model: int, d_exp: int, n_experts: int, topk: int,
                 eps: float = 1e-6, blob=None, expert_ptrs=None, keep=()):
        self.d_model, self.d_exp, self.n_experts, self.topk, self.enc, self.eps = (
            d_model, d_exp, n_experts, topk, enc, eps)
        mat = d_exp * d_model // 32 * GROUP_BYTES[enc]
        self.mat_bytes, self.region_bytes = mat, 3 * mat
        if expert_ptrs is None:
            base = blob.data_ptr()
            expert_ptrs = [base + e * 3 * mat + k * mat for e in range(n_experts) for k in range(3)]
        tab = (Tensor * (3 * n_experts))()
        for i, p in enumerate(expert_ptrs):
            tab[i] = Tensor(p, enc)
        desc = MoeDesc(d_model, d_exp, n_experts, topk, eps, ln2.data_ptr(), Tensor(wgate.data_ptr(), ENC_F32),
                       ctypes.cast(tab, ctypes.POINTER(Tensor)))
        h = ctypes.c_void_p()
        check(lib().cpg_moe_layer_create(ctypes.byref(desc), ctypes.byref(h)))
        self.handle = h
        self._keep = (ln2, wgate, blob, tab) + tuple(keep)   # keep device memory alive

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                lib().cpg_moe_layer_destroy(h)
            except Exception:
                pass
            self.handle = None

    def workspace_bytes(self, max_T: int) -> int:
        return int(lib().cpg_moe_workspace_bytes(self.handle, max_T))

    def workspace(self, max_T: int):
        torch = _torch()
        return torch.zeros(self.workspace_bytes(max_T), dtype=torch.uint8, device="cuda")

    def forward(self, x, attn=None, *, ws=None, mlp=None, want_x_out=True, stream=None,
                check_status=True) -> MoEOutputs:
        """qwen3_layer_kv's MoE half for x (T, d_model) on the device."""
        torch = _torch()
        x = x.contiguous()
        T = x.shape[0]
        if ws is None:
            ws = self.workspace(T)
        dev = x.device
        router = torch.empty((T, self.n_experts), dtype=torch.float32, device=dev)
        topk = torch.empty((T, self.topk), dtype=torch.int32, device=dev)
        wt = torch.empty((T, self.topk), dtype=torch.float32, device=dev)
        if mlp is None:
            mlp = torch.zeros((T, self.d_model), dtype=torch.float32, device=dev)
        x_out = torch.empty_like(x) if want_x_out else None
        sp = _stream_ptr(stream)
        check(lib().cpg_moe_forward(self.handle, x.data_ptr(), None if attn is None else attn.contiguous().data_ptr(),
                                    T, mlp.data_ptr(), None if x_out is None else x_out.data_ptr(),
                                    topk.data_ptr(), wt.data_ptr(), router.data_ptr(), ws.data_ptr(),
                                    ws.numel(), sp))
        if check_status:
            check(lib().cpg_moe_check(ws.data_ptr(), sp))
        return MoEOutputs(mlp, x_out, router, topk, wt)


def moe_apply(layer: "MoELayer", xn, topk_idx, wt, *, ws=None, mlp=None, stream=None, check_status=True,
              phase_ms=None):
    """Routed experts on the tensor cores (prefill): mlp += sum_j wt[t,j] * expert_j(xn[t]).
    phase_ms: optional list, receives [sort, gate_up, down, combine] in ms (synchronising)."""
    torch = _torch()
    xn = xn.contiguous()
    T = xn.shape[0]
    idx = topk_idx.to(torch.int32).contiguous()
    wt = wt.to(torch.float32).contiguous()
    if ws is None:
        ws = torch.empty(int(lib().cpg_moe_apply_workspace_bytes(layer.handle, T)), dtype=torch.uint8,
                         device=xn.device)
    if mlp is None:
        mlp = torch.zeros((T, layer.d_model), dtype=torch.float32, device=xn.device)
    sp = _stream_ptr(stream)
    if phase_ms is None:
        check(lib().cpg_moe_apply(layer.handle, xn.data_ptr(), T, idx.data_ptr(), wt.data_ptr(), mlp.data_ptr(),
                                  ws.data_ptr(), ws.numel(), sp))
    else:
        ph = (ctypes.c_float * 4)()
        check(lib().cpg_moe_apply_profile(layer.handle, xn.data_ptr(), T, idx.data_ptr(), wt.data_ptr(),
                                          mlp.data_ptr(), ws.data_ptr(), ws.numel(), sp, ph))
        phase_ms[:] = list(ph)
    if check_status:
        check(lib().cpg_moe_apply_check(ws.data_ptr(), sp))
    return mlp


def moe_apply_rows(layer: "MoELayer", rows_f16, slot_expert, slot_wt, *, ws=None, out=None, stream=None,
                   check_status=True):
    """cpg_moe_apply_rows: out[r] = sum over the valid slots (id >= 0) of wt * expert(rows[r])."""
    torch = _torch()
    rows = rows_f16.contiguous()
    R = rows.shape[0]
    ide = slot_expert.to(torch.int32).contiguous()
    wt = slot_wt.to(torch.float32).contiguous()
    if ws is None:
        ws = torch.empty(int(lib().cpg_moe_apply_workspace_bytes(layer.handle, R)), dtype=torch.uint8,
                         device=rows.device)
    if out is None:
        out = torch.empty((R, layer.d_model), dtype=torch.float32, device=rows.device)
    sp = _stream_ptr(stream)
    check(lib().cpg_moe_apply_rows(layer.handle, rows.data_ptr(), R, ide.data_ptr(), wt.data_ptr(), out.data_ptr(),
                                   ws.data_ptr(), ws.numel(), sp))
    if check_status:
        check(lib().cpg_moe_apply_check(ws.data_ptr(), sp))
    return out


class PeerLost(RuntimeError):
    """A rank of the expert-parallel group left or stopped answering its heartbeat."""


class EpHeartbeat:
    """Host-side liveness of an expert-parallel group, over a key-value store every rank reaches
    (torch.distributed.TCPStore / FileStore or anything with set(key, value) and check(keys)).

    Before each step (e.g. each batch through the stacked layers) every rank calls step(): it
    publishes that it reached the step and waits, up to `timeout_s`, until every peer has too.
    A peer that called leave() is noticed at once, one that died is noticed at the deadline;
    either way step() raises PeerLost BEFORE this rank enqueues the step's collectives, so no
    NCCL transfer is ever posted towards a peer that is gone (the caller then aborts its
    communicator with ExpertParallel.abort()). The reference engine is single-process and has
    no counterpart; its error contract (NULL + message or rc < 0, never a hang,
    engine/api/cachepotato.h:44-69) is the model."""

    def __init__(self, store, rank: int, nranks: int, timeout_s: float = 30.0, prefix: str = "cpg_ep"):
        self.store, self.rank, self.nranks = store, rank, nranks
        self.timeout_s, self.prefix, self.n = float(timeout_s), prefix, 0

    def _key(self, what: str, r: int) -> str:
        return f"{self.prefix}/{what}/{r}"

    def step(self) -> int:
        import time
        n = self.n
        self.store.set(self._key(f"step{n}", self.rank), "1")
        peers = [p for p in range(self.nranks) if p != self.rank]
        want = [self._key(f"step{n}", p) for p in peers]
        t0 = time.monotonic()
        while True:
            if not want or self.store.check(want):
                self.n += 1
                return n
            gone = [p for p in peers if self.store.check([self._key("left", p)])]
            if gone:
                raise PeerLost(f"rank(s) {gone} left the expert-parallel group before step {n}")
            if time.monotonic() - t0 > self.timeout_s:
                late = [p for p in peers if not self.store.check([self._key(f"step{n}", p)])]
                raise PeerLost(f"rank(s) {late} did not reach step {n} within {self.timeout_s:.1f} s")
            time.sleep(0.001)

    def leave(self) -> None:
        """Announce that this rank takes no further steps (call between steps)."""
        self.store.set(self._key("left", self.rank), "1")


class ExpertParallel:
    """cpg_ep: one rank of an expert-parallel group (one process per GPU). Rank r's local layer
    holds experts [r*E_l, (r+1)*E_l) of the full layer; every rank passes the same T."""

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().cpg_ep_unique_id(buf))
        return buf.raw

    def __init__(self, nranks: int, rank: int, uid: bytes, timeout_ms: int | None = None):
        assert len(uid) == 128
        h = ctypes.c_void_p()
        check(lib().cpg_ep_create(nranks, rank, ctypes.create_string_buffer(uid, 128), ctypes.byref(h)))
        self.handle, self.nranks, self.rank = h, nranks, rank
        if timeout_ms is not None:
            check(lib().cpg_ep_set_timeout(self.handle, int(timeout_ms)))

    def workspace(self, local_layer: "MoELayer", T: int):
        torch = _torch()
        return torch.empty(int(lib().cpg_ep_workspace_bytes(self.handle, local_layer.handle, T)), dtype=torch.uint8,
                           device="cuda")

    def forward(self, local_layer: "MoELayer", xn, topk_idx, wt, *, mlp=None, ws=None, stream=None,
                check_status=True, phase_ms=None):
        """mlp += the MoE block over this rank's T tokens (global expert ids in topk_idx).
        phase_ms: a list to receive the five phase times (plan + pack, dispatch, owner experts,
        return, combine; synchronising)."""
        torch = _torch()
        xn = xn.contiguous()
        T = xn.shape[0]
        idx = topk_idx.to(torch.int32).contiguous()
        wt = wt.to(torch.float32).contiguous()
        if ws is None:
            ws = self.workspace(local_layer, T)
        if mlp is None:
            mlp = torch.zeros((T, local_layer.d_model), dtype=torch.float32, device=xn.device)
        sp = _stream_ptr(stream)
        if phase_ms is not None:
            ph = (ctypes.c_float * 5)()
            check(lib().cpg_moe_ep_profile(self.handle, local_layer.handle, xn.data_ptr(), T, idx.data_ptr(),
                                           wt.data_ptr(), mlp.data_ptr(), ws.data_ptr(), ws.numel(), sp, ph))
            phase_ms[:] = list(ph)
        else:
            check(lib().cpg_moe_ep(self.handle, local_layer.handle, xn.data_ptr(), T, idx.data_ptr(), wt.data_ptr(),
                                   mlp.data_ptr(), ws.data_ptr(), ws.numel(), sp))
        if check_status:
            self.wait(stream)
            check(lib().cpg_moe_ep_check(ws.data_ptr(), sp))
        return mlp

    def wait(self, stream=None) -> None:
        """Bounded wait for this rank's enqueued EP work (aborts the communicator at the deadline)."""
        check(lib().cpg_ep_wait(self.handle, _stream_ptr(stream)))

    def abort(self) -> None:
        """ncclCommAbort: for a rank that learned (EpHeartbeat) that a peer is gone."""
        if self.handle is not None and self.handle.value:
            check(lib().cpg_ep_abort(self.handle))

    def close(self) -> None:
        if self.handle is not None and self.handle.value:
            lib().cpg_ep_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Qwen3Model:
    """cpg_qwen3: the whole model on one device (embed_rows, run_layers, apply_head and the greedy
    loop of cp_chat, engine/api/cachepotato.c:108-166, 315-378).

    attn: per layer a dict of device tensors ln1, q_norm, k_norm (f32) and wq, wk, wv, wo
    (uint8 blocks in attn_enc); moe: per layer a MoELayer; embed / lm_head: device blocks in
    their encodings; final_norm f32."""

    def __init__(self, *, d_model, n_heads, n_kv, head_dim, vocab, max_ctx, attn, moe, attn_enc,
                 embed, embed_enc, lm_head, head_enc, final_norm, rope_theta=1e6, rms_eps=1e-6):
        L = len(attn)
        tab = (Qwen3Attn * L)()
        for i, a in enumerate(attn):
            tab[i] = Qwen3Attn(a["ln1"].data_ptr(), a["q_norm"].data_ptr(), a["k_norm"].data_ptr(),
                               Tensor(a["wq"].data_ptr(), attn_enc), Tensor(a["wk"].data_ptr(), attn_enc),
                               Tensor(a["wv"].data_ptr(), attn_enc), Tensor(a["wo"].data_ptr(), attn_enc))
        moes = (ctypes.c_void_p * L)(*[m.handle.value for m in moe])
        desc = Qwen3Desc(d_model, n_heads, n_kv, head_dim, vocab, L, max_ctx, rope_theta, rms_eps,
                         Tensor(embed.data_ptr(), embed_enc), Tensor(lm_head.data_ptr(), head_enc),
                         final_norm.data_ptr(), tab, moes)
        h = ctypes.c_void_p()
        check(lib().cpg_qwen3_create(ctypes.byref(desc), ctypes.byref(h)))
        self.handle, self.vocab = h, vocab
        self._keep = (attn, moe, embed, lm_head, final_norm, tab, moes)

    def prefill(self, ids) -> int:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        nxt = ctypes.c_int()
        check(lib().cpg_qwen3_prefill(self.handle, ids.ctypes.data, len(ids), ctypes.byref(nxt)))
        return nxt.value

    def step(self, token: int) -> int:
        nxt = ctypes.c_int()
        check(lib().cpg_qwen3_step(self.handle, int(token), ctypes.byref(nxt)))
        return nxt.value

    def generate(self, prompt, n_new: int) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_new + 1, np.int32)
        check(lib().cpg_qwen3_generate(self.handle, prompt.ctypes.data, len(prompt), n_new, out.ctypes.data))
        return out

    def logits(self):
        """The last position's logits as a device tensor (a view; valid until the next call)."""
        torch = _torch()
        from .workload import device_view
        return device_view(torch, int(lib().cpg_qwen3_logits(self.handle)), self.vocab * 4, "f4")

    def stream_ptr(self) -> int:
        return int(lib().cpg_qwen3_stream(self.handle) or 0)

    def close(self) -> None:
        if self.handle is not None and self.handle.value:
            lib().cpg_qwen3_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Qwen3Batch:
    """cpg_qwen3_batch: n_slots sequences over one Qwen3Model's weights (continuous batching).
    Each slot has its own KV cache and position; prefill(slot, prompt) starts a sequence in a
    slot, step(slots, ids) advances the named slots by one token each, generate(slots, ids, n)
    runs n such steps feeding each argmax back on the device."""

    def __init__(self, model: Qwen3Model, n_slots: int, max_ctx: int):
        h = ctypes.c_void_p()
        check(lib().cpg_qwen3_batch_create(model.handle, n_slots, max_ctx, ctypes.byref(h)))
        self.handle, self.model, self.vocab, self.n_slots = h, model, model.vocab, n_slots

    def prefill(self, slot: int, ids) -> int:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        nxt = ctypes.c_int()
        check(lib().cpg_qwen3_batch_prefill(self.handle, int(slot), ids.ctypes.data, len(ids), ctypes.byref(nxt)))
        return nxt.value

    def step(self, slots, ids) -> np.ndarray:
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        assert len(slots) == len(ids)
        out = np.zeros(len(slots), np.int32)
        check(lib().cpg_qwen3_batch_step(self.handle, slots.ctypes.data, ids.ctypes.data, len(slots), out.ctypes.data))
        return out

    def generate(self, slots, ids, n_steps: int) -> np.ndarray:
        """(n_steps, len(slots)) ids: row s = the ids step s produced."""
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        assert len(slots) == len(ids)
        out = np.zeros((n_steps, len(slots)), np.int32)
        check(lib().cpg_qwen3_batch_generate(self.handle, slots.ctypes.data, ids.ctypes.data, len(slots), n_steps,
                                             out.ctypes.data))
        return out

    def position(self, slot: int) -> int:
        return int(lib().cpg_qwen3_batch_position(self.handle, int(slot)))

    def logits(self):
        """The last call's logits as a (rows, vocab) device tensor (a view; valid until the next call)."""
        torch = _torch()
        from .workload import device_view
        rows = ctypes.c_int()
        p = int(lib().cpg_qwen3_batch_logits(self.handle, ctypes.byref(rows)))
        return device_view(torch, p, rows.value * self.vocab * 4, "f4").view(rows.value, self.vocab)

    def close(self) -> None:
        if self.handle is not None and self.handle.value:
            lib().cpg_qwen3_batch_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DecodeContext:
    """cpg_ctx: the host-buffer decode loop (run_layers' MoE half, cachepotato.c:149-166)."""

    def __init__(self, shape_layer: MoELayer, max_T: int, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().cpg_ctx_create(device, max_T, shape_layer.handle, ctypes.byref(h)))
        self.handle = h
        self.topk = shape_layer.topk

    def stream_ptr(self) -> int:
        return int(lib().cpg_ctx_stream(self.handle) or 0)

    def run(self, layers, x: np.ndarray, want_topk: bool = False):
        """x (T, d_model) host f32 (ideally pinned), updated in place: x += mlp_l per layer."""
        assert x.dtype == np.float32 and x.flags.c_contiguous
        L, T = len(layers), x.shape[0]
        arr = (ctypes.c_void_p * L)(*[l.handle.value for l in layers])
        topk = np.empty((L, T, self.topk), np.int32) if want_topk else None
        check(lib().cpg_run_moe_layers(self.handle, arr, L, x.ctypes.data, T,
                                       None if topk is None else topk.ctypes.data))
        return topk

    @staticmethod
    def layer_array(layers):
        return (ctypes.c_void_p * len(layers))(*[l.handle.value for l in layers])

    def run_host_ptr(self, arr, L: int, x_ptr: int, T: int) -> None:
        """cpg_run_moe_layers on a host pointer (e.g. a pinned torch tensor)."""
        check(lib().cpg_run_moe_layers(self.handle, arr, L, x_ptr, T, None))

    def run_device(self, arr, L: int, T: int) -> None:
        """cpg_ctx_run: the layers on the context's device activations, no copies, no sync."""
        check(lib().cpg_ctx_run(self.handle, arr, L, T))

    def x_ptr(self) -> int:
        return int(lib().cpg_ctx_x(self.handle))

    def topk_ptr(self) -> int:
        return int(lib().cpg_ctx_topk(self.handle))

    def profile(self, on: bool) -> None:
        check(lib().cpg_ctx_profile(self.handle, 1 if on else 0))

    def phase_ms(self):
        out = (ctypes.c_float * 4)()
        check(lib().cpg_ctx_phase_ms(self.handle, out))
        return [float(v) for v in out]

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                lib().cpg_ctx_destroy(h)
            except Exception:
                pass
            self.handle = None
