"""ctypes bindings for the parity checkers.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
reference legs import this module. It wraps two CPU libraries built by oracle/Makefile:

  _build/libcpg_oracle.so   the C restatement of the reference path (cpg_oracle.c)
  _ref/libcpref.so          the reference engine's own sources + our harness (ref_harness.c);
                            built only where the reference tree exists, then shipped as a
                            prebuilt .so (it may be absent on a fresh checkout)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libcpg_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libcpref.so")
REF_TREE = os.environ.get("CPG_REFERENCE_TREE", "/root/reference")

ENC_F32, ENC_Q8, ENC_Q4 = 0, 8, 4
GROUP_BYTES = {ENC_Q4: 18, ENC_Q8: 34}

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_vpp = ctypes.POINTER(ctypes.c_void_p)


def build(ref: bool = True) -> None:
    """Compile the checkers (the restatement always; the reference when its tree is here)."""
    targets = ["oracle"]
    if ref and os.path.isdir(os.path.join(REF_TREE, "engine")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REF_TREE}", *targets], check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def row_bytes(enc: int, n_in: int) -> int:
    if enc == ENC_F32:
        return 4 * n_in
    return (n_in // 32) * GROUP_BYTES[enc]


class Oracle:
    """The C restatement. Every method takes/returns numpy arrays."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        L = ctypes.CDLL(path)
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        for n in ("orc_q8_dequant_row", "orc_q4_dequant_row"):
            getattr(L, n).argtypes = [_u8p, _f32p, ctypes.c_long]
        for n in ("orc_quantize_q8_0", "orc_quantize_q4_0"):
            getattr(L, n).argtypes = [_f32p, ctypes.c_long, _u8p, ctypes.c_int]
        L.orc_fill_normal.argtypes = [_f32p, ctypes.c_long, ctypes.c_uint64, ctypes.c_float,
                                      ctypes.c_int]
        L.orc_mm.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
        L.orc_silu.restype = ctypes.c_float
        L.orc_silu.argtypes = [ctypes.c_float]
        L.orc_qwen3_moe.restype = ctypes.c_int
        L.orc_qwen3_moe.argtypes = [
            _f32p, ctypes.c_void_p, ctypes.c_int, _vpp, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
            _f32p, _f32p, ctypes.c_int, _f32p, _f32p, _i32p, _f32p, _f32p]
        L.orc_moe_apply.restype = ctypes.c_int
        L.orc_moe_apply.argtypes = [_vpp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p,
                                    ctypes.c_int, ctypes.c_int, _i32p, _f32p, _f32p]
        self.L = L

    # -- format
    def quantize(self, x: np.ndarray, enc: int, nthreads: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert x.size % 32 == 0
        out = np.empty(x.size // 32 * GROUP_BYTES[enc], dtype=np.uint8)
        fn = self.L.orc_quantize_q4_0 if enc == ENC_Q4 else self.L.orc_quantize_q8_0
        nt = nthreads or (os.cpu_count() or 1)
        fn(_ptr(x, _f32p), x.size, _ptr(out, _u8p), nt)
        return out

    def dequant(self, blocks: np.ndarray, n: int, enc: int) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty(n, dtype=np.float32)
        fn = self.L.orc_q4_dequant_row if enc == ENC_Q4 else self.L.orc_q8_dequant_row
        fn(_ptr(blocks, _u8p), _ptr(out, _f32p), n)
        return out

    def normal(self, n: int, seed: int, std: float = 1.0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.L.orc_fill_normal(_ptr(out, _f32p), n, seed, std, os.cpu_count() or 1)
        return out

    # -- kernels
    def mm(self, w: np.ndarray, enc: int, x: np.ndarray, n_in: int, n_out: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(n_out, dtype=np.float32)
        self.L.orc_mm(w.ctypes.data, enc, _ptr(out, _f32p), _ptr(x, _f32p), n_in, n_out)
        return out

    def rmsnorm(self, x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        g = np.ascontiguousarray(g, dtype=np.float32)
        out = np.empty_like(x)
        self.L.orc_rmsnorm(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(g, _f32p), x.size, eps)
        return out

    # -- block
    def qwen3_moe(self, layer: "SynthLayer", x: np.ndarray, attn: np.ndarray | None = None):
        """Returns dict(mlp, router, topk_idx, wt, xn) for tokens x (T, d_model)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, D = x.shape
        E, K = layer.n_experts, layer.topk
        mlp = np.zeros((T, D), np.float32)
        router = np.empty((T, E), np.float32)
        idx = np.empty((T, K), np.int32)
        wt = np.empty((T, K), np.float32)
        xn = np.empty((T, D), np.float32)
        ptrs = layer.expert_ptrs()
        a = None if attn is None else np.ascontiguousarray(attn, dtype=np.float32)
        rc = self.L.orc_qwen3_moe(
            _ptr(layer.ln2, _f32p), layer.wgate.ctypes.data, ENC_F32, ptrs, layer.enc,
            D, layer.d_exp, E, K, layer.eps, _ptr(x, _f32p),
            None if a is None else _ptr(a, _f32p), T,
            _ptr(mlp, _f32p), _ptr(router, _f32p), _ptr(idx, _i32p), _ptr(wt, _f32p),
            _ptr(xn, _f32p))
        assert rc == 0
        return dict(mlp=mlp, router=router, topk_idx=idx, wt=wt, xn=xn)

    def moe_apply(self, layer: "SynthLayer", xn: np.ndarray, idx: np.ndarray, wt: np.ndarray):
        xn = np.ascontiguousarray(xn, dtype=np.float32)
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        wt = np.ascontiguousarray(wt, dtype=np.float32)
        T, D = xn.shape
        mlp = np.zeros((T, D), np.float32)
        rc = self.L.orc_moe_apply(layer.expert_ptrs(), layer.enc, D, layer.d_exp,
                                  _ptr(xn, _f32p), T, idx.shape[1], _ptr(idx, _i32p),
                                  _ptr(wt, _f32p), _ptr(mlp, _f32p))
        assert rc == 0
        return mlp


class Reference:
    """The reference engine itself (oracle/_ref/libcpref.so). Raises if it was never built."""

    def __init__(self, path: str = REF_SO, threads: int = 0):
        if not os.path.exists(path):
            build(ref=True)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path}: reference engine not built (no reference tree)")
        L = ctypes.CDLL(path)
        L.refh_init_threads.restype = ctypes.c_int
        L.refh_init_threads.argtypes = [ctypes.c_int]
        L.refh_qwen3_moe.restype = ctypes.c_int
        L.refh_qwen3_moe.argtypes = [
            _f32p, _f32p, _vpp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_float, _f32p, ctypes.c_int, _f32p, _f32p, _i32p]
        L.refh_moe_apply.restype = ctypes.c_int
        L.refh_moe_apply.argtypes = [_vpp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p,
                                     ctypes.c_int, ctypes.c_int, _i32p, _f32p, _f32p]
        for n in ("matmul_wx_q4", "matmul_wx_q8"):
            getattr(L, n).argtypes = [_f32p, _f32p, _u8p, ctypes.c_int, ctypes.c_int]
        L.matmul_wx.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        for n in ("q4_dequant_row", "q8_dequant_row"):
            getattr(L, n).argtypes = [_u8p, _f32p, ctypes.c_int]
        # the pool is process-global and only the first initialisation counts (parallel.c:126-132)
        self.threads = L.refh_init_threads(threads or (os.cpu_count() or 1))
        self.L = L

    def dequant(self, blocks: np.ndarray, n: int, enc: int) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty(n, dtype=np.float32)
        fn = self.L.q4_dequant_row if enc == ENC_Q4 else self.L.q8_dequant_row
        fn(_ptr(blocks, _u8p), _ptr(out, _f32p), n)
        return out

    def mm(self, w: np.ndarray, enc: int, x: np.ndarray, n_in: int, n_out: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(n_out, dtype=np.float32)
        if enc == ENC_Q4:
            self.L.matmul_wx_q4(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(w, _u8p), n_in, n_out)
        elif enc == ENC_Q8:
            self.L.matmul_wx_q8(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(w, _u8p), n_in, n_out)
        else:
            self.L.matmul_wx(_ptr(out, _f32p), _ptr(x, _f32p), _ptr(w, _f32p), n_in, n_out)
        return out

    def qwen3_moe(self, layer: "SynthLayer", x: np.ndarray):
        """The unmodified qwen3_layer_kv on x (T, d_model); returns dict(mlp, router, topk_idx)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, D = x.shape
        E, K = layer.n_experts, layer.topk
        mlp = np.zeros((T, D), np.float32)
        router = np.empty((T, E), np.float32)
        idx = np.empty((T, K), np.int32)
        rc = self.L.refh_qwen3_moe(_ptr(layer.ln2, _f32p), _ptr(layer.wgate, _f32p),
                                   layer.expert_ptrs(), layer.enc, D, layer.d_exp, E, K,
                                   layer.eps, _ptr(x, _f32p), T, _ptr(mlp, _f32p),
                                   _ptr(router, _f32p), _ptr(idx, _i32p))
        assert rc == 0, rc
        return dict(mlp=mlp, router=router, topk_idx=idx)

    def moe_apply(self, layer: "SynthLayer", xn: np.ndarray, idx: np.ndarray, wt: np.ndarray):
        xn = np.ascontiguousarray(xn, dtype=np.float32)
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        wt = np.ascontiguousarray(wt, dtype=np.float32)
        T, D = xn.shape
        mlp = np.zeros((T, D), np.float32)
        rc = self.L.refh_moe_apply(layer.expert_ptrs(), layer.enc, D, layer.d_exp,
                                   _ptr(xn, _f32p), T, idx.shape[1], _ptr(idx, _i32p),
                                   _ptr(wt, _f32p), _ptr(mlp, _f32p))
        assert rc == 0
        return mlp


def reference_available() -> bool:
    return os.path.exists(REF_SO) or os.path.isdir(os.path.join(REF_TREE, "engine"))


class SynthLayer:
    """One Qwen3-MoE layer held in host memory: f32 router, f32 ln2, and per-expert regions
    laid out as in a CPW1 v4 file (Wg, Wu, Wd contiguous per expert; models/qwen3-30b-a3b
    convert.py:182-237), quantised with the oracle's encoder."""

    def __init__(self, d_model: int, d_exp: int, n_experts: int, topk: int, enc: int,
                 seed: int, eps: float = 1e-6, router_scale: np.ndarray | None = None,
                 oracle: Oracle | None = None, std: float = 0.02):
        self.d_model, self.d_exp, self.n_experts, self.topk = d_model, d_exp, n_experts, topk
        self.enc, self.eps = enc, eps
        orc = oracle or Oracle()
        self.ln2 = np.ones(d_model, np.float32)
        self.wgate = orc.normal(n_experts * d_model, seed * 2 + 1, std).reshape(n_experts, d_model)
        if router_scale is not None:
            self.wgate *= router_scale.astype(np.float32)[:, None]
        self.wgate = np.ascontiguousarray(self.wgate, dtype=np.float32)
        n_mat = d_exp * d_model
        self.mat_bytes = n_mat // 32 * GROUP_BYTES[enc]
        self.region_bytes = 3 * self.mat_bytes
        w = orc.normal(n_experts * 3 * n_mat, seed * 2 + 2, std)
        # (e, kind, rows, cols): gate/up are (d_exp, d_model), down is (d_model, d_exp); the
        # flat order per expert is Wg | Wu | Wd, each row-major
        self.blob = orc.quantize(w, enc)
        del w
        self._ptrs = None

    def expert_ptrs(self):
        if self._ptrs is None:
            base = self.blob.ctypes.data
            arr = (ctypes.c_void_p * (self.n_experts * 3))()
            for e in range(self.n_experts):
                for k in range(3):
                    arr[e * 3 + k] = base + e * self.region_bytes + k * self.mat_bytes
            self._ptrs = arr
        return ctypes.cast(self._ptrs, _vpp)

    def expert_matrix(self, e: int, kind: int) -> np.ndarray:
        o = e * self.region_bytes + kind * self.mat_bytes
        return self.blob[o:o + self.mat_bytes]

    def shard(self, r: int, G: int) -> "SynthLayer":
        """Experts [r*E/G, (r+1)*E/G) as a layer of their own (the local layer of rank r of an
        expert-parallel group); the blob is a view of this layer's."""
        assert self.n_experts % G == 0
        E_l = self.n_experts // G
        sub = object.__new__(SynthLayer)
        sub.__dict__.update(self.__dict__)
        sub.n_experts = E_l
        sub.wgate = np.ascontiguousarray(self.wgate[r * E_l:(r + 1) * E_l])
        sub.blob = self.blob[r * E_l * self.region_bytes:(r + 1) * E_l * self.region_bytes]
        sub._ptrs = None
        return sub
