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
REF_GPU_SO = os.path.join(HERE, "_ref", "libcpref_gpu.so")
REF_API_SO = os.path.join(HERE, "_ref", "libcpref_api.so")    # the reference's cachepotato.h engine (CPU)
REF_TOK_SO = os.path.join(HERE, "_ref", "libcpref_tok.so")    # its tokenizer module alone
# The reference source tree: CPG_REFERENCE_TREE, else a `reference` checkout beside this
# repository (where the build environment keeps it). Absent on machines that only run the
# prebuilt checkers.
REF_TREE = os.environ.get("CPG_REFERENCE_TREE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")

ENC_F32, ENC_Q8, ENC_Q4 = 0, 8, 4
GROUP_BYTES = {ENC_Q4: 18, ENC_Q8: 34}

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_vpp = ctypes.POINTER(ctypes.c_void_p)


def build(ref: bool = True) -> None:
    """Compile the checkers (the restatement always; the reference when its tree is here, and
    its drop-in build linked to libcpg_b200.so when that library exists)."""
    targets = ["oracle"]
    if ref and os.path.isdir(os.path.join(REF_TREE, "engine")):
        targets += ["ref", "ref_api"]
        if os.path.exists(os.path.join(os.path.dirname(HERE), "cachepotato_b200", "_build", "libcpg_b200.so")):
            targets.append("ref_gpu")
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
        L.refh_qwen3_generate.restype = ctypes.c_int
        L.refh_qwen3_generate.argtypes = ([ctypes.c_int] * 9 + [ctypes.c_float] * 2 +
                                          [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, _f32p] +
                                          [_vpp] * 8 + [ctypes.c_int, _vpp, _vpp, ctypes.c_int] +
                                          [_i32p, ctypes.c_int, ctypes.c_int, _i32p, _f32p])
        if hasattr(L, "refh_v4_generate"):
            L.refh_v4_generate.restype = ctypes.c_int
            L.refh_v4_generate.argtypes = [ctypes.c_char_p, _i32p, ctypes.c_int, ctypes.c_int, _i32p, _f32p, _i32p]
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

    def qwen3_generate(self, model: "SynthModel", prompt, n_new: int):
        """The reference engine over a whole model: the prompt in one pass, then n_new greedy
        steps. Returns (ids of the n_new + 1 argmaxes, logits of the last step)."""
        m = model
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        ids = np.zeros(n_new + 1, np.int32)
        logits = np.zeros(m.vocab, np.float32)

        def arr(xs):
            a = (ctypes.c_void_p * len(xs))(*[x.ctypes.data for x in xs])
            keep.append(a)
            return ctypes.cast(a, _vpp)
        keep = []
        exp = (ctypes.c_void_p * (m.n_layers * m.n_experts * 3))()
        for l, ly in enumerate(m.layers):
            for e in range(m.n_experts):
                for k in range(3):
                    exp[(l * m.n_experts + e) * 3 + k] = ly.blob.ctypes.data + e * ly.region_bytes + k * ly.mat_bytes
        rc = self.L.refh_qwen3_generate(
            m.d_model, m.n_heads, m.n_kv, m.head_dim, m.d_exp, m.n_experts, m.topk, m.vocab, m.n_layers,
            m.rope_theta, m.eps, m.embed.ctypes.data, m.embed_enc, m.lm_head.ctypes.data, m.head_enc,
            _ptr(m.final_norm, _f32p), arr(m.ln1), arr([ly.ln2 for ly in m.layers]), arr(m.q_norm), arr(m.k_norm),
            arr(m.wq), arr(m.wk), arr(m.wv), arr(m.wo), m.attn_enc, arr([ly.wgate for ly in m.layers]),
            ctypes.cast(exp, _vpp), m.layers[0].enc, _ptr(prompt, _i32p), len(prompt), n_new,
            _ptr(ids, _i32p), _ptr(logits, _f32p))
        assert rc == 0
        return ids, logits

    def v4_generate(self, path: str, prompt, n_new: int):
        """A CPW1 v4 file through the reference's own loader and generate loop. Returns (ids of
        the n_new + 1 argmaxes, the last step's logits, [layers, d_model, vocab, experts, topk,
        d_exp])."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        ids = np.zeros(n_new + 1, np.int32)
        meta = np.zeros(6, np.int32)
        logits = np.zeros(151936 * 2, np.float32)          # the loader's vocabulary (qwen3_moe.c:401), with room
        rc = self.L.refh_v4_generate(path.encode(), _ptr(prompt, _i32p), len(prompt), n_new, _ptr(ids, _i32p),
                                     _ptr(logits, _f32p), _ptr(meta, _i32p))
        assert rc == 0, rc
        return ids, logits[:meta[2]].copy(), meta

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


class SynthModel:
    """A whole Qwen3-MoE model in host memory (the whole-model benchmark shape or smaller): per layer an
    attention half (ln1, Wq/Wk/Wv/Wo in attn_enc, q_norm/k_norm) and a SynthLayer MoE half, plus
    embed and lm_head (head_enc) and the final norm. Norm gains are 1 + norm_jitter·N(0,1)."""

    def __init__(self, d_model, n_heads, n_kv, head_dim, d_exp, n_experts, topk, vocab, n_layers, seed,
                 attn_enc=ENC_Q4, exp_enc=ENC_Q4, head_enc=ENC_Q8, rope_theta=1e6, eps=1e-6, norm_jitter=0.0,
                 oracle: Oracle | None = None, std: float = 0.02):
        orc = oracle or Oracle()
        self.d_model, self.n_heads, self.n_kv, self.head_dim = d_model, n_heads, n_kv, head_dim
        self.d_exp, self.n_experts, self.topk, self.vocab, self.n_layers = d_exp, n_experts, topk, vocab, n_layers
        self.rope_theta, self.eps = rope_theta, eps
        self.attn_enc, self.head_enc, self.embed_enc = attn_enc, head_enc, head_enc
        qd, kd = n_heads * head_dim, n_kv * head_dim

        def gain(n, s):
            g = np.ones(n, np.float32)
            if norm_jitter:
                g += norm_jitter * orc.normal(n, s, 1.0)
            return np.ascontiguousarray(g, dtype=np.float32)

        def mat(rows, cols, s, enc):
            w = orc.normal(rows * cols, s, std)
            return w if enc == ENC_F32 else orc.quantize(w, enc)
        self.layers, self.ln1, self.q_norm, self.k_norm = [], [], [], []
        self.wq, self.wk, self.wv, self.wo = [], [], [], []
        for l in range(n_layers):
            b = seed * 1000 + 20 * l
            ly = SynthLayer(d_model, d_exp, n_experts, topk, exp_enc, seed=b + 1, oracle=orc, std=std)
            ly.ln2 = gain(d_model, b + 2)
            self.layers.append(ly)
            self.ln1.append(gain(d_model, b + 3))
            self.q_norm.append(gain(head_dim, b + 4))
            self.k_norm.append(gain(head_dim, b + 5))
            self.wq.append(mat(qd, d_model, b + 6, attn_enc))
            self.wk.append(mat(kd, d_model, b + 7, attn_enc))
            self.wv.append(mat(kd, d_model, b + 8, attn_enc))
            self.wo.append(mat(d_model, qd, b + 9, attn_enc))
        self.embed = mat(vocab, d_model, seed * 1000 + 991, head_enc)
        self.lm_head = mat(vocab, d_model, seed * 1000 + 992, head_enc)
        self.final_norm = gain(d_model, seed * 1000 + 993)


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
