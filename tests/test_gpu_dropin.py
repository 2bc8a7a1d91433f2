"""The drop-in, proven on the reference engine itself: the reference's own qwen3_moe.c compiled
with qwen3_mm's kernel calls (qwen3_moe.c:36-40) routed to this library by compiler flags alone
(-Dmatmul_wx_q4=cpg_matmul_wx_q4 -Dmatmul_wx_q8=cpg_matmul_wx_q8 -Dmatmul_wx=cpg_matmul_wx; no
reference file edited; oracle/Makefile target ref_gpu), linked to libcpg_b200.so. The unmodified
qwen3_layer_kv then runs its router and every expert GEMV on the GPU, reading the weights from
the HBM region store that mirrors the host mapping (cpg_store_open_v4), while the plain CPU
build of the same sources computes the reference answer on the same mapping.

Bar: identical expert ids (tie-aware), router logits and block output within 1e-5 (the f32
matvec kernel gate, tools/verify_q8_kernels.py)."""
import ctypes
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_rel
from helpers import KERNEL_TOL, check_topk

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


class _Mapped:
    """A SynthLayer whose tensors all live in one host buffer laid out like a v4 data section
    (ln2 | router | expert regions, 64-byte aligned), so the store can mirror it."""

    def __init__(self, L):
        self.__dict__.update({k: v for k, v in L.__dict__.items() if k != "_ptrs"})
        parts = [L.ln2.view(np.uint8), L.wgate.reshape(-1).view(np.uint8), L.blob]
        offs, o = [], 0
        for p in parts:
            offs.append(o)
            o = (o + p.nbytes + 63) // 64 * 64
        self.mapping = np.zeros(o + 64, np.uint8)
        base = (-self.mapping.ctypes.data) % 64
        self.mapping = self.mapping[base:base + o]
        for p, off in zip(parts, offs):
            self.mapping[off:off + p.nbytes] = p
        self.ln2 = self.mapping[offs[0]:offs[0] + L.ln2.nbytes].view(np.float32)
        self.wgate = self.mapping[offs[1]:offs[1] + L.wgate.nbytes].view(np.float32).reshape(L.wgate.shape)
        self.blob = self.mapping[offs[2]:offs[2] + L.blob.nbytes]
        self._ptrs = None

    expert_ptrs = O.SynthLayer.expert_ptrs


@pytest.mark.parametrize("enc,T", [(O.ENC_Q4, 1), (O.ENC_Q4, 3), (O.ENC_Q8, 2)])
def test_reference_engine_runs_on_gpu_dropins(orc, enc, T):
    from cachepotato_b200 import _lib
    if not os.path.exists(O.REF_GPU_SO):
        pytest.skip("the drop-in build of the reference engine was not built (no reference tree)")
    lib = _lib.lib()
    ref_cpu = O.Reference(threads=8)
    ref_gpu = O.Reference(path=O.REF_GPU_SO, threads=8)
    D, F, E, K = 2048, 768, 128, 8
    L = _Mapped(O.SynthLayer(D, F, E, K, enc, seed=60 + enc + T, oracle=orc))
    x = orc.normal(T * D, 61 + T, 1.0).reshape(T, D)
    want = ref_cpu.qwen3_moe(L, x)
    _lib.check(lib.cpg_store_open_v4(ctypes.c_void_p(L.mapping.ctypes.data), L.mapping.nbytes, 0))
    try:
        # the layer's tensors resolve to resident device copies (no per-call upload)
        for p in (L.wgate.ctypes.data, L.blob.ctypes.data, L.blob.ctypes.data + L.blob.nbytes - 1):
            assert lib.cpg_store_translate(ctypes.c_void_p(p))
        got = ref_gpu.qwen3_moe(L, x)
    finally:
        lib.cpg_store_close()
    assert _lib.last_error() == ""
    assert max_rel(got["router"], want["router"]) <= KERNEL_TOL
    bad = check_topk(got["topk_idx"], want["topk_idx"], want["router"], K)
    assert not bad, bad
    ok = np.all(got["topk_idx"] == want["topk_idx"], axis=1)
    assert max_rel(got["mlp"][ok], want["mlp"][ok]) <= KERNEL_TOL
