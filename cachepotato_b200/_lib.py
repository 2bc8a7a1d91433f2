"""ctypes binding of libcpg_b200.so (include/cpg.h).

There is no fallback: if the CUDA library is missing or fails to load, importing the API
raises. Device pointers are plain integers (e.g. torch.Tensor.data_ptr()).
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB

CPG_OK, CPG_EINVAL, CPG_ECUDA, CPG_ETIMEOUT, CPG_ENOMEM, CPG_ENCCL, CPG_ESTATE = 0, -1, -2, -3, -4, -5, -6
ENC_F32, ENC_Q8, ENC_Q4 = 0, 8, 4
GROUP_BYTES = {ENC_Q4: 18, ENC_Q8: 34}

# every symbol include/cpg.h declares (tests check the library exports each one)
EXPORTS = [
    "cpg_last_error", "cpg_version",
    "cpg_matmul_wx", "cpg_matmul_wx_q8", "cpg_matmul_wx_q4", "cpg_q8_dequant_row", "cpg_q4_dequant_row",
    "cpg_dequant", "cpg_quantize", "cpg_matvec",
    "cpg_store_open_v4", "cpg_store_open", "cpg_store_add_region", "cpg_store_region_get",
    "cpg_store_translate", "cpg_store_base", "cpg_store_bytes", "cpg_store_totals", "cpg_store_close",
    "cpg_store_verify", "cpg_crc32", "cpg_route_check",
    "cpg_moe_layer_create", "cpg_moe_layer_destroy", "cpg_moe_workspace_bytes", "cpg_moe_forward",
    "cpg_moe_check", "cpg_moe_forward_noalloc",
    "cpg_ctx_create", "cpg_ctx_destroy", "cpg_ctx_stream", "cpg_run_moe_layers",
    "cpg_ctx_run", "cpg_ctx_x", "cpg_ctx_topk", "cpg_ctx_profile", "cpg_ctx_phase_ms",
    "cpg_moe_apply_workspace_bytes", "cpg_moe_apply", "cpg_moe_apply_check", "cpg_moe_apply_profile",
    "cpg_moe_apply_rows", "cpg_ep_unique_id", "cpg_ep_create", "cpg_ep_destroy", "cpg_ep_workspace_bytes",
    "cpg_moe_ep", "cpg_moe_ep_check", "cpg_moe_ep_profile", "cpg_ep_set_timeout", "cpg_ep_abort", "cpg_ep_wait",
    "cpg_qwen3_create", "cpg_qwen3_destroy", "cpg_qwen3_prefill", "cpg_qwen3_step", "cpg_qwen3_generate",
    "cpg_qwen3_append", "cpg_qwen3_rewind",
    "cpg_qwen3_logits", "cpg_qwen3_stream", "cpg_qwen3_position",
    "cpg_qwen3_batch_create", "cpg_qwen3_batch_destroy", "cpg_qwen3_batch_prefill", "cpg_qwen3_batch_step",
    "cpg_qwen3_batch_generate", "cpg_qwen3_batch_position", "cpg_qwen3_batch_logits",
]


class CpgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"cpg error {code}: {msg}")
        self.code = code


class Tensor(ctypes.Structure):
    """cpg_tensor / QW3T: pointer + encoding."""
    _fields_ = [("p", ctypes.c_void_p), ("enc", ctypes.c_int)]


class MoeDesc(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int), ("d_exp", ctypes.c_int), ("n_experts", ctypes.c_int),
                ("topk", ctypes.c_int), ("rms_eps", ctypes.c_float), ("ln2", ctypes.c_void_p),
                ("wgate", Tensor), ("experts", ctypes.POINTER(Tensor))]


class Qwen3Attn(ctypes.Structure):
    _fields_ = [("ln1", ctypes.c_void_p), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("wq", Tensor), ("wk", Tensor), ("wv", Tensor), ("wo", Tensor)]


class Qwen3Desc(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int), ("n_heads", ctypes.c_int), ("n_kv", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("vocab", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("max_ctx", ctypes.c_int), ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float),
                ("embed", Tensor), ("lm_head", Tensor), ("final_norm", ctypes.c_void_p),
                ("attn", ctypes.POINTER(Qwen3Attn)), ("moe", ctypes.POINTER(ctypes.c_void_p))]


class StoreTotals(ctypes.Structure):
    _fields_ = [("regions", ctypes.c_long), ("expert_regions", ctypes.c_long),
                ("resident_bytes", ctypes.c_long), ("h2d_bytes", ctypes.c_long)]


_vp, _i, _l, _sz, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_size_t, ctypes.c_float
_SIGS = {
    "cpg_last_error": (ctypes.c_char_p, []),
    "cpg_version": (_i, []),
    "cpg_matmul_wx": (None, [_vp, _vp, _vp, _i, _i]),
    "cpg_matmul_wx_q8": (None, [_vp, _vp, _vp, _i, _i]),
    "cpg_matmul_wx_q4": (None, [_vp, _vp, _vp, _i, _i]),
    "cpg_q8_dequant_row": (None, [_vp, _vp, _i]),
    "cpg_q4_dequant_row": (None, [_vp, _vp, _i]),
    "cpg_dequant": (_i, [_vp, _vp, _i, _l, _vp]),
    "cpg_quantize": (_i, [_vp, _vp, _i, _l, _vp]),
    "cpg_matvec": (_i, [_vp, _vp, Tensor, _i, _i, _i, _vp]),
    "cpg_store_open_v4": (_i, [_vp, _sz, _sz]),
    "cpg_store_open": (_i, [_sz]),
    "cpg_store_add_region": (_i, [_sz, _sz, _i]),
    "cpg_store_region_get": (_vp, [_i]),
    "cpg_store_translate": (_vp, [_vp]),
    "cpg_store_base": (_vp, []),
    "cpg_store_bytes": (_sz, []),
    "cpg_store_totals": (_i, [ctypes.POINTER(StoreTotals)]),
    "cpg_store_close": (None, []),
    "cpg_store_verify": (_i, [_vp, _i, ctypes.POINTER(_i)]),
    "cpg_crc32": (_i, [_vp, _sz, ctypes.POINTER(ctypes.c_uint32), _vp]),
    "cpg_route_check": (_i, [_vp, _vp, _vp, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(ctypes.c_double), _vp]),
    "cpg_moe_layer_create": (_i, [ctypes.POINTER(MoeDesc), ctypes.POINTER(_vp)]),
    "cpg_moe_layer_destroy": (None, [_vp]),
    "cpg_moe_workspace_bytes": (_sz, [_vp, _i]),
    "cpg_moe_forward": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "cpg_moe_check": (_i, [_vp, _vp]),
    "cpg_moe_forward_noalloc": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "cpg_ctx_create": (_i, [_i, _i, _vp, ctypes.POINTER(_vp)]),
    "cpg_ctx_destroy": (None, [_vp]),
    "cpg_ctx_stream": (_vp, [_vp]),
    "cpg_run_moe_layers": (_i, [_vp, ctypes.POINTER(_vp), _i, _vp, _i, _vp]),
    "cpg_ctx_run": (_i, [_vp, ctypes.POINTER(_vp), _i, _i]),
    "cpg_moe_apply_workspace_bytes": (_sz, [_vp, _i]),
    "cpg_moe_apply": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _sz, _vp]),
    "cpg_moe_apply_check": (_i, [_vp, _vp]),
    "cpg_moe_apply_profile": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _sz, _vp, ctypes.POINTER(ctypes.c_float)]),
    "cpg_moe_apply_rows": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _sz, _vp]),
    "cpg_ep_unique_id": (_i, [_vp]),
    "cpg_ep_create": (_i, [_i, _i, _vp, ctypes.POINTER(_vp)]),
    "cpg_ep_destroy": (None, [_vp]),
    "cpg_ep_workspace_bytes": (_sz, [_vp, _vp, _i]),
    "cpg_moe_ep": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _sz, _vp]),
    "cpg_moe_ep_check": (_i, [_vp, _vp]),
    "cpg_moe_ep_profile": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _sz, _vp, ctypes.POINTER(ctypes.c_float)]),
    "cpg_ep_set_timeout": (_i, [_vp, _i]),
    "cpg_ep_abort": (_i, [_vp]),
    "cpg_ep_wait": (_i, [_vp, _vp]),
    "cpg_qwen3_create": (_i, [ctypes.POINTER(Qwen3Desc), ctypes.POINTER(_vp)]),
    "cpg_qwen3_destroy": (None, [_vp]),
    "cpg_qwen3_prefill": (_i, [_vp, _vp, _i, ctypes.POINTER(_i)]),
    "cpg_qwen3_step": (_i, [_vp, _i, ctypes.POINTER(_i)]),
    "cpg_qwen3_append": (_i, [_vp, _vp, _i, ctypes.POINTER(_i)]),
    "cpg_qwen3_rewind": (_i, [_vp, _i]),
    "cpg_qwen3_generate": (_i, [_vp, _vp, _i, _i, _vp]),
    "cpg_qwen3_logits": (_vp, [_vp]),
    "cpg_qwen3_stream": (_vp, [_vp]),
    "cpg_qwen3_position": (_i, [_vp]),
    "cpg_qwen3_batch_create": (_i, [_vp, _i, _i, ctypes.POINTER(_vp)]),
    "cpg_qwen3_batch_destroy": (None, [_vp]),
    "cpg_qwen3_batch_prefill": (_i, [_vp, _i, _vp, _i, ctypes.POINTER(_i)]),
    "cpg_qwen3_batch_step": (_i, [_vp, _vp, _vp, _i, _vp]),
    "cpg_qwen3_batch_generate": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "cpg_qwen3_batch_position": (_i, [_vp, _i]),
    "cpg_qwen3_batch_logits": (_vp, [_vp, ctypes.POINTER(_i)]),
    "cpg_ctx_x": (_vp, [_vp]),
    "cpg_ctx_topk": (_vp, [_vp]),
    "cpg_ctx_profile": (_i, [_vp, _i]),
    "cpg_ctx_phase_ms": (_i, [_vp, ctypes.POINTER(ctypes.c_float)]),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load libcpg_b200.so (raises if it was never built: there is no CPU fallback)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB):
            raise ImportError(f"{LIB} is missing: build it with `python -m cachepotato_b200.build`")
        L = ctypes.CDLL(LIB)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def last_error() -> str:
    return (lib().cpg_last_error() or b"").decode()


def check(rc: int) -> None:
    if rc != CPG_OK:
        raise CpgError(rc, last_error())
