"""cachepotato_b200 — the Qwen3-MoE expert hot path of CachePotato, native on B200 (sm_100a).

The product is libcpg_b200.so (C ABI in include/cpg.h); this package builds it, binds it with
ctypes and mirrors the reference interface (cachepotato_b200.qwen3). There is no CPU fallback.
"""
from ._lib import CpgError, ENC_F32, ENC_Q4, ENC_Q8, lib  # noqa: F401

__all__ = ["CpgError", "ENC_F32", "ENC_Q4", "ENC_Q8", "lib"]
