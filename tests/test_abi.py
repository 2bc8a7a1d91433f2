"""CPU-side checks of the C ABI: the library loads without a GPU and exports every symbol that
include/cpg.h declares; host-side helpers (router calibration) behave."""
import os
import re

import numpy as np

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "cpg.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cpg_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    import ctypes
    from cachepotato_b200 import _lib
    L = _lib.lib()
    declared = _declared()
    assert len(declared) >= 30
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing
    assert set(declared) == set(_lib.EXPORTS), set(declared) ^ set(_lib.EXPORTS)
    assert L.cpg_version() == 100


def test_errors_without_a_gpu_are_reported_not_crashes():
    import ctypes
    from cachepotato_b200 import _lib
    L = _lib.lib()
    # argument validation happens before any CUDA call
    assert L.cpg_dequant(None, None, 4, 64, None) == _lib.CPG_EINVAL
    assert "null" in _lib.last_error()
    assert L.cpg_quantize(1 << 20, 1 << 20, 4, 33, None) == _lib.CPG_EINVAL
    assert "multiple of 32" in _lib.last_error()
    assert L.cpg_store_add_region(0, 16, 1) == _lib.CPG_ESTATE
    assert L.cpg_store_region_get(0) is None
    assert L.cpg_store_verify(None, 0, None) == _lib.CPG_ESTATE          # no store open
    out = ctypes.c_uint32(5)
    assert L.cpg_crc32(None, 0, ctypes.byref(out), None) == 0 and out.value == 0   # zlib.crc32(b"")
    assert L.cpg_crc32(None, 5, ctypes.byref(out), None) == _lib.CPG_EINVAL
    st, er = (ctypes.c_int * 3)(), (ctypes.c_double * 2)()
    assert L.cpg_route_check(None, None, None, 0, 128, 8, st, er, None) == 0 and st[2] == -1
    assert L.cpg_route_check(None, None, None, 4, 300, 8, st, er, None) == _lib.CPG_EINVAL


def test_router_calibration_is_deterministic_and_skewed():
    from cachepotato_b200.workload import calibrate_router_scales, load_stats, rmsnorm_rows, topk_counts
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 2048)).astype(np.float32)
    W = (rng.standard_normal((128, 2048)) * 0.02).astype(np.float32)
    z = rmsnorm_rows(x) @ W.T
    s1 = calibrate_router_scales(z, 8, 1.1, seed=3)
    s2 = calibrate_router_scales(z, 8, 1.1, seed=3)
    assert np.array_equal(s1, s2)
    c = topk_counts(z, s1, 8)
    c0 = topk_counts(z, np.ones(128), 8)
    assert c.sum() == 64 * 8 and c.max() >= 3 * c0.max() // 2
    assert 80 <= load_stats(np.argsort(-(z * s1), 1)[:, :8], 128)["distinct_experts"] <= 128
