"""CPU-side checks of libcachepotato_b200.so, the engine's public API (include/cpg_chat.h,
engine/api/cachepotato.h) over the GPU model: with the reference's tokenizer module loaded, as a
front-end links it, the library loads without a GPU and exports every function the header
declares; errors before any device work are reported, not crashes; the machine probes and
the defaults agree with the reference's own cachepotato.c (oracle/_ref/libcpref_api.so)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

CHAT_SO = os.path.join(ROOT, "cachepotato_b200", "_build", "libcachepotato_b200.so")
REF_API = os.path.join(ROOT, "oracle", "_ref", "libcpref_api.so")
REF_TOK = os.path.join(ROOT, "oracle", "_ref", "libcpref_tok.so")


def _declared():
    src = open(os.path.join(ROOT, "include", "cpg_chat.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cp_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def libs():
    if not (os.path.exists(CHAT_SO) and os.path.exists(REF_API) and os.path.exists(REF_TOK)):
        pytest.skip("libcachepotato_b200.so or the reference's API / tokenizer build is missing")
    ctypes.CDLL(REF_TOK, mode=ctypes.RTLD_GLOBAL)
    return ctypes.CDLL(CHAT_SO), ctypes.CDLL(REF_API)


def test_exports_every_declared_function(libs):
    ours, ref = libs
    names = _declared()
    assert len(names) == 9, names
    assert not [n for n in names if not hasattr(ours, n)]
    assert not [n for n in names if not hasattr(ref, n)]          # the same API as the reference


def test_defaults_and_probes_match_the_reference(libs):
    ours, ref = libs

    class Options(ctypes.Structure):
        _fields_ = [("budget_mb", ctypes.c_long), ("threads", ctypes.c_int), ("pin_cores", ctypes.c_int),
                    ("max_ctx", ctypes.c_int), ("tokenizer_dir", ctypes.c_char_p)]
    a, b = Options(), Options()
    ours.cp_options_default(ctypes.byref(a))
    ref.cp_options_default(ctypes.byref(b))
    assert bytes(a) == bytes(b)
    assert ours.cp_physical_cores() == ref.cp_physical_cores() >= 1
    for lib in (ours, ref):
        lib.cp_auto_budget_mb.restype = ctypes.c_long
        lib.cp_auto_budget_mb.argtypes = [ctypes.c_longlong]
        lib.cp_mem_available_mb.restype = ctypes.c_long
    for size in (0, 1 << 20, 16 << 30, 1 << 45):
        assert ours.cp_auto_budget_mb(size) == ref.cp_auto_budget_mb(size)
    assert abs(ours.cp_mem_available_mb() - ref.cp_mem_available_mb()) < 512


def test_open_errors_are_reported(libs, tmp_path):
    ours, _ = libs
    ours.cp_open.restype = ctypes.c_void_p
    ours.cp_open.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    err = ctypes.create_string_buffer(256)
    assert not ours.cp_open(str(tmp_path / "missing.v4cp").encode(), None, err, 256)
    assert b"cannot open model file" in err.value
    model = tmp_path / "model.v4cp"
    model.write_bytes(b"\0" * 128)
    assert not ours.cp_open(str(model).encode(), None, err, 256)     # no tokenizer beside it
    assert b"tokenizer files" in err.value
