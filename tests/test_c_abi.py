"""include/cpg.h from plain C: a C11 program (tests/c/abi_smoke.c) compiled with gcc against the
header and linked to libcpg_b200.so, as the reference's C engine would link it. CPU only: it
calls the entry points that return before any CUDA work."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "cachepotato_b200", "_build")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_header_compiles_as_c11_and_links():
    if not os.path.exists(os.path.join(LIBDIR, "libcpg_b200.so")):
        pytest.skip("library not built")
    out_dir = os.path.join(ROOT, "tests", "c", "_build")      # git-ignored, inside the tree
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "abi_smoke")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "abi_smoke.c"), "-L", LIBDIR, "-lcpg_b200",
                    "-Wl,-rpath," + LIBDIR, "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", (out.stdout, out.stderr)
