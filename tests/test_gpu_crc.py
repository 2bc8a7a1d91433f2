"""CRC-32 of device memory, the CPW1 v4 region digest, against zlib.crc32: the reference writer's
own definition (format/v4_writer.py:248, "the single definition" the loader must match), and the
region store's digest check through the C ABI."""
import ctypes
import time
import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _crc(L, ptr, n):
    from cachepotato_b200 import _lib
    out = ctypes.c_uint32()
    _lib.check(L.cpg_crc32(ptr, n, ctypes.byref(out), None))
    return out.value


def test_crc32_matches_zlib():
    from cachepotato_b200 import _lib
    L = _lib.lib()
    chk = torch.tensor(list(b"123456789"), dtype=torch.uint8, device="cuda")
    assert _crc(L, chk.data_ptr(), 9) == 0xCBF43926 == zlib.crc32(b"123456789")
    host = np.random.default_rng(7).integers(0, 256, 3_000_100, dtype=np.uint8)
    dev = torch.from_numpy(host).cuda()
    # piece (512 B) and segment (64 KiB) boundaries, unaligned starts
    for n in (0, 1, 3, 4, 5, 511, 512, 513, 65535, 65536, 65537, 131072 + 7, 3_000_001):
        for off in (0, 1, 3, 16):
            assert _crc(L, dev.data_ptr() + off, n) == zlib.crc32(host[off:off + n].tobytes()), (n, off)


def test_crc32_large_buffer():
    """1 GiB: the result against zlib, and the device rate (printed)."""
    from cachepotato_b200 import _lib
    L = _lib.lib()
    n = 1 << 30
    dev = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    _crc(L, dev.data_ptr(), 4096)                       # tables uploaded outside the timing
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    got = _crc(L, dev.data_ptr(), n)
    dt = time.perf_counter() - t0
    assert got == zlib.crc32(dev.cpu().numpy().tobytes())
    print(f"cpg_crc32: 1 GiB in {dt * 1e3:.2f} ms ({n / dt / 1e9:.1f} GB/s, host call included)")


def test_store_verify_reports_the_first_bad_region():
    from cachepotato_b200 import _lib
    L = _lib.lib()
    sizes = [1000, 2_654_208, 0, 17, 70_000, 65_536]  # an expert region of the Qwen3 shape among them
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]) + 64
    mapping = np.random.default_rng(11).integers(0, 256, int(offs[-1] + sizes[-1] + 100), dtype=np.uint8)
    L.cpg_store_close()
    _lib.check(L.cpg_store_open_v4(mapping.ctypes.data, mapping.size, 0))
    try:
        for i, (o, n) in enumerate(zip(offs, sizes)):
            assert L.cpg_store_add_region(int(o), int(n), 1) == i
        digests = np.array([zlib.crc32(mapping[o:o + n].tobytes()) for o, n in zip(offs, sizes)], np.uint64)
        first = ctypes.c_int(7)
        _lib.check(L.cpg_store_verify(digests.ctypes.data, len(sizes), ctypes.byref(first)))
        assert first.value == -1
        bad = digests.copy()
        bad[3] ^= np.uint64(1)                          # a wrong digest, planted on the host
        assert L.cpg_store_verify(bad.ctypes.data, len(sizes), ctypes.byref(first)) == _lib.CPG_EINVAL
        assert first.value == 3 and "region 3" in _lib.last_error()
        assert L.cpg_store_verify(digests.ctypes.data, len(sizes) - 1, None) == _lib.CPG_EINVAL
    finally:
        L.cpg_store_close()
