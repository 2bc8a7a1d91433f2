"""Parity of the format and matvec kernels on the GPU, called through the C ABI.

Dequantisation and encoding are bit-exact (against the reference's own KATs and the oracle);
fp32 matvec agrees with the reference engine's kernels within rel 1e-5, the reference's own
kernel-gate tolerance (tools/verify_q8_kernels.py)."""
import hashlib

import numpy as np
import pytest

import oracle as O
import make_golden as MG
from conftest import max_rel
from helpers import KERNEL_TOL

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def q():
    from cachepotato_b200 import qwen3
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    return qwen3


@pytest.mark.parametrize("tag,enc", [("q4", O.ENC_Q4), ("q8", O.ENC_Q8)])
def test_dequant_reference_kats(q, golden, tag, enc):
    kats = golden("decode_kats.npz")
    for key in [str(k) for k in kats[tag + "_cases"]]:
        blocks = torch.from_numpy(kats[key + "_blocks"]).cuda()
        n = int(kats[key + "_n"])
        got = q.dequant(blocks, n, enc).cpu().numpy()
        assert hashlib.sha256(got.astype("<f4").tobytes()).hexdigest() == str(kats[key + "_dec_sha256"]), key
        # the host drop-in (kernels.h signature) too
        out = np.empty(n, np.float32)
        (q.q4_dequant_row if enc == O.ENC_Q4 else q.q8_dequant_row)(kats[key + "_blocks"], out, n)
        assert np.array_equal(out.view(np.uint32), got.view(np.uint32)), key


@pytest.mark.parametrize("enc", [O.ENC_Q4, O.ENC_Q8])
def test_dequant_random_blocks_bit_exact(q, orc, enc):
    """Arbitrary bytes, including fp16 subnormal / inf / NaN scales, decode bit-exactly."""
    rng = np.random.default_rng(7)
    gb = O.GROUP_BYTES[enc]
    blocks = rng.integers(0, 256, size=4096 * gb, dtype=np.uint8)
    got = q.dequant(torch.from_numpy(blocks).cuda(), 4096 * 32, enc).cpu().numpy()
    want = orc.dequant(blocks, 4096 * 32, enc)
    diff = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    assert diff.size == 0, (diff.size, [(hex(got.view(np.uint32)[i]), hex(want.view(np.uint32)[i])) for i in diff[:4]])


@pytest.mark.parametrize("tag,enc", [("q4", O.ENC_Q4), ("q8", O.ENC_Q8)])
def test_quantize_reference_kats(q, golden, tag, enc):
    kats = golden("decode_kats.npz")
    for key in [str(k) for k in kats[tag + "_cases"]]:
        if key + "_x" not in kats:
            continue
        got = q.quantize(torch.from_numpy(kats[key + "_x"]).cuda(), enc).cpu().numpy()
        want = kats[key + "_blocks"]
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (key, bad.size, bad[:8].tolist(), got[bad[:8]].tolist(), want[bad[:8]].tolist())


@pytest.mark.parametrize("enc", [O.ENC_Q4, O.ENC_Q8])
def test_quantize_matches_oracle_at_scale(q, orc, enc):
    x = orc.normal(1 << 22, 99, 0.02)
    x[:32] = 0.0                                       # all-zero group
    x[32:64] = np.arange(32, dtype=np.float32) / 8.0   # ties
    x[64:96] *= 1e4                                    # saturating
    x[96:128] = 1e-9                                   # scale rounds to fp16 zero
    got = q.quantize(torch.from_numpy(x).cuda(), enc).cpu().numpy()
    want = orc.quantize(x, enc)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (bad.size, bad[:8].tolist(), got[bad[:8]].tolist(), want[bad[:8]].tolist())


@pytest.mark.parametrize("case", MG.MATVEC_CASES, ids=[c[0] for c in MG.MATVEC_CASES])
def test_matvec_vs_reference_engine(q, orc, golden, case):
    name, enc, n_in, n_out, seed = case
    w, x = MG.matvec_inputs(enc, n_in, n_out, seed, orc)
    want = golden("matvec_ref.npz")[name]
    out = np.empty(n_out, np.float32)
    {O.ENC_Q4: q.matmul_wx_q4, O.ENC_Q8: q.matmul_wx_q8, O.ENC_F32: q.matmul_wx}[enc](out, x, w, n_in, n_out)
    assert max_rel(out, want) <= KERNEL_TOL
    dev = q.qwen3_mm(torch.from_numpy(np.ascontiguousarray(w)).cuda(), enc, torch.from_numpy(x).cuda(), n_in, n_out)
    assert max_rel(dev.cpu().numpy()[0], want) <= KERNEL_TOL


@pytest.mark.parametrize("enc", [O.ENC_Q4, O.ENC_Q8])
@pytest.mark.parametrize("T", [1, 5, 13])
def test_matvec_batched_vs_oracle(q, orc, enc, T):
    n_in, n_out = 2048, 512
    w = orc.quantize(orc.normal(n_in * n_out, 5 + T, 0.02), enc)
    x = orc.normal(T * n_in, 6 + T, 1.0).reshape(T, n_in)
    got = q.qwen3_mm(torch.from_numpy(w).cuda(), enc, torch.from_numpy(x).cuda(), n_in, n_out).cpu().numpy()
    for t in range(T):
        assert max_rel(got[t], orc.mm(w, enc, x[t], n_in, n_out)) <= KERNEL_TOL


def test_matvec_odd_group_count(q, orc):
    """n_in = 32 * odd: rows are not 4-byte aligned; the byte-load path handles them."""
    n_in, n_out = 96, 37
    for enc in (O.ENC_Q4, O.ENC_Q8):
        w = orc.quantize(orc.normal(n_in * n_out, 11, 0.02), enc)
        x = orc.normal(n_in, 12, 1.0)
        out = np.empty(n_out, np.float32)
        (q.matmul_wx_q4 if enc == O.ENC_Q4 else q.matmul_wx_q8)(out, x, w, n_in, n_out)
        assert max_rel(out, orc.mm(w, enc, x, n_in, n_out)) <= KERNEL_TOL


def test_bad_arguments_raise(q):
    from cachepotato_b200 import CpgError
    out = np.empty(8, np.float32)
    with pytest.raises(CpgError):
        q.matmul_wx_q4(out, np.zeros(33, np.float32), np.zeros(64, np.uint8), 33, 8)


def test_region_store_translates_host_mapping(q, orc):
    """cpg_store_open_v4 mirrors a host 'mapping' into HBM; region ids index the table as
    pager_add_region's do; host pointers inside the mapping resolve to the resident copy."""
    import ctypes
    from cachepotato_b200 import _lib
    L = _lib.lib()
    n_in, n_out = 2048, 768
    w = orc.quantize(orc.normal(n_in * n_out, 3, 0.02), O.ENC_Q4)
    header = 4096
    mapping = np.zeros(header + 2 * w.size, np.uint8)
    mapping[header:header + w.size] = w
    mapping[header + w.size:] = w[::-1]
    L.cpg_store_close()
    _lib.check(L.cpg_store_open_v4(mapping.ctypes.data, mapping.size, header))
    try:
        assert L.cpg_store_add_region(0, w.size, 1) == 0
        assert L.cpg_store_add_region(w.size, w.size, 1) == 1
        assert L.cpg_store_add_region(2 * w.size, 16, 0) == _lib.CPG_EINVAL
        tot = _lib.StoreTotals()
        _lib.check(L.cpg_store_totals(ctypes.byref(tot)))
        assert tot.regions == 2 and tot.expert_regions == 2 and tot.h2d_bytes == 2 * w.size
        r1 = L.cpg_store_region_get(1)
        assert r1 == L.cpg_store_translate(mapping.ctypes.data + header + w.size)
        assert L.cpg_store_translate(mapping.ctypes.data) is None
        # the drop-in reads the resident copy when given the mapping address
        x = orc.normal(n_in, 4, 1.0)
        out = np.empty(n_out, np.float32)
        view = mapping[header:header + w.size]
        q.matmul_wx_q4(out, x, view, n_in, n_out)
        assert max_rel(out, orc.mm(w, O.ENC_Q4, x, n_in, n_out)) <= KERNEL_TOL
        # region 1 holds the reversed bytes: decode it in place and compare
        n = (w.size // 18) * 32
        out_dev = torch.empty(n, dtype=torch.float32, device="cuda")
        _lib.check(L.cpg_dequant(out_dev.data_ptr(), r1, O.ENC_Q4, n, None))
        torch.cuda.synchronize()
        want = orc.dequant(np.ascontiguousarray(w[::-1]), n, O.ENC_Q4)     # NaN scales possible
        assert np.array_equal(out_dev.cpu().numpy().view(np.uint32), want.view(np.uint32))
    finally:
        L.cpg_store_close()


@pytest.mark.parametrize("n_in,n_out,shift", [(2, 2048, 0), (37, 19, 1), (2048, 2, 3)])
def test_f32_matvec_any_shape(q, orc, n_in, n_out, shift):
    """matmul_wx takes any n_in and any row alignment (kernels.c:84-95; the reference's own
    attention uses (D, 2) f32 tensors): odd widths and weights shifted off 16 bytes."""
    ref = O.Reference(threads=8)
    buf = orc.normal(n_in * n_out + shift, 70 + n_in, 0.02)
    w = buf[shift:]                                   # shift floats: 4-byte aligned only
    x = orc.normal(n_in, 71 + n_in, 1.0)
    out = np.empty(n_out, np.float32)
    q.matmul_wx(out, x, w, n_in, n_out)
    assert max_rel(out, ref.mm(np.ascontiguousarray(w), O.ENC_F32, x, n_in, n_out)) <= KERNEL_TOL
