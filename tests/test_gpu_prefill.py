"""The prefill path: externally routed experts through the tcgen05 grouped GEMM (cpg_moe_apply),
against the reference's own expert loop (golden) and the oracle.

Bar: max|d|/max|ref| <= 1e-3 per block (fp16 weights q*d rounded once, fp16 activations, fp32
accumulation in tensor memory)."""
import numpy as np
import pytest

import oracle as O
import make_golden as MG
from conftest import max_rel
from helpers import BLOCK_TOL, device_layer
from cachepotato_b200.workload import zipf_assignment

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _apply(dl, xn, idx, wt):
    from cachepotato_b200.qwen3 import moe_apply
    return moe_apply(dl, torch.from_numpy(xn).cuda(), torch.from_numpy(idx).cuda(),
                     torch.from_numpy(wt).cuda()).cpu().numpy()


def test_apply_vs_reference_expert_loop(orc, golden):
    name, D, F, E, K, enc, T, seed = MG.APPLY_CASE
    g = golden("apply_ref.npz")
    L = O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc)
    xn = MG.moe_inputs(D, T, seed, orc)
    got = _apply(device_layer(L), xn, g["idx"], g["wt"])
    assert max_rel(got, g["mlp"]) <= BLOCK_TOL


@pytest.mark.parametrize("T", [1, 37, 1000])
def test_apply_vs_oracle_small(orc, T):
    D, F, E, K = 256, 256, 16, 4
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=500, oracle=orc)
    xn = orc.normal(T * D, 600 + T, 1.0).reshape(T, D)
    idx, wt = MG.apply_routing(T, E, K, 700 + T)
    got = _apply(device_layer(L), xn, idx, wt)
    assert max_rel(got, orc.moe_apply(L, xn, idx, wt)) <= BLOCK_TOL


def test_apply_full_shape_zipf_sampled(orc):
    """Qwen3 shape, Zipf-Mandelbrot routed batch (uneven groups, several token tiles per expert);
    per-token outputs are independent, so a sample of tokens is checked against the oracle."""
    D, F, E, K, T = 2048, 768, 128, 8, 1024
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=901, oracle=orc)
    xn = orc.normal(T * D, 902, 1.0).reshape(T, D)
    idx, wt = zipf_assignment(T, E, K, 1.2, 20.0, 903)
    got = _apply(device_layer(L), xn, idx, wt)
    sample = np.random.default_rng(4).choice(T, 24, replace=False)
    want = orc.moe_apply(L, xn[sample], idx[sample], wt[sample])
    assert max_rel(got[sample], want) <= BLOCK_TOL
    counts = np.bincount(idx.ravel(), minlength=E)
    assert counts.max() > 128                       # experts spanning several token tiles


def test_apply_deterministic_and_accumulates(orc):
    from cachepotato_b200.qwen3 import moe_apply
    D, F, E, K, T = 256, 256, 16, 4, 300
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=510, oracle=orc)
    dl = device_layer(L)
    xn = torch.from_numpy(orc.normal(T * D, 511, 1.0).reshape(T, D)).cuda()
    idx, wt = MG.apply_routing(T, E, K, 512)
    idx, wt = torch.from_numpy(idx).cuda(), torch.from_numpy(wt).cuda()
    a = moe_apply(dl, xn, idx, wt)
    b = moe_apply(dl, xn, idx, wt)
    assert torch.equal(a, b)
    base = torch.ones_like(a)
    c = moe_apply(dl, xn, idx, wt, mlp=base.clone())
    assert torch.allclose(c - 1.0, a, rtol=0, atol=1e-6)


def test_apply_rejects_bad_expert_ids(orc):
    from cachepotato_b200 import CpgError
    from cachepotato_b200.qwen3 import moe_apply
    D, F, E, K, T = 256, 256, 16, 4, 8
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=520, oracle=orc)
    xn = orc.normal(T * D, 521, 1.0).reshape(T, D)
    idx, wt = MG.apply_routing(T, E, K, 522)
    idx[3, 1] = E + 5                                  # planted on the host, checked on the device
    with pytest.raises(CpgError):
        moe_apply(device_layer(L), torch.from_numpy(xn).cuda(), torch.from_numpy(idx).cuda(),
                  torch.from_numpy(wt).cuda())


def test_apply_bench_config_T4096_sampled():
    """The prefill benchmark's own batch: 4096 tokens routed by zipf_assignment(4096, 128, 8, 1.2,
    20.0, seed 1234 + 77) (groups of about 90-890 tokens, up to four 256-token tiles per expert),
    checked on 320 tokens against the reference engine's expert loop (qwen3_moe.c:199-222 with
    the routing given): every token of the largest group's last token tile, and random others."""
    ref = O.Reference(threads=16)
    orc = O.Oracle()
    D, F, E, K, T = 2048, 768, 128, 8, 4096
    L = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=1277, oracle=orc)
    xn = orc.normal(T * D, 1278, 1.0).reshape(T, D)
    idx, wt = zipf_assignment(T, E, K, 1.2, 20.0, 1234 + 77)
    got = _apply(device_layer(L), xn, idx, wt)
    counts = np.bincount(idx.ravel(), minlength=E)
    big = int(counts.argmax())
    members = np.nonzero((idx == big).any(1))[0]               # tokens ascending, as the sort keeps them
    last_tile = members[(len(members) - 1) // 256 * 256:]
    assert counts.max() > 768 and len(last_tile) > 0           # a fourth token tile exists
    rest = np.setdiff1d(np.arange(T), last_tile)
    sample = np.sort(np.concatenate([last_tile, np.random.default_rng(6).choice(rest, 320 - len(last_tile),
                                                                                 replace=False)]))
    want = ref.moe_apply(L, xn[sample], idx[sample], wt[sample])
    assert max_rel(got[sample], want) <= BLOCK_TOL
