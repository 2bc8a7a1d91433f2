"""Parity of the MoE block (router, experts, combine) on the GPU against the reference engine
(golden fixtures) and the oracle, through the C ABI.

Bars: router logits rel 1e-5 (fp32 GEMV, different summation order); expert ids identical
except where the top-k probability margin is below 1e-6; routing weights rel 1e-5; block
output max|d|/max|ref| <= 1e-5 (the experts run on fp16 tensor cores with exact Q4/Q8 integers
and f32 activations carried as fp16 hi + lo halves, fp32 accumulation)."""
import numpy as np
import pytest

import oracle as O
import make_golden as MG
from conftest import max_rel
from helpers import DECODE_TOL, check_topk, device_layer

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

FULL = [c for c in MG.MOE_CASES if c[0].startswith("full")]


@pytest.fixture(scope="module")
def layers(orc):
    cache = {}

    def get(D, F, E, K, enc, seed, scale=None):
        key = (D, F, E, K, enc, seed, None if scale is None else scale.tobytes())
        if key not in cache:
            L = O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc, router_scale=scale)
            cache[key] = (L, device_layer(L))
        return cache[key]
    return get


def _compare(got, want, K, logits_tol=1e-5):
    assert max_rel(got.router.cpu().numpy(), want["router"]) <= logits_tol
    idx = got.topk_idx.cpu().numpy()
    bad = check_topk(idx, want["topk_idx"], want["router"], K)
    assert not bad, f"tokens with unexplained routing differences: {bad}"
    ok = np.all(idx == want["topk_idx"], axis=1)
    if "wt" in want:
        assert max_rel(got.wt.cpu().numpy()[ok], want["wt"][ok]) <= 1e-5
    err = max_rel(got.mlp.cpu().numpy()[ok], want["mlp"][ok])
    assert err <= DECODE_TOL, err
    return err


@pytest.mark.parametrize("case", FULL, ids=[c[0] for c in FULL])
def test_block_vs_reference_engine(orc, golden, layers, case):
    """The reference's own qwen3_layer_kv outputs (tests/golden/moe_ref.npz)."""
    name, D, F, E, K, enc, T, seed = case
    g = golden("moe_ref.npz")
    L, dl = layers(D, F, E, K, enc, seed)
    x = MG.moe_inputs(D, T, seed, orc)
    got = dl.forward(torch.from_numpy(x).cuda())
    want = {k: g[f"{name}_{k}"] for k in ("router", "topk_idx", "mlp")}
    _compare(got, want, K)
    # residual: x_out = x + (0 + mlp)
    assert np.allclose(got.x_out.cpu().numpy(), x + got.mlp.cpu().numpy(), rtol=0, atol=0)


@pytest.mark.parametrize("enc", [O.ENC_Q4, O.ENC_Q8])
@pytest.mark.parametrize("T", [1, 3, 8, 17, 64, 200, 300])
def test_block_vs_oracle_small(orc, layers, enc, T):
    # T·K ≤ 1024 pairs are grouped by the gate/up kernel itself (T = 200: 7 mask words per
    # expert), larger batches (T = 300) by the separate grouping kernel
    D, F, E, K = 256, 256, 16, 4
    L, dl = layers(D, F, E, K, enc, 100 + enc)
    x = orc.normal(T * D, 1000 + T, 1.0).reshape(T, D)
    got = dl.forward(torch.from_numpy(x).cuda())
    _compare(got, orc.qwen3_moe(L, x), K)


def test_block_batched_zipf_vs_oracle(orc, layers):
    """Batched decode (T = 64) with a Zipf-calibrated router: experts shared by many tokens."""
    from cachepotato_b200.workload import calibrate_router_scales, rmsnorm_rows
    D, F, E, K, T = 2048, 768, 128, 8, 64
    x = orc.normal(T * D, 4242, 1.0).reshape(T, D)
    L0 = O.SynthLayer(D, F, E, K, O.ENC_Q4, seed=77, oracle=orc)
    scale = calibrate_router_scales(rmsnorm_rows(x) @ L0.wgate.T, K, 1.1, seed=5)
    L, dl = layers(D, F, E, K, O.ENC_Q4, 77, scale)
    got = dl.forward(torch.from_numpy(x).cuda())
    want = orc.qwen3_moe(L, x)
    _compare(got, want, K)
    counts = np.bincount(want["topk_idx"].ravel(), minlength=E)
    assert counts.max() >= 16            # the calibrated router does share experts


def test_attn_input_and_mlp_accumulation(orc, layers):
    D, F, E, K, T = 256, 256, 16, 4, 5
    L, dl = layers(D, F, E, K, O.ENC_Q4, 300)
    x = orc.normal(T * D, 1, 1.0).reshape(T, D)
    attn = orc.normal(T * D, 2, 0.5).reshape(T, D)
    mlp0 = orc.normal(T * D, 3, 0.1).reshape(T, D)
    got = dl.forward(torch.from_numpy(x).cuda(), torch.from_numpy(attn).cuda(),
                     mlp=torch.from_numpy(mlp0.copy()).cuda())
    want = orc.qwen3_moe(L, x, attn)                       # oracle mlp starts at zero
    assert max_rel(got.mlp.cpu().numpy() - mlp0, want["mlp"]) <= DECODE_TOL
    assert np.array_equal(got.topk_idx.cpu().numpy(), want["topk_idx"])
    xo = got.x_out.cpu().numpy()
    assert np.array_equal(xo, (x + (attn + got.mlp.cpu().numpy())).astype(np.float32))


def test_deterministic_bitwise(orc, layers):
    D, F, E, K, T = 2048, 768, 128, 8, 64
    L, dl = layers(D, F, E, K, O.ENC_Q4, 21)
    x = torch.from_numpy(orc.normal(T * D, 9, 1.0).reshape(T, D)).cuda()
    a = dl.forward(x)
    b = dl.forward(x)
    assert torch.equal(a.mlp, b.mlp) and torch.equal(a.topk_idx, b.topk_idx)


def test_decode_context_chains_layers(orc, layers):
    """cpg_run_moe_layers (host buffers, CUDA graph) == chaining cpg_moe_forward by hand."""
    from cachepotato_b200.qwen3 import DecodeContext
    D, F, E, K, T = 2048, 768, 128, 8, 4
    ls = [layers(D, F, E, K, O.ENC_Q4, s)[1] for s in (21, 22, 23)]
    x = orc.normal(T * D, 31, 1.0).reshape(T, D)
    xd = torch.from_numpy(x).cuda()
    for l in ls:
        xd = l.forward(xd).x_out
    ctx = DecodeContext(ls[0], max_T=8)
    xh = x.copy()
    topk = ctx.run(ls, xh, want_topk=True)
    assert np.array_equal(xh, xd.cpu().numpy())
    assert topk.shape == (3, T, K)
    xh2 = x.copy()
    ctx.run(ls, xh2)                                    # graph replay
    assert np.array_equal(xh, xh2)


def test_phase_profile(orc, layers):
    from cachepotato_b200.qwen3 import DecodeContext
    D, F, E, K, T = 2048, 768, 128, 8, 64
    l = layers(D, F, E, K, O.ENC_Q4, 21)[1]
    ctx = DecodeContext(l, max_T=T)
    ctx.profile(True)
    xh = orc.normal(T * D, 5, 1.0).reshape(T, D)
    ctx.run([l, l], xh)
    ms = ctx.phase_ms()
    # T=64: gate/up and down items share one launch (timed as the gate/up phase)
    assert ms[0] > 0 and ms[1] > 0 and ms[2] >= 0 and ms[3] > 0 and ms[1] > ms[3]


def test_block_zipf_t64_vs_reference_engine(orc, golden):
    """The headline batch (64 tokens, Zipf(1.1)-calibrated router, full shape, Q4_0) against the
    reference engine's own qwen3_layer_kv output (tests/golden/moe_zipf_ref.npz)."""
    g = golden("moe_zipf_ref.npz")
    L, x, _ = MG.zipf_case_layer(orc, scale=g["router_scale"])
    got = device_layer(L).forward(torch.from_numpy(x).cuda())
    want = {k: g[k] for k in ("router", "topk_idx", "mlp")}
    err = _compare(got, want, L.topk)
    counts = np.bincount(want["topk_idx"].ravel(), minlength=L.n_experts)
    assert counts.max() > 32 and err <= DECODE_TOL     # experts spanning several token chunks


@pytest.mark.parametrize("T,bad", [(1, 0), (3, 2)])
def test_nan_token_routes_like_the_reference(orc, layers, T, bad):
    """A token whose activations hold a NaN has NaN logits: the reference's scan
    (qwen3_moe.c:184-194) then keeps its starting candidate, the lowest untaken id, in every
    slot. The device routes it the same way (one-token and batched paths) and the tokens before
    it are unaffected (in the reference harness later tokens see the NaN token's keys through
    its zero attention, 0 * NaN = NaN, so only earlier tokens are compared)."""
    ref = O.Reference(threads=8)
    D, F, E, K = 256, 256, 16, 4
    L, dl = layers(D, F, E, K, O.ENC_Q4, 310)
    x = orc.normal(T * D, 311, 1.0).reshape(T, D)
    x[bad, 17] = np.nan
    want = ref.qwen3_moe(L, x)
    got = dl.forward(torch.from_numpy(x).cuda())
    idx = got.topk_idx.cpu().numpy()
    assert idx[bad].tolist() == want["topk_idx"][bad].tolist() == list(range(K))
    good = list(range(bad))
    if good:
        assert np.array_equal(idx[good], want["topk_idx"][good])
        assert max_rel(got.mlp.cpu().numpy()[good], want["mlp"][good]) <= DECODE_TOL
