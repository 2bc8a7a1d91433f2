"""The oracle is pinned before it is trusted: against the reference's own decoder KATs and
against outputs of the reference engine itself (tests/golden/, made by make_golden.py)."""
import hashlib

import numpy as np
import pytest

import oracle as O
import make_golden as MG
from conftest import max_rel


def _kat_cases(kats, tag):
    return [str(n) for n in kats[tag + "_cases"]]


@pytest.mark.parametrize("tag,enc", [("q4", O.ENC_Q4), ("q8", O.ENC_Q8)])
def test_decoder_kats_bit_exact(orc, golden, tag, enc):
    kats = golden("decode_kats.npz")
    for key in _kat_cases(kats, tag):
        blocks = kats[key + "_blocks"]
        n = int(kats[key + "_n"])
        dec = orc.dequant(blocks, n, enc)
        assert hashlib.sha256(dec.astype("<f4").tobytes()).hexdigest() == str(kats[key + "_dec_sha256"]), key
        if key + "_dec" in kats:
            assert np.array_equal(dec.view(np.uint32), kats[key + "_dec"].view(np.uint32)), key


@pytest.mark.parametrize("tag,enc", [("q4", O.ENC_Q4), ("q8", O.ENC_Q8)])
def test_encoder_kats_bit_exact(orc, golden, tag, enc):
    kats = golden("decode_kats.npz")
    for key in _kat_cases(kats, tag):
        if key + "_x" not in kats:
            continue
        x = kats[key + "_x"]
        assert np.array_equal(orc.quantize(x, enc), kats[key + "_blocks"]), key


def test_f16_conversion_roundtrip(orc):
    """Every finite fp16 survives f16 -> f32 -> f16; subnormals and signed zero included."""
    L = orc.L
    for h in list(range(0, 0x7C00, 7)) + [0x0001, 0x03FF, 0x0400, 0x7BFF, 0x8001, 0x8000]:
        f = L.orc_f16_to_f32(h)
        assert L.orc_f32_to_f16(f) == h, hex(h)
        assert np.float32(f) == np.float16(np.uint16(h).view(np.float16)).astype(np.float32)


def test_f32_to_f16_matches_numpy(orc):
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(2000) * s for s in (1e-8, 1e-6, 1e-4, 1e-2, 1, 1e3, 7e4)])
    vals = vals.astype(np.float32)
    want = vals.astype(np.float16).view(np.uint16)
    got = np.array([orc.L.orc_f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("case", MG.MATVEC_CASES, ids=[c[0] for c in MG.MATVEC_CASES])
def test_matvec_vs_reference(orc, golden, case):
    """Oracle (scalar order) vs the reference's threaded AVX2 kernels: rel 1e-5, the tolerance
    of tools/verify_q8_kernels.py."""
    name, enc, n_in, n_out, seed = case
    w, x = MG.matvec_inputs(enc, n_in, n_out, seed, orc)
    got = orc.mm(w, enc, x, n_in, n_out)
    assert max_rel(got, golden("matvec_ref.npz")[name]) <= 1e-5


@pytest.mark.parametrize("case", MG.MOE_CASES[:3], ids=[c[0] for c in MG.MOE_CASES[:3]])
def test_moe_block_vs_reference(orc, golden, case):
    name, D, F, E, K, enc, T, seed = case
    g = golden("moe_ref.npz")
    layer = O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc)
    x = MG.moe_inputs(D, T, seed, orc)
    r = orc.qwen3_moe(layer, x)
    assert np.array_equal(r["topk_idx"], g[name + "_topk_idx"])
    assert max_rel(r["router"], g[name + "_router"]) <= 1e-6
    assert max_rel(r["mlp"], g[name + "_mlp"]) <= 1e-5


def test_moe_apply_vs_reference(orc, golden):
    name, D, F, E, K, enc, T, seed = MG.APPLY_CASE
    g = golden("apply_ref.npz")
    layer = O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc)
    xn = MG.moe_inputs(D, T, seed, orc)
    idx, wt = MG.apply_routing(T, E, K, seed)
    assert np.array_equal(idx, g["idx"])
    mlp = orc.moe_apply(layer, xn, idx, wt)
    assert max_rel(mlp, g["mlp"]) <= 1e-5


def test_topk_tie_rule(orc):
    """Equal probabilities: the lower expert id wins, output in descending order
    (qwen3_moe.c:184-194). The mistake is planted in the oracle's input, on the CPU."""
    import ctypes
    E, K, D = 16, 4, 32
    w = np.zeros((E, D), np.float32)
    w[[3, 9, 12, 5], 0] = [2.0, 2.0, 1.0, 2.0]     # experts 3, 5, 9 tie; 12 next
    xn = np.zeros(D, np.float32); xn[0] = 1.0
    logits = np.empty(E, np.float32); probs = np.empty(E, np.float32)
    idx = np.empty(K, np.int32); wt = np.empty(K, np.float32)
    f = ctypes.POINTER(ctypes.c_float); i = ctypes.POINTER(ctypes.c_int)
    orc.L.orc_route(w.ctypes.data_as(ctypes.c_void_p), O.ENC_F32, xn.ctypes.data_as(f), D, E, K,
                    logits.ctypes.data_as(f), probs.ctypes.data_as(f), idx.ctypes.data_as(i),
                    wt.ctypes.data_as(f))
    assert list(idx) == [3, 5, 9, 12]
    assert abs(float(wt.sum()) - 1.0) < 1e-6


def test_route_check_oracle_matches_reference_verdicts(golden):
    """The tie-aware agreement oracle against the reference's own checker
    (tools/check_qwen3_baseline.py run on the same trace: tests/golden/make_route_golden.py)."""
    import route_check as RC
    g = golden("route_check.npz")
    L = int(g["n_layers"])
    mismatch, ties, sum_err, w_err = [], 0, 0.0, 0.0
    for i in range(L):
        r = RC.route_check(g[f"logits{i}"], g[f"topk{i}"], g[f"wt{i}"])
        if r["bad"]:
            mismatch.append(i)
            ties += int(r["tie"][:r["first_bad"]].sum())     # the reference stops a layer there
        else:
            ties += r["ties"]
        sum_err, w_err = max(sum_err, r["sum_err"]), max(w_err, r["w_err"])
    assert mismatch == g["ref_mismatch"].tolist() == [3, 4]
    assert ties == int(g["ref_ties"]) and ties > 0
    assert abs(w_err - float(g["ref_w_err"])) <= 0.01 * float(g["ref_w_err"])   # printed to 3 digits
    assert sum_err <= 1e-6 and float(g["ref_sum_err"]) <= 1e-6                 # float32 weights


def test_routing_agreement_excuses_only_near_tied_swaps():
    """The parity helper accepts an id difference only where the two experts that traded places
    have reference probabilities within 1e-6 (a planted near-tie elsewhere excuses nothing)."""
    from helpers import check_topk
    E, K = 16, 4
    logits = np.zeros((1, E), np.float32)
    logits[0, :6] = [5.0, 4.0, 3.0, 2.0, 2.0, 1.0]          # experts 3 and 4 tie exactly
    logits[0, 10] = 3.0 + 1e-3                                # a clear 3rd place, not a tie with 2
    want = np.array([[0, 1, 10, 2]], np.int32)
    assert check_topk(want, want, logits, K) == []
    # 2nd/3rd swapped: probabilities differ by far more than 1e-6
    assert check_topk(np.array([[0, 10, 1, 2]], np.int32), want, logits, K) == [0]
    # the 4th slot taken by a non-tied expert, although a tie exists among 3 / 4
    assert check_topk(np.array([[0, 1, 10, 3]], np.int32), want, logits, K) == [0]
    logits2 = logits.copy()
    logits2[0, 10] = 0.0
    want2 = np.array([[0, 1, 2, 3]], np.int32)
    # the boundary tie 3 / 4 may go either way
    assert check_topk(np.array([[0, 1, 2, 4]], np.int32), want2, logits2, K) == []
    # a repeated id is never accepted
    assert check_topk(np.array([[0, 1, 2, 2]], np.int32), want2, logits2, K) == [0]


def test_oracle_zipf_t64_vs_reference_engine(orc, golden):
    """The C restatement on the headline 64-token Zipf batch against the reference engine."""
    import make_golden as MG
    g = golden("moe_zipf_ref.npz")
    L, x, _ = MG.zipf_case_layer(orc, scale=g["router_scale"])
    r = orc.qwen3_moe(L, x)
    assert np.array_equal(r["topk_idx"], g["topk_idx"])
    assert np.abs(r["mlp"] - g["mlp"]).max() / np.abs(g["mlp"]).max() <= 1e-5
