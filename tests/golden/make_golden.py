"""Generates the committed golden fixtures in tests/golden/ (run here, where the reference tree
and its compiled engine exist; the GPU box only reads the .npz files).

  decode_kats.npz   the reference's own decoder known-answer cases, regenerated exactly as
                    tools/verify_q4_decode.py:48-55 and tools/verify_q8_decode.py:48-58 build
                    them (seed 20261017), encoded AND decoded by the reference's Python format
                    module (format/q4.py, format/q8.py)
  matvec_ref.npz    the reference engine's matmul_wx_q4 / matmul_wx_q8 / matmul_wx
                    (engine/kernels/kernels.c) run multi-threaded (its AVX2 production path)
                    on seeded synthetic inputs
  moe_ref.npz       the reference engine's qwen3_layer_kv (engine/blocks/qwen3_moe.c:87-229)
                    on seeded synthetic layers: router logits, top-k ids, MoE output
  moe_zipf_ref.npz  the same for the 64-token headline batch (Zipf(1.1)-calibrated router, its
                    per-expert router scales stored with the outputs)
  apply_ref.npz     the reference's expert loop on externally drawn routing

Synthetic weights and activations come from the oracle's counter-based generator
(orc_fill_normal, seed-keyed) and the oracle encoder, which decode_kats pins bit-exactly to
the reference encoder; only seeds and outputs are stored, so the fixtures stay small.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

REF_TREE = O.REF_TREE
REF_THREADS = 8

# (name, d_model, d_exp, n_experts, topk, enc, T, seed)
MOE_CASES = [
    ("small_q4", 256, 64, 16, 4, O.ENC_Q4, 3, 11),
    ("small_q8", 256, 64, 16, 4, O.ENC_Q8, 3, 12),
    ("full_q4_t1", 2048, 768, 128, 8, O.ENC_Q4, 1, 21),
    ("full_q4_t4", 2048, 768, 128, 8, O.ENC_Q4, 4, 21),
    ("full_q8_t1", 2048, 768, 128, 8, O.ENC_Q8, 1, 22),
    ("full_q8_t2", 2048, 768, 128, 8, O.ENC_Q8, 2, 22),
]
# (name, enc, n_in, n_out, seed)
MATVEC_CASES = [
    ("q4_gate", O.ENC_Q4, 2048, 768, 31),
    ("q4_down", O.ENC_Q4, 768, 2048, 32),
    ("q4_small", O.ENC_Q4, 64, 40, 33),
    ("q4_wide", O.ENC_Q4, 4096, 2048, 34),
    ("q8_gate", O.ENC_Q8, 2048, 768, 35),
    ("q8_down", O.ENC_Q8, 768, 2048, 36),
    ("q8_small", O.ENC_Q8, 64, 40, 37),
    ("f32_router", O.ENC_F32, 2048, 128, 38),
]
APPLY_CASE = ("apply_q4", 256, 256, 16, 4, O.ENC_Q4, 40, 41)
# the headline decode batch: 64 tokens, full shape, Q4_0, router rows scaled so the top-8 load
# follows Zipf(1.1) (scales computed here and stored, so the GPU test rebuilds the same layer)
ZIPF_CASE = ("zipf_q4_t64", 2048, 768, 128, 8, O.ENC_Q4, 64, 77)


def zipf_case_layer(orc, scale=None):
    """The ZIPF_CASE layer and its input x; with scale None the scales are calibrated here."""
    sys.path.insert(0, ROOT)
    from cachepotato_b200.workload import calibrate_router_scales, rmsnorm_rows
    name, D, F, E, K, enc, T, seed = ZIPF_CASE
    x = orc.normal(T * D, 4242, 1.0).reshape(T, D)
    if scale is None:
        L0 = O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc)
        scale = calibrate_router_scales(rmsnorm_rows(x) @ L0.wgate.T, K, 1.1, seed=5)
    return O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc, router_scale=scale), x, scale


def moe_inputs(d_model, T, seed, orc):
    return orc.normal(T * d_model, seed * 7 + 3, 1.0).reshape(T, d_model)


def matvec_inputs(enc, n_in, n_out, seed, orc):
    w32 = orc.normal(n_in * n_out, seed * 5 + 1, 0.02)
    w = w32 if enc == O.ENC_F32 else orc.quantize(w32, enc)
    x = orc.normal(n_in, seed * 5 + 2, 1.0)
    return w, x


def apply_routing(T, E, K, seed):
    """K distinct experts per token and renormalised weights, from a numpy Generator."""
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    wt = rng.random((T, K)).astype(np.float32) + np.float32(0.1)
    wt /= wt.sum(1, keepdims=True)
    return idx, wt.astype(np.float32)


def decode_kats():
    sys.path.insert(0, os.path.join(REF_TREE, "format"))
    import q4  # the reference's own format module
    import q8
    out = {}
    rng = np.random.default_rng(20261017)              # verify_q4_decode.py:48-55
    q4_cases = [
        ("random", rng.standard_normal(32 * 64).astype(np.float32) * 0.05),
        ("zeros", np.zeros(64, dtype=np.float32)),
        ("saturating", rng.standard_normal(64).astype(np.float32) * 100),
        ("ties", (np.arange(64, dtype=np.float32) / 8.0) - 4.0),
        ("neg_extremes", -np.abs(rng.standard_normal(64).astype(np.float32))),
    ]
    rng = np.random.default_rng(20261017)              # verify_q8_decode.py:48-58
    q8_cases = [
        ("random_small", rng.standard_normal(32 * 40).astype(np.float32) * 0.05),
        ("random_large", rng.standard_normal(768 * 192).astype(np.float32) * 0.02),
        ("all_zeros", np.zeros(64, dtype=np.float32)),
        ("exact_powers", np.arange(64, dtype=np.float32) / 64.0),
        ("large_dynamic_range", np.concatenate([rng.standard_normal(32).astype(np.float32),
                                                rng.standard_normal(32).astype(np.float32) * 1000])),
    ]
    for tag, mod, cases, enc_fn in (("q4", q4, q4_cases, q4.encode_q4_0),
                                    ("q8", q8, q8_cases, q8.encode_q8_0)):
        names = []
        for name, x in cases:
            x = np.ascontiguousarray(x, dtype=np.float32)
            blocks, shape = enc_fn(x)
            dec = (mod.decode_q4_0 if tag == "q4" else mod.decode_q8_0)(blocks, shape)
            key = f"{tag}_{name}"
            names.append(key)
            out[key + "_blocks"] = np.frombuffer(blocks, np.uint8).copy()
            out[key + "_x_sha256"] = np.array(hashlib.sha256(x.tobytes()).hexdigest())
            out[key + "_dec_sha256"] = np.array(hashlib.sha256(dec.astype("<f4").tobytes()).hexdigest())
            out[key + "_n"] = np.array(x.size)
            if x.size <= 4096:                          # small cases keep x and y themselves
                out[key + "_x"] = x
                out[key + "_dec"] = dec.astype(np.float32)
        out[tag + "_cases"] = np.array(names)
    np.savez_compressed(os.path.join(HERE, "decode_kats.npz"), **out)


def main():
    O.build(ref=True)
    orc = O.Oracle()
    ref = O.Reference(threads=REF_THREADS)
    decode_kats()

    mv = {"threads": np.array(ref.threads)}
    for name, enc, n_in, n_out, seed in MATVEC_CASES:
        w, x = matvec_inputs(enc, n_in, n_out, seed, orc)
        mv[name] = ref.mm(w, enc, x, n_in, n_out)
    np.savez_compressed(os.path.join(HERE, "matvec_ref.npz"), **mv)

    moe = {"threads": np.array(ref.threads)}
    for name, D, F, E, K, enc, T, seed in MOE_CASES:
        layer = O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc)
        x = moe_inputs(D, T, seed, orc)
        r = ref.qwen3_moe(layer, x)
        for k, v in r.items():
            moe[f"{name}_{k}"] = v
    np.savez_compressed(os.path.join(HERE, "moe_ref.npz"), **moe)

    layer, x, scale = zipf_case_layer(orc)
    r = ref.qwen3_moe(layer, x)
    np.savez_compressed(os.path.join(HERE, "moe_zipf_ref.npz"), threads=np.array(ref.threads),
                        router_scale=scale.astype(np.float32), **r)

    name, D, F, E, K, enc, T, seed = APPLY_CASE
    layer = O.SynthLayer(D, F, E, K, enc, seed=seed, oracle=orc)
    xn = moe_inputs(D, T, seed, orc)
    idx, wt = apply_routing(T, E, K, seed)
    np.savez_compressed(os.path.join(HERE, "apply_ref.npz"), idx=idx, wt=wt,
                        mlp=ref.moe_apply(layer, xn, idx, wt))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
