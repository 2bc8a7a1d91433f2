"""The whole Qwen3-MoE model (config 3 path): prompt in one pass, then greedy decode, against the
reference engine itself (qwen3_layer_kv per layer with real attention and KV cache, embed_rows /
apply_head / argmax as cp_chat runs them, engine/api/cachepotato.c:108-166, 315-378).

Bar: the same greedy ids at every step, and the last step's logits within max|d|/max|ref| ≤ 1e-3."""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel
from helpers import BLOCK_TOL, device_model

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ref():
    return O.Reference(threads=8)


@pytest.mark.parametrize("n_prompt,n_new", [(1, 4), (7, 6), (33, 3)])
def test_small_model_generate(orc, ref, n_prompt, n_new):
    m = O.SynthModel(256, 4, 2, 128, 256, 16, 4, 512, 2, seed=5, norm_jitter=0.1, oracle=orc)
    prompt = np.random.default_rng(n_prompt).integers(0, m.vocab, n_prompt).astype(np.int32)
    want_ids, want_logits = ref.qwen3_generate(m, prompt, n_new)
    gm = device_model(m, max_ctx=n_prompt + n_new + 1)
    try:
        got_ids = gm.generate(prompt, n_new)
        got_logits = gm.logits().cpu().numpy()
    finally:
        gm.close()
    assert got_ids.tolist() == want_ids.tolist()
    assert max_rel(got_logits, want_logits) <= BLOCK_TOL


def test_qwen3_shape_two_layers(orc, ref):
    """Qwen3-30B-A3B widths (32 query / 4 KV heads, 128 experts top-8, d_exp 768), 2 layers,
    vocab cut to 4096."""
    m = O.SynthModel(2048, 32, 4, 128, 768, 128, 8, 4096, 2, seed=9, norm_jitter=0.05, oracle=orc)
    prompt = np.random.default_rng(3).integers(0, m.vocab, 12).astype(np.int32)
    want_ids, want_logits = ref.qwen3_generate(m, prompt, 4)
    gm = device_model(m, max_ctx=32)
    try:
        got_ids = gm.generate(prompt, 4)
        got_logits = gm.logits().cpu().numpy()
    finally:
        gm.close()
    assert got_ids.tolist() == want_ids.tolist()
    assert max_rel(got_logits, want_logits) <= BLOCK_TOL


def test_qwen3_shape_prompt_on_tensor_cores(orc, ref):
    """A 64-token prompt at Qwen3-30B-A3B widths: the prompt pass runs the attention projections
    on the tcgen05 GEMM (fp16 operands, fp32 accumulation); same ids, logits within the bar."""
    m = O.SynthModel(2048, 32, 4, 128, 768, 128, 8, 4096, 2, seed=11, norm_jitter=0.05, oracle=orc)
    prompt = np.random.default_rng(4).integers(0, m.vocab, 64).astype(np.int32)
    want_ids, want_logits = ref.qwen3_generate(m, prompt, 3)
    gm = device_model(m, max_ctx=80)
    try:
        got_ids = gm.generate(prompt, 3)
        got_logits = gm.logits().cpu().numpy()
    finally:
        gm.close()
    assert got_ids.tolist() == want_ids.tolist()
    assert max_rel(got_logits, want_logits) <= BLOCK_TOL


def test_long_context_attention_fallback(orc, ref):
    """max_ctx 2048: the prompt attention's score rows no longer fit in shared memory, so a
    40-token prompt takes the one-query-per-block kernel; decode steps keep the split kernel."""
    m = O.SynthModel(256, 4, 2, 128, 256, 16, 4, 512, 2, seed=7, norm_jitter=0.1, oracle=orc)
    prompt = np.random.default_rng(40).integers(0, m.vocab, 40).astype(np.int32)
    want_ids, want_logits = ref.qwen3_generate(m, prompt, 3)
    gm = device_model(m, max_ctx=2048)
    try:
        got_ids = gm.generate(prompt, 3)
        got_logits = gm.logits().cpu().numpy()
    finally:
        gm.close()
    assert got_ids.tolist() == want_ids.tolist()
    assert max_rel(got_logits, want_logits) <= BLOCK_TOL


def test_step_matches_generate(orc):
    m = O.SynthModel(256, 4, 2, 128, 256, 16, 4, 512, 2, seed=6, oracle=orc)
    prompt = np.array([5, 100, 7], np.int32)
    gm = device_model(m, max_ctx=16)
    try:
        ids = gm.generate(prompt, 3)
        nxt = gm.prefill(prompt)
        seq = [nxt]
        for _ in range(3):
            nxt = gm.step(nxt)
            seq.append(nxt)
    finally:
        gm.close()
    assert seq == ids.tolist()


def test_rejects_bad_ids(orc):
    from cachepotato_b200 import CpgError
    m = O.SynthModel(256, 4, 2, 128, 256, 16, 4, 512, 1, seed=7, oracle=orc)
    gm = device_model(m, max_ctx=8)
    try:
        with pytest.raises(CpgError):
            gm.prefill(np.array([1, 512], np.int32))
        with pytest.raises(CpgError):
            gm.prefill(np.arange(9, dtype=np.int32))       # longer than max_ctx
    finally:
        gm.close()
