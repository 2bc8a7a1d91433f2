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


def _first_divergence_explained(ref, m, prompt, j, got_id, want_id):
    """Ids first differ at step j: true only if the reference's own logits at that step put the
    two ids within the logits tolerance of each other (a near-tie the bar cannot separate)."""
    _, lg = ref.qwen3_generate(m, prompt, j)
    return abs(float(lg[got_id]) - float(lg[want_id])) <= BLOCK_TOL * float(np.abs(lg).max())


def test_qwen3_full_vocab_512_prompt(orc, ref):
    """configs[2]'s vocabulary (151,936, Q8_0 embed and lm_head) and its 512-token prompt through
    two Qwen3-30B-A3B-shaped layers: the two-stage argmax over the full vocabulary, the prompt
    attention's 512-key tiles and the tensor-core projections at 512 tokens."""
    m = O.SynthModel(2048, 32, 4, 128, 768, 128, 8, 151936, 2, seed=13, norm_jitter=0.05, oracle=orc)
    prompt = np.random.default_rng(13).integers(0, m.vocab, 512).astype(np.int32)
    want_ids, want_logits = ref.qwen3_generate(m, prompt, 4)
    gm = device_model(m, max_ctx=520)
    try:
        got_ids = gm.generate(prompt, 4)
        got_logits = gm.logits().cpu().numpy()
    finally:
        gm.close()
    assert got_ids.tolist() == want_ids.tolist()
    assert max_rel(got_logits, want_logits) <= BLOCK_TOL


def _mem_available_gb():
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) / 2**20
    except OSError:
        pass
    return 0.0


def test_bench_full_model_first_ids(ref):
    """The benchmark's own configs[2] model (48 layers, its seeds: bench.expert_blob and
    bench.full_model_parts) and 512-token prompt: the first 8 greedy ids on the GPU against the
    reference engine's generate loop (engine/api/cachepotato.c:315-378) on copies of the same
    weights. A first difference is accepted only where the reference's logits at that step tie
    the two ids within the logits tolerance."""
    from types import SimpleNamespace
    import bench
    from cachepotato_b200 import _lib
    from cachepotato_b200 import qwen3 as Q
    if _mem_available_gb() < 48:
        pytest.skip("needs about 20 GB of host memory for the weight copies")
    lib = _lib.lib()
    seed, L, n_new = 1234, 48, 7
    D, F, E, K = 2048, 768, 128, 8
    blobs = [bench.expert_blob(torch, lib, Q, seed, l) for l in range(L)]
    P = bench.full_model_parts(torch, lib, Q, seed, L)
    moe = [Q.MoELayer(P["ln2"], P["routers"][l], O.ENC_Q4, D, F, E, K, blob=blobs[l]) for l in range(L)]
    gm = Q.Qwen3Model(d_model=D, n_heads=P["H"], n_kv=P["KVH"], head_dim=P["HD"], vocab=P["V"],
                      max_ctx=len(P["prompt"]) + n_new + 1, attn=P["attn"], moe=moe, attn_enc=O.ENC_Q4,
                      embed=P["embed"], embed_enc=O.ENC_Q8, lm_head=P["head"], head_enc=O.ENC_Q8,
                      final_norm=P["final_norm"])
    try:
        got = gm.generate(P["prompt"], n_new).tolist()
    finally:
        gm.close()
    host = lambda t: np.ascontiguousarray(t.cpu().numpy())
    ones_d, ones_h = np.ones(D, np.float32), np.ones(P["HD"], np.float32)
    mat = F * D // 32 * 18
    layers = [SimpleNamespace(blob=host(b), region_bytes=3 * mat, mat_bytes=mat, ln2=ones_d,
                              wgate=host(P["routers"][l]), enc=O.ENC_Q4) for l, b in enumerate(blobs)]
    del blobs
    m = SimpleNamespace(d_model=D, n_heads=P["H"], n_kv=P["KVH"], head_dim=P["HD"], d_exp=F, n_experts=E, topk=K,
                        vocab=P["V"], n_layers=L, rope_theta=1e6, eps=1e-6, embed=host(P["embed"]),
                        embed_enc=O.ENC_Q8, lm_head=host(P["head"]), head_enc=O.ENC_Q8, final_norm=ones_d,
                        ln1=[ones_d] * L, q_norm=[ones_h] * L, k_norm=[ones_h] * L,
                        wq=[host(a["wq"]) for a in P["attn"]], wk=[host(a["wk"]) for a in P["attn"]],
                        wv=[host(a["wv"]) for a in P["attn"]], wo=[host(a["wo"]) for a in P["attn"]],
                        attn_enc=O.ENC_Q4, layers=layers)
    want, _ = ref.qwen3_generate(m, P["prompt"], n_new)
    want = want.tolist()
    if got != want:
        j = next(i for i in range(len(got)) if got[i] != want[i])
        assert _first_divergence_explained(ref, m, P["prompt"], j, got[j], want[j]), (got, want)
        assert got[:j] == want[:j]
