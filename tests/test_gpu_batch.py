"""Several sequences decoded together (cpg_qwen3_batch, continuous batching).

The reference engine decodes one sequence at a time (engine/api/cachepotato.h:12-16), so the
oracle for a batch is that engine's own greedy loop (cp_chat, engine/api/cachepotato.c:315-378,
through oracle/ref_harness.c) run on each sequence alone: every slot must produce exactly the ids
the reference produces for its prompt, however the slots are grouped into steps, and each slot's
last logits must stay within max|d|/max|ref| <= 1e-3 of the reference's."""
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


def _small(orc, seed):
    return O.SynthModel(256, 4, 2, 128, 256, 16, 4, 512, 2, seed=seed, norm_jitter=0.1, oracle=orc)


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).astype(np.int32) for n in lens]


def test_batch_matches_reference_per_sequence(orc, ref):
    from cachepotato_b200.qwen3 import Qwen3Batch
    m = _small(orc, 21)
    prompts = _prompts(m.vocab, [1, 5, 9, 3], 22)
    n_new = 5
    gm = device_model(m, max_ctx=32)
    b = Qwen3Batch(gm, 4, 24)
    try:
        first = [b.prefill(j, p) for j, p in enumerate(prompts)]
        out = b.generate([0, 1, 2, 3], first, n_new)
        lg = b.logits().cpu().numpy()
        for j, p in enumerate(prompts):
            want_ids, want_logits = ref.qwen3_generate(m, p, n_new)
            got = [first[j]] + out[:, j].tolist()
            assert got == want_ids.tolist(), f"slot {j}"
            assert max_rel(lg[j], want_logits) <= BLOCK_TOL
            assert b.position(j) == len(p) + n_new
    finally:
        b.close()
        gm.close()


@pytest.mark.parametrize("n", [7, 12])
def test_batch_on_dense_kernel(orc, ref, n):
    """7 and 12 sequences: the step's projections and lm_head run on the dense tensor-core kernel
    (5 to 64 token rows: decode tile copies, fp16 hi + lo activations, f32 group scales); 7 rows
    leave a partly filled four-token column tile."""
    from cachepotato_b200.qwen3 import Qwen3Batch
    m = _small(orc, 41)
    prompts = _prompts(m.vocab, list(range(1, n + 1)), 42)
    n_new = 4
    gm = device_model(m, max_ctx=32)
    b = Qwen3Batch(gm, n, 20)
    try:
        first = [b.prefill(j, p) for j, p in enumerate(prompts)]
        slots = np.arange(n)[::-1].copy()                        # reversed slot order
        out = b.generate(slots, [first[j] for j in slots], n_new)
        lg = b.logits().cpu().numpy()
        for r, j in enumerate(slots):
            want_ids, want_logits = ref.qwen3_generate(m, prompts[j], n_new)
            assert [first[j]] + out[:, r].tolist() == want_ids.tolist(), f"slot {j}"
            assert max_rel(lg[r], want_logits) <= BLOCK_TOL
    finally:
        b.close()
        gm.close()


def test_continuous_batching_join_and_leave(orc, ref):
    """Sequences join (prefill into a free slot) and leave between steps, in changing orders; a
    finished sequence's slot is reused. Each sequence's ids equal the reference's for its prompt."""
    from cachepotato_b200.qwen3 import Qwen3Batch
    m = _small(orc, 23)
    A, B, C, D = _prompts(m.vocab, [4, 2, 7, 3], 24)
    gm = device_model(m, max_ctx=32)
    b = Qwen3Batch(gm, 3, 24)
    got = {k: [] for k in "ABCD"}
    nxt = {}
    try:
        def prefill(key, slot, prompt):
            nxt[key] = b.prefill(slot, prompt)
            got[key].append(nxt[key])

        def step(pairs):                              # [(key, slot), ...] in step order
            ids = b.step([s for _, s in pairs], [nxt[k] for k, _ in pairs])
            for (k, _), i in zip(pairs, ids.tolist()):
                nxt[k] = i
                got[k].append(i)

        prefill("A", 0, A)
        prefill("B", 1, B)
        for _ in range(3):
            step([("A", 0), ("B", 1)])
        prefill("C", 2, C)
        for _ in range(2):
            step([("B", 1), ("C", 2), ("A", 0)])
        for _ in range(2):                            # A has left
            step([("C", 2), ("B", 1)])
        prefill("D", 0, D)                            # D reuses A's slot
        for _ in range(2):
            step([("D", 0), ("C", 2)])
        out = b.generate([1, 0], [nxt["B"], nxt["D"]], 2)
        got["B"] += out[:, 0].tolist()
        got["D"] += out[:, 1].tolist()
    finally:
        b.close()
        gm.close()
    for key, prompt in zip("ABCD", (A, B, C, D)):
        want, _ = ref.qwen3_generate(m, prompt, len(got[key]) - 1)
        assert got[key] == want.tolist(), key


def test_batch_leaves_the_models_own_sequence_alone(orc):
    from cachepotato_b200.qwen3 import Qwen3Batch
    m = _small(orc, 25)
    p, q = _prompts(m.vocab, [6, 3], 26)
    gm = device_model(m, max_ctx=32)
    try:
        plain = gm.generate(p, 4).tolist()
        b = Qwen3Batch(gm, 2, 16)
        try:
            seq = [gm.prefill(p)]
            b.prefill(1, q)
            for _ in range(4):
                seq.append(gm.step(seq[-1]))
                b.step([1], [seq[-1] % m.vocab])
        finally:
            b.close()
    finally:
        gm.close()
    assert seq == plain


def test_batch_qwen3_widths_on_tensor_cores(orc, ref):
    """Qwen3-30B-A3B widths, 40 sequences: the step's projections run on the tcgen05 GEMM
    (32 tokens or more) and the MoE block on the batched expert kernel, each token's attention on
    its own slot. Every slot agrees with the single-sequence path; a sample with the reference."""
    from cachepotato_b200.qwen3 import Qwen3Batch
    m = O.SynthModel(2048, 32, 4, 128, 768, 128, 8, 4096, 2, seed=27, norm_jitter=0.05, oracle=orc)
    S, n_new = 40, 3
    lens = np.random.default_rng(28).integers(1, 7, S)
    prompts = _prompts(m.vocab, lens, 29)
    gm = device_model(m, max_ctx=48)
    b = Qwen3Batch(gm, S, 16)
    try:
        first = [b.prefill(j, p) for j, p in enumerate(prompts)]
        order = np.random.default_rng(30).permutation(S)             # any slot order
        out = b.generate(order, [first[j] for j in order], n_new)
        lg = b.logits().cpu().numpy()
        for r, j in enumerate(order):
            want = gm.generate(prompts[j], n_new)
            want_lg = gm.logits().cpu().numpy()
            assert [first[j]] + out[:, r].tolist() == want.tolist(), f"slot {j}"
            assert max_rel(lg[r], want_lg) <= BLOCK_TOL
        for j in (0, 17):
            want_ids, want_logits = ref.qwen3_generate(m, prompts[j], n_new)
            r = int(np.nonzero(order == j)[0][0])
            assert [first[j]] + out[:, r].tolist() == want_ids.tolist()
            assert max_rel(lg[r], want_logits) <= BLOCK_TOL
    finally:
        b.close()
        gm.close()


def test_batch_rejects_bad_requests(orc):
    from cachepotato_b200 import CpgError
    from cachepotato_b200.qwen3 import Qwen3Batch
    m = _small(orc, 31)
    gm = device_model(m, max_ctx=16)
    b = Qwen3Batch(gm, 3, 8)
    try:
        n0 = b.prefill(0, np.array([1, 2, 3], np.int32))
        with pytest.raises(CpgError):
            b.step([1], [n0])                                  # slot 1 holds no sequence
        with pytest.raises(CpgError):
            b.step([0, 0], [n0, n0])                           # a slot named twice
        with pytest.raises(CpgError):
            b.step([3], [n0])                                  # no such slot
        with pytest.raises(CpgError):
            b.step([0], [m.vocab])                             # id out of range
        with pytest.raises(CpgError):
            b.prefill(1, np.arange(8, dtype=np.int32))         # no room left in max_ctx 8
        with pytest.raises(CpgError):
            b.generate([0], [n0], 6)                           # 3 + 6 positions > 8
        assert b.position(0) == 3 and b.position(1) == -1
        b.generate([0], [n0], 5)                               # exactly fills the slot
        assert b.position(0) == 8
        with pytest.raises(CpgError):
            Qwen3Batch(gm, 3, 17)                              # longer than the model's max_ctx
    finally:
        b.close()
        gm.close()
