"""Test helpers: put an oracle SynthLayer on the device and compare routing by the reference's
agreement rule (expert ids identical except where the top-k margin is below 1e-6)."""
import numpy as np

TOPK_MARGIN = 1e-6     # routing agreement: ids may differ only where the margin is below this
BLOCK_TOL = 1e-3       # max|d| / max|ref| for block outputs on fp16 operand rows (the tcgen05
                       # prefill and expert-parallel paths: the benchmark's bf16-class config)
DECODE_TOL = 1e-5      # max|d| / max|ref| for the decode MoE block (f32 activations carried as
                       # fp16 hi + lo halves; the kernel gate of tools/verify_q8_kernels.py)
KERNEL_TOL = 1e-5      # fp32 matvec kernels (tools/verify_q8_kernels.py tolerance)


def device_layer(layer, torch=None):
    """MoELayer over a copy of SynthLayer `layer` in device memory."""
    import torch as _t
    from cachepotato_b200.qwen3 import MoELayer
    torch = torch or _t
    ln2 = torch.from_numpy(layer.ln2).cuda()
    wg = torch.from_numpy(layer.wgate).cuda()
    blob = torch.from_numpy(layer.blob).cuda()
    return MoELayer(ln2, wg, layer.enc, layer.d_model, layer.d_exp, layer.n_experts, layer.topk,
                    eps=layer.eps, blob=blob)


def probs_from_logits(logits):
    z = logits.astype(np.float64)
    z = np.exp(z - z.max(-1, keepdims=True))
    return z / z.sum(-1, keepdims=True)


def check_topk(got_idx, want_idx, want_logits, K):
    """Per token: same ordered ids, or every differing slot explained by a sub-1e-6 probability
    margin between the two experts that swapped there (the reference's top-k picks by strict '>'
    in descending order, qwen3_moe.c:184-194, so only near-equal probabilities can trade places,
    within the top k or across the k-th / (k+1)-th boundary)."""
    p = probs_from_logits(want_logits)
    bad = []
    for t in range(got_idx.shape[0]):
        g, w = np.asarray(got_idx[t]), np.asarray(want_idx[t])
        if np.array_equal(g, w):
            continue
        diff = np.nonzero(g != w)[0]
        ok = len(set(g.tolist())) == len(g) and all(
            0 <= g[j] < p.shape[1] and abs(p[t, g[j]] - p[t, w[j]]) < TOPK_MARGIN for j in diff)
        if not ok:
            bad.append(t)
    return bad


def device_model(model, max_ctx, torch=None):
    """cachepotato_b200 Qwen3Model over a copy of oracle SynthModel `model` in device memory."""
    import torch as _t
    from cachepotato_b200.qwen3 import Qwen3Model
    torch = torch or _t
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    attn = [dict(ln1=dev(model.ln1[l]), q_norm=dev(model.q_norm[l]), k_norm=dev(model.k_norm[l]),
                 wq=dev(model.wq[l]), wk=dev(model.wk[l]), wv=dev(model.wv[l]), wo=dev(model.wo[l]))
            for l in range(model.n_layers)]
    moe = [device_layer(ly) for ly in model.layers]
    return Qwen3Model(d_model=model.d_model, n_heads=model.n_heads, n_kv=model.n_kv, head_dim=model.head_dim,
                      vocab=model.vocab, max_ctx=max_ctx, attn=attn, moe=moe, attn_enc=model.attn_enc,
                      embed=dev(model.embed), embed_enc=model.embed_enc, lm_head=dev(model.lm_head),
                      head_enc=model.head_enc, final_norm=dev(model.final_norm), rope_theta=model.rope_theta,
                      rms_eps=model.eps)
