"""A synthetic Qwen3-MoE checkpoint and the CPW1 v4 file the reference builds from it.

TEST INFRASTRUCTURE. The reference converts a HuggingFace checkpoint to CPW1 v4 with
models/qwen3-30b-a3b/convert.py through format/v4_writer.py. Neither the real weights nor the
reference tree exist on the GPU box, so the end-to-end file test needs the file's exact bytes
without them:

  write_checkpoint(dir)  the checkpoint the reference converter reads: config.json,
                         model.safetensors and its index, every tensor drawn from a seeded
                         generator (a Qwen3-30B-A3B-shaped model cut to width 256 and 2 layers;
                         vocabulary 151,936, top-8, RoPE theta 1e6 and eps 1e-6 are what the
                         reference loader assumes, qwen3_moe.c:397-401)
  write_v4(path)         the same model written as the reference converter writes it with
                         --quant q8_0 --quant-experts q4_0 --quant-attn q4_0 (the benchmark's
                         encodings): our own writer of the format (format/SPEC.md) that follows
                         the converter's tensor order, blocks and regions (convert.py:166-237)
                         and the writer's layout rules (v4_writer.py:197-299: f32 tensors placed
                         first, 64-byte alignment, CRC-32 region digests over the payload and its
                         padding). tests/golden/make_v4_golden.py checks that both routes give the
                         same bytes (sha256 stored in v4_ref.npz).

Quantisation uses the oracle's encoder, pinned bit-exact to format/q4.py and format/q8.py by
the reference's decoder KATs.
"""
from __future__ import annotations

import json
import os
import struct
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))

CFG = dict(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, head_dim=128, num_experts=16,
           num_experts_per_tok=8, moe_intermediate_size=256, vocab_size=151936, rope_theta=1000000.0,
           rms_norm_eps=1e-6, num_hidden_layers=2)
# the public-API tests' model: 128 experts, as the reference engine's cp_open expects (its
# layer binding clears a 128-entry expert-region table, qwen3_moe.c:462-586)
CHAT_CFG = dict(CFG, num_experts=128)
SEED = 20261202
EMBED_ROWS = 1024                       # the converter's default region granularity of the embed table

# format constants (format/SPEC.md; the values v4_writer.py writes)
MAGIC, VERSION, HDR_BYTES, ALIGN = 0x34575043, 4, 88, 64
KIND_EMBED, KIND_ATTN, KIND_MOE = 1, 0x10, 0x20
R_EMBED, R_NORM, R_ATTN, R_ROUTER, R_EXPERT, R_HEAD = 1, 2, 3, 4, 5, 8
REGION_TENSOR, REGION_EXPERT = 0, 1
NO_BLOCK = 0xFFFFFFFF
ENC_DESC = {"f32": (0, 0, 0, 4, 1, 0, 4, "f32"), "q8_0": (1, 3, 32, 34, 1, 3, 64, "Q8_0"),
            "q4_0": (1, 4, 32, 18, 1, 3, 64, "Q4_0")}


def hf_tensors(c=None):
    """(HF name, shape, kind) in a fixed order; kind: 'norm' (1 + 0.05 N(0,1)) or 'mat' (0.02 N)."""
    c = c or CFG
    D, H, KV, HD, E, F, V = (c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"],
                             c["num_experts"], c["moe_intermediate_size"], c["vocab_size"])
    out = [("model.embed_tokens.weight", (V, D), "mat")]
    for l in range(c["num_hidden_layers"]):
        p = f"model.layers.{l}."
        out += [(p + "input_layernorm.weight", (D,), "norm"), (p + "post_attention_layernorm.weight", (D,), "norm"),
                (p + "self_attn.q_norm.weight", (HD,), "norm"), (p + "self_attn.k_norm.weight", (HD,), "norm"),
                (p + "self_attn.q_proj.weight", (H * HD, D), "mat"), (p + "self_attn.k_proj.weight", (KV * HD, D), "mat"),
                (p + "self_attn.v_proj.weight", (KV * HD, D), "mat"), (p + "self_attn.o_proj.weight", (D, H * HD), "mat"),
                (p + "mlp.gate.weight", (E, D), "mat")]
        for e in range(E):
            for k, shp in (("gate_proj", (F, D)), ("up_proj", (F, D)), ("down_proj", (D, F))):
                out.append((p + f"mlp.experts.{e}.{k}.weight", shp, "mat"))
    out += [("model.norm.weight", (D,), "norm"), ("lm_head.weight", (V, D), "mat")]
    return out


def tensor_value(name, shape, kind):
    """Deterministic f32 values of one checkpoint tensor (seeded by its name)."""
    rng = np.random.default_rng([SEED, zlib.crc32(name.encode())])
    v = rng.standard_normal(int(np.prod(shape)), dtype=np.float32)
    v = v * np.float32(0.05) + np.float32(1.0) if kind == "norm" else v * np.float32(0.02)
    return v.astype(np.float32).reshape(shape)


def write_checkpoint(d):
    """The HuggingFace-layout checkpoint the reference converter reads (one safetensors shard)."""
    from safetensors.numpy import save_file
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(CFG, f)
    tens = {n: tensor_value(n, s, k) for n, s, k in hf_tensors()}
    save_file(tens, os.path.join(d, "model.safetensors"))
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": {n: "model.safetensors" for n in tens}}, f)


def _layout(c=None):
    """The converter's tensors in registration order: (name, hf name, shape, role, encoding)."""
    c = c or CFG
    D, H, KV, HD, E, F, V, L = (c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"],
                                c["num_experts"], c["moe_intermediate_size"], c["vocab_size"], c["num_hidden_layers"])
    t = []
    for ci, r0 in enumerate(range(0, V, EMBED_ROWS)):
        t.append((f"embed.{ci}", "model.embed_tokens.weight", (min(r0 + EMBED_ROWS, V) - r0, D), R_EMBED, "q8_0", r0))
    for l in range(L):
        p = f"model.layers.{l}."
        t += [(f"ln1.{l}", p + "input_layernorm.weight", (D,), R_NORM, "f32", None),
              (f"ln2.{l}", p + "post_attention_layernorm.weight", (D,), R_NORM, "f32", None),
              (f"q_norm.{l}", p + "self_attn.q_norm.weight", (HD,), R_NORM, "f32", None),
              (f"k_norm.{l}", p + "self_attn.k_norm.weight", (HD,), R_NORM, "f32", None)]
        for nm, key in (("Wq", "q_proj"), ("Wk", "k_proj"), ("Wv", "v_proj"), ("Wo", "o_proj")):
            shp = (H * HD, D) if nm == "Wq" else (KV * HD, D) if nm in ("Wk", "Wv") else (D, H * HD)
            t.append((f"{nm}.{l}", p + f"self_attn.{key}.weight", shp, R_ATTN, "q4_0", None))
        t.append((f"Wgate.{l}", p + "mlp.gate.weight", (E, D), R_ROUTER, "f32", None))
        for e in range(E):
            for nm, key in (("Wg", "gate_proj"), ("Wu", "up_proj"), ("Wd", "down_proj")):
                shp = (D, F) if nm == "Wd" else (F, D)
                t.append((f"expert.{l}.{e}.{nm}", p + f"mlp.experts.{e}.{key}.weight", shp, R_EXPERT, "q4_0", None))
    t += [("final_norm", "model.norm.weight", (D,), R_NORM, "f32", None),
          ("lm_head", "lm_head.weight", (V, D), R_HEAD, "q8_0", None)]
    return t


def _nbytes(shape, enc):
    n = int(np.prod(shape))
    return n // 32 * 34 if enc == "q8_0" else n // 32 * 18 if enc == "q4_0" else n * 4


def write_v4(path, c=None):
    """The CPW1 v4 file of the checkpoint, byte for byte as the reference converter writes it
    (c: another configuration of the same family, CFG by default)."""
    import oracle as O
    orc = O.Oracle()
    c = c or CFG
    kinds = {n: k for n, _, k in hf_tensors(c)}
    hf_shape = {n: s for n, s, _ in hf_tensors(c)}
    tensors = _layout(c)
    cache = {}

    def payload(i):
        name, src, shape, role, enc, r0 = tensors[i]
        if src not in cache:
            cache.clear()
            cache[src] = tensor_value(src, hf_shape[src], kinds[src])
        a = cache[src]
        if r0 is not None:
            a = a[r0:r0 + shape[0]]
        a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
        if enc == "f32":
            return a.tobytes()
        return orc.quantize(a, O.ENC_Q8 if enc == "q8_0" else O.ENC_Q4).tobytes()

    encs = []
    for t in tensors:
        if t[4] not in encs:
            encs.append(t[4])
    # physical placement: f32 tensors first, then the rest, each group in registration order
    order = [i for i, t in enumerate(tensors) if t[4] == "f32"] + [i for i, t in enumerate(tensors) if t[4] != "f32"]
    off, pads, offs = 0, {}, {}
    for i in order:
        nb = _nbytes(tensors[i][2], tensors[i][4])
        offs[i], pads[i] = off, (-nb) % ALIGN
        off += nb + pads[i]
    tid = {t[0]: i for i, t in enumerate(tensors)}

    def u16(v): return struct.pack("<H", v & 0xFFFF)
    def u32(v): return struct.pack("<I", v & 0xFFFFFFFF)
    def u64(v): return struct.pack("<Q", v & 0xFFFFFFFFFFFFFFFF)
    def string(s): return u16(len(s.encode())) + s.encode()

    enc_b = b"".join(u32(k) + bytes([d[0], d[1]]) + u16(d[2]) + u16(d[3]) + bytes([d[4], d[5], d[6]]) + string(d[7])
                     for k, d in ((k, ENC_DESC[e]) for k, e in enumerate(encs)))
    tens_b = u32(len(tensors))
    for i, (name, _, shape, role, enc, _) in enumerate(tensors):
        tens_b += string(name) + u32(encs.index(enc)) + bytes([len(shape)]) + b"".join(u32(d) for d in shape)
        tens_b += u64(offs[i]) + u64(_nbytes(shape, enc)) + u32(NO_BLOCK) + u16(role)
    L, E, K = c["num_hidden_layers"], c["num_experts"], c["num_experts_per_tok"]
    blocks = [(KIND_EMBED, 0xFFFFFFFF, [tid[t[0]] for t in tensors if t[0].startswith("embed.")],
               [c["vocab_size"], c["hidden_size"], 0])]
    theta = struct.unpack("<I", struct.pack("<f", c["rope_theta"]))[0]
    one = struct.unpack("<I", struct.pack("<f", 1.0))[0]
    for l in range(L):
        blocks.append((KIND_ATTN, l, [tid[f"{n}.{l}"] for n in ("Wq", "Wk", "Wv", "Wo", "q_norm", "k_norm")],
                       [c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"], theta, 1, 0]))
        blocks.append((KIND_MOE, l, [tid[f"Wgate.{l}"]], [E, K, 0, 1, 0, one, 0, 0, 0, 1]))
    blk_b = u32(len(blocks)) + b"".join(bytes([k]) + u32(ly) + bytes([len(r)]) + b"".join(u32(x) for x in r) +
                                        bytes([len(p)]) + b"".join(u32(x) for x in p) for k, ly, r, p in blocks)
    regions = []
    for l in range(L):
        for e in range(E):
            ids = [tid[f"expert.{l}.{e}.{n}"] for n in ("Wg", "Wu", "Wd")]
            regions.append((min(ids), max(ids) + 1, REGION_EXPERT, l, e, e + 1))
    for i, t in enumerate(tensors):
        if not t[0].startswith("expert."):
            regions.append((i, i + 1, REGION_TENSOR, 0xFFFF, 0, 1))
    reg_b = u32(len(regions))
    for lo, hi, kind, slot, mlo, mhi in regions:
        crc = 0
        for i in range(lo, hi):
            crc = zlib.crc32(payload(i) + b"\0" * pads[i], crc)
        length = offs[hi - 1] + _nbytes(tensors[hi - 1][2], tensors[hi - 1][4]) - offs[lo]
        reg_b += u64(offs[lo]) + u64(length) + u32(lo) + u32(hi) + bytes([kind]) + u16(slot) + u32(mlo) + u32(mhi)
        reg_b += u64(crc)
    off_enc = HDR_BYTES
    off_tens = off_enc + len(enc_b)
    off_blk = off_tens + len(tens_b)
    off_reg = off_blk + len(blk_b)
    off_data = (off_reg + len(reg_b) + ALIGN - 1) // ALIGN * ALIGN
    hdr = struct.pack("<IIII", MAGIC, VERSION, HDR_BYTES, 0)
    hdr += struct.pack("<IIII", len(tensors), len(blocks), len(regions), len(encs))
    hdr += struct.pack("<QQQQQ", off_enc, off_tens, off_blk, off_reg, off_data)
    hdr += struct.pack("<IIII", 0, 0, 0, 0)
    with open(path, "wb") as f:
        f.write(hdr + enc_b + tens_b + blk_b + reg_b)
        f.write(b"\0" * (off_data - f.tell()))
        for i in sorted(range(len(tensors)), key=lambda k: offs[k]):
            f.write(payload(i) + b"\0" * pads[i])
    return off_data


def sha256(path):
    import hashlib
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()
