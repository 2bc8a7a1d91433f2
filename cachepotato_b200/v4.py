"""CPW1 v4 model files on the device: the loader half of the reference engine for this path.

The reference maps the file and walks its tables in C: qwen3_map_ex reads the header, the
encoding table, the block table (layer count) and the region table (engine/blocks/
qwen3_moe.c:318-459), qwen3_bind_layer resolves each layer's tensors by name (462-586), and
the pager serves region ids that are region-table indices (engine/pager/pager.h:51-86). Here:

  V4File    parses the same tables from a read-only mapping of the file (format/SPEC.md; tensor
            offsets are relative to the data section, as the writer emits them)
  V4Model   copies the data section into the HBM region store once (cpg_store_open_v4), adds
            every region in table order so ids are table indices (cpg_store_add_region),
            checks every region's CRC-32 digest on the device against the table
            (cpg_store_verify / cpg_crc32: the digests the writer stores are zlib.crc32 over
            each region's tensors including their alignment padding, format/v4_writer.py:
            235-250), binds every layer from the resident copy and builds the whole model
            (cpg_qwen3) with one MoE layer (cpg_moe_layer) per attention block.

Model facts the reference loader fixes rather than reads (qwen3_moe.c:397-401): top-k 8 and
RMSNorm eps 1e-6; the RoPE theta is read here from the attention block's parameters (the
reference uses 1e6, which is what its converter writes). One store per process, like the pager.
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np

from . import _lib
from ._lib import ENC_F32, ENC_Q4, ENC_Q8, check, lib

MAGIC, VERSION = 0x34575043, 4
KIND_EMBED, KIND_ATTN, KIND_MOE = 1, 0x10, 0x20
REGION_EXPERT = 1
_TOPK, _EPS = 8, 1e-6


class _Reader:
    def __init__(self, buf: np.ndarray, pos: int):
        self.b, self.p = buf, pos

    def take(self, fmt: str):
        n = struct.calcsize(fmt)
        v = struct.unpack_from(fmt, self.b, self.p)
        self.p += n
        return v if len(v) > 1 else v[0]

    def string(self) -> str:
        n = self.take("<H")
        s = bytes(self.b[self.p:self.p + n]).decode()
        self.p += n
        return s


class V4File:
    """A CPW1 v4 file's tables over a read-only mapping (numpy memmap)."""

    def __init__(self, path: str):
        self.path = path
        self.map = np.memmap(path, dtype=np.uint8, mode="r")
        b = self.map
        magic, version, hdr_bytes, _ = struct.unpack_from("<IIII", b, 0)
        if magic != MAGIC or version != VERSION:
            raise ValueError(f"{path}: not a CPW1 v4 file (magic {magic:#x}, version {version})")
        n_tens, n_blk, n_reg, n_enc = struct.unpack_from("<IIII", b, 16)
        off_enc, off_tens, off_blk, off_reg, off_data = struct.unpack_from("<QQQQQ", b, 32)
        self.off_data = off_data
        r = _Reader(b, off_enc)
        self.encodings = []                       # engine code per encoding index
        for _ in range(n_enc):
            r.take("<I")
            kind, scalar = r.take("<BB")
            r.take("<HHBBB")
            r.string()
            self.encodings.append(ENC_F32 if kind == 0 else ENC_Q8 if scalar == 3 else ENC_Q4 if scalar == 4 else -1)
        r = _Reader(b, off_tens)
        if r.take("<I") != n_tens:
            raise ValueError(f"{path}: tensor table count differs from the header")
        self.tensors = []
        for _ in range(n_tens):
            name = r.string()
            eidx = r.take("<I")
            nd = r.take("<B")
            dims = [r.take("<I") for _ in range(nd)]
            off, nbytes = r.take("<QQ")
            r.take("<IH")
            enc = self.encodings[eidx] if eidx < n_enc else -1
            self.tensors.append(dict(name=name, enc=enc, dims=dims, off=off, nbytes=nbytes))
        self.by_name = {t["name"]: t for t in self.tensors}
        r = _Reader(b, off_blk)
        if r.take("<I") != n_blk:
            raise ValueError(f"{path}: block table count differs from the header")
        self.blocks = []
        for _ in range(n_blk):
            kind, layer, nref = r.take("<BIB")
            refs = [r.take("<I") for _ in range(nref)]
            npar = r.take("<B")
            params = [r.take("<I") for _ in range(npar)]
            self.blocks.append(dict(kind=kind, layer=layer, refs=refs, params=params))
        r = _Reader(b, off_reg)
        if r.take("<I") != n_reg:
            raise ValueError(f"{path}: region table count differs from the header")
        self.regions = []
        for _ in range(n_reg):
            off, length, lo, hi = r.take("<QQII")
            kind, slot, mlo, mhi, digest = r.take("<BHIIQ")
            self.regions.append(dict(off=off, len=length, lo=lo, hi=hi, kind=kind, digest=digest))
        self.n_layers = sum(1 for bl in self.blocks if bl["kind"] == KIND_ATTN)

    def digest_len(self, region) -> int:
        """Bytes the region's digest covers: its tensors including each one's alignment padding
        (the writer pads every tensor to the table's alignment, 64 bytes)."""
        last = self.tensors[region["hi"] - 1]
        end = last["off"] + last["nbytes"]
        end += (-end) % 64
        return end - region["off"]

    def tensor(self, name: str):
        t = self.by_name.get(name)
        if t is None:
            raise KeyError(f"{self.path}: no tensor {name!r}")
        return t


class DevAddr:
    """A device address where the model wrappers expect a tensor (they only call data_ptr())."""

    def __init__(self, p: int):
        self.p = int(p)

    def data_ptr(self) -> int:
        return self.p


class V4Model:
    """A CPW1 v4 Qwen3-MoE file resident in HBM and bound as a whole model (cpg_qwen3)."""

    def __init__(self, path: str, max_ctx: int, verify: bool = True):
        from .qwen3 import MoELayer, Qwen3Model
        self.file = f = V4File(path)
        L = lib()
        L.cpg_store_close()
        check(L.cpg_store_open_v4(ctypes.c_void_p(f.map.ctypes.data), f.map.size, f.off_data))
        self.store_open = True
        for i, rg in enumerate(f.regions):
            rid = L.cpg_store_add_region(rg["off"], rg["len"], int(rg["kind"] == REGION_EXPERT))
            if rid != i:
                raise RuntimeError(f"region {i} got id {rid}: region ids must be table indices")
        self.verified = False
        if verify:
            self.verify()
        base = int(L.cpg_store_base())
        dev = lambda name: DevAddr(base + f.tensor(name)["off"])
        attn_blk = next(bl for bl in f.blocks if bl["kind"] == KIND_ATTN)
        moe_blk = next((bl for bl in f.blocks if bl["kind"] == KIND_MOE), None)
        H, KV, HD, theta_bits = attn_blk["params"][:4]
        theta = struct.unpack("<f", struct.pack("<I", theta_bits))[0]
        D = f.tensor("final_norm")["dims"][0]
        E = moe_blk["params"][0] if moe_blk else f.tensor("Wgate.0")["dims"][0]
        K = moe_blk["params"][1] if moe_blk and len(moe_blk["params"]) > 1 else _TOPK
        F = f.tensor("expert.0.0.Wg")["dims"][0]
        # the embed table: one tensor, or row chunks (embed.0, embed.1, ...) that lie back to back
        if "embed" in f.by_name:
            emb = f.tensor("embed")
            V = emb["dims"][0]
        else:
            chunks = sorted((t for t in f.tensors if t["name"].startswith("embed.")), key=lambda t: int(t["name"][6:]))
            for a, b in zip(chunks, chunks[1:]):
                if a["off"] + a["nbytes"] != b["off"]:
                    raise ValueError("embed chunks are not contiguous in the data section")
            emb = chunks[0]
            V = sum(t["dims"][0] for t in chunks)
        head = f.tensor("lm_head")
        self.dims = dict(n_layers=f.n_layers, d_model=D, n_heads=H, n_kv=KV, head_dim=HD, vocab=V, n_experts=E,
                         topk=K, d_exp=F, rope_theta=theta)
        attn, moe = [], []
        for l in range(f.n_layers):
            attn.append(dict(ln1=dev(f"ln1.{l}"), q_norm=dev(f"q_norm.{l}"), k_norm=dev(f"k_norm.{l}"),
                             wq=dev(f"Wq.{l}"), wk=dev(f"Wk.{l}"), wv=dev(f"Wv.{l}"), wo=dev(f"Wo.{l}")))
            enc = f.tensor(f"expert.{l}.0.Wg")["enc"]
            ptrs = [base + f.tensor(f"expert.{l}.{e}.{m}")["off"] for e in range(E) for m in ("Wg", "Wu", "Wd")]
            moe.append(MoELayer(dev(f"ln2.{l}"), dev(f"Wgate.{l}"), enc, D, F, E, K, eps=_EPS, expert_ptrs=ptrs))
        attn_enc = f.tensor("Wq.0")["enc"]
        self.model = Qwen3Model(d_model=D, n_heads=H, n_kv=KV, head_dim=HD, vocab=V, max_ctx=max_ctx, attn=attn,
                                moe=moe, attn_enc=attn_enc, embed=DevAddr(base + emb["off"]), embed_enc=emb["enc"],
                                lm_head=DevAddr(base + head["off"]), head_enc=head["enc"],
                                final_norm=dev("final_norm"), rope_theta=theta, rms_eps=_EPS)

    def verify(self) -> None:
        """Every region's CRC-32 on the device against the region table (raises on a mismatch)."""
        f, L = self.file, lib()
        lens = [f.digest_len(rg) for rg in f.regions]
        if all(n == rg["len"] for n, rg in zip(lens, f.regions)):
            digests = (ctypes.c_uint64 * len(f.regions))(*[rg["digest"] for rg in f.regions])
            bad = ctypes.c_int(-1)
            rc = L.cpg_store_verify(digests, len(f.regions), ctypes.byref(bad))
            if rc != _lib.CPG_OK:
                raise _lib.CpgError(rc, f"region {bad.value}: digest mismatch ({_lib.last_error()})")
        else:
            base = int(L.cpg_store_base())
            for i, (rg, n) in enumerate(zip(f.regions, lens)):
                crc = ctypes.c_uint32()
                check(L.cpg_crc32(ctypes.c_void_p(base + rg["off"]), n, ctypes.byref(crc), None))
                if crc.value != rg["digest"]:
                    raise _lib.CpgError(_lib.CPG_EINVAL, f"region {i}: digest {crc.value:#x} != {rg['digest']:#x}")
        self.verified = True

    def generate(self, prompt, n_new: int):
        return self.model.generate(prompt, n_new)

    def logits(self):
        return self.model.logits()

    def close(self) -> None:
        if getattr(self, "model", None) is not None:
            self.model.close()
            self.model = None
        if getattr(self, "store_open", False):
            lib().cpg_store_close()
            self.store_open = False
