"""CPW1 v4 files without a GPU: the file the reference converter writes from the synthetic
checkpoint (tests/golden/v4_synth.py) is reproduced byte for byte (sha256 recorded by
tests/golden/make_v4_golden.py from the reference's own convert.py + v4_writer.py), and the
loader's table walk (cachepotato_b200.v4.V4File) reads it as the reference reader does
(engine/blocks/qwen3_moe.c:318-586): layer count from the attention blocks, region ids =
table indices, tensor offsets relative to the data section, region digests = zlib.crc32 of
the region's bytes (format/v4_writer.py:235-250)."""
import os
import tempfile
import zlib

import numpy as np
import pytest

import v4_synth as S


@pytest.fixture(scope="module")
def v4_path():
    d = tempfile.mkdtemp(prefix="cpg_v4_")
    p = os.path.join(d, "model.v4cp")
    S.write_v4(p)
    yield p
    os.unlink(p)
    os.rmdir(d)


def test_writer_reproduces_the_reference_converter(golden, v4_path):
    g = golden("v4_ref.npz")
    assert os.path.getsize(v4_path) == int(g["size"])
    assert S.sha256(v4_path) == str(g["sha256"])


def test_table_walk_matches_the_reference_reader(golden, v4_path):
    from cachepotato_b200.v4 import V4File, REGION_EXPERT
    g = golden("v4_ref.npz")
    f = V4File(v4_path)
    L, D, V, E, K, F = (int(v) for v in g["meta"])          # what the reference loader read
    assert f.n_layers == L == S.CFG["num_hidden_layers"]
    assert f.tensor("final_norm")["dims"] == [D] and f.tensor("expert.0.0.Wg")["dims"][0] == F
    assert f.tensor("Wgate.1")["dims"] == [E, D]
    assert sum(t["dims"][0] for t in f.tensors if t["name"].startswith("embed.")) == V
    experts = [r for r in f.regions if r["kind"] == REGION_EXPERT]
    assert len(experts) == L * E
    data = np.asarray(f.map)
    for i, r in enumerate(f.regions):
        assert f.digest_len(r) == r["len"]                     # every tensor here is 64-byte sized
        lo = f.off_data + r["off"]
        assert zlib.crc32(data[lo:lo + r["len"]].tobytes()) == r["digest"], i
    # an expert region is its three matrices back to back (qwen3_moe.c:208-216 relies on it)
    r = experts[5]
    names = [f.tensors[i]["name"] for i in range(r["lo"], r["hi"])]
    assert names == ["expert.0.5.Wg", "expert.0.5.Wu", "expert.0.5.Wd"]
    assert f.tensors[r["lo"]]["off"] == r["off"]
