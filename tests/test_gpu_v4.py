"""A CPW1 v4 file end to end on the GPU: the bytes the reference converter writes (regenerated
by tests/golden/v4_synth.py and checked against the recorded sha256), loaded by
cachepotato_b200.v4.V4Model: data section copied once into the HBM region store, region ids =
table indices, every region's CRC-32 digest verified on the device, every layer bound from the
resident copy, then a 24-token prompt and 4 greedy steps. Compared with the reference engine
run through its own loader on the same file (tests/golden/v4_ref.npz): identical greedy ids and
the last step's logits within max|d|/max|ref| <= 1e-3."""
import os
import tempfile

import numpy as np
import pytest

import v4_synth as S
from helpers import BLOCK_TOL

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_v4_file_end_to_end(golden):
    from cachepotato_b200 import _lib
    from cachepotato_b200.v4 import V4Model
    g = golden("v4_ref.npz")
    d = tempfile.mkdtemp(prefix="cpg_v4_")
    path = os.path.join(d, "model.v4cp")
    try:
        S.write_v4(path)
        assert S.sha256(path) == str(g["sha256"])
        m = V4Model(path, max_ctx=64)
        try:
            assert m.verified
            assert m.dims["n_layers"] == int(g["meta"][0]) and m.dims["vocab"] == int(g["meta"][2])
            ids = m.generate(g["prompt"], len(g["ids"]) - 1)
            logits = m.logits().cpu().numpy()
        finally:
            m.close()
        assert ids.tolist() == g["ids"].tolist()
        got = logits[g["logit_pos"]]
        assert np.abs(got - g["logits"]).max() / float(g["logit_max"]) <= BLOCK_TOL
    finally:
        if os.path.exists(path):
            os.unlink(path)
        os.rmdir(d)


def test_v4_digest_mismatch_is_reported(golden):
    """One flipped byte inside an expert region: the device check names that region."""
    from cachepotato_b200 import CpgError
    from cachepotato_b200.v4 import V4File, V4Model
    d = tempfile.mkdtemp(prefix="cpg_v4_")
    path = os.path.join(d, "model.v4cp")
    try:
        S.write_v4(path)
        f = V4File(path)
        r = next(i for i, rg in enumerate(f.regions) if rg["kind"] == 1 and i == 7)
        pos = f.off_data + f.regions[r]["off"] + 1000
        del f
        with open(path, "r+b") as fh:
            fh.seek(pos)
            b = fh.read(1)
            fh.seek(pos)
            fh.write(bytes([b[0] ^ 0x5A]))
        with pytest.raises(CpgError, match=f"region {r}"):
            V4Model(path, max_ctx=16)
        from cachepotato_b200 import _lib
        _lib.lib().cpg_store_close()
    finally:
        if os.path.exists(path):
            os.unlink(path)
        os.rmdir(d)
