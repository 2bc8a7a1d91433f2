"""The engine's public API on the GPU (libcachepotato_b200.so, include/cpg_chat.h) against the
reference's own cachepotato.c on the CPU (engine/api/cachepotato.c:205-378, compiled from its
sources into oracle/_ref/libcpref_api.so): the same CPW1 v4 file (the reference converter's bytes,
tests/golden/v4_synth.py, 128 experts), the same synthetic tokenizer files, the same conversation of six turns
(a turn stopped by the callback, cp_reset, a context restart at max_ctx 128). Every turn must
stream the same token bytes and report the same prompt / context / generated counts, restart flag
and stop reason; a second cp_open in the process must be refused by both."""
import json
import os
import subprocess
import sys
import tempfile

import pytest

import chat_synth
import v4_synth as S

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _drive(kind, model, out):
    r = subprocess.run([sys.executable, os.path.join(HERE, "chat_driver.py"), kind, model, out],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    with open(out) as f:
        return json.load(f)


def test_chat_turns_match_the_reference_engine():
    d = tempfile.mkdtemp(prefix="cpg_chat_")
    model = os.path.join(d, "model.v4cp")
    S.write_v4(model, S.CHAT_CFG)
    chat_synth.write(d)
    ref = _drive("ref", model, os.path.join(d, "ref.json"))
    gpu = _drive("gpu", model, os.path.join(d, "gpu.json"))
    assert "error" not in ref, ref
    assert "error" not in gpu, gpu
    assert gpu["second_open_refused"] and ref["second_open_refused"]
    assert gpu["stats"] == ref["stats"]
    stops = set()
    for i, (a, b) in enumerate(zip(ref["turns"], gpu["turns"])):
        assert a == b, f"turn {i}: reference {a} vs gpu {b}"
        stops.add(a["stop"])
    assert any(t["context_reset"] for t in ref["turns"])          # the restart path ran
    assert 3 in stops                                              # CP_STOP_CALLER ran
