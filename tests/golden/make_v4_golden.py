"""Golden fixture for the CPW1 v4 end-to-end test (tests/golden/v4_ref.npz). Run where the
reference tree exists:

    python tests/golden/make_v4_golden.py

1. writes the synthetic checkpoint of v4_synth.py and converts it with the reference's own
   models/qwen3-30b-a3b/convert.py (unmodified; --quant q8_0 --quant-experts q4_0
   --quant-attn q4_0), which writes through format/v4_writer.py;
2. writes the same model with v4_synth.write_v4 and requires identical bytes;
3. runs the reference engine on the reference-written file through its own loader
   (qwen3_map_ex / qwen3_bind_layer, harness refh_v4_generate): a 24-token prompt, then 4
   greedy steps.
Stored: the file's sha256 and size, the prompt, the greedy ids, the last step's logits at 4096
fixed positions plus their maximum, and the model dimensions the loader read.
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
import oracle as O  # noqa: E402
import v4_synth as S  # noqa: E402

PROMPT_SEED, N_PROMPT, N_NEW, N_LOGITS = 77, 24, 4, 4096


def prompt():
    return np.random.default_rng(PROMPT_SEED).integers(0, S.CFG["vocab_size"], N_PROMPT).astype(np.int32)


def logit_positions():
    return np.sort(np.random.default_rng(PROMPT_SEED + 1).choice(S.CFG["vocab_size"], N_LOGITS, replace=False))


def main():
    O.build(ref=True)
    ref = O.Reference(threads=8)
    with tempfile.TemporaryDirectory() as d:
        ck = os.path.join(d, "ckpt")
        S.write_checkpoint(ck)
        a, b = os.path.join(d, "ref.v4cp"), os.path.join(d, "ours.v4cp")
        subprocess.run([sys.executable, os.path.join(O.REF_TREE, "models", "qwen3-30b-a3b", "convert.py"),
                        "--model", ck, "--out", a, "--quant", "q8_0", "--quant-experts", "q4_0",
                        "--quant-attn", "q4_0"], check=True)
        S.write_v4(b)
        ha, hb = S.sha256(a), S.sha256(b)
        assert ha == hb, f"v4_synth.write_v4 differs from the reference converter: {hb} != {ha}"
        ids, logits, meta = ref.v4_generate(a, prompt(), N_NEW)
        pos = logit_positions()
        np.savez_compressed(os.path.join(HERE, "v4_ref.npz"), sha256=np.array(ha), size=np.array(os.path.getsize(a)),
                            prompt=prompt(), ids=ids, logit_pos=pos, logits=logits[pos],
                            logit_max=np.array(float(np.abs(logits).max()), np.float32), meta=meta)
        print("v4 golden:", ha, os.path.getsize(a), "ids", ids.tolist(), "meta", meta.tolist())


if __name__ == "__main__":
    main()
