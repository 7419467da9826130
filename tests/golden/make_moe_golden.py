"""Generate tests/golden/moe_a3b_width.npz: qwen35moe at BASELINE config 4's
layer widths, from the FP64 restatement oracle/moe_fp64.py.

The reference has no CPU qwen35moe path (its MoE backend is Metal-only), so
its formulas are restated in float64 over the reference-exact FP32 weight
values; this fixture lets the GPU test compare a full-width model without
running the FP64 restatement on the GPU host.  The model is
synth_gguf.a3b_width_spec(): 4 layers (3 DeltaNet, 1 gated attention) with
every config-4 width, vocabulary 4096.  Stored: the GGUF SHA-256, the prompt,
greedy tokens and full logits of the prefill and 4 decode steps, and the
top-1 / top-2 margin per step.

    python tests/golden/make_moe_golden.py
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from myllm_b200 import synth_gguf as sg  # noqa: E402
from oracle.moe_fp64 import MoeFP64  # noqa: E402


def main():
    spec = sg.a3b_width_spec()
    prompt = sg.prompt_ids(spec.seed, 12, spec.vocab)
    with tempfile.TemporaryDirectory(dir=os.environ.get("MYLLM_GOLDEN_TMP")) as tmp:
        path = os.path.join(tmp, "a3b_width.gguf")
        sha = sg.write_moe(spec, path)
        ref = MoeFP64(path, max_sequence=64)
        tok, logits = ref.prefill(prompt)
        toks, all_logits = [tok], [logits]
        for _ in range(4):
            tok, logits = ref.decode(tok)
            toks.append(tok)
            all_logits.append(logits)
    lg = np.stack(all_logits).astype(np.float32)
    top2 = np.sort(np.stack(all_logits), axis=1)[:, -2:]
    np.savez_compressed(os.path.join(HERE, "moe_a3b_width.npz"), sha256=np.array(sha), prompt=prompt,
                        tokens=np.array(toks), logits=lg, margin=top2[:, 1] - top2[:, 0])
    print("tokens", toks, "margins", top2[:, 1] - top2[:, 0])


if __name__ == "__main__":
    main()
