"""Generate the golden fixtures of tests/golden from the reference itself.

Runs the reference's own CPU path (CPULLM's sequence through
oracle/ref_harness.cpp, built from the reference sources by oracle/Makefile)
on seeded synthetic GGUF models written by myllm_b200.synth_gguf, and
stores tokens and logits.  The GGUF SHA-256 is stored with each fixture so a
test can tell when the generator no longer reproduces the same file.

    python tests/golden/make_golden.py [--skip-05b] [--only-7b]

Fixtures:
  tiny_s{seed}.npz   every format on some tensor (hidden 256, 2 layers),
                     prompt 8 and 40 tokens, prefill + 4 greedy decodes, full
                     logits from the reference.
  blocks.npz         per format: native rows and the reference's dequantized
                     FP32 values (known-answer vectors for the block decoders).
  qwen2_05b.npz      BASELINE config 0 (Qwen2.5-0.5B shape): 16-token prompt,
                     prefill + 4 decodes; tokens, top-64 logits, every 16th
                     logit, max |logit| and the top-1/top-2 margin per step.
  qwen2_7b.npz       BASELINE config 2 (Qwen2.5-7B shape, the bench workload's
                     model): 8-token prompt, prefill + 2 decodes, the same
                     summary as qwen2_05b.  The reference holds ~35 GB of FP32
                     weights, so the harness and the CPULLM cross-check run
                     one after the other (--only-7b makes just this one).
  q4km_d128.npz      a small model with the 7B's structure (Q4_K_M layout,
                     head_dim 128, 7 query heads per KV head; 3 layers):
                     prompts of 8 and 1100 tokens (the long one spans 16
                     attention key splits of two 64-key tiles each), prefill
                     + 4 greedy decodes, full logits (--only-small).
  qwen2_7b_long.npz  BASELINE config 2 at its full length: the bench's
                     512-token prompt, prefill + 128 greedy decodes, the same
                     summary (--only-7b-long).  The harness's fixture is
                     written as soon as it finishes (cpullm_checked = 0), then
                     rewritten with cpullm_checked = 1 once CPULLM itself has
                     produced the same tokens (about 40 minutes of one core
                     for each of the two runs).
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from myllm_b200 import synth_gguf as sg  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def run_reference(path: str, prompt: np.ndarray, steps: int):
    ref = oracle.ReferenceCPU(path)
    tok, lg = ref.prefill(prompt)
    tokens, logits = [tok], [lg]
    for _ in range(steps):
        tok, lg = ref.decode(tok)
        tokens.append(tok)
        logits.append(lg)
    # the harness's argmax must equal CPULLM's own token sequence
    cpu = oracle.ReferenceCPULLM(path)
    t = [cpu.prefill(prompt)]
    for _ in range(steps):
        t.append(cpu.decode(t[-1]))
    assert t == tokens, (t, tokens)
    cpu.close()
    return ref, np.array(tokens, dtype=np.int32), np.stack(logits)


def run_reference_sequential(path: str, prompt: np.ndarray, steps: int):
    """run_reference for models whose FP32 weights fit in host memory only
    once: the harness is closed before CPULLM cross-checks its tokens."""
    ref = oracle.ReferenceCPU(path)
    tok, lg = ref.prefill(prompt)
    tokens, logits = [tok], [lg]
    for _ in range(steps):
        tok, lg = ref.decode(tok)
        tokens.append(tok)
        logits.append(lg)
    ref.close()
    cpu = oracle.ReferenceCPULLM(path)
    t = [cpu.prefill(prompt)]
    for _ in range(steps):
        t.append(cpu.decode(t[-1]))
    cpu.close()
    assert t == tokens, (t, tokens)
    return np.array(tokens, dtype=np.int32), np.stack(logits)


def summary(logits: np.ndarray) -> dict:
    order = np.argsort(-logits, axis=1, kind="stable")[:, :64]
    srt = np.sort(logits, axis=1)
    return dict(top_idx=order.astype(np.int32), top_val=np.take_along_axis(logits, order, axis=1).astype(np.float32),
                stride16=logits[:, ::16].astype(np.float32), maxabs=np.abs(logits).max(axis=1).astype(np.float32),
                margin=(srt[:, -1] - srt[:, -2]).astype(np.float32))


def qwen2_7b(tmp: str) -> None:
    spec = sg.CONFIGS["qwen2.5-7b"]
    path = os.path.join(tmp, "q7b.gguf")
    sha = sg.write_qwen2(spec, path)
    prompt = sg.prompt_ids(spec.seed, 8, spec.vocab)
    toks, logits = run_reference_sequential(path, prompt, 2)
    np.savez_compressed(os.path.join(HERE, "qwen2_7b.npz"), sha256=np.array(sha), prompt=prompt, tokens=toks,
                        **summary(logits))


def qwen2_7b_long(tmp: str, prompt_len: int = 512, steps: int = 128) -> None:
    """The bench workload end to end: the same prompt bench.py prefills
    (prompt_ids(seed, 512)), then `steps` greedy decodes."""
    spec = sg.CONFIGS["qwen2.5-7b"]
    path = os.path.join(tmp, "q7b.gguf")
    sha = sg.write_qwen2(spec, path)
    prompt = sg.prompt_ids(spec.seed, prompt_len, spec.vocab)
    out = os.path.join(HERE, "qwen2_7b_long.npz")
    ref = oracle.ReferenceCPU(path)
    tok, lg = ref.prefill(prompt)
    tokens, logits = [tok], [lg]
    for _ in range(steps):
        tok, lg = ref.decode(tok)
        tokens.append(tok)
        logits.append(lg)
    ref.close()
    toks = np.array(tokens, dtype=np.int32)
    summ = summary(np.stack(logits))
    np.savez_compressed(out, sha256=np.array(sha), prompt=prompt, tokens=toks, cpullm_checked=np.array(0),
                        **summ)
    cpu = oracle.ReferenceCPULLM(path)
    t = [cpu.prefill(prompt)]
    for _ in range(steps):
        t.append(cpu.decode(t[-1]))
    cpu.close()
    assert t == tokens, (t, tokens)
    np.savez_compressed(out, sha256=np.array(sha), prompt=prompt, tokens=toks, cpullm_checked=np.array(1),
                        **summ)


def q4km_small(tmp: str) -> None:
    spec = sg.q4km_small_spec()
    path = os.path.join(tmp, "q4km_d128.gguf")
    sha = sg.write_qwen2(spec, path)
    out = {"sha256": np.array(sha)}
    for n in (8, 1100):
        prompt = sg.prompt_ids(spec.seed, n, spec.vocab)
        ref, toks, logits = run_reference(path, prompt, 4)
        ref.close()
        out[f"prompt{n}"] = prompt
        out[f"tokens{n}"] = toks
        out[f"logits{n}"] = logits.astype(np.float32)
        out[f"margin{n}"] = summary(logits)["margin"]
    np.savez_compressed(os.path.join(HERE, "q4km_d128.npz"), **out)


def tiny(seed: int, tmp: str) -> None:
    spec = sg.tiny_spec(seed=seed)
    path = os.path.join(tmp, f"tiny{seed}.gguf")
    sha = sg.write_qwen2(spec, path)
    out = {"sha256": np.array(sha), "seed": np.array(seed)}
    for n in (8, 40):
        prompt = sg.prompt_ids(spec.seed, n, spec.vocab)
        ref, toks, logits = run_reference(path, prompt, 4)
        out[f"prompt{n}"] = prompt
        out[f"tokens{n}"] = toks
        out[f"logits{n}"] = logits.astype(np.float32)
        ref.close()
    np.savez_compressed(os.path.join(HERE, f"tiny_s{seed}.npz"), **out)


def blocks(tmp: str) -> None:
    spec = sg.tiny_spec(seed=7)
    path = os.path.join(tmp, "tiny7.gguf")
    if not os.path.exists(path):
        sg.write_qwen2(spec, path)
    ref = oracle.ReferenceCPU(path)
    out = {}
    picks = {sg.Q4_K: (0, "attn_q"), sg.Q6_K: (0, "attn_v"), sg.Q5_0: (1, "attn_q"), sg.Q8_0: (1, "attn_v")}
    for gtype, (layer, name) in picks.items():
        vals = ref.tensor(layer, name)[:4]
        rows, cols = 4, vals.shape[1]
        full_rows = ref.tensor(layer, name).shape[0]
        key = sg.stream_key(spec.seed, f"blk.{layer}.{name}.weight")
        raw = sg.fill(gtype, full_rows, cols, key, 0.0, spec.weight_std)[:rows]
        out[f"raw_{sg.TYPE_NAMES[gtype]}"] = raw
        out[f"ref_{sg.TYPE_NAMES[gtype]}"] = vals
    ref.close()
    np.savez_compressed(os.path.join(HERE, "blocks.npz"), **out)


def qwen2_05b(tmp: str) -> None:
    spec = sg.CONFIGS["qwen2.5-0.5b"]
    path = os.path.join(tmp, "q05b.gguf")
    sha = sg.write_qwen2(spec, path)
    prompt = sg.prompt_ids(spec.seed, 16, spec.vocab)
    ref, toks, logits = run_reference(path, prompt, 4)
    ref.close()
    order = np.argsort(-logits, axis=1, kind="stable")[:, :64]
    top_vals = np.take_along_axis(logits, order, axis=1)
    srt = np.sort(logits, axis=1)
    np.savez_compressed(os.path.join(HERE, "qwen2_05b.npz"), sha256=np.array(sha), prompt=prompt, tokens=toks,
                        top_idx=order.astype(np.int32), top_val=top_vals.astype(np.float32),
                        stride16=logits[:, ::16].astype(np.float32),
                        maxabs=np.abs(logits).max(axis=1).astype(np.float32),
                        margin=(srt[:, -1] - srt[:, -2]).astype(np.float32))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-05b", action="store_true")
    ap.add_argument("--only-7b", action="store_true")
    ap.add_argument("--only-7b-long", action="store_true")
    ap.add_argument("--only-small", action="store_true")
    args = ap.parse_args()
    if not oracle.ref_available():
        oracle.build()
    if args.only_small:
        with tempfile.TemporaryDirectory() as tmp:
            q4km_small(tmp)
        return
    if args.only_7b_long:
        with tempfile.TemporaryDirectory(dir=os.environ.get("MYLLM_GOLDEN_TMP")) as tmp:
            qwen2_7b_long(tmp)
        return
    if args.only_7b:
        with tempfile.TemporaryDirectory(dir=os.environ.get("MYLLM_GOLDEN_TMP")) as tmp:
            qwen2_7b(tmp)
        return
    with tempfile.TemporaryDirectory() as tmp:
        for seed in (7, 11):
            tiny(seed, tmp)
        blocks(tmp)
        if not args.skip_05b:
            qwen2_05b(tmp)


if __name__ == "__main__":
    main()
