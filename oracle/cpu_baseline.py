"""ORACLE — test infrastructure: times the reference's own CPULLM
(oracle/_ref/libref_cpu.so, compiled from the reference sources) on a bounded
sample of the benchmark workload: a short prefill and a few greedy decode
steps, each timed with a monotonic clock around the call as chat.cpp:852-871
does.  CPULLM is single-threaded, so one host core is used.

qwen35moe has no reference CPU path; with --moe the sample runs the
reference's own Metal kernels compiled for the host
(oracle/_ref/libref_metal.so) chained in its forward's layer order
(oracle.metal_ref.MoeReference), one token per step, on one host core.

    python -m oracle.cpu_baseline --model M.gguf --prompt 4 --decode 2 [--warmup 1] [--moe]
"""
from __future__ import annotations

import argparse
import json
import os
import time


def measure(path: str, prompt: int = 4, decode: int = 2, warmup: int = 0) -> dict:
    import oracle
    from myllm_b200 import synth_gguf as sg
    if not oracle.ref_available():
        return {"value": None, "unavailable": "oracle/_ref/libref_cpu.so was not built (no reference sources)"}
    cores = os.cpu_count()
    t0 = time.perf_counter()
    llm = oracle.ReferenceCPULLM(path, 0)
    load_s = time.perf_counter() - t0
    ids = sg.uniform_ids(prompt, 12345, 1000)
    t0 = time.perf_counter()
    tok = llm.prefill(ids)
    prefill_s = time.perf_counter() - t0
    for _ in range(warmup):
        tok = llm.decode(tok)
    t0 = time.perf_counter()
    for _ in range(decode):
        tok = llm.decode(tok)
    dec_s = time.perf_counter() - t0
    llm.close()
    return {"value": decode / dec_s, "unit": "tokens/s", "cores": 1, "host_cores": cores, "kind": "reference",
            "sample": f"reference CPULLM: prefill {prompt} tokens then {warmup}+{decode} greedy decode steps "
                      f"(timed: {decode}); load {load_s:.1f} s not timed",
            "prefill_tokens_per_s": prompt / prefill_s, "load_s": load_s}


def measure_moe(path: str, prompt: int = 2, decode: int = 2, warmup: int = 0) -> dict:
    import numpy as np
    from myllm_b200 import synth_gguf as sg
    from oracle import metal_ref
    if not metal_ref.available():
        return {"value": None, "unavailable": "oracle/_ref/libref_metal.so was not built (no reference sources)"}
    cores = os.cpu_count()
    t0 = time.perf_counter()
    ref = metal_ref.MoeReference(path, prompt + warmup + decode + 1)
    load_s = time.perf_counter() - t0
    ids = sg.uniform_ids(prompt, 12345, 1000)
    t0 = time.perf_counter()
    for t in ids:
        logits = ref.step(int(t))
    prefill_s = time.perf_counter() - t0
    for _ in range(warmup):
        logits = ref.step(int(np.argmax(logits)))
    t0 = time.perf_counter()
    for _ in range(decode):
        logits = ref.step(int(np.argmax(logits)))
    dec_s = time.perf_counter() - t0
    return {"value": decode / dec_s, "unit": "tokens/s", "cores": 1, "host_cores": cores, "kind": "reference",
            "sample": f"the reference's Metal kernels compiled for the host, chained in its forward's layer order "
                      f"(the reference has no CPU qwen35moe path): {prompt} prompt tokens one step each, then "
                      f"{warmup}+{decode} greedy steps (timed: {decode}); open {load_s:.1f} s not timed",
            "prefill_tokens_per_s": prompt / prefill_s, "load_s": load_s}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--prompt", type=int, default=4)
    ap.add_argument("--decode", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=0)
    ap.add_argument("--moe", action="store_true", help="qwen35moe: time the reference kernels on the host")
    a = ap.parse_args()
    run = measure_moe if a.moe else measure
    print(json.dumps(run(a.model, a.prompt, a.decode, a.warmup)))


if __name__ == "__main__":
    main()
