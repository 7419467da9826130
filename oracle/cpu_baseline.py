"""ORACLE — test infrastructure: times the reference's own CPULLM
(oracle/_ref/libref_cpu.so, compiled from the reference sources) on a bounded
sample of the benchmark workload: a short prefill and a few greedy decode
steps, each timed with a monotonic clock around the call as chat.cpp:852-871
does.  CPULLM is single-threaded, so one host core is used.

    python -m oracle.cpu_baseline --model M.gguf --prompt 4 --decode 2 [--warmup 1]
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--prompt", type=int, default=4)
    ap.add_argument("--decode", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=0)
    a = ap.parse_args()
    print(json.dumps(measure(a.model, a.prompt, a.decode, a.warmup)))


if __name__ == "__main__":
    main()
