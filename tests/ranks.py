"""Run one process per rank for the multi-rank tests, and stop them all as
soon as one fails.

`run_workers(target, world, args)` spawns `target(rank, world, *args, queue)`
for every rank; each worker puts `(rank, payload, None)` on success or
`(rank, None, message)` on failure.  When a rank fails, or exits without
reporting (a crash), the other ranks may be blocked in a collective with it:
they are killed at once instead of being left to a collective timeout, and
the failure is raised in the parent.

`run_ranks` is the multi-GPU use: one CudaLLM per GPU with the shared NCCL
id, prefill and `steps` greedy decode steps, tokens and logits per rank.
"""
import multiprocessing as mp
import queue as queue_mod
import time

import numpy as np


def run_workers(target, world, args, timeout=300):
    """{rank: payload} for ranks 0..world-1; raises AssertionError naming the
    first rank that failed, exited without a result, or ran out of time."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world) + tuple(args) + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    out, errors = {}, []
    silent = {}  # rank -> polls since it exited without a result
    deadline = time.monotonic() + timeout
    try:
        while len(out) < world and not errors:
            try:
                r, payload, err = q.get(timeout=1.0)
            except queue_mod.Empty:
                for r, p in enumerate(procs):
                    if r not in out and p.exitcode is not None:
                        # its result may still be in the pipe: allow one more poll
                        silent[r] = silent.get(r, 0) + 1
                        if silent[r] >= 2:
                            errors.append(f"rank {r}: exited with code {p.exitcode} without a result")
                            break
                if not errors and time.monotonic() > deadline:
                    errors.append(f"ranks {sorted(set(range(world)) - set(out))}: no result within {timeout} s")
                continue
            if err:
                errors.append(f"rank {r}: {err}")
                silent[r] = -1  # reported
            else:
                out[r] = payload
        if errors:
            # name the ranks that had already died: often the cause of the
            # error another rank reported (a broken connection)
            for r, p in enumerate(procs):
                if r not in out and silent.get(r, 0) >= 0 and p.exitcode not in (None, 0) and \
                        not any(e.startswith(f"rank {r}: exited") for e in errors):
                    errors.append(f"rank {r}: exited with code {p.exitcode} without a result")
    finally:
        for p in procs:
            if errors:
                p.kill()
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert not errors, errors
    return out


def _rank_worker(rank, world, nccl_id, path, prompt, steps, max_seq, queue):
    from myllm_b200 import CudaLLM
    try:
        llm = CudaLLM(path, max_sequence=max_seq, device=rank, rank=rank, world=world, nccl_id=nccl_id)
        toks = [llm.prefill(prompt)]
        logits = [llm.last_logits()]
        for _ in range(steps):
            toks.append(llm.decode(toks[-1]))
            logits.append(llm.last_logits())
        llm.close()
        queue.put((rank, (toks, np.stack(logits)), None))
    except Exception as e:  # reported to the parent, which fails the test
        queue.put((rank, None, f"{type(e).__name__}: {e}"))


def run_ranks(world, path, prompt, steps, max_seq=64, timeout=300):
    """{rank: (tokens, logits [steps + 1, vocab])} for ranks 0..world-1."""
    from myllm_b200 import nccl_unique_id
    return run_workers(_rank_worker, world, (nccl_unique_id(), path, [int(t) for t in prompt], steps, max_seq),
                       timeout)
