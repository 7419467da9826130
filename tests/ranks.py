"""Run one CudaLLM per GPU as spawned processes (multi-GPU tests).

Each rank builds its model with the shared NCCL id, runs prefill and
`steps` greedy decode steps, and reports its tokens and logits.
"""
import multiprocessing as mp

import numpy as np


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
        queue.put((rank, toks, np.stack(logits), None))
    except Exception as e:  # reported to the parent, which fails the test
        queue.put((rank, None, None, f"{type(e).__name__}: {e}"))


def run_ranks(world, path, prompt, steps, max_seq=64, timeout=300):
    """{rank: (tokens, logits [steps + 1, vocab])} for ranks 0..world-1."""
    from myllm_b200 import nccl_unique_id
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_rank_worker, args=(r, world, nid, path, [int(t) for t in prompt], steps, max_seq, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out, errors = {}, []
    try:
        for _ in range(world):
            r, t, l, err = q.get(timeout=timeout)
            if err:
                # the other ranks may be blocked in a collective with the
                # failed one: stop them now instead of waiting for a timeout
                errors.append(f"rank {r}: {err}")
                break
            out[r] = (t, l)
    finally:
        for p in procs:
            if errors:
                p.kill()
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert not errors, errors
    return out
