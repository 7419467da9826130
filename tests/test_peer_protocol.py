"""The exchange protocol of cl_peer_allreduce (csrc/kernels/peer.cu), model-
checked on the CPU.

The kernel's steps per block b of rank r, for one call: read the block's own
call counter e (after the previous call of rank r has finished: stream
order), store r's vector into rank b's slot [e % 2][r], release-store e into
rank b's flag [e % 2][r], wait until every flag [e % 2][s] of r's own buffer
has reached e, read the slots, store e as the block's counter.  Here every
rank's blocks run those steps in random interleavings; the checks are that no
slot is overwritten before its reader has read it, that every read sees
exactly that call's vector of that rank, and that no interleaving deadlocks.
"""
import random

import pytest


def run(world, calls, seed):
    rng = random.Random(seed)
    epoch = [[0] * world for _ in range(world)]                   # [rank][block]
    flag = [[[0] * world for _ in range(2)] for _ in range(world)]  # [rank][parity][src]
    slot = [[[None] * world for _ in range(2)] for _ in range(world)]
    unread = {}  # (owner, parity, src) -> blocks of the owner yet to read the slot
    call = [0] * world          # call in progress on each rank
    left = [world] * world      # blocks of that call not finished

    def block(r, b):
        e = epoch[r][b] + 1
        assert e == call[r] + 1
        p = e % 2
        yield
        # store r's vector into rank b's slot [p][r]: its previous content must be read
        assert not unread.get((b, p, r)), (r, b, e)
        slot[b][p][r] = (r, e)
        unread[(b, p, r)] = set(range(world))
        yield
        flag[b][p][r] = e
        yield
        while any(flag[r][p][s] < e for s in range(world)):
            yield "wait"
        for s in range(world):
            assert slot[r][p][s] == (s, e), (r, b, s, e, slot[r][p][s])
            unread[(r, p, s)].discard(b)
        yield
        epoch[r][b] = e

    running = {}
    for r in range(world):
        for b in range(world):
            running[(r, b)] = block(r, b)
    while running:
        keys = list(running)
        rng.shuffle(keys)
        progressed = False
        for key in keys:
            try:
                step = next(running[key])
            except StopIteration:
                del running[key]
                r, _ = key
                left[r] -= 1
                if left[r] == 0:
                    call[r] += 1
                    if call[r] < calls:  # stream order: the next call starts after this one ends
                        left[r] = world
                        for b in range(world):
                            running[(r, b)] = block(r, b)
                progressed = True
                break
            if step != "wait":
                progressed = True
                break
        assert progressed, "deadlock"
    assert call == [calls] * world


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_exchange_protocol_random_interleavings(world):
    for seed in range(40 if world < 8 else 8):
        run(world, 12, seed)
