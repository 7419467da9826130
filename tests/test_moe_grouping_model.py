"""The route bucketing of the grouped prefill expert GEMV (moe.cu:
route_group_kernel), model-checked on the CPU: the kernel's own scan layout
(thread t of 1024 owns local experts [4t, 4t + 4), a 32-lane inclusive scan
per warp, then the warp totals) and scatter must give, for any routes,
offsets that are the exclusive prefix sums of the per-expert counts and a
list holding each of this rank's routes exactly once, under its expert.

The GPU tests check the kernel at the config-4 widths; this walks the same
index rules at up to 4095 local experts, with empty and crowded buckets,
ids of other ranks and ids out of range (skipped).
"""
import random

THREADS, MAX_EXPERTS = 1024, 4096
PER = MAX_EXPERTS // THREADS


def group_routes(ids, n_local, rank, world):
    def mine(e):
        return e >= 0 and e % world == rank and e // world < n_local

    cnt = [0] * MAX_EXPERTS
    for e in ids:
        if mine(e):
            cnt[e // world] += 1
    own, run = [], []
    for t in range(THREADS):
        o, r = [], 0
        for i in range(PER):
            o.append(r)
            r += cnt[PER * t + i]
        own.append(o)
        run.append(r)
    incl = [0] * THREADS
    for w in range(THREADS // 32):  # __shfl_up_sync inclusive scan, lane by lane
        vals = run[32 * w:32 * w + 32]
        for o in (1, 2, 4, 8, 16):
            vals = [vals[l] + (vals[l - o] if l >= o else 0) for l in range(32)]
        incl[32 * w:32 * w + 32] = vals
    warp_tot = [incl[32 * w + 31] for w in range(THREADS // 32)]
    offsets = [0] * (n_local + 1)
    cursor = [0] * MAX_EXPERTS
    for t in range(THREADS):
        base = sum(warp_tot[:t // 32]) + incl[t] - run[t]
        for i in range(PER):
            e = PER * t + i
            cursor[e] = base + own[t][i]
            if e <= n_local:
                offsets[e] = base + own[t][i]
    lst = [None] * len(ids)
    for r, e in enumerate(ids):
        if mine(e):
            lst[cursor[e // world]] = r
            cursor[e // world] += 1
    return offsets, lst


def check(ids, n_local, rank, world):
    offsets, lst = group_routes(ids, n_local, rank, world)
    mine = [r for r, e in enumerate(ids) if e >= 0 and e % world == rank and e // world < n_local]
    assert offsets[0] == 0 and offsets[n_local] == len(mine)
    assert all(offsets[e] <= offsets[e + 1] for e in range(n_local))
    assert sorted(lst[:len(mine)]) == mine
    for le in range(n_local):
        bucket = lst[offsets[le]:offsets[le + 1]]
        assert len(bucket) == sum(1 for r in mine if ids[r] // world == le)
        assert all(ids[r] // world == le for r in bucket)


def test_config4_chunks():
    rng = random.Random(3)
    for tokens in (1, 64, 512):
        ids = [e for _ in range(tokens) for e in rng.sample(range(256), 8)]
        check(ids, 256, 0, 1)
        for world in (2, 4, 8):
            for rank in range(world):
                check(ids, len(range(rank, 256, world)), rank, world)


def test_largest_expert_table_and_crowded_buckets():
    rng = random.Random(5)
    check([rng.randrange(4095) for _ in range(3000)], 4095, 0, 1)
    check([7] * 500 + [4094] * 300 + [0] * 2, 4095, 0, 1)  # two crowded buckets at both ends
    check([1, 3, 5], 4095, 1, 2)


def test_ids_outside_the_table_are_skipped():
    check([-1, 300, 2, 9999, 2], 256, 0, 1)
    check([5, 6, 7], 2, 0, 1)  # every id beyond n_local: empty buckets, offsets all zero
