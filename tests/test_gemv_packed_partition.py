"""The work split of the packed decode GEMV (gemv_pk.cu), model-checked on the
CPU: for every launch shape, every output tile must be written exactly once,
from exactly its own units.

This restates the kernel's index rules (the CTA ranges, whole tiles or
stream-K; a CTA's shared first and last tile; the warps' intervals; the slot
rule of a split tile; the ticket count and the combiner's read order) and
walks them for random shapes and for the 7B / 14B decode shapes at 148 CTAs
of 12 warps.  The GPU tests check the arithmetic; this checks that no unit is
lost or counted twice at any shape the GPU tests do not reach.
"""
import random

KW = 12  # warps per CTA (gemv_pk.cu kW)


def range_begin(U, w, G):
    return U * w // G


def warp_of(U, u, G):
    return ((u + 1) * G - 1) // U


def simulate(U, nb, grid):
    tiles_total = U // nb
    whole = tiles_total >= grid
    G = min(grid, tiles_total if whole else U)
    writes, gpart, tickets, finishes = {}, {}, {}, []
    for c in range(G):
        if whole:
            cb, ce = tiles_total * c // G * nb, tiles_total * (c + 1) // G * nb
        else:
            cb, ce = range_begin(U, c, G), range_begin(U, c + 1, G)
        assert cb < ce
        tf, tl = cb // nb, (ce - 1) // nb
        f_shared = cb % nb != 0 or ce < tf * nb + nb
        l_shared = tl != tf and ce % nb != 0
        a0b, a0e = cb, (min(ce, tf * nb + nb) if f_shared else cb)
        a1b, a1e = (tl * nb if l_shared else ce), ce
        ob, oe = a0e, a1b
        n_a, n_b = (a0e - a0b) + (a1e - a1b), oe - ob
        red_a, red_b, spans = {}, {}, []
        for w in range(KW):
            i0, i1, la = n_a * w // KW, n_a * (w + 1) // KW, a0e - a0b
            sp = [(a0b + min(i0, la), a0b + min(i1, la)), (a1b + max(i0 - la, 0), a1b + max(i1 - la, 0)),
                  (ob + n_b * w // KW, ob + n_b * (w + 1) // KW)]
            spans.append(sp)
            wb, we = sp[2]
            for k, (b, e) in enumerate(sp):
                u = b
                while u < e:
                    t = u // nb
                    end = min(e, t * nb + nb)
                    units = set(range(u, end))
                    if k < 2:
                        assert (w, k) not in red_a
                        red_a[(w, k)] = (t, units)
                    elif t * nb >= wb and t * nb + nb <= we:
                        assert t not in writes
                        writes[t] = units
                    else:
                        slot = 1 if wb < t * nb else 0
                        assert (w, slot) not in red_b
                        red_b[(w, slot)] = (t, units)
                    u = end
        for which, t, shared in ((0, tf, f_shared), (1, tl, l_shared)):
            if shared:
                units = set()
                for w in range(KW):
                    if (w, which) in red_a:
                        tt, us = red_a[(w, which)]
                        assert tt == t
                        units |= us
                gpart[(c, which)] = (t, units)
                finishes.append(t)
        for w in range(KW):
            wb, we = spans[w][2]
            if wb >= we:
                continue
            for slot in (0, 1):
                if slot == 0:
                    if wb % nb != 0 or wb + nb <= we:
                        continue
                    ub = wb
                else:
                    ub = (we - 1) // nb * nb
                    if ub <= wb or ub + nb <= we:
                        continue
                t, units = red_b[(w, slot)]
                assert t == ub // nb
                units = set(units)
                for w2 in range(w + 1, KW):
                    b2, e2 = spans[w2][2]
                    if b2 >= ub + nb:
                        break
                    if b2 < e2:
                        tt, us = red_b[(w2, 0)]
                        assert tt == t
                        units |= us
                assert t not in writes
                writes[t] = units
    for t in finishes:  # the tickets: the last sharing CTA sums in CTA order
        ub = t * nb
        c0, c1 = warp_of(U, ub, G), warp_of(U, ub + nb - 1, G)
        tickets[t] = tickets.get(t, 0) + 1
        if tickets[t] == c1 - c0 + 1:
            tt, units = gpart[(c0, 1 if range_begin(U, c0, G) < ub else 0)]
            assert tt == t
            units = set(units)
            for c in range(c0 + 1, c1 + 1):
                tt, us = gpart[(c, 0)]
                assert tt == t
                units |= us
            assert t not in writes
            writes[t] = units
    for t in range(tiles_total):
        assert writes.get(t) == set(range(t * nb, t * nb + nb)), (U, nb, grid, t)


def test_decode_shapes_at_148_ctas():
    # (tiles, super-blocks per row): 7B / 14B q+k+v, o, gate/up pairs, down, LM head
    for tiles, nb in ((288, 14), (224, 14), (2368, 14), (224, 74), (9504, 14), (400, 20), (1728, 20),
                      (320, 54), (9504, 20), (32, 14), (1, 1)):
        simulate(tiles * nb, nb, 148)


def test_random_shapes_and_grids():
    rng = random.Random(7)
    for _ in range(600):
        nb = rng.choice([1, 2, 3, 14, 20, 54, 74])
        simulate(rng.randint(1, 300) * nb, nb, rng.choice([1, 2, 5, 37, 148]))
