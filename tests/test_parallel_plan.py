"""Multi-GPU placement on the CPU: the shard plans the C++ loaders use
(cudallm_tp_plan / cudallm_ep_plan), checked for coverage at every world size
the configs allow, then driven through one decode step by world-size 2 and 4
`gloo` process groups.

The gloo ranks restate, in float64 NumPy, what each GPU rank computes with its
shard and which exchange follows (the reference runs on one device, so the
single-rank result is the target):
  * qwen2 tensor parallel: Q/K/V rows of the local heads, local GQA attention,
    the o_proj column share (after an all-gather of the attention output when
    the plan says gather_attn), gate/up rows and ffn_down columns of the FFN
    share, rank 0 adding the residual, an all-reduce (sum) after each
    row-split product, and the LM head's (value, index) records merged with
    the lowest index on ties (cpu_llm.cpp:34-48);
  * qwen35moe expert parallel: router softmax, top-k with the lower expert id
    on ties and renormalisation (metal_llm.metal:1424-1474), each rank's routed
    experts read from its stacked tensors at the planned local index, the
    shared expert on its planned rank, one all-reduce (sum).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from myllm_b200 import InvalidArgument, ep_plan, tp_plan
from myllm_b200 import synth_gguf as sg


def o_block_of(spec):
    return max(sg.BLOCK[spec.types(l, "attn_output")][0] for l in range(spec.layers))


def specs():
    return [sg.tiny_spec(seed=7)] + [sg.CONFIGS[n] for n in ("qwen2.5-0.5b", "qwen2.5-7b", "qwen2.5-14b")]


def partition(ranges, total):
    """Ranges in rank order tile [0, total) with no gap or overlap."""
    pos = 0
    for r in ranges:
        assert r.start == pos, (r, pos)
        pos = r.stop
    assert pos == total


@pytest.mark.parametrize("spec", specs(), ids=lambda s: s.name)
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_tp_plan_covers_every_row_and_column_once(spec, world):
    hq, hkv, d, F, V = spec.heads, spec.kv_heads, spec.hidden // spec.heads, spec.ffn, spec.vocab
    ob = o_block_of(spec)
    if hq % world or hkv % world:
        with pytest.raises(InvalidArgument):
            tp_plan(F, V, hq, hkv, d, ob, world, 0)
        return
    plans = [tp_plan(F, V, hq, hkv, d, ob, world, r) for r in range(world)]
    partition([p.q_heads for p in plans], hq)
    partition([p.kv_heads for p in plans], hkv)
    partition([p.ffn_rows for p in plans], F)
    partition([p.o_cols for p in plans], hq * d)
    partition([p.vocab_rows for p in plans], V)
    for p in plans:
        # each rank's query heads read only its own KV heads (GQA group hq / hkv)
        group = hq // hkv
        assert p.q_heads.start // group == p.kv_heads.start and len(p.q_heads) == group * len(p.kv_heads)
        if world > 1:
            assert p.ffn_rows.start % 256 == 0 and len(p.ffn_rows) % 256 == 0
        assert p.o_cols.start % ob == 0 and len(p.o_cols) % ob == 0
        if not p.gather_attn:
            assert p.o_cols == range(p.q_heads.start * d, p.q_heads.stop * d)
        assert abs(len(p.vocab_rows) - V / world) < 1
    # rank 0 adds the residual: it always has a share of every split
    assert len(plans[0].ffn_rows) and len(plans[0].o_cols) and len(plans[0].vocab_rows)
    assert len({p.gather_attn for p in plans}) == 1


def test_tp_plan_14b_eight_way_gathers_the_attention_output():
    s = sg.CONFIGS["qwen2.5-14b"]
    p = tp_plan(s.ffn, s.vocab, s.heads, s.kv_heads, 128, 256, 8, 0)
    # 5 heads x 128 columns are not on the 256-column grid of the Q4_K o_proj
    assert p.gather_attn and p.o_cols == range(0, 768)
    # Q5_0 o_proj (32-column blocks): the 0.5B shape's 7 heads x 64 columns split cleanly
    s = sg.CONFIGS["qwen2.5-0.5b"]
    p = tp_plan(s.ffn, s.vocab, s.heads, s.kv_heads, 64, 32, 2, 1)
    assert not p.gather_attn and p.o_cols == range(448, 896)


def test_tp_plan_rejects_bad_ranks_and_shapes():
    with pytest.raises(InvalidArgument):
        tp_plan(512, 1000, 4, 2, 64, 256, 2, 2)
    with pytest.raises(InvalidArgument):
        tp_plan(512, 1000, 4, 2, 64, 256, 0, 0)
    with pytest.raises(InvalidArgument):
        tp_plan(500, 1000, 4, 2, 64, 256, 2, 0)  # FFN not on the 256 grid
    with pytest.raises(InvalidArgument):
        tp_plan(512, 1000, 4, 2, 48, 256, 1, 0)  # o_proj width 192 off its block grid


@pytest.mark.parametrize("world", [1, 2, 3, 8, 300])
def test_ep_plan_places_every_expert_once(world):
    E, L = 256, 40
    er, el, sr = ep_plan(E, L, world)
    for r in range(world):
        mine = np.flatnonzero(er == r)
        # stacked in expert order: local indices 0, 1, 2, ...
        assert list(el[mine]) == list(range(len(mine)))
    assert ((er >= 0) & (er < world)).all() and ((sr >= 0) & (sr < world)).all()
    counts = np.bincount(er, minlength=world)
    assert counts.max() - counts.min() <= 1
    assert len(set(sr[:world])) == min(world, L)  # shared experts spread over ranks


# --------------------------------------------------------------- gloo ranks

def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_gloo(fn, world, *args):
    port = free_port()
    mp.spawn(_gloo_entry, args=(world, port, fn, args), nprocs=world, join=True)


def _gloo_entry(rank, world, port, fn, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


def rmsnorm(x, g, eps=1e-6):
    return x / np.sqrt((x * x).mean() + eps) * g


def silu(x):
    return x / (1.0 + np.exp(-x))


def qwen2_layer_model(hq, hkv, d, F, V, past, seed):
    rng = np.random.default_rng(seed)
    H = hq * d
    n = lambda *s: rng.standard_normal(s) * 0.2  # noqa: E731
    return dict(h=n(H) * 5, g1=1 + n(H), g2=1 + n(H), g3=1 + n(H), wq=n(hq * d, H), bq=n(hq * d),
                wk=n(hkv * d, H), bk=n(hkv * d), wv=n(hkv * d, H), bv=n(hkv * d), wo=n(H, H), wg=n(F, H),
                wu=n(F, H), wd=n(H, F), wout=n(V, H), kc=n(past, hkv * d) * 5, vc=n(past, hkv * d))


def attention(q, k, v, kc, vc, nq, nkv, d):
    """Decode attention of nq query heads over the cache plus the new row."""
    K = np.vstack([kc, k[None]]).reshape(-1, nkv, d)
    Vv = np.vstack([vc, v[None]]).reshape(-1, nkv, d)
    out = np.empty(nq * d)
    for h in range(nq):
        kh = h // (nq // nkv)
        s = K[:, kh] @ q[h * d:(h + 1) * d] / np.sqrt(d)
        p = np.exp(s - s.max())
        out[h * d:(h + 1) * d] = (p / p.sum()) @ Vv[:, kh]
    return out


def qwen2_step_full(m, hq, hkv, d):
    a = rmsnorm(m["h"], m["g1"])
    q, k, v = m["wq"] @ a + m["bq"], m["wk"] @ a + m["bk"], m["wv"] @ a + m["bv"]
    h = m["h"] + m["wo"] @ attention(q, k, v, m["kc"], m["vc"], hq, hkv, d)
    f = rmsnorm(h, m["g2"])
    h = h + m["wd"] @ (silu(m["wg"] @ f) * (m["wu"] @ f))
    return h, head(m["wout"], rmsnorm(h, m["g3"]))


def head(w, y):
    """Logits with one summation order per row, whatever slice of rows it is
    given: identical rows give bit-identical logits (planted ties stay ties)."""
    return (w * y).sum(axis=1)


def greedy(logits):
    return int(np.argmax(logits))  # numpy: first (lowest) index of the maximum


def _tp_rank(rank, world, hq, hkv, d, F, V, o_block, seed, tie):
    m = qwen2_layer_model(hq, hkv, d, F, V, 7, seed)
    h_ref, logits_ref = qwen2_step_full(m, hq, hkv, d)
    if tie:
        # the same largest logit at one row of the first and one of the last shard
        y = rmsnorm(h_ref, m["g3"])
        big = y / (y @ y) * (np.abs(logits_ref).max() + 10.0)
        m["wout"][[3, V - 2]] = big
        logits_ref = head(m["wout"], y)
    p = tp_plan(F, V, hq, hkv, d, o_block, world, rank)
    qs = slice(p.q_heads.start * d, p.q_heads.stop * d)
    ks = slice(p.kv_heads.start * d, p.kv_heads.stop * d)
    a = rmsnorm(m["h"], m["g1"])
    q = m["wq"][qs] @ a + m["bq"][qs]
    k = m["wk"][ks] @ a + m["bk"][ks]
    v = m["wv"][ks] @ a + m["bv"][ks]
    att = attention(q, k, v, m["kc"][:, ks], m["vc"][:, ks], len(p.q_heads), len(p.kv_heads), d)
    if p.gather_attn:
        parts = [torch.zeros(att.size, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(att))
        att_in = torch.cat(parts).numpy()[p.o_cols.start:p.o_cols.stop]
    else:
        att_in = att
    res = m["h"] if rank == 0 else 0.0
    part = torch.from_numpy(m["wo"][:, p.o_cols.start:p.o_cols.stop] @ att_in + res)
    dist.all_reduce(part)
    h = part.numpy()
    f = rmsnorm(h, m["g2"])
    fr = slice(p.ffn_rows.start, p.ffn_rows.stop)
    act = silu(m["wg"][fr] @ f) * (m["wu"][fr] @ f)
    part = torch.from_numpy(m["wd"][:, fr] @ act + (h if rank == 0 else 0.0))
    dist.all_reduce(part)
    h = part.numpy()
    np.testing.assert_allclose(h, h_ref, rtol=0, atol=1e-11 * np.abs(h_ref).max())
    # LM head: local (value, global index) record, all-gathered, merged
    local = head(m["wout"][p.vocab_rows.start:p.vocab_rows.stop], rmsnorm(h, m["g3"]))
    i = int(np.argmax(local))
    rec = torch.tensor([local[i], p.vocab_rows.start + i], dtype=torch.float64)
    recs = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(recs, rec)
    best = max(recs, key=lambda r: (r[0].item(), -r[1].item()))
    token = int(best[1].item())
    assert token == greedy(logits_ref)
    if tie:
        assert token == 3


@pytest.mark.parametrize("world,o_block,tie", [(2, 256, False), (2, 32, True), (4, 256, True), (4, 32, False)])
def test_tensor_parallel_step_on_gloo_ranks(world, o_block, tie):
    # 12 query / 4 KV heads of 64 (768 columns = 3 blocks of 256): 2-way and
    # 4-way head shares (384 / 192 columns) are off the 256 grid (gather; at
    # 4-way rank 3's o_proj share is empty) and on the 32 grid (local heads);
    # FFN 1280 = 5 blocks gives uneven shares; vocabulary 1001 is uneven
    run_gloo(_tp_rank, world, 12, 4, 64, 1280, 1001, o_block, 11, tie)


def moe_model(E, H, FF, SFF, seed):
    rng = np.random.default_rng(seed)
    n = lambda *s: rng.standard_normal(s) * 0.3  # noqa: E731
    return dict(x=n(H) * 3, router=n(E, H), gate=n(E, FF, H), up=n(E, FF, H), down=n(E, H, FF), wsh=n(H),
                sg=n(SFF, H), su=n(SFF, H), sd=n(H, SFF))


def route(logits, k):
    p = np.exp(logits - logits.max())
    p /= p.sum()
    ids = sorted(range(len(p)), key=lambda e: (-p[e], e))[:k]
    w = p[ids]
    return ids, w / w.sum()


def expert(m, e, x, gate, up, down):
    return down[e] @ (silu(gate[e] @ x) * (up[e] @ x))


def _ep_rank(rank, world, E, K, layer, seed):
    H, FF, SFF = 32, 16, 24
    m = moe_model(E, H, FF, SFF, seed)
    logits = m["router"] @ m["x"]
    logits[[1, E - 1]] = logits.max() + 1.0  # a tie at the top: expert 1 before E - 1
    ids, w = route(logits, K)
    assert ids[:2] == [1, E - 1]
    shared = 1.0 / (1.0 + np.exp(-(m["wsh"] @ m["x"]))) * (m["sd"] @ (silu(m["sg"] @ m["x"]) * (m["su"] @ m["x"])))
    ref = sum(wi * expert(m, e, m["x"], m["gate"], m["up"], m["down"]) for e, wi in zip(ids, w)) + shared
    er, el, sr = ep_plan(E, layer + 1, world)
    mine = np.flatnonzero(er == rank)
    # this rank's stacked expert tensors, indexed by the planned local index
    stack = {t: m[t][mine] for t in ("gate", "up", "down")}
    part = np.zeros(H)
    for e, wi in zip(ids, w):
        if er[e] == rank:
            part += wi * expert(stack, el[e], m["x"], stack["gate"], stack["up"], stack["down"])
    if sr[layer] == rank:
        part += shared
    t = torch.from_numpy(part)
    dist.all_reduce(t)
    np.testing.assert_allclose(t.numpy(), ref, rtol=0, atol=1e-12 * np.abs(ref).max())


@pytest.mark.parametrize("world,experts,layer", [(2, 16, 5), (4, 16, 2), (4, 3, 3)])
def test_expert_parallel_step_on_gloo_ranks(world, experts, layer):
    # (4, 3): more ranks than experts, rank 3 holds none
    run_gloo(_ep_rank, world, experts, min(4, experts), layer, 5)
