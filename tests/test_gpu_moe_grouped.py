"""Grouped prefill expert GEMV (moe.cu: cl_moe_group_routes +
cl_moe_expert_gemv_grouped) against the per-route prefill kernel
(cl_moe_expert_gemv_rows) on the same routes, and against float64 products
of the exact dequantized experts (the oracle's decoders, model.cpp:581-683).

The grouped kernel forms the same unit dots in the same order as the
per-route kernel, so the two agree to the last bit on the rows this rank
owns, and the test requires that.  Against float64 the
tolerance is the decode GEMV's, 2e-5 of the largest output.  Routes follow
the prefill layout: token t owns routes [t * top_k, (t + 1) * top_k) and its
top_k experts are distinct; one case sends every token to the same expert
(one expert with a route per token, walked in several chunks), one leaves
most experts without a route.
"""
import numpy as np
import pytest
import torch

import oracle
from oracle.moe_fp64 import _silu
from myllm_b200 import kernels as K
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def experts(gtype, e, rows, cols, seed):
    return sg.fill(gtype, e * rows, cols, sg.stream_key(seed, f"grp{gtype}_{e}_{rows}_{cols}"), 0.0, 0.02)


def route_ids(tokens, n_experts, top_k, seed, mode="random"):
    rng = np.random.default_rng(seed)
    ids = np.empty((tokens, top_k), np.int32)
    for t in range(tokens):
        if mode == "hot":  # expert 3 on every token, the rest random
            rest = rng.permutation([e for e in range(n_experts) if e != 3])[:top_k - 1]
            ids[t] = np.concatenate([[3], rest])
        elif mode == "few":  # only experts 0 .. 2 * top_k - 1
            ids[t] = rng.permutation(2 * top_k)[:top_k]
        else:
            ids[t] = rng.permutation(n_experts)[:top_k]
    return ids.reshape(-1)


def local_rows(native, rows, n_experts, rank, world):
    return np.concatenate([native[e * rows:(e + 1) * rows] for e in range(n_experts) if e % world == rank])


CASES = [
    # (gate/up type, down type, experts, hidden, expert ffn, tokens, top_k, world, rank, mode)
    (sg.Q4_K, sg.Q6_K, 256, 2048, 512, 64, 8, 1, 0, "random"),   # config 4's widths, a 64-token chunk
    (sg.Q4_K, sg.Q4_K, 256, 2048, 512, 40, 8, 2, 1, "hot"),
    (sg.Q4_K, sg.Q6_K, 64, 512, 256, 33, 8, 4, 2, "random"),
    (sg.Q5_K, sg.Q8_0, 32, 512, 256, 17, 4, 1, 0, "few"),
    (sg.Q8_0, sg.Q5_0, 16, 256, 128, 9, 2, 2, 0, "hot"),
]


@pytest.mark.parametrize("gt,dt,E,H,FF,T,KR,world,rank,mode", CASES)
def test_grouped_matches_per_route_and_float64(cuda, gt, dt, E, H, FF, T, KR, world, rank, mode):
    gate, up, down = experts(gt, E, FF, H, 1), experts(gt, E, FF, H, 2), experts(dt, E, H, FF, 3)
    gd = K.repack(gt, local_rows(gate, FF, E, rank, world), H)
    ud = K.repack(gt, local_rows(up, FF, E, rank, world), H)
    dd = K.repack(dt, local_rows(down, H, E, rank, world), FF)
    n_local = len(range(rank, E, world))
    ids_np = route_ids(T, E, KR, 4 + T, mode)
    ids = torch.from_numpy(ids_np).cuda()
    x = sg.normal(T * H, sg.stream_key(5, f"grpx{T}_{H}"), 0.0, 1.0).reshape(T, H)
    xd = cu(x)
    R = T * KR
    groups = K.moe_group_routes(ids, n_local, rank, world)
    off, lst = groups[0].cpu().numpy(), groups[1].cpu().numpy()
    mine = [r for r in range(R) if ids_np[r] % world == rank]
    # the buckets: every route of this rank once, under its local expert
    assert off[0] == 0 and off[-1] == len(mine) and np.all(np.diff(off) >= 0)
    assert sorted(lst[:len(mine)].tolist()) == mine
    for le in range(n_local):
        assert all(ids_np[r] // world == le for r in lst[off[le]:off[le + 1]])

    act_rows = K.moe_expert_gemv_rows(gt, gd, FF, H, xd, ids, H, KR, w_up=ud, rank=rank, world=world)
    act = K.moe_expert_gemv_grouped(gt, gd, FF, H, xd, ids, H, KR, n_local, w_up=ud, rank=rank, world=world,
                                    groups=groups)
    y_rows = K.moe_expert_gemv_rows(dt, dd, H, FF, act_rows, ids, FF, 1, rank=rank, world=world)
    y = K.moe_expert_gemv_grouped(dt, dd, H, FF, act, ids, FF, 1, n_local, rank=rank, world=world, groups=groups)
    a_g, a_r = act.cpu().numpy()[mine], act_rows.cpu().numpy()[mine]
    y_g, y_r = y.cpu().numpy()[mine], y_rows.cpu().numpy()[mine]
    assert np.array_equal(a_g, a_r) and np.array_equal(y_g, y_r)

    # float64 products of a few of this rank's routes (first, last, and the busiest expert's)
    busiest = int(np.argmax(np.diff(off)))
    sample = sorted({mine[0], mine[-1], *lst[off[busiest]:off[busiest + 1]][:3].tolist()})
    for r in sample:
        e = int(ids_np[r])
        G = oracle.dequant(gt, gate[e * FF:(e + 1) * FF], FF, H).astype(np.float64)
        U = oracle.dequant(gt, up[e * FF:(e + 1) * FF], FF, H).astype(np.float64)
        D = oracle.dequant(dt, down[e * H:(e + 1) * H], H, FF).astype(np.float64)
        xt = x[r // KR].astype(np.float64)
        a = _silu(G @ xt) * (U @ xt)
        assert rel_err(act.cpu().numpy()[r], a) <= 5e-5, r
        # the down product of the device's own activation row
        assert rel_err(y.cpu().numpy()[r], D @ act.cpu().numpy()[r].astype(np.float64)) <= 2e-5, r


def test_grouped_repeats_on_reused_scratch(cuda):
    """Two calls in a row on one planes buffer and one bucket set give the
    same rows (the scratch holds only the current call's encoding)."""
    E, H, FF, T, KR = 32, 512, 256, 24, 4
    gate = experts(sg.Q4_K, E, FF, H, 7)
    gd = K.repack(sg.Q4_K, gate, H)
    ids = torch.from_numpy(route_ids(T, E, KR, 8)).cuda()
    groups = K.moe_group_routes(ids, E)
    planes = torch.empty(K._native.lib().cl_moe_xq_planes_bytes(T, H), dtype=torch.uint8, device="cuda")
    xa = cu(sg.normal(T * H, sg.stream_key(9, "grpa"), 0.0, 1.0).reshape(T, H))
    xb = cu(sg.normal(T * H, sg.stream_key(9, "grpb"), 0.0, 3.0).reshape(T, H))
    ya = K.moe_expert_gemv_grouped(sg.Q4_K, gd, FF, H, xa, ids, H, KR, E, groups=groups, planes=planes)
    yb = K.moe_expert_gemv_grouped(sg.Q4_K, gd, FF, H, xb, ids, H, KR, E, groups=groups, planes=planes)
    ya2 = K.moe_expert_gemv_grouped(sg.Q4_K, gd, FF, H, xa, ids, H, KR, E, groups=groups, planes=planes)
    assert np.array_equal(ya.cpu().numpy(), ya2.cpu().numpy())
    rb = K.moe_expert_gemv_rows(sg.Q4_K, gd, FF, H, xb, ids, H, KR)
    assert np.array_equal(yb.cpu().numpy(), rb.cpu().numpy())
