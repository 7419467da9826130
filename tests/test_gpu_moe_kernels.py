"""qwen35moe kernels against FP64 restatements of the reference formulas
(the same helpers the FP64 oracle uses, oracle/moe_fp64.py).

Tolerances: FP32 device arithmetic vs FP64 math, max |err| / max |ref|.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from oracle.moe_fp64 import _rmsnorm, _sigmoid, _silu, _softplus
from myllm_b200 import kernels as K
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu


def rel_err(got, ref):
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


def rnd(n, seed, std=1.0, shape=None):
    v = sg.normal(int(np.prod(shape or (n,))), sg.stream_key(seed, f"moe{n}"), 0.0, std)
    return v.reshape(shape) if shape else v


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_gemv_f32(cuda):
    w = rnd(0, 1, 0.02, (300, 2048))
    x = rnd(2048, 2)
    got = K.gemv_f32(cu(w), cu(x)).cpu().numpy()
    assert rel_err(got, w.astype(np.float64) @ x) <= 1e-5


def route_ref(logits, k):
    e = np.exp(logits - logits.max())
    p = e / e.sum()
    order = sorted(range(len(p)), key=lambda i: (-p[i], i))[:k]
    return np.array(order), p[order] / p[order].sum()


@pytest.mark.parametrize("ne,k", [(256, 8), (16, 4), (60, 1)])
def test_moe_route(cuda, ne, k):
    # well-separated logits (no near-ties between FP32 and FP64), shuffled
    logits = np.linspace(-3.0, 3.0, ne)[np.argsort(rnd(ne, 3))]
    ids, wts = K.moe_route(cu(logits), k)
    rid, rw = route_ref(logits.astype(np.float64), k)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    assert rel_err(wts.cpu().numpy(), rw) <= 1e-6


def test_moe_route_ties_prefer_lower_ids(cuda):
    logits = np.zeros(64)
    logits[[5, 9, 40, 41]] = 1.0
    ids, wts = K.moe_route(cu(logits), 6)
    # four equal maxima in id order, then the lowest ids of the rest
    np.testing.assert_array_equal(ids.cpu().numpy(), [5, 9, 40, 41, 0, 1])
    assert abs(float(wts.sum()) - 1.0) < 1e-6


def experts(gtype, e, rows, cols, seed):
    return sg.fill(gtype, e * rows, cols, sg.stream_key(seed, f"exp{gtype}_{rows}_{cols}"), 0.0, 0.02)


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q6_K, sg.Q8_0])
@pytest.mark.parametrize("world,rank", [(1, 0), (2, 1), (4, 2)])
def test_moe_experts_end_to_end(cuda, gtype, world, rank):
    """gate/up SwiGLU product, per-route down product and the combine, with
    the experts of one rank resident (expert e on rank e % world)."""
    E, H, F = 16, 512, 256
    ids = np.array([3, 15, 0, 7, 10, 6], dtype=np.int32)
    wts = np.array([0.3, 0.2, 0.15, 0.15, 0.1, 0.1])
    gate, up = experts(gtype, E, F, H, 10), experts(gtype, E, F, H, 11)
    down = experts(gtype, E, H, F, 12)
    local = [e for e in range(E) if e % world == rank]
    pick = lambda m, rows: np.concatenate([m[e * rows:(e + 1) * rows] for e in local])
    gd, ud, dd = (K.repack(gtype, pick(m, r), c) for m, r, c in ((gate, F, H), (up, F, H), (down, H, F)))
    x = rnd(H, 13)
    idd, wd = torch.from_numpy(ids).cuda(), cu(wts)
    act = K.moe_expert_gemv(gtype, gd, F, H, cu(x), idd, w_up=ud, rank=rank, world=world)
    y = K.moe_expert_gemv(gtype, dd, H, F, act, idd, x_stride=F, rank=rank, world=world)
    shared_y, shared_logit, res = rnd(H, 14), np.array([0.7]), rnd(H, 15)
    out = K.moe_combine(y, idd, wd, cu(shared_y), cu(shared_logit), cu(res), rank=rank, world=world)
    G, U, D = (oracle.dequant(gtype, m, m.shape[0], c).astype(np.float64) for m, c in ((gate, H), (up, H), (down, F)))
    ref = np.zeros(H)
    for e, wt in zip(ids, wts):
        if e % world != rank:
            continue
        a = _silu(G[e * F:(e + 1) * F] @ x) * (U[e * F:(e + 1) * F] @ x)
        np.testing.assert_allclose(act[list(ids).index(e)].cpu().numpy(), a, rtol=0, atol=2e-5 * np.abs(a).max())
        ref += wt * (D[e * H:(e + 1) * H] @ a)
    ref = res + (ref + shared_y * _sigmoid(shared_logit[0]))
    assert rel_err(out.cpu().numpy(), ref) <= 2e-5


# small heads, then config 4's widths (16 key / 32 value heads, 128 x 128 state)
@pytest.mark.parametrize("G,R,D", [(2, 4, 64), (16, 32, 128)])
def test_gdn_prep_and_step(cuda, G, R, D):
    KC, eps = 4, 1e-6
    W = (2 * G + R) * D
    qkv, alpha, beta_raw = rnd(W, 20), rnd(R, 21), rnd(R, 22)
    conv_w = rnd(0, 23, 0.5, (W, KC))
    hist = rnd(0, 24, 1.0, (KC - 1, W))
    dt, a = rnd(R, 25, 0.1), -np.exp(rnd(R, 26, 0.5))
    z, gamma = rnd(R * D, 27), 1.0 + rnd(D, 28, 0.02)
    state = rnd(0, 29, 0.1, (R, D, D))
    hist_d, state_d = cu(hist), cu(state)
    act, decay, beta = K.gdn_prep(cu(qkv), cu(alpha), cu(beta_raw), cu(conv_w), hist_d, cu(dt), cu(a), G, R, D, eps)
    out = K.gdn_step(act, decay, beta, cu(z), cu(gamma), state_d, G, R, D, eps)
    # FP64 reference (the formulas of oracle/moe_fp64.py, one token)
    cat = np.concatenate([hist, qkv[None, :]], axis=0)
    conv = _silu(np.einsum("tc,ct->c", cat, conv_w))
    kw = G * D
    q, k, v = conv[:kw].reshape(G, D), conv[kw:2 * kw].reshape(G, D), conv[2 * kw:].reshape(R, D)
    q = q / np.sqrt((q * q).sum(1, keepdims=True) + eps)
    k = k / np.sqrt((k * k).sum(1, keepdims=True) + eps)
    ref_act = np.concatenate([q.reshape(-1), k.reshape(-1), v.reshape(-1)])
    assert rel_err(act.cpu().numpy(), ref_act) <= 1e-5
    dec = np.exp(_softplus(alpha + dt) * a)
    assert rel_err(decay.cpu().numpy(), dec) <= 1e-5
    assert rel_err(beta.cpu().numpy(), _sigmoid(beta_raw)) <= 1e-6
    np.testing.assert_allclose(hist_d.cpu().numpy(), cat[1:], rtol=0, atol=0)
    S = state.astype(np.float64).copy()
    ref = np.empty((R, D))
    for h in range(R):
        kh = h % G
        S[h] *= dec[h]
        delta = _sigmoid(beta_raw[h]) * (v[h] - S[h].T @ k[kh])
        S[h] += np.outer(k[kh], delta)
        ref[h] = _rmsnorm(S[h].T @ q[kh] / math.sqrt(D), gamma, eps)
    ref = ref.reshape(-1) * _silu(z)
    assert rel_err(out.cpu().numpy(), ref) <= 2e-5
    assert rel_err(state_d.cpu().numpy(), S) <= 2e-5


# small heads, then config 4's gated attention (16 / 2 heads of 256, RoPE on 64)
@pytest.mark.parametrize("hq,hkv,d,rot", [(4, 2, 64, 32), (16, 2, 256, 64)])
def test_attn_gate_prep(cuda, hq, hkv, d, rot):
    eps, pos, cap = 1e-6, 5, 8
    mixed, kr, vr = rnd(2 * hq * d, 30), rnd(hkv * d, 31), rnd(hkv * d, 32)
    qn, kn = 1.0 + rnd(d, 33, 0.02), 1.0 + rnd(d, 34, 0.02)
    theta = 1e7
    half = rot // 2
    ang = np.arange(cap)[:, None] * theta ** (-2.0 * np.arange(half)[None, :] / rot)
    table = np.stack([np.cos(ang), np.sin(ang)], axis=-1)  # [cap][half][2]
    kc = torch.zeros(cap, hkv * d, device="cuda")
    vc = torch.zeros_like(kc)
    q, gate = K.attn_gate_prep(cu(mixed), cu(kr), cu(vr), cu(qn), cu(kn), hq, hkv, d, rot, cu(table), pos, eps, kc, vc)

    def rope(x):
        c, s = table[pos, :, 0], table[pos, :, 1]
        y = x.copy()
        y[:half] = x[:half] * c - x[half:rot] * s
        y[half:rot] = x[:half] * s + x[half:rot] * c
        return y
    m = mixed.reshape(hq, 2, d)
    ref_q = np.concatenate([rope(_rmsnorm(m[h, 0], qn, eps)) for h in range(hq)])
    ref_k = np.concatenate([rope(_rmsnorm(kr.reshape(hkv, d)[g], kn, eps)) for g in range(hkv)])
    assert rel_err(q.cpu().numpy(), ref_q) <= 1e-5
    np.testing.assert_array_equal(gate.cpu().numpy(), m[:, 1, :].reshape(-1).astype(np.float32))
    assert rel_err(kc[pos].cpu().numpy(), ref_k) <= 1e-5
    np.testing.assert_array_equal(vc[pos].cpu().numpy(), vr.astype(np.float32))
    assert float(kc[pos - 1].abs().sum()) == 0.0


def test_mul_sigmoid(cuda):
    a, g = rnd(1000, 40), rnd(1000, 41, 10.0)
    got = K.mul_sigmoid(cu(a), cu(g)).cpu().numpy()
    assert rel_err(got, a * _sigmoid(g)) <= 1e-6
