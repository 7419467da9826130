"""GPU parity of the individual kernels against the oracle (CPU restatement
of the reference arithmetic) or, for floating-point activation kernels, a
plain FP64/FP32 restatement of the reference formula.

Tolerances: GEMV/GEMM |y - y_ref| <= 2e-5 * max|y_ref| (the XQ activation
encoding is exact to max|x_block| * 2^-22; the rest is FP32 summation order);
activation kernels are compared at FP32 rounding level.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from myllm_b200 import kernels as K
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu

FORMATS = [sg.Q4_K, sg.Q5_K, sg.Q6_K, sg.Q5_0, sg.Q8_0]
# BASELINE config 1 sweep shapes (N x K); K-quants skip K = 896.
SWEEP = [(896, 896), (4864, 896), (896, 4864), (18944, 3584), (3584, 18944), (13824, 5120)]


def weights(gtype, n, k, seed=1):
    return sg.fill(gtype, n, k, sg.stream_key(seed, f"w{gtype}_{n}_{k}"), 0.0, 0.02)


def xvec(k, m=1, seed=2, std=1.0):
    return sg.normal(m * k, sg.stream_key(seed, f"x{k}_{m}"), 0.0, std).reshape(m, k)


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def applicable(gtype, k):
    return k % sg.BLOCK[gtype][0] == 0


@pytest.mark.parametrize("gtype", FORMATS)
@pytest.mark.parametrize("n,k", SWEEP)
def test_gemv_sweep(cuda, gtype, n, k):
    if not applicable(gtype, k):
        pytest.skip("K not a multiple of the block size")
    w = weights(gtype, n, k)
    x = xvec(k)
    ref = oracle.gemm(gtype, w, n, k, x)[0]
    wd = K.repack(gtype, w, k)
    got = K.gemv(gtype, wd, n, k, torch.from_numpy(x[0]).cuda()).cpu().numpy()
    assert rel_err(got, ref) <= 2e-5


@pytest.mark.parametrize("gtype", FORMATS)
def test_gemv_bias_residual_and_ragged_rows(cuda, gtype):
    n, k = 333, 512  # n not a multiple of any CTA row tile
    w = weights(gtype, n, k, seed=3)
    x = xvec(k, seed=4)
    bias = sg.normal(n, sg.stream_key(5, "b"), 0.0, 0.5)
    res = sg.normal(n, sg.stream_key(6, "r"), 0.0, 1.0)
    ref = oracle.gemm(gtype, w, n, k, x, bias)[0] + res
    wd = K.repack(gtype, w, k)
    got = K.gemv(gtype, wd, n, k, torch.from_numpy(x[0]).cuda(), torch.from_numpy(bias).cuda(),
                 torch.from_numpy(res).cuda())
    assert rel_err(got.cpu().numpy(), ref) <= 2e-5
    # in place: y aliases the residual
    r = torch.from_numpy(res).cuda()
    K.gemv(gtype, wd, n, k, torch.from_numpy(x[0]).cuda(), torch.from_numpy(bias).cuda(), r, out=r)
    assert rel_err(r.cpu().numpy(), ref) <= 2e-5


def test_gemv_multi_segments_mixed_formats(cuda):
    k = 512
    x = xvec(k, seed=8)
    segs, refs = [], []
    for i, (gtype, n) in enumerate([(sg.Q4_K, 300), (sg.Q6_K, 64), (sg.Q8_0, 70), (sg.Q5_0, 33)]):
        w = weights(gtype, n, k, seed=10 + i)
        b = sg.normal(n, sg.stream_key(20 + i, "b"), 0.0, 0.1)
        refs.append(oracle.gemm(gtype, w, n, k, x, b)[0])
        out = torch.empty(n, device="cuda")
        segs.append((gtype, K.repack(gtype, w, k), n, torch.from_numpy(b).cuda(), None, out))
    K.gemv_multi(segs, k, torch.from_numpy(x[0]).cuda())
    for s, ref in zip(segs, refs):
        assert rel_err(s[5].cpu().numpy(), ref) <= 2e-5


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q5_0])
def test_gemv_swiglu(cuda, gtype):
    n, k = 1000, 1024
    wg, wu = weights(gtype, n, k, seed=30), weights(gtype, n, k, seed=31)
    x = xvec(k, seed=32)
    g = oracle.gemm(gtype, wg, n, k, x)[0].astype(np.float64)
    u = oracle.gemm(gtype, wu, n, k, x)[0].astype(np.float64)
    ref = g / (1.0 + np.exp(-g)) * u
    got = K.gemv_swiglu(gtype, K.repack(gtype, wg, k), K.repack(gtype, wu, k), n, k,
                        torch.from_numpy(x[0]).cuda()).cpu().numpy()
    assert rel_err(got, ref) <= 5e-5


def rmsnorm_ref(x, g, eps):
    """cpu_llm.cpp:156-165 in numpy: double sum of squares, float mean/inv."""
    ss = (x.astype(np.float64) ** 2).sum(axis=-1)
    inv = (np.float32(1.0) / np.sqrt((ss / x.shape[-1]).astype(np.float32) + np.float32(eps))).astype(np.float32)
    return (x * (inv[..., None] * g)).astype(np.float32)


@pytest.mark.parametrize("k", [896, 3584, 18944])
def test_gemv_fused_rmsnorm(cuda, k):
    gtype = sg.Q8_0 if k == 896 else sg.Q4_K
    n = 700
    w = weights(gtype, n, k, seed=33)
    x = xvec(k, seed=34, std=3.0)
    g = sg.normal(k, sg.stream_key(35, "g"), 1.0, 0.02)
    ref = oracle.gemm(gtype, w, n, k, rmsnorm_ref(x, g, 1e-6))[0]
    out = torch.empty(n, device="cuda")
    K.gemv_multi([(gtype, K.repack(gtype, w, k), n, None, None, out)], k, torch.from_numpy(x[0]).cuda(),
                 torch.from_numpy(g).cuda(), 1e-6)
    assert rel_err(out.cpu().numpy(), ref) <= 2e-5
    gate = K.gemv_swiglu(gtype, K.repack(gtype, w, k), K.repack(gtype, w, k), n, k, torch.from_numpy(x[0]).cuda(),
                         torch.from_numpy(g).cuda(), 1e-6).cpu().numpy().astype(np.float64)
    r = ref.astype(np.float64)
    assert rel_err(gate, r / (1.0 + np.exp(-r)) * r) <= 5e-5


def test_gemv_rejects_unsupported_width(cuda):
    w = torch.zeros((4, K.row_stride(sg.Q4_K, 32768)), dtype=torch.uint8, device="cuda")
    from myllm_b200._native import KernelError
    with pytest.raises(KernelError):
        K.gemv(sg.Q4_K, w, 4, 32768, torch.zeros(32768, device="cuda"))


def test_no_device_error_recorded(cuda):
    assert K.device_error() == 0


def test_xq_encoding_precision(cuda):
    x = torch.from_numpy(xvec(4096, seed=40, std=3.0)[0]).cuda()
    x[:32] = 0.0  # an all-zero block
    xq = K.quantize_xq(x).cpu().numpy()
    k = 4096
    limbs = xq[: k // 16 * 48].view(np.int8).reshape(k // 16, 3, 16).astype(np.float64)
    off = ((k // 16 * 48) + ((k // 16 * 8 + 15) // 16 * 16))
    scale = xq[off: off + k // 32 * 4].view(np.float32).astype(np.float64)
    t = limbs[:, 0] * 16384 + limbs[:, 1] * 128 + limbs[:, 2]
    xr = (t.reshape(k // 32, 32) * scale[:, None]).reshape(-1)
    xa = x.cpu().numpy().astype(np.float64)
    bmax = np.abs(xa.reshape(-1, 32)).max(axis=1).repeat(32)
    assert np.all(np.abs(xr - xa) <= bmax * 2.0 ** -21 + 1e-30)
    assert np.all(xr[:32] == 0.0)


@pytest.mark.parametrize("gtype", FORMATS)
@pytest.mark.parametrize("m", [1, 7, 128])
def test_gemm_small(cuda, gtype, m):
    n, k = 384, 512
    w = weights(gtype, n, k, seed=50)
    x = xvec(k, m, seed=51)
    b = sg.normal(n, sg.stream_key(52, "b"), 0.0, 0.1)
    r = xvec(n, m, seed=53)
    ref = oracle.gemm(gtype, w, n, k, x, b) + r
    got = K.gemm(gtype, K.repack(gtype, w, k), n, k, torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda(),
                 torch.from_numpy(r).cuda())
    assert rel_err(got.cpu().numpy(), ref) <= 2e-5


def test_rmsnorm_matches_reference_formula(cuda):
    rows, k = 5, 3584
    x = xvec(k, rows, seed=60)
    g = sg.normal(k, sg.stream_key(61, "g"), 1.0, 0.02)
    eps = 1e-6
    # cpu_llm.cpp:156-165
    ss = (x.astype(np.float64) ** 2).sum(axis=1)
    inv = (np.float32(1.0) / np.sqrt((ss / k).astype(np.float32) + np.float32(eps))).astype(np.float32)
    ref = x * (inv[:, None] * g[None, :])
    y, xq = K.rmsnorm(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(), eps, want_xq=True)
    np.testing.assert_array_equal(y.cpu().numpy(), ref.astype(np.float32))


def rope_ref(vec, pos, theta, rot):
    v = vec.copy()
    half = rot // 2
    for p in range(half):
        f = np.float32(theta) ** np.float32(-2.0 * p / rot)
        a = np.float32(pos) * np.float32(f)
        c, s = np.float32(math.cos(a)), np.float32(math.sin(a))
        x0, x1 = v[p], v[p + half]
        v[p] = x0 * c - x1 * s
        v[p + half] = x0 * s + x1 * c
    return v


@pytest.mark.parametrize("d,rot", [(64, 64), (128, 128), (256, 64)])
def test_rope_kv_append(cuda, d, rot):
    rows, hq, hkv, cap, pos0, theta = 3, 4, 2, 16, 5, 1e6
    half = rot // 2
    table = np.zeros((cap, half, 2), dtype=np.float32)
    for pos in range(cap):
        for p in range(half):
            f = np.float32(theta) ** np.float32(-2.0 * p / rot)
            a = np.float32(pos) * f
            table[pos, p] = (np.cos(a), np.sin(a))
    q = xvec(hq * d, rows, seed=70)
    k = xvec(hkv * d, rows, seed=71)
    v = xvec(hkv * d, rows, seed=72)
    qt, kt, vt = (torch.from_numpy(a.copy()).cuda() for a in (q, k, v))
    kc = torch.zeros(cap, hkv * d, device="cuda")
    vc = torch.zeros(cap, hkv * d, device="cuda")
    K.rope_kv(qt, kt, vt, rows, hq, hkv, d, rot, torch.from_numpy(table).cuda(), pos0, kc, vc)
    for r in range(rows):
        for h in range(hq):
            want = rope_ref(q[r, h * d:(h + 1) * d], pos0 + r, theta, rot)
            np.testing.assert_allclose(qt[r, h * d:(h + 1) * d].cpu().numpy(), want, rtol=0, atol=2e-6)
        for h in range(hkv):
            want = rope_ref(k[r, h * d:(h + 1) * d], pos0 + r, theta, rot)
            np.testing.assert_allclose(kc[pos0 + r, h * d:(h + 1) * d].cpu().numpy(), want, rtol=0, atol=2e-6)
        np.testing.assert_array_equal(vc[pos0 + r].cpu().numpy(), v[r])


def attention_ref(q, kc, vc, hq, hkv, d, length):
    out = np.zeros(hq * d, dtype=np.float64)
    grp = hq // hkv
    for h in range(hq):
        g = h // grp
        kk = kc[:length, g * d:(g + 1) * d].astype(np.float64)
        s = kk @ q[h * d:(h + 1) * d].astype(np.float64) / math.sqrt(d)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * d:(h + 1) * d] = p @ vc[:length, g * d:(g + 1) * d]
    return out


@pytest.mark.parametrize("hq,hkv,d,length,cap", [(14, 2, 64, 17, 1024), (28, 4, 128, 600, 1024),
                                                 (16, 2, 256, 300, 1024), (5, 1, 128, 1, 1024),
                                                 (32, 2, 96, 77, 100), (28, 4, 128, 4096, 4096),
                                                 (40, 8, 128, 5, 4096), (16, 2, 256, 2500, 4096)])
def test_attention_decode(cuda, hq, hkv, d, length, cap):
    q = xvec(hq * d, seed=80)[0]
    kc = xvec(hkv * d, cap, seed=81)
    vc = xvec(hkv * d, cap, seed=82)
    ref = attention_ref(q, kc, vc, hq, hkv, d, length)
    got = K.attn_decode(torch.from_numpy(q).cuda(), torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda(),
                        length, cap, hq, hkv, d, 1.0 / math.sqrt(d))
    assert rel_err(got.cpu().numpy(), ref) <= 1e-5


def test_attention_decode_reuses_workspace(cuda):
    """One workspace across calls of different lengths (as in a captured
    decode graph replayed at growing positions)."""
    import ctypes
    from myllm_b200 import _native
    lib = _native.lib()
    hq, hkv, d, cap = 28, 4, 128, 2048
    q = xvec(hq * d, seed=85)[0]
    kc = xvec(hkv * d, cap, seed=86)
    vc = xvec(hkv * d, cap, seed=87)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
    wsb = int(lib.cl_attn_decode_workspace_bytes(hq, d, cap))
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    out = torch.empty(hq * d, device="cuda")
    for length in (2048, 3, 555, 1, 1200):
        ln = torch.tensor([length], dtype=torch.int32, device="cuda")
        rc = lib.cl_attn_decode(K._p(qd), K._p(kd), K._p(vd), K._p(ln), cap, hq, hkv, d,
                                ctypes.c_float(1.0 / math.sqrt(d)), K._p(out), None, K._p(ws), wsb, K._stream())
        assert rc == 0
        ref = attention_ref(q, kc, vc, hq, hkv, d, length)
        assert rel_err(out.cpu().numpy(), ref) <= 1e-5, length


@pytest.mark.parametrize("hq,hkv,d,pos0,rows", [(4, 2, 64, 0, 40), (28, 4, 128, 0, 70), (8, 8, 128, 33, 20)])
def test_attention_prefill(cuda, hq, hkv, d, pos0, rows):
    cap = pos0 + rows
    q = xvec(hq * d, rows, seed=90)
    kc = xvec(hkv * d, cap, seed=91)
    vc = xvec(hkv * d, cap, seed=92)
    got = K.attn_prefill(torch.from_numpy(q).cuda(), torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda(),
                         pos0, rows, hq, hkv, d).cpu().numpy()
    for r in range(rows):
        ref = attention_ref(q[r], kc, vc, hq, hkv, d, pos0 + r + 1)
        assert rel_err(got[r], ref) <= 1e-5, r


def causal_attention_ref(q, kc, vc, hq, hkv, d, pos0, rows):
    """float64 causal GQA attention of query rows at positions pos0.. against
    cache rows 0..pos0+rows-1 (cpu_llm.cpp:816-827), all rows at once."""
    out = np.zeros((rows, hq * d), dtype=np.float64)
    grp = hq // hkv
    n = pos0 + rows
    mask = np.arange(n)[None, :] > (pos0 + np.arange(rows))[:, None]
    for h in range(hq):
        g = h // grp
        qq = q[:, h * d:(h + 1) * d].astype(np.float64)
        kk = kc[:n, g * d:(g + 1) * d].astype(np.float64)
        s = qq @ kk.T / math.sqrt(d)
        s[mask] = -np.inf
        p = np.exp(s - s.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        out[:, h * d:(h + 1) * d] = p @ vc[:n, g * d:(g + 1) * d].astype(np.float64)
    return out


@pytest.mark.parametrize("tc", [False, True, "split"])
@pytest.mark.parametrize("hq,hkv,d,pos0,rows", [
    (28, 4, 128, 0, 512),    # BASELINE config 2 (7B shape): the bench's 512-token prompt
    (40, 8, 128, 0, 1024),   # BASELINE config 3 (14B shape): the 1024-token prompt
    (28, 4, 128, 512, 256),  # a later chunk of a chunked prefill
    (14, 2, 128, 37, 100),   # ragged: a chunk starting mid-tile, rows not a multiple of 64
    (28, 4, 128, 0, 8),      # a short prompt: fewer rows than one warp's 16
    (28, 4, 128, 0, 1),      # one row
    (28, 4, 128, 5, 3),      # a short chunk after earlier rows
])
def test_attention_prefill_long(cuda, hq, hkv, d, pos0, rows, tc):
    """Causal prefill attention at the prompt lengths the benchmarks prefill:
    the FP32 kernel and the split-FP16 tensor-core kernel at 1e-5, the FP16
    tensor-core kernel at 5e-3 (operands and probabilities rounded to 11-bit
    significands) of each row's scale."""
    cap = pos0 + rows
    q = xvec(hq * d, rows, seed=93)
    kc = xvec(hkv * d, cap, seed=94)
    vc = xvec(hkv * d, cap, seed=95)
    got = K.attn_prefill(torch.from_numpy(q).cuda(), torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda(),
                         pos0, rows, hq, hkv, d, tensor_cores=tc).cpu().numpy()
    ref = causal_attention_ref(q, kc, vc, hq, hkv, d, pos0, rows)
    err = np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert err.max() <= (5e-3 if tc is True else 1e-5), (int(err.argmax()), float(err.max()))


def test_argmax_lowest_index_on_ties(cuda):
    n = 152064
    x = torch.from_numpy(xvec(n, seed=100)[0]).cuda()
    ws = K.argmax_workspace(n)
    assert int(K.argmax(x, ws)) == int(torch.argmax(x))
    x[7] = 1e6
    x[100000] = 1e6
    x[150000] = 1e6
    assert int(K.argmax(x, ws)) == 7  # workspace re-armed by the previous call
    x.fill_(0.5)
    assert int(K.argmax(x, ws)) == 0


@pytest.mark.parametrize("gtype", FORMATS)
def test_embedding_rows_are_reference_values(cuda, gtype):
    vocab, k = 50, 512
    w = weights(gtype, vocab, k, seed=110)
    ref = oracle.dequant(gtype, w, vocab, k)
    ids = torch.tensor([3, 0, 49, 3, 60, -1], dtype=torch.int32, device="cuda")
    out, flag = K.embed(gtype, K.repack(gtype, w, k), vocab, k, ids)
    out = out.cpu().numpy()
    for i, t in enumerate([3, 0, 49, 3]):
        np.testing.assert_array_equal(out[i], ref[t])
    assert np.all(out[4:] == 0) and int(flag) == 1


@pytest.mark.parametrize("hq,hkv,d,rot,pos,cap", [(28, 4, 128, 128, 549, 4096), (28, 4, 128, 128, 0, 4096),
                                                  (14, 2, 64, 64, 63, 512), (8, 2, 64, 32, 200, 256),
                                                  (28, 4, 128, 128, 2047, 2048)])
def test_attention_decode_with_fused_rope_matches_separate_calls(cuda, hq, hkv, d, rot, pos, cap):
    """cl_attn_decode_rope = cl_rope_kv (one row) + cl_attn_decode, exactly:
    same outputs bit for bit and the same cache row written."""
    g = torch.Generator(device="cpu").manual_seed(pos + d)
    q = torch.randn(hq * d, generator=g).cuda()
    kn = torch.randn(hkv * d, generator=g).cuda()
    vn = torch.randn(hkv * d, generator=g).cuda()
    kc = torch.randn(cap, hkv * d, generator=g).cuda()
    vc = torch.randn(cap, hkv * d, generator=g).cuda()
    ang = torch.arange(cap, dtype=torch.float64)[:, None] * 1e6 ** (-2.0 * torch.arange(rot // 2, dtype=torch.float64) / rot)
    table = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).float().cuda()  # [cap][rot/2][2]
    scale = 1.0 / math.sqrt(d)
    # separate: RoPE + append, then attention
    q1, kc1, vc1 = q.clone(), kc.clone(), vc.clone()
    K.rope_kv(q1, kn, vn, 1, hq, hkv, d, rot, table, pos, kc1, vc1)
    want = K.attn_decode(q1, kc1, vc1, pos + 1, cap, hq, hkv, d, scale)
    # fused
    kc2, vc2 = kc.clone(), vc.clone()
    got = K.attn_decode_rope(q, kn, vn, table, pos, rot, kc2, vc2, cap, hq, hkv, d, scale)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)


def test_attention_decode_clamps_length_to_capacity(cuda):
    """A device-side length beyond the cache capacity is clamped to it (the
    kernel never reads outside the caches): same result as length = capacity."""
    hq, hkv, d, cap = 8, 2, 64, 96
    g = torch.Generator(device="cpu").manual_seed(5)
    q = torch.randn(hq * d, generator=g).cuda()
    kc = torch.randn(cap, hkv * d, generator=g).cuda()
    vc = torch.randn(cap, hkv * d, generator=g).cuda()
    scale = 1.0 / math.sqrt(d)
    want = K.attn_decode(q, kc, vc, cap, cap, hq, hkv, d, scale)
    got = K.attn_decode(q, kc, vc, cap + 100, cap, hq, hkv, d, scale)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
