"""Decode GEMV over fragment-packed K-quant weights (gemv_pk.cu:
cl_gemv_pack + cl_gemv_packed) against the oracle's FP32 GEMV over the exact
dequantized weights (gevmt, cpu_llm.cpp:512-547) and against the ring GEMV
(gemv_mma.cu) on the same inputs.

The products are the same exact integer dots of the XQ4 limbs as the ring
GEMV, so the tolerance is the GEMV tolerance of every other decode GEMV test:
|y - y_ref| <= 2e-5 * max|y_ref|.  Shapes cover the 7B and 14B decode
matrices, ragged row counts (zero-padded tiles), tiles shared by several
warps (the ticketed partial sums) and tiles owned by one warp.
"""
import numpy as np
import pytest
import torch

import oracle
from myllm_b200 import kernels as K
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu

TOL = 2e-5


def weights(gtype, n, k, seed):
    return sg.fill(gtype, n, k, sg.stream_key(seed, f"pk{gtype}_{n}_{k}"), 0.0, 0.02)


def vec(n, seed, std=1.0):
    return sg.normal(n, sg.stream_key(seed, f"pkv{n}"), 0.0, std)


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def rmsnorm_ref(x, g, eps):
    ss = (x.astype(np.float64) ** 2).sum()
    inv = np.float32(1.0) / np.sqrt(np.float32(ss / x.shape[-1]) + np.float32(eps))
    return (x * (inv * g)).astype(np.float32)


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q6_K])
@pytest.mark.parametrize("n,k", [(3584, 3584), (512, 3584), (1000, 512), (3584, 18944), (5120, 13824), (17, 256)])
def test_packed_gemv_matches_oracle(cuda, gtype, n, k):
    w = weights(gtype, n, k, 1)
    x = vec(k, 2)
    b = vec(n, 3, 0.1)
    r = vec(n, 4, 0.5)
    ref = oracle.gemm(gtype, w, n, k, x[None, :], b)[0] + r
    wd = K.repack(gtype, w, k)
    pk = K.gemv_pack(gtype, wd, n, k)
    y = torch.empty(n, device="cuda")
    K.gemv_packed([(gtype, pk, n, cu(b), cu(r), y)], k, cu(x))
    got = y.cpu().numpy()
    assert rel_err(got, ref) <= TOL
    # the ring GEMV on the same device-layout rows agrees as closely
    ring = K.gemv(gtype, wd, n, k, cu(x), cu(b), cu(r)).cpu().numpy()
    assert rel_err(got, ring) <= TOL


def test_mixed_segments_with_norm_one_launch(cuda):
    """q / k / v segments (Q4_K, Q4_K, Q6_K; biases) sharing an RMS-normalised
    x: one launch picks the format per unit."""
    k = 3584
    x = vec(k, 10, 2.0)
    g = 1.0 + vec(k, 11, 0.05)
    xn = rmsnorm_ref(x, g, 1e-6)
    segs, refs = [], []
    for i, (gtype, n) in enumerate([(sg.Q4_K, 3584), (sg.Q4_K, 512), (sg.Q6_K, 512)]):
        w = weights(gtype, n, k, 20 + i)
        b = vec(n, 30 + i, 0.1)
        refs.append(oracle.gemm(gtype, w, n, k, xn[None, :], b)[0])
        pk = K.gemv_pack(gtype, K.repack(gtype, w, k), n, k)
        segs.append((gtype, pk, n, cu(b), None, torch.empty(n, device="cuda")))
    K.gemv_packed(segs, k, cu(x), cu(g), 1e-6)
    for s, ref in zip(segs, refs):
        assert rel_err(s[5].cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("gtype,n,k", [(sg.Q4_K, 18944, 3584), (sg.Q6_K, 700, 3584), (sg.Q4_K, 13824, 5120)])
def test_packed_swiglu_with_norm(cuda, gtype, n, k):
    wg, wu = weights(gtype, n, k, 40), weights(gtype, n, k, 41)
    x, gm = vec(k, 42, 3.0), 1.0 + vec(k, 43, 0.02)
    xn = rmsnorm_ref(x, gm, 1e-6)[None, :]
    a = oracle.gemm(gtype, wg, n, k, xn)[0].astype(np.float64)
    b = oracle.gemm(gtype, wu, n, k, xn)[0].astype(np.float64)
    ref = a / (1.0 + np.exp(-a)) * b
    pk = K.gemv_pack(gtype, K.repack(gtype, wg, k), n, k, K.repack(gtype, wu, k))
    y = torch.empty(n, device="cuda")
    K.gemv_packed([(gtype, pk, n, None, None, y)], k, cu(x), cu(gm), 1e-6, swiglu=True)
    assert rel_err(y.cpu().numpy(), ref) <= 5e-5


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q6_K])
def test_activation_outliers(cuda, gtype):
    """A few channels 1000x larger than the rest share 256-column blocks with
    ordinary values (the fourth limb keeps the small ones FP32-grade)."""
    n, k = 512, 3584
    w = weights(gtype, n, k, 50)
    x = vec(k, 51)
    x[[7, 300, 2049]] *= 1000.0
    ref = oracle.gemm(gtype, w, n, k, x[None, :])[0]
    y = torch.empty(n, device="cuda")
    K.gemv_packed([(gtype, K.gemv_pack(gtype, K.repack(gtype, w, k), n, k), n, None, None, y)], k, cu(x))
    assert rel_err(y.cpu().numpy(), ref) <= TOL


def test_deterministic_and_workspace_rearmed(cuda):
    """Repeated launches on one workspace give bit-identical rows (the partial
    sums are added in warp order and the tickets re-arm themselves)."""
    n, k = 3584, 18944
    w = weights(sg.Q4_K, n, k, 60)
    pk = K.gemv_pack(sg.Q4_K, K.repack(sg.Q4_K, w, k), n, k)
    ws = K.gemv_packed_workspace((n + 15) // 16)
    x = cu(vec(k, 61))
    outs = []
    for _ in range(3):
        y = torch.empty(n, device="cuda")
        K.gemv_packed([(sg.Q4_K, pk, n, None, None, y)], k, x, ws=ws)
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
    ref = oracle.gemm(sg.Q4_K, w, n, k, x.cpu().numpy()[None, :])[0]
    assert rel_err(outs[0], ref) <= TOL

