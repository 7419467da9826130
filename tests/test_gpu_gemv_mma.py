"""Tensor-core decode GEMV (gemv_mma.cu: Q4_K / Q6_K on mma.sync) against the
oracle's FP32 GEMV over the exact dequantized weights (gevmt,
cpu_llm.cpp:512-547).

The kernel encodes x with one scale per 256 columns and four int8 limbs
(absolute error below max|x_block| * 2^-29), so the products are exact in
integers; tolerance |y - y_ref| <= 2e-5 * max|y_ref| as for every GEMV.
"""
import numpy as np
import pytest
import torch

import oracle
from myllm_b200 import _native
from myllm_b200 import kernels as K
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu

TOL = 2e-5


def weights(gtype, n, k, seed):
    return sg.fill(gtype, n, k, sg.stream_key(seed, f"mma{gtype}_{n}_{k}"), 0.0, 0.02)


def vec(n, seed, std=1.0):
    return sg.normal(n, sg.stream_key(seed, f"mmav{n}"), 0.0, std)


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def rmsnorm_ref(x, g, eps):
    ss = (x.astype(np.float64) ** 2).sum()
    inv = np.float32(1.0) / np.sqrt(np.float32(ss / x.shape[-1]) + np.float32(eps))
    return (x * (inv * g)).astype(np.float32)


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_interleaved_q4k_q6k_segments_one_launch(cuda):
    """q/k/v-like segments of both formats, ragged row counts, biases and a
    fused RMSNorm: one launch picks the format per 16-row tile."""
    k = 3584
    x = vec(k, 1, 2.0)
    g = 1.0 + vec(k, 2, 0.05)
    xn = rmsnorm_ref(x, g, 1e-6)
    segs, refs = [], []
    for i, (gtype, n) in enumerate([(sg.Q4_K, 300), (sg.Q6_K, 77), (sg.Q4_K, 16), (sg.Q6_K, 1)]):
        w = weights(gtype, n, k, 10 + i)
        b = vec(n, 20 + i, 0.1)
        refs.append(oracle.gemm(gtype, w, n, k, xn[None, :], b)[0])
        segs.append((gtype, K.repack(gtype, w, k), n, cu(b), None, torch.empty(n, device="cuda")))
    K.gemv_multi(segs, k, cu(x), cu(g), 1e-6)
    for s, ref in zip(segs, refs):
        assert rel_err(s[5].cpu().numpy(), ref) <= TOL


def test_q6k_swiglu_with_norm(cuda):
    n, k = 700, 3584
    wg, wu = weights(sg.Q6_K, n, k, 30), weights(sg.Q6_K, n, k, 31)
    x, gm = vec(k, 32, 3.0), 1.0 + vec(k, 33, 0.02)
    xn = rmsnorm_ref(x, gm, 1e-6)[None, :]
    a = oracle.gemm(sg.Q6_K, wg, n, k, xn)[0].astype(np.float64)
    b = oracle.gemm(sg.Q6_K, wu, n, k, xn)[0].astype(np.float64)
    ref = a / (1.0 + np.exp(-a)) * b
    got = K.gemv_swiglu(sg.Q6_K, K.repack(sg.Q6_K, wg, k), K.repack(sg.Q6_K, wu, k), n, k, cu(x), cu(gm), 1e-6)
    assert rel_err(got.cpu().numpy(), ref) <= 5e-5


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q6_K])
def test_activation_outliers(cuda, gtype):
    """A few channels 1000x larger than the rest (the outlier pattern of real
    LLM activations) share 256-column blocks with ordinary values."""
    n, k = 512, 3584
    w = weights(gtype, n, k, 40)
    x = vec(k, 41)
    x[[5, 300, 301, 2049]] = [1500.0, -900.0, 1200.0, -2000.0]
    ref = oracle.gemm(gtype, w, n, k, x[None, :])[0]
    got = K.gemv(gtype, K.repack(gtype, w, k), n, k, cu(x)).cpu().numpy()
    assert rel_err(got, ref) <= TOL
    # and the same blocks without their outliers (the scale shrinks back)
    x2 = x.copy()
    x2[[5, 300, 301, 2049]] = 0.0
    ref2 = oracle.gemm(gtype, w, n, k, x2[None, :])[0]
    got2 = K.gemv(gtype, K.repack(gtype, w, k), n, k, cu(x2)).cpu().numpy()
    assert rel_err(got2, ref2) <= TOL


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q6_K])
def test_single_row_and_widest_rows(cuda, gtype):
    # one row: a 16-row tile with 15 rows unused
    k = 1024
    w = weights(gtype, 1, k, 50)
    x = vec(k, 51)
    got = K.gemv(gtype, K.repack(gtype, w, k), 1, k, cu(x)).cpu().numpy()
    assert rel_err(got, oracle.gemm(gtype, w, 1, k, x[None, :])[0]) <= TOL
    # the widest rows the tensor-core path takes (96 blocks of 256: six per
    # consumer warp in the x encoding), split into several stages per tile
    k = 24576
    w = weights(gtype, 40, k, 52)
    x = vec(k, 53)
    got = K.gemv(gtype, K.repack(gtype, w, k), 40, k, cu(x)).cpu().numpy()
    assert rel_err(got, oracle.gemm(gtype, w, 40, k, x[None, :])[0]) <= TOL


def test_rows_wider_than_both_paths_are_rejected(cuda):
    k = 24832  # 97 blocks: beyond the tensor-core path; beyond the dp4a path's 23552
    w = torch.zeros((4, K.row_stride(sg.Q6_K, k)), dtype=torch.uint8, device="cuda")
    with pytest.raises(_native.KernelError):
        K.gemv(sg.Q6_K, w, 4, k, torch.zeros(k, device="cuda"))


def test_no_device_error(cuda):
    torch.cuda.synchronize()
    assert K.device_error() == 0
