"""The 16-bit tensor-core prefill GEMM (cl_dequant16 + cl_gemm16_run).

Reference: metal_gemm_*_f32 / gemmtb (metal_llm.metal:621-704,
cpu_llm.cpp:591-653), an FP32 product of the dequantized weights.  The
oracle is the reference-exact dequantization (oracle.dequant) multiplied in
float64.  The operands are rounded once to FP16 (11-bit significands) or
BF16 (8-bit), so the bar is max|err| / max|ref| <= 2e-3 (FP16) and 1.5e-2
(BF16); the north-star tolerance for logits is 1e-2.  The split form
(GEMM_F16X3: FP16 hi + lo parts, three MMAs per step) is FP32-grade: 5e-5,
the bar of the split-TF32 path's tests.  The dequantization itself is
checked exactly: every element equals the FP32 reference value rounded once
to the 16-bit format (and, split, lo = the FP16 rounding of value - hi).
"""
import numpy as np
import pytest
import torch

import oracle
from myllm_b200 import kernels as K
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu

TOL = {K.GEMM_F16: 2e-3, K.GEMM_BF16: 1.5e-2, K.GEMM_F16X3: 5e-5}


def weights(gtype, n, k, seed):
    return sg.fill(gtype, n, k, sg.stream_key(seed, f"g16_{gtype}_{n}_{k}"), 0.0, 0.02)


def xmat(m, k, seed):
    return sg.normal(m * k, sg.stream_key(seed, f"g16x_{m}_{k}"), 0.0, 1.0).reshape(m, k)


def rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("fmt", [K.GEMM_F16, K.GEMM_BF16])
@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q6_K, sg.Q8_0, sg.Q5_0])
def test_dequant16_rounds_the_reference_values_once(cuda, gtype, fmt):
    n, k = 96, 1024
    w = weights(gtype, n, k, 1)
    ref = oracle.dequant(gtype, w, n, k)
    got = K.dequant16(gtype, K.repack(gtype, w, k), n, k, fmt).float().cpu().numpy()
    want = torch.from_numpy(ref).to(torch.bfloat16 if fmt == K.GEMM_BF16 else torch.float16).float().numpy()
    assert np.array_equal(got, want)


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q6_K, sg.Q8_0, sg.Q5_0])
def test_dequant16_split_form(cuda, gtype):
    """Rows [hi | lo] of the values times 2^e, e putting the largest
    magnitude in [2^13, 2^14): hi = FP16(v), lo = FP16(v - hi) (both
    exact steps in FP32); the maximum is the device's."""
    n, k = 96, 1024
    w = weights(gtype, n, k, 1)
    ref = oracle.dequant(gtype, w, n, k).astype(np.float32)

    def split(v, amax):
        e = 14 - np.frexp(np.float32(amax))[1]
        sv = torch.from_numpy((v * np.float32(2.0 ** e)).astype(np.float32))
        hi = sv.to(torch.float16)
        return hi, (sv - hi.float()).to(torch.float16), e

    got, amax = K.dequant16(gtype, K.repack(gtype, w, k), n, k, K.GEMM_F16X3)
    assert float(amax.item()) == float(np.abs(ref).max())
    hi, lo, e = split(ref, np.abs(ref).max())
    assert 2 ** 13 <= np.abs(ref).max() * 2.0 ** e < 2 ** 14
    got = got.cpu()
    assert torch.equal(got[:, :k], hi) and torch.equal(got[:, k:], lo)
    x = xmat(7, k, 9).astype(np.float32)
    xs, xm = K.convert16(torch.from_numpy(x).cuda(), K.GEMM_F16X3)
    assert float(xm.item()) == float(np.abs(x).max())
    xh, xl, _ = split(x, np.abs(x).max())
    xs = xs.cpu()
    assert torch.equal(xs[:, :k], xh) and torch.equal(xs[:, k:], xl)


@pytest.mark.parametrize("fmt", [K.GEMM_F16, K.GEMM_F16X3])
@pytest.mark.parametrize("gtype,n,k,m", [
    (sg.Q4_K, 18944, 3584, 512),   # 7B gate / up at the bench prompt
    (sg.Q6_K, 3584, 18944, 512),   # 7B down (Q6_K layers): K split
    (sg.Q4_K, 3584, 3584, 128),    # 7B q / o, one row tile
    (sg.Q4_K, 13824, 5120, 2048),  # 14B gate at config 1's largest M
    (sg.Q5_0, 4864, 896, 16),      # 0.5B gate at its 16-token prompt (partial row tile, N tail)
    (sg.Q8_0, 896, 4864, 200),     # 0.5B down (partial tiles both ways)
])
def test_gemm16_against_float64(cuda, gtype, n, k, m, fmt):
    w = weights(gtype, n, k, 2)
    x = xmat(m, k, 3)
    wd = oracle.dequant(gtype, w, n, k).astype(np.float64)
    ref = x.astype(np.float64) @ wd.T
    got = K.gemm16(gtype, K.repack(gtype, w, k), n, k, torch.from_numpy(x).cuda(), fmt=fmt).cpu().numpy()
    assert rel(got, ref) <= TOL[fmt], rel(got, ref)
    assert K.device_error() == 0


def test_gemm16_bf16(cuda):
    n, k, m = 4864, 3584, 256
    w = weights(sg.Q4_K, n, k, 4)
    x = xmat(m, k, 5)
    ref = x.astype(np.float64) @ oracle.dequant(sg.Q4_K, w, n, k).astype(np.float64).T
    got = K.gemm16(sg.Q4_K, K.repack(sg.Q4_K, w, k), n, k, torch.from_numpy(x).cuda(), fmt=K.GEMM_BF16).cpu().numpy()
    assert rel(got, ref) <= TOL[K.GEMM_BF16], rel(got, ref)


@pytest.mark.parametrize("fmt", [K.GEMM_F16, K.GEMM_F16X3])
def test_gemm16_split_and_unsplit_agree_with_bias_residual_segments(cuda, fmt):
    """Three column ranges (a fused Q/K/V product) with biases, a residual on
    the last, through the K-split path and unsplit."""
    n0, n1, n2, k, m = 3584, 512, 512, 3584, 300
    n = n0 + n1 + n2
    w = weights(sg.Q4_K, n, k, 6)
    x = xmat(m, k, 7)
    ref = x.astype(np.float64) @ oracle.dequant(sg.Q4_K, w, n, k).astype(np.float64).T
    g = torch.Generator().manual_seed(8)
    biases = [torch.randn(c, generator=g).cuda() for c in (n0, n1, n2)]
    res = torch.randn(m, n2, generator=g).cuda()
    w16 = K.dequant16(sg.Q4_K, K.repack(sg.Q4_K, w, k), n, k, fmt)
    x16 = K.convert16(torch.from_numpy(x).cuda(), fmt)
    for split in (True, False):
        ys = [torch.empty(m, c, device="cuda") for c in (n0, n1, n2)]
        K.gemm16_run(w16, x16, [(ys[0], biases[0], None, 0, n0), (ys[1], biases[1], None, n0, n1),
                                (ys[2], biases[2], res, n0 + n1, n2)], fmt=fmt, split=split)
        got = torch.cat(ys, dim=1).cpu().numpy().astype(np.float64)
        want = ref + torch.cat(biases).cpu().numpy()[None, :]
        want[:, n0 + n1:] += res.cpu().numpy()
        assert rel(got, want) <= TOL[fmt], (split, rel(got, want))
    assert K.device_error() == 0
