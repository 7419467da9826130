"""Tensor-core (tcgen05) prefill GEMM against the oracle's FP32 GEMM.

The reference's prefill GEMMs (gemmtb, cpu_llm.cpp:631-653; metal_gemm_*_f32,
metal_llm.metal:621-704) compute in FP32 from the exact dequantized weights.
CL_GEMM_TF32X3 must stay within the FP32 bar of the CUDA-core kernel
(max |err| <= 2e-5 max |ref|); CL_GEMM_F16 rounds both operands to FP16 once
and is held to 3e-3.
"""
import numpy as np
import pytest
import torch

import oracle
from myllm_b200 import _native
from myllm_b200 import kernels as K
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu

TOL = {"tf32x3": 2e-5, "f16": 3e-3}
ALL = [sg.Q4_K, sg.Q5_K, sg.Q6_K, sg.Q5_0, sg.Q8_0, sg.F32, sg.F16]


def weights(gtype, n, k, seed):
    return sg.fill(gtype, n, k, sg.stream_key(seed, f"tcw{gtype}_{n}_{k}"), 0.0, 0.02)


def xmat(m, k, seed, std=1.0):
    return sg.normal(m * k, sg.stream_key(seed, f"tcx{m}_{k}"), 0.0, std).reshape(m, k)


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def run(gtype, n, k, m, path, seed=7, bias=False, residual=False):
    w = weights(gtype, n, k, seed)
    x = xmat(m, k, seed + 1)
    b = sg.normal(n, sg.stream_key(seed + 2, "tcb"), 0.0, 0.1) if bias else None
    r = xmat(m, n, seed + 3) if residual else None
    ref = oracle.gemm(gtype, w, n, k, x, b)
    if r is not None:
        ref = ref + r
    wd = K.repack(gtype, w, k)
    got = K.gemm(gtype, wd, n, k, torch.from_numpy(x).cuda(), None if b is None else torch.from_numpy(b).cuda(),
                 None if r is None else torch.from_numpy(r).cuda(), path=path)
    return got.cpu().numpy(), ref


@pytest.mark.parametrize("path", ["tf32x3", "f16"])
@pytest.mark.parametrize("gtype", ALL)
def test_gemm_tc_formats(cuda, gtype, path):
    got, ref = run(gtype, 384, 512, 200, path)
    assert rel_err(got, ref) <= TOL[path]


@pytest.mark.parametrize("path", ["tf32x3", "f16"])
@pytest.mark.parametrize("m,n,k", [(1, 128, 256), (7, 200, 768), (128, 128, 1024), (300, 520, 256),
                                   (129, 4864, 896)])
def test_gemm_tc_ragged_shapes(cuda, path, m, n, k):
    gtype = sg.Q8_0 if k % 256 else sg.Q4_K
    got, ref = run(gtype, n, k, m, path, seed=11)
    assert rel_err(got, ref) <= TOL[path]


@pytest.mark.parametrize("gtype", [sg.Q6_K, sg.Q5_0])
def test_gemm_tc_bias_residual_in_place(cuda, gtype):
    n = k = 768 if gtype == sg.Q6_K else 640
    m = 150
    w = weights(gtype, n, k, 21)
    x = xmat(m, k, 22)
    b = sg.normal(n, sg.stream_key(23, "tcb"), 0.0, 0.1)
    r = xmat(m, n, 24)
    ref = oracle.gemm(gtype, w, n, k, x, b) + r
    y = torch.from_numpy(r.copy()).cuda()  # residual and output alias
    K.gemm(gtype, K.repack(gtype, w, k), n, k, torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda(), y,
           path="tf32x3", out=y)
    assert rel_err(y.cpu().numpy(), ref) <= TOL["tf32x3"]


def test_gemm_tc_qwen_7b_shapes(cuda):
    # q_proj and down_proj of the 7B config at a 256-token chunk
    for n, k, gtype in [(3584, 3584, sg.Q4_K), (3584, 18944, sg.Q6_K)]:
        got, ref = run(gtype, n, k, 256, "tf32x3", seed=31)
        assert rel_err(got, ref) <= TOL["tf32x3"], (n, k)


def test_gemm_auto_uses_tensor_path_and_falls_back(cuda):
    n, k, m = 256, 512, 64
    w = weights(sg.Q4_K, n, k, 41)
    wd = K.repack(sg.Q4_K, w, k)
    x = torch.from_numpy(xmat(m, k, 42)).cuda()
    auto = K.gemm(sg.Q4_K, wd, n, k, x, path="auto")
    tc = K.gemm(sg.Q4_K, wd, n, k, x, path="tf32x3")
    assert torch.equal(auto, tc)
    # K not a multiple of 32 (F32 weights): cl_gemm takes the CUDA-core kernel
    k2 = 40
    w2 = weights(sg.F32, n, k2, 43)
    x2 = xmat(m, k2, 44)
    got = K.gemm(sg.F32, K.repack(sg.F32, w2, k2), n, k2, torch.from_numpy(x2).cuda())
    assert rel_err(got.cpu().numpy(), oracle.gemm(sg.F32, w2, n, k2, x2)) <= 2e-5


def test_gemm_tc_rejects_unsupported(cuda):
    n, k, m = 128, 96, 8  # Q8_0 rows of 96: fine for TF32X3 (k % 32), not for F16 (k % 64)
    w = weights(sg.Q8_0, n, k, 51)
    wd = K.repack(sg.Q8_0, w, k)
    x = torch.from_numpy(xmat(m, k, 52)).cuda()
    with pytest.raises(_native.KernelError):
        K.gemm(sg.Q8_0, wd, n, k, x, path="f16")
    got = K.gemm(sg.Q8_0, wd, n, k, x, path="tf32x3")
    assert rel_err(got.cpu().numpy(), oracle.gemm(sg.Q8_0, w, n, k, xmat(m, k, 52))) <= 2e-5
    lib = _native.lib()
    y = torch.empty(m * n, device="cuda")
    assert lib.cl_gemm_tc(sg.Q8_0, K._p(wd), wd.stride(0), n, k, K._p(x), m, None, None, K._p(y), 7,
                          K._stream()) == 2
    torch.cuda.synchronize()


def test_gemm_tc_no_device_error(cuda):
    torch.cuda.synchronize()
    code = K.device_error()
    assert code == 0
