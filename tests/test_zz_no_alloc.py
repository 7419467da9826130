"""The no-allocation decode-attention entry point, called through the C-ABI.

cl_attn_decode_noalloc exists for callers that cannot allocate device memory
when they run decode attention (for example inside a stream capture that
refuses cudaMalloc, or under a fixed device-memory budget): its scratch is a
fixed array inside the library instead of a caller workspace.  This test
checks that it returns what the workspace entry point (cl_attn_decode)
returns, on two calls in a row with different inputs, that both agree with
a float64 restatement of the attention formula (score = q.k / sqrt(d),
softmax over the live keys, weighted sum of V; cpu_llm.cpp:888-903), and
that a request larger than the fixed array is refused with CL_ERR_LIMIT.  It is collected
last, and it works both alone in a fresh process (the first call performs
the per-device set-up) and after the other tests.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from myllm_b200 import _native

pytestmark = pytest.mark.gpu

CL_ERR_LIMIT = 5


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(seed, hq, hkv, d, cap):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(hq * d, generator=g).cuda()
    kc = torch.randn(cap, hkv * d, generator=g).cuda()
    vc = torch.randn(cap, hkv * d, generator=g).cuda()
    return q, kc, vc


def _attention_f64(q, kc, vc, hq, hkv, d, length):
    """float64 GQA decode attention over cache rows 0..length-1."""
    out = np.zeros(hq * d, dtype=np.float64)
    grp = hq // hkv
    for h in range(hq):
        g = h // grp
        kk = kc[:length, g * d:(g + 1) * d].astype(np.float64)
        s = kk @ q[h * d:(h + 1) * d].astype(np.float64) / math.sqrt(d)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * d:(h + 1) * d] = p @ vc[:length, g * d:(g + 1) * d].astype(np.float64)
    return out


def test_noalloc_attention_matches_workspace_entry_point(cuda):
    lib = _native.lib()
    hq, hkv, d, cap = 28, 4, 128, 4096
    scale = 1.0 / math.sqrt(d)
    wsb = int(lib.cl_attn_decode_workspace_bytes(hq, d, cap))
    assert 0 < wsb <= int(lib.cl_attn_decode_noalloc_limit_bytes())
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    for call, (seed, length) in enumerate([(1, 577), (2, 33)]):
        q, kc, vc = _inputs(seed, hq, hkv, d, cap)
        ln = torch.tensor([length], dtype=torch.int32, device="cuda")
        want = torch.empty(hq * d, device="cuda")
        got = torch.empty(hq * d, device="cuda")
        rc = lib.cl_attn_decode(_p(q), _p(kc), _p(vc), _p(ln), cap, hq, hkv, d, scale, _p(want), None, _p(ws), wsb,
                                _stream())
        assert rc == 0
        rc = lib.cl_attn_decode_noalloc(_p(q), _p(kc), _p(vc), _p(ln), cap, hq, hkv, d, scale, _p(got), _stream())
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        w, g = want.cpu().numpy(), got.cpu().numpy()
        # same kernels on the same inputs: within the attention tests' 1e-5
        assert np.abs(g - w).max() <= 1e-5 * np.abs(w).max(), f"call {call}"
        # and both against float64, at the attention tests' 1e-5
        ref = _attention_f64(q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy(), hq, hkv, d, length)
        assert np.abs(g - ref).max() <= 1e-5 * np.abs(ref).max(), f"call {call}"


def test_noalloc_attention_refuses_requests_beyond_the_fixed_scratch(cuda):
    lib = _native.lib()
    limit = int(lib.cl_attn_decode_noalloc_limit_bytes())
    # A long context uses the full split count, so the need grows with the
    # query heads: take the fewest heads (a multiple of the 8 KV heads) whose
    # need, as the library computes it, exceeds the fixed array.
    d, max_len = 256, 4096
    hq = 8
    while int(lib.cl_attn_decode_workspace_bytes(hq, d, max_len)) <= limit:
        hq += 8
    assert hq // 8 <= 16, "the refused request must be valid in every other respect"
    assert int(lib.cl_attn_decode_workspace_bytes(hq - 8, d, max_len)) <= limit
    dummy = torch.zeros(16, device="cuda")
    ln = torch.ones(1, dtype=torch.int32, device="cuda")
    rc = lib.cl_attn_decode_noalloc(_p(dummy), _p(dummy), _p(dummy), _p(ln), max_len, hq, 8, d, 1.0, _p(dummy),
                                    _stream())
    assert rc == CL_ERR_LIMIT
    assert lib.cl_status_string(rc) == b"request exceeds the fixed no-allocation scratch size"
