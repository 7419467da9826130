"""The peer all-reduce's bounded wait, made to run out on one GPU.

cl_peer_allreduce waits for every rank's flag with a wall-clock limit; a
rank that never arrives must not hang the others.  Here rank 0 of a
two-rank exchange runs alone: its second exchange buffer is an ordinary
local buffer that no kernel ever writes a flag into, so the wait for rank 1
runs out.  The test shortens the limit to 50 ms, checks that the kernel
returns, that the status word reads non-zero and that the sum was skipped,
then re-initialises the buffer and checks that the context still works.
No second process is involved and nothing faults: the wait ends by its own
limit.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from myllm_b200 import _native

pytestmark = pytest.mark.gpu

STATUS_OFFSET = 4 * (8 + 2 * 8)  # header: u32 epoch[8], u32 flag[2][8], u32 status


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_missing_rank_ends_the_wait_with_a_status(cuda):
    lib = _native.lib()
    n = 1024
    nbytes = int(lib.cl_peer_exchange_bytes(n))
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    for b in bufs:
        assert lib.cl_peer_exchange_init(_p(b), n, _stream()) == 0
    addr = (ctypes.c_void_p * 2)(bufs[0].data_ptr(), bufs[1].data_ptr())
    status_ptr = lib.cl_peer_exchange_status(_p(bufs[0]))
    assert status_ptr == bufs[0].data_ptr() + STATUS_OFFSET
    x = torch.randn(n, device="cuda")
    out = torch.full((n,), 7.0, device="cuda")
    try:
        assert lib.cl_peer_set_wait_limit_ns(50 * 10 ** 6) == 0
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        assert lib.cl_peer_allreduce(_p(x), _p(out), n, n, 0, 2, addr, _stream()) == 0  # rank 1 never calls
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        status = int(bufs[0][STATUS_OFFSET:STATUS_OFFSET + 4].view(torch.int32).item())
        assert status != 0, "the wait for the missing rank must report through the status word"
        assert elapsed < 5.0, elapsed
        assert bool((out == 7.0).all()), "a failed exchange must not write a partial sum"

        # the context is still usable: re-initialise and exchange with one rank
        assert lib.cl_peer_exchange_init(_p(bufs[0]), n, _stream()) == 0
        assert lib.cl_peer_allreduce(_p(x), _p(out), n, n, 0, 1, addr, _stream()) == 0
        torch.cuda.synchronize()
        assert int(bufs[0][STATUS_OFFSET:STATUS_OFFSET + 4].view(torch.int32).item()) == 0
        np.testing.assert_array_equal(out.cpu().numpy(), x.cpu().numpy())
    finally:
        lib.cl_peer_set_wait_limit_ns(20 * 10 ** 9)
