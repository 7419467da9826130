"""Tensor parallel (qwen2) on 2 GPUs of one box: the column/row splits with
one NCCL all-reduce after o_proj and down, and the vocab-split LM head with
the (value, index) merge, give the reference CPULLM's tokens and logits."""
import os

import numpy as np
import pytest
import torch  # noqa: F401  (the skipif condition below is evaluated in this namespace)

from myllm_b200 import synth_gguf as sg
from ranks import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.skipif("torch.cuda.device_count() < 2")]

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("n", [8, 40])
def test_tensor_parallel_two_gpus_matches_reference(model_dir, cuda, monkeypatch, n):
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", "tf32x3")  # FP32-grade prefill: the 1e-4 bar
    d = np.load(os.path.join(GOLDEN, "tiny_s7.npz"))
    path = os.path.join(model_dir, "tiny_s7.gguf")
    assert sg.write_qwen2(sg.tiny_spec(seed=7), path) == str(d["sha256"])
    got = run_ranks(2, path, d[f"prompt{n}"], 4)
    for r in (0, 1):
        toks, logits = got[r]
        assert toks == list(d[f"tokens{n}"]), r
        for i, ref in enumerate(d[f"logits{n}"]):
            assert rel(logits[i], ref) <= 1e-4, (r, i)


def test_tensor_parallel_peer_allreduce(model_dir, cuda, monkeypatch):
    """The decode all-reduces through cl_peer_allreduce (exchange buffers
    mapped by CUDA IPC, rank-order sum) instead of NCCL: the same tokens and
    logits as the reference, and bit-identical logits on both ranks."""
    monkeypatch.setenv("CUDALLM_ALLREDUCE", "p2p")  # inherited by the spawned ranks
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", "tf32x3")
    d = np.load(os.path.join(GOLDEN, "tiny_s7.npz"))
    path = os.path.join(model_dir, "tiny_s7.gguf")
    assert sg.write_qwen2(sg.tiny_spec(seed=7), path) == str(d["sha256"])
    got = run_ranks(2, path, d["prompt8"], 4)
    for r in (0, 1):
        toks, logits = got[r]
        assert toks == list(d["tokens8"]), r
        for i, ref in enumerate(d["logits8"]):
            assert rel(logits[i], ref) <= 1e-4, (r, i)
    assert np.array_equal(got[0][1], got[1][1])


def test_one_process_drives_two_devices(model_dir, cuda, monkeypatch):
    """One process, one model per device (a host thread per GPU is not
    needed: each CudaLLM makes its device current for its calls).  The
    kernels' shared-memory limits and SM counts are set up per device, so
    the model on the second device runs the same kernels as the first and
    both give the reference's tokens and logits; a GEMV that needs the raised
    shared-memory limit then still launches on device 0."""
    import torch
    from myllm_b200 import CudaLLM
    from myllm_b200 import kernels as K
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", "tf32x3")
    d = np.load(os.path.join(GOLDEN, "tiny_s7.npz"))
    path = os.path.join(model_dir, "tiny_s7.gguf")
    assert sg.write_qwen2(sg.tiny_spec(seed=7), path) == str(d["sha256"])
    llms = [CudaLLM(path, max_sequence=64, device=dev) for dev in (0, 1)]
    for llm in llms:
        toks = [llm.prefill(d["prompt8"])]
        logits = [llm.last_logits()]
        for _ in range(3):
            toks.append(llm.decode(toks[-1]))
            logits.append(llm.last_logits())
        assert toks == list(d["tokens8"])[:4]
        for i, lg in enumerate(logits):
            assert rel(lg, d["logits8"][i]) <= 1e-4, i
    for llm in llms:
        llm.close()
    torch.cuda.set_device(0)
    n, k = 3584, 18944  # the widest decode GEMV: its launch needs the raised shared-memory limit
    w = K.repack(sg.Q4_K, sg.fill(sg.Q4_K, n, k, sg.stream_key(3, "two_dev"), 0.0, 0.02), k)
    y = K.gemv(sg.Q4_K, w, n, k, torch.ones(k, device="cuda"))
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
