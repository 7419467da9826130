"""B200-native CUDA backend for MyLLM-style GGUF inference.

``CudaLLM`` is the qwen2 backend with the reference backends' contract
(reset / prefill / decode -> greedy token).  Compute lives in the in-tree
``lib/libcudallm.so`` (sm_100a kernels + C++17 host); this package is the
Python mirror of that interface.
"""
from .llm import (BackendError, CudaLLM, InvalidArgument, LengthError, MemoryStats, ModelConfig, OutOfRange,
                  TensorParallelShard, ep_plan, nccl_unique_id, tp_plan)

__all__ = ["CudaLLM", "InvalidArgument", "OutOfRange", "LengthError", "BackendError", "MemoryStats",
           "ModelConfig", "nccl_unique_id", "TensorParallelShard", "tp_plan", "ep_plan"]
