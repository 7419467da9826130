"""Build recipe for the native libraries, in-tree under ``myllm_b200/lib``.

* ``libcudallm.so``: the sm_100a kernels, the ``cl_*`` kernel C-ABI, the C++17
  host (GGUF reader, ``CudaLLM`` / ``CudaMoeLLM``) and the ``cudallm_*``
  backend C-ABI.  Built with nvcc for ``arch=compute_100a,code=sm_100a``.
* ``libsynth.so``: the seeded synthetic-weight generator used to write test
  and benchmark GGUF files.

Each library is rebuilt only when a source is newer than it.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "lib")
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def _nccl_dir():
    """The NCCL that PyTorch ships, so that one libnccl.so.2 serves both."""
    try:
        import nvidia.nccl  # type: ignore
        d = os.path.join(list(nvidia.nccl.__path__)[0], "lib")
        if os.path.exists(os.path.join(d, "libnccl.so.2")):
            return d
    except ImportError:
        pass
    return None
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _newer(target: str, sources) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd, cwd=None):
    res = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} (exit {res.returncode})")
    return res


def build_synth(force: bool = False) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    out = os.path.join(LIB_DIR, "libsynth.so")
    src = os.path.join(CSRC, "synth", "synth.c")
    if force or _newer(out, [src]):
        tmp = out + ".tmp"
        _run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-o", tmp, src, "-lm"])
        os.replace(tmp, out)
    return out


def cuda_sources():
    ks = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    hs = sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    hdr = sorted(glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True) +
                 glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True) +
                 glob.glob(os.path.join(INCLUDE, "*.h")))
    return ks, hs, hdr


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    """Compile every kernel and host source into libcudallm.so for sm_100a."""
    os.makedirs(LIB_DIR, exist_ok=True)
    out = os.path.join(LIB_DIR, "libcudallm.so")
    ks, hs, hdr = cuda_sources()
    if not (force or _newer(out, ks + hs + hdr)):
        return out
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    inc = ["-I", INCLUDE, "-I", os.path.join(CSRC, "kernels"), "-I", os.path.join(CSRC, "host")]
    objs = []
    procs = []
    for src in ks + hs:
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        if not force and not _newer(obj, [src] + hdr):
            continue
        if src.endswith(".cu"):
            cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                   *inc, "-c", src, "-o", obj]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
        else:
            cmd = [NVCC, "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler",
                   "-fvisibility=hidden", "-Xcompiler", "-Wall", *inc, "-c", src, "-o", obj]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                            stderr=subprocess.STDOUT, text=True)))
    failed = []
    for cmd, p in procs:
        text, _ = p.communicate()
        if p.returncode != 0 or (verbose and text):
            sys.stderr.write(" ".join(cmd) + "\n" + text)
        if p.returncode != 0:
            failed.append(cmd[-3])
    if failed:
        raise RuntimeError("CUDA build failed for: " + ", ".join(failed))
    tmp = out + ".tmp"
    nd = _nccl_dir()
    nccl = ["-L", nd, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + nd] if nd else ["-lnccl"]
    _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, *nccl, "-lpthread", "-ldl", "-lrt"])
    os.replace(tmp, out)
    return out


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_cuda(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("built", LIB_DIR)
