"""Source check of the launch-order rule in csrc/kernels/common.cuh: data an
earlier kernel wrote is never read on the non-coherent load path.

Every kernel of this library is launched with programmatic dependent launch,
so it may start before the kernel that writes its inputs has finished; a line
of a buffer every layer reuses can then still sit in the SM's read-only cache.
The split tensor-core prefill attention read Q and the KV cache through
const __restrict__ pointers (which the compiler may read with ld.global.nc)
and produced a different wrong prefill each run on B200 until those reads
went through L2.  This test keeps activation, cache and index parameters of
every __global__ function free of __restrict__ and keeps __ldg / .nc loads
away from them; weights and tables keep both.
"""
import glob
import os
import re

KERNELS = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "myllm_b200", "csrc", "kernels")

# parameter names that carry data an earlier kernel (or a copy) wrote
ACTIVATIONS = {"x", "q", "kc", "vc", "k", "v", "len_dev", "part", "out", "g", "u", "o", "b", "token", "value",
               "rec", "ids", "index", "logits", "y", "wts", "shared_y", "shared_logit", "qkv", "alpha", "beta_raw",
               "act", "decay", "beta", "z", "state", "mixed", "k_raw", "v_raw", "pos_dev", "in", "xq", "amax",
               "hist", "res", "residual"}
# the DeltaNet A parameter of these kernels is a weight
WEIGHT_NAMED_A = {"gdn_prep_kernel", "gdn_prep_rows_kernel"}


def kernel_signatures():
    for f in sorted(glob.glob(os.path.join(KERNELS, "*.cu"))):
        text = open(f).read()
        for m in re.finditer(r"__global__[^{;]*?(\w+)\s*\(([^)]*)\)\s*\{", text, re.S):
            yield os.path.basename(f), m.group(1), m.group(2)


def test_kernels_were_found():
    names = {k for _, k, _ in kernel_signatures()}
    assert {"attn_prefill_tc_kernel", "attn_decode_split", "rope_kv_kernel", "gemv_pk_kernel"} <= names


def test_no_restrict_on_data_written_by_earlier_kernels():
    bad = []
    for f, kname, params in kernel_signatures():
        for pm in re.finditer(r"([\w:]+\s*\*\s*)__restrict__\s+(\w+)", params):
            kind, name = pm.group(1), pm.group(2)
            if "uint8_t" in kind:  # quantized weights
                continue
            if name in ACTIVATIONS or (name == "a" and kname not in WEIGHT_NAMED_A):
                bad.append(f"{f}:{kname}:{name}")
    assert not bad, bad


def test_explicit_noncoherent_loads_read_weights_only():
    """__ldg of a maximum or activation is what the 16-bit GEMM used to do
    for the activation maximum; only weight maxima and weight rows may."""
    bad = []
    for f in sorted(glob.glob(os.path.join(KERNELS, "*.cu"))):
        for ln, line in enumerate(open(f), 1):
            for m in re.finditer(r"__ldg\(([^;]*?)\)", line):
                arg = m.group(1)
                if re.search(r"\b(xmax|amax|x|x4|q|kc|vc|act|part)\b", arg) and "wmax" not in arg:
                    bad.append(f"{os.path.basename(f)}:{ln}: {line.strip()}")
    assert not bad, bad
