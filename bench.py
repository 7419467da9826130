#!/usr/bin/env python
"""Benchmark of the CudaLLM hot path (BASELINE metric: batch-1 decode tok/s,
prefill tok/s, GEMV HBM GB/s against the measured HBM peak).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

Workload: N = 1 runs BASELINE config 2 (Qwen2.5-7B architecture, Q4_K_M
layout, 512-token prompt, greedy decode against a 4096-slot KV cache); N > 1
runs config 3 (Qwen2.5-14B architecture) tensor-parallel over the N ranks.
`--model qwen3.6-35b-a3b --prompt 64 --steps 64 --max-sequence 1024` runs
config 4 (qwen35moe), expert-parallel over the N ranks.
Weights are seeded synthetic values (no public checkpoint is involved).  A
step is one greedy decode token; `value` is decode tokens/s of the whole job
from device time (CUDA events, max over ranks); `e2e` is the same metric from
the public CudaLLM.decode() call, host to host.  The 4.4 GB (7B) weight set is
far larger than the 126 MB L2, so no flush is needed between steps.  The
N = 1 line also carries `scaling_base`: the N > 1 workload (14B) on one GPU,
the same-model denominator for the scaling series.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MODEL_DIR = os.environ.get("MYLLM_MODEL_DIR", "/tmp/myllm_b200_models")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--prompt", type=int, default=None,
                    help="prompt tokens (default: the BASELINE config's: 512 for the 7B shape, 1024 for the "
                         "14B shape, 64 for qwen3.6-35b-a3b)")
    ap.add_argument("--max-sequence", type=int, default=None,
                    help="KV capacity (default: 4096, or 1024 for qwen3.6-35b-a3b)")
    ap.add_argument("--model", default=None, help="synthetic config name (default by --gpus)")
    ap.add_argument("--kernel-iters", type=int, default=40)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config-1 kernel sweep (N = 1 only)")
    ap.add_argument("--no-scaling-base", action="store_true",
                    help="skip the single-GPU run of the N > 1 workload (N = 1 only)")
    ap.add_argument("--allreduce", choices=["nccl", "p2p"], default=None,
                    help="tensor-parallel decode all-reduce: NCCL (default) or the peer-memory kernel")
    ap.add_argument("--no-parity", action="store_true",
                    help="N > 1: skip the check of the sharded run's tokens and logits against one GPU")
    args = ap.parse_args()
    return args


# Prompt length and KV capacity of each BASELINE config (configs 2, 3, 4).
CONFIG_RUN = {"qwen2.5-7b": (512, 4096), "qwen2.5-14b": (1024, 4096), "qwen3.6-35b-a3b": (64, 1024)}


def model_name(args, world):
    if args.model:
        return args.model
    return "qwen2.5-7b" if world == 1 else "qwen2.5-14b"


def for_model(args, name):
    """A copy of args with prompt / max_sequence resolved for model `name`:
    the flags where given, else the BASELINE config's values."""
    import copy
    prompt, cap = CONFIG_RUN.get(name, (512, 4096))
    out = copy.copy(args)
    out.prompt = args.prompt if args.prompt is not None else prompt
    out.max_sequence = args.max_sequence if args.max_sequence is not None else cap
    return out


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None, "samples": len(sm),
                "reasons": sorted(reasons)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peaks():
    """(sustained, burst) dense bf16 TFLOP/s of one GPU and where they come
    from: the measured cuBLAS GEMM, else the earlier pool measurement."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops_sustained" in d and "bf16_tflops" in d:
            return float(d["bf16_tflops_sustained"]), float(d["bf16_tflops"]), "measured"
    return 1400.0, 1590.0, "fallback"


def prefill_flops(spec, tokens: int) -> int:
    """Useful FLOPs of a qwen2 prefill of `tokens` tokens from position 0
    (2 per multiply-add): every layer's q/k/v/o and gate/up/down products
    over all rows, causal attention (row i scores and mixes keys 0..i), and
    the LM head on the last row only (prefill returns the next token)."""
    H, F, T = spec.hidden, spec.ffn, tokens
    d = H // spec.heads
    kvd = spec.kv_heads * d
    per_row = 2 * (H * H + 2 * kvd * H + H * H + 2 * F * H + H * F)
    attn = 2 * 2 * spec.heads * d * (T * (T + 1) // 2)
    return spec.layers * (T * per_row + attn) + 2 * spec.vocab * H


def profile_traffic(kernel: str, shape=None, algorithmic=None):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summaries
    (profiles/traffic.json: the shape each was captured at, its DRAM bytes and
    algorithmic bytes).  At another shape of the same kernel the measured
    traffic / algorithmic ratio is applied to this launch's algorithmic bytes
    (the kernel streams each weight byte once, so traffic grows in
    proportion).  Returns (bytes or None, where the number comes from)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None, "no ncu capture committed"
    with open(p) as f:
        e = json.load(f).get(kernel)
    if not isinstance(e, dict):
        return None, f"no ncu capture of {kernel}"
    if shape is None or shape == e["shape"] or not algorithmic:
        return e["traffic"], f"measured at {e['shape']} ({e['source']})"
    ratio = e["traffic"] / e["algorithmic"]
    return ratio * algorithmic, f"scaled: {ratio:.3f} x the algorithmic bytes, as measured at {e['shape']}"


# ---------------------------------------------------------------------------
FUSED_PAIRS = {(12, 14), (6, 8)}  # GGML ids: (Q4_K, Q6_K), (Q5_0, Q8_0)


def gemv_launches(types) -> int:
    """Launches cl_gemv_multi makes for consecutive segments of these types:
    runs of one format, or of a fused pair of formats, share a launch."""
    n, i = 0, 0
    while i < len(types):
        j, other = i + 1, None
        while j < len(types):
            t = types[j]
            if t == types[i] or t == other:
                j += 1
            elif other is None and (min(t, types[i]), max(t, types[i])) in FUSED_PAIRS:
                other = t
                j += 1
            else:
                break
        n += 1
        i = j
    return n


def decode_bytes_per_token(spec, position: int) -> int:
    """Algorithmic HBM bytes of one decode token at `position`: every weight
    matrix once (native GGML bytes), one embedding row, the norms and biases,
    and the K/V rows 0..position of every layer."""
    from myllm_b200 import synth_gguf as sg
    total = 0
    H, F = spec.hidden, spec.ffn
    kvd = spec.kv_heads * (H // spec.heads)
    types = spec.types
    for l in range(spec.layers):
        total += H * sg.row_bytes(types(l, "attn_q"), H) + kvd * sg.row_bytes(types(l, "attn_k"), H)
        total += kvd * sg.row_bytes(types(l, "attn_v"), H) + H * sg.row_bytes(types(l, "attn_output"), H)
        total += F * sg.row_bytes(types(l, "ffn_gate"), H) + F * sg.row_bytes(types(l, "ffn_up"), H)
        total += H * sg.row_bytes(types(l, "ffn_down"), F)
        total += 4 * (2 * H + H + 2 * kvd)            # norms + biases
        total += 2 * (position + 1) * kvd * 4          # K and V rows read
    out_t = spec.output_type if spec.output_type is not None else spec.embed_type
    total += spec.vocab * sg.row_bytes(out_t, H) + sg.row_bytes(spec.embed_type, H) + 4 * H
    return total


def prefill_roofline(spec, tokens: int, prefill_ms: float, world: int, moe: bool):
    """The prefill as a tensor-bound job: useful TFLOP/s per GPU against the
    measured dense bf16 GEMM peak (sustained; the burst fraction beside it)."""
    if moe:
        return {"unavailable": "qwen35moe prefill: the routed experts and the DeltaNet scan are not GEMM-shaped "
                               "work; no tensor roofline is stated for them"}
    sus, burst, kind = measured_tensor_peaks()
    flops = prefill_flops(spec, tokens)
    ach = flops / world / (prefill_ms * 1e-3) / 1e12 if prefill_ms > 0 else 0.0
    return {"bound": "tensor", "achieved": ach, "peak": sus, "unit": "TFLOP/s", "frac": ach / sus,
            "burst_peak": burst, "burst_frac": ach / burst, "flops": flops,
            "peak_kind": f"{kind} bf16_tflops_sustained (cuBLAS bf16 GEMM, seconds-long loop), per GPU",
            "note": "useful FLOPs (2 per multiply-add: layer GEMMs, causal attention, last-row LM head); the "
                    "default FP32-grade path (split FP16) issues three tensor-core products per useful one"}


def moe_decode_bytes(spec, position: int):
    """Algorithmic HBM bytes of one qwen35moe decode token at `position`, as
    (replicated, expert): `replicated` is read by every expert-parallel rank
    (embedding row, attention / DeltaNet weights, the F32 router, norms, the
    LM head, the KV rows 0..position of the attention layers, each DeltaNet
    state and convolution history read and written once); `expert` is the
    top-k routed experts' gate/up/down rows plus the shared expert, spread
    over the ranks."""
    from myllm_b200 import synth_gguf as sg
    t = sg.moe_a3b_types
    H, E, FF, SFF = spec.hidden, spec.experts, spec.expert_ffn, spec.shared_ffn
    qw, kvw = spec.heads * spec.head_dim, spec.kv_heads * spec.head_dim
    rep = sg.row_bytes(sg.Q4_K, H) + spec.vocab * sg.row_bytes(sg.Q6_K, H) + 4 * H
    exp = 0
    for l in range(spec.layers):
        rep += 4 * 2 * H + E * H * 4                          # norms + F32 router
        if spec.is_attention(l):
            rep += 2 * qw * sg.row_bytes(t(l, "attn_q"), H) + kvw * sg.row_bytes(t(l, "attn_k"), H)
            rep += kvw * sg.row_bytes(t(l, "attn_v"), H) + H * sg.row_bytes(t(l, "attn_output"), qw)
            rep += 4 * 2 * spec.head_dim + 2 * (position + 1) * kvw * 4
        else:
            rep += spec.qkv_width * sg.row_bytes(t(l, "attn_qkv"), H)
            rep += spec.ssm_inner * sg.row_bytes(t(l, "attn_gate"), H)
            rep += 2 * spec.ssm_rank * H * 4 + spec.qkv_width * spec.conv_kernel * 4
            rep += 4 * (2 * spec.ssm_rank + spec.ssm_state)
            rep += H * sg.row_bytes(t(l, "ssm_out"), spec.ssm_inner)
            rep += 2 * 4 * spec.ssm_rank * spec.ssm_state * spec.ssm_state  # state read + write
            rep += 2 * 4 * (spec.conv_kernel - 1) * spec.qkv_width          # conv history
        exp += spec.experts_used * (FF * sg.row_bytes(t(l, "ffn_gate_exps"), H)
                                    + FF * sg.row_bytes(t(l, "ffn_up_exps"), H)
                                    + H * sg.row_bytes(t(l, "ffn_down_exps"), FF))
        exp += 4 * H + SFF * sg.row_bytes(t(l, "ffn_gate_shexp"), H) + SFF * sg.row_bytes(t(l, "ffn_up_shexp"), H)
        exp += H * sg.row_bytes(t(l, "ffn_down_shexp"), SFF)
    return rep, exp


def moe_launches_per_step(spec, world: int, rank: int) -> int:
    """Kernels one qwen35moe decode step launches on `rank` (NCCL's own
    kernels not counted): the graph recorded by CudaMoeLLM's decode."""
    from myllm_b200 import synth_gguf as sg
    t = sg.moe_a3b_types
    n = 1                                                       # embed
    for l in range(spec.layers):
        if spec.is_attention(l):
            # q/gate + k + v GEMV (input norm fused), gate prep, attention split + combine, gate, o_proj
            n += gemv_launches([t(l, "attn_q"), t(l, "attn_k"), t(l, "attn_v")]) + 1 + 2 + 1 + 1
        else:
            # attn_norm, qkv + z GEMV, alpha | beta, prep, recurrence step, out GEMV
            n += 1 + gemv_launches([t(l, "attn_qkv"), t(l, "attn_gate")]) + 1 + 1 + 1 + 1
        n += 1 + 1 + 1                                          # post norm, router | shared gate, top-k
        if any(e % world == rank for e in range(spec.experts)):
            n += 2                                              # routed gate/up, down
        if l % world == rank:
            n += 2                                              # shared gate/up, down
        n += 1 if world == 1 else 2                             # combine (+ residual add)
    return n + 3                                                # head GEMV, argmax, counter


def time_head_kernel(spec, iters: int):
    """Device time of the LM-head GEMV (RMSNorm fused; the largest single
    weight read of a qwen35moe token) timed alone with CUDA events on the
    launching stream; two weight copies alternate (2 x 417 MB > 126 MB L2)."""
    import torch
    from myllm_b200 import kernels as K
    from myllm_b200 import synth_gguf as sg
    H, V, gtype = spec.hidden, spec.vocab, sg.Q6_K
    w = K.repack(gtype, sg.fill(gtype, V, H, sg.stream_key(spec.seed, "bench_head"), 0.0, 0.02), H)
    ws = [w, w.clone()]
    x = torch.randn(H, device="cuda")
    gamma = torch.ones(H, device="cuda")
    y = torch.empty(V, device="cuda")
    for i in range(4):
        K.gemv_multi([(gtype, ws[i % 2], V, None, None, y)], H, x, gamma, 1e-6)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(iters):
        K.gemv_multi([(gtype, ws[i % 2], V, None, None, y)], H, x, gamma, 1e-6)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    algo = V * sg.row_bytes(gtype, H) + 2 * 4 * H + 4 * V
    del ws, w
    return {"kernel": "gemv_mma_kernel<Q6_K> (RMSNorm + LM-head GEMV on mma.sync)",
            "shape": f"[{V},{H}] Q6_K", "bytes_per_launch": algo, "avg_launch_us": ms * 1e3,
            "gbs": algo / (ms * 1e-3) / 1e9}


def time_gateup_kernel(spec, iters: int):
    """Device time of the dominant decode kernel (fused gate/up GEMV with
    SwiGLU over the FFN rows) on the model's shapes and formats, timed alone
    with CUDA events on the launching stream; 4 weight copies rotate so each
    launch streams from HBM (4 x 2 x 38 MB > 126 MB L2)."""
    import torch
    from myllm_b200 import kernels as K
    from myllm_b200 import synth_gguf as sg
    H, F = spec.hidden, spec.ffn
    gtype = spec.types(1, "ffn_gate")
    wn = sg.fill(gtype, F, H, sg.stream_key(spec.seed, "bench_gate"), 0.0, 0.02)
    base = K.repack(gtype, wn, H)
    copies = [(base.clone(), base.clone()) for _ in range(4)]
    x = torch.randn(H, device="cuda")
    gamma = torch.ones(H, device="cuda")
    for i in range(8):
        g, u = copies[i % 4]
        K.gemv_swiglu(gtype, g, u, F, H, x, gamma, 1e-6)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(iters):
        g, u = copies[i % 4]
        K.gemv_swiglu(gtype, g, u, F, H, x, gamma, 1e-6)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    algo = 2 * F * sg.row_bytes(gtype, H) + 2 * 4 * H + 4 * F  # weights + x, gamma + y
    del copies
    name = ("gemv_mma_kernel<Q4_K,swiglu> (RMSNorm + gate/up GEMV on mma.sync + SwiGLU)" if gtype == sg.Q4_K
            else "gemv_tma_kernel<swiglu> (RMSNorm + gate/up GEMV + SwiGLU)")
    return {"kernel": name, "shape": f"2x[{F},{H}] {sg.TYPE_NAMES[gtype]}",
            "bytes_per_launch": algo, "avg_launch_us": ms * 1e3, "gbs": algo / (ms * 1e-3) / 1e9}


# GEMV shapes (N x K) per format, GEMM at M in {128, 512, 2048}
SWEEP_SHAPES = [(896, 896), (4864, 896), (896, 4864), (18944, 3584), (3584, 18944), (13824, 5120)]


def graph_time_us(fn, iters: int) -> float:
    """Average device time of fn(i) over `iters` calls captured in one CUDA
    graph (replayed after a warm-up), so the host call cost is not timed."""
    import torch
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def kernel_sweep(peak_gbs: float, seed: int):
    """Config 1: decode GEMV GB/s over the sweep shapes and formats (weights
    rotate over copies whose total exceeds the 126 MB L2 where memory allows;
    `l2_resident` marks the small shapes whose copies fit in L2), and the
    prefill GEMM at M = 128 / 512 / 2048 on every one of those weights."""
    import math
    import torch
    from myllm_b200 import kernels as K
    from myllm_b200 import synth_gguf as sg
    gemv, gemm = [], []
    for gtype in (sg.Q4_K, sg.Q6_K, sg.Q5_0, sg.Q8_0):
        for n, k in SWEEP_SHAPES:
            if k % sg.BLOCK[gtype][0]:
                continue  # K-quants need K % 256 == 0 (n/a at K = 896)
            w = K.repack(gtype, sg.fill(gtype, n, k, sg.stream_key(seed, f"sweep{gtype}_{n}_{k}"), 0.0, 0.02), k)
            nbytes = n * sg.row_bytes(gtype, k) + 4 * k + 4 * n
            copies = max(2, min(64, math.ceil(300e6 / nbytes)))
            ws = [w] + [w.clone() for _ in range(copies - 1)]
            x = torch.randn(k, device="cuda")
            y = torch.empty(n, device="cuda")
            us = graph_time_us(lambda i: K.gemv(gtype, ws[i % copies], n, k, x, out=y), 40)
            entry = {"type": sg.TYPE_NAMES[gtype], "n": n, "k": k, "us": round(us, 2),
                     "gbs": round(nbytes / us / 1e3, 1), "frac": round(nbytes / us / 1e3 / peak_gbs, 3),
                     "l2_resident": copies * nbytes < 126e6}
            if gtype in (sg.Q4_K, sg.Q6_K):
                # the same product on the fragment-packed GEMV (cl_gemv_packed)
                pks = [K.gemv_pack(gtype, wi, n, k) for wi in ws]
                pws = K.gemv_packed_workspace((n + 15) // 16)
                us = graph_time_us(lambda i: K.gemv_packed([(gtype, pks[i % copies], n, None, None, y)], k, x, ws=pws),
                                   40)
                entry.update(packed_us=round(us, 2), packed_gbs=round(nbytes / us / 1e3, 1))
                del pks
            gemv.append(entry)
            del ws
            # prefill GEMM on the same weights at the config's batch sizes
            for m in (128, 512, 2048):
                entry = {"type": sg.TYPE_NAMES[gtype], "n": n, "k": k, "m": m}
                try:
                    xm = torch.randn(m, k, device="cuda")
                    out = torch.empty(m * n, device="cuda")
                    us = graph_time_us(lambda i: K.gemm(gtype, w, n, k, xm, out=out), 5)
                    entry.update(us=round(us, 1), tflops=round(2 * m * n * k / us / 1e6, 1))
                    del xm, out
                except Exception as e:  # recorded; the other entries stand
                    entry["error"] = f"{type(e).__name__}: {e}"
                gemm.append(entry)
            del w
    # the 7B LM head (the largest decode matrix), where the decode graph uses the packed GEMV
    head = None
    try:
        V, H = 152064, 3584
        wn = sg.fill(sg.Q6_K, V, H, sg.stream_key(seed, "sweep_head"), 0.0, 0.02)
        w = K.repack(sg.Q6_K, wn, H)
        pk = K.gemv_pack(sg.Q6_K, w, V, H)
        ws2, pk2 = [w, w.clone()], [pk, pk.clone()]
        x = torch.randn(H, device="cuda")
        gm = torch.ones(H, device="cuda")
        y = torch.empty(V, device="cuda")
        pws = K.gemv_packed_workspace((V + 15) // 16)
        nbytes = V * sg.row_bytes(sg.Q6_K, H) + 8 * H + 4 * V
        ring = graph_time_us(lambda i: K.gemv_multi([(sg.Q6_K, ws2[i % 2], V, None, None, y)], H, x, gm, 1e-6), 20)
        pkd = graph_time_us(lambda i: K.gemv_packed([(sg.Q6_K, pk2[i % 2], V, None, None, y)], H, x, gm, 1e-6,
                                                    ws=pws), 20)
        head = {"shape": f"[{V},{H}] Q6_K + RMSNorm", "ring_us": round(ring, 2),
                "ring_gbs": round(nbytes / ring / 1e3, 1), "packed_us": round(pkd, 2),
                "packed_gbs": round(nbytes / pkd / 1e3, 1)}
        del ws2, pk2, w, pk
    except Exception as e:
        head = {"error": f"{type(e).__name__}: {e}"}
    return {"gemv": gemv, "gemm": gemm, "lm_head_7b": head,
            "note": "GEMV frac of the measured HBM copy peak (packed_*: the fragment-packed GEMV on the same "
                    "weights); GEMM (cl_gemm, the path prefill uses: split-TF32 "
                    "tcgen05 where the shape allows, else FP32 CUDA cores) TFLOP/s of useful work (2 M N K); "
                    "split-TF32 issues three tensor-core products per useful one"}


def reference_host_bytes(spec) -> int:
    """Host memory the reference CPULLM holds for a qwen2 model: every tensor
    dequantized to FP32 plus the file image it reads whole (model.cpp:392)."""
    from myllm_b200 import synth_gguf as sg
    tensors = sg.qwen2_tensors(spec)
    return sum(4 * t.rows * t.cols + t.nbytes for t in tensors)


def mem_available():
    """MemAvailable of this host in bytes, or None where /proc/meminfo is absent."""
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return None


def moe_kernel_times(peak_gbs: float, seed: int):
    """Config 4's decode kernels timed alone at its widths (hidden 2048, 256
    experts top-8 of FFN 512, DeltaNet 16 / 32 heads with a 128 x 128 state,
    gated attention 16 / 2 heads of 256 over 512 keys), each captured in a
    CUDA graph and replayed; inputs rotate over copies larger than L2 (all 256
    experts through 32 disjoint route sets, 96 DeltaNet states, 64 KV caches),
    as the weights of a whole token would evict them.  GB/s of algorithmic
    bytes; every kernel is guarded on its own."""
    import ctypes
    import torch
    from myllm_b200 import _native
    from myllm_b200 import kernels as K
    from myllm_b200 import synth_gguf as sg
    lib = _native.lib()
    p = K._p
    st = K._stream
    spec = sg.MOE_CONFIGS["qwen3.6-35b-a3b"]
    H, E, Kr, FF = spec.hidden, spec.experts, spec.experts_used, spec.expert_ffn
    G, R, D, KC = spec.ssm_groups, spec.ssm_rank, spec.ssm_state, spec.conv_kernel
    hq, hkv, d, rot, L, cap = spec.heads, spec.kv_heads, spec.head_dim, spec.rot_dim, 512, 1024
    out = {}

    def timed(name, fn, iters, nbytes):
        try:
            us = graph_time_us(fn, iters)
            out[name] = {"us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1),
                         "frac": round(nbytes / us / 1e3 / peak_gbs, 3), "bytes": int(nbytes)}
        except Exception as e:  # recorded; the other kernels stand
            out[name] = {"error": f"{type(e).__name__}: {e}"}

    # router: F32 [256, 2048] product, then softmax / top-8 / renormalise
    rw = [torch.randn(E, H, device="cuda") / H ** 0.5 for _ in range(64)]
    xn = torch.randn(H, device="cuda")
    logits = torch.empty(E, device="cuda")
    ids = torch.empty(Kr, dtype=torch.int32, device="cuda")
    wts = torch.empty(Kr, device="cuda")
    timed("router_gemv_f32", lambda i: K.check(lib.cl_gemv_f32(p(rw[i % 64]), E, H, p(xn), p(logits), st()), "gemv_f32"),
          40, E * H * 4 + 4 * H + 4 * E)
    timed("route_topk", lambda i: K.check(lib.cl_moe_route(p(logits), E, Kr, p(ids), p(wts), st()), "route"),
          40, 4 * E + 8 * Kr)
    # routed experts: gate/up with SwiGLU, then down, Q4_K as in the recipe
    try:
        q4 = sg.Q4_K
        gate = K.repack(q4, sg.fill(q4, E * FF, H, sg.stream_key(seed, "mk_gate"), 0.0, 0.02), H)
        up = K.repack(q4, sg.fill(q4, E * FF, H, sg.stream_key(seed, "mk_up"), 0.0, 0.02), H)
        down = K.repack(q4, sg.fill(q4, E * H, FF, sg.stream_key(seed, "mk_down"), 0.0, 0.02), FF)
        sets = [torch.arange(j, E, E // Kr, dtype=torch.int32, device="cuda")[:Kr] for j in range(E // Kr)]
        act = torch.empty(Kr, FF, device="cuda")
        ey = torch.empty(Kr, H, device="cuda")
        gu_bytes = Kr * 2 * FF * sg.row_bytes(q4, H) + 4 * H + 4 * Kr * FF
        dn_bytes = Kr * H * sg.row_bytes(q4, FF) + 4 * Kr * FF + 4 * Kr * H
        timed("expert_gate_up_swiglu", lambda i: K.check(lib.cl_moe_expert_gemv(
            q4, p(gate), p(up), gate.stride(0), FF, H, p(xn), 0, p(sets[i % len(sets)]), Kr, 0, 1, p(act), st()),
            "experts"), 32, gu_bytes)
        timed("expert_down", lambda i: K.check(lib.cl_moe_expert_gemv(
            q4, p(down), None, down.stride(0), H, FF, p(act), FF, p(sets[i % len(sets)]), Kr, 0, 1, p(ey), st()),
            "experts"), 32, dn_bytes)
        # prefill: one layer's routed experts (gate/up + SwiGLU, down) for a
        # chunk of T tokens, per route (cl_moe_expert_gemv_rows) and grouped by
        # expert (cl_moe_group_routes + cl_moe_expert_gemv_grouped); the two
        # forms' rows compared bit for bit
        pre = {}
        for T in (64, 512):
            rng = torch.Generator().manual_seed(seed + T)
            pids = torch.stack([torch.randperm(E, generator=rng)[:Kr] for _ in range(T)]).reshape(-1).to(
                dtype=torch.int32, device=xn.device)
            px = torch.randn(T, H, device="cuda")
            rt = T * Kr
            a_r, y_r = torch.empty(rt, FF, device="cuda"), torch.empty(rt, H, device="cuda")
            a_g, y_g = torch.empty(rt, FF, device="cuda"), torch.empty(rt, H, device="cuda")
            offs = torch.empty(E + 1, dtype=torch.int32, device="cuda")
            lst = torch.empty(rt, dtype=torch.int32, device="cuda")
            nbp = max(int(lib.cl_moe_xq_planes_bytes(T, H)), int(lib.cl_moe_xq_planes_bytes(rt, FF)))
            planes = torch.empty(nbp, dtype=torch.uint8, device="cuda")

            def per_route(i, px=px, pids=pids, rt=rt, a_r=a_r, y_r=y_r):
                K.check(lib.cl_moe_expert_gemv_rows(q4, p(gate), p(up), gate.stride(0), FF, H, p(px), H, Kr,
                                                    p(pids), rt, 0, 1, p(a_r), st()), "experts_rows")
                K.check(lib.cl_moe_expert_gemv_rows(q4, p(down), None, down.stride(0), H, FF, p(a_r), FF, 1,
                                                    p(pids), rt, 0, 1, p(y_r), st()), "experts_rows")

            def grouped(i, px=px, pids=pids, rt=rt, a_g=a_g, y_g=y_g, offs=offs, lst=lst, planes=planes, nbp=nbp):
                K.check(lib.cl_moe_group_routes(p(pids), rt, E, 0, 1, p(offs), p(lst), st()), "group_routes")
                K.check(lib.cl_moe_expert_gemv_grouped(q4, p(gate), p(up), gate.stride(0), FF, H, p(px), H, Kr,
                                                       p(pids), rt, 0, 1, p(offs), p(lst), E, p(planes), nbp,
                                                       p(a_g), st()), "experts_grouped")
                K.check(lib.cl_moe_expert_gemv_grouped(q4, p(down), None, down.stride(0), H, FF, p(a_g), FF, 1,
                                                       p(pids), rt, 0, 1, p(offs), p(lst), E, p(planes), nbp,
                                                       p(y_g), st()), "experts_grouped")
            try:
                t_r, t_g = graph_time_us(per_route, 4), graph_time_us(grouped, 4)
                pre[str(T)] = {"routes_us": round(t_r, 1), "grouped_us": round(t_g, 1),
                               "speedup": round(t_r / t_g, 2),
                               "bit_identical": bool(torch.equal(a_r, a_g) and torch.equal(y_r, y_g))}
            except Exception as e:
                pre[str(T)] = {"error": f"{type(e).__name__}: {e}"}
        out["prefill_experts"] = pre
        del gate, up, down
    except Exception as e:
        out["experts"] = {"error": f"{type(e).__name__}: {e}"}
    # DeltaNet: conv + L2 norms + decay / beta, then the delta-rule step
    W = (2 * G + R) * D
    qkv, z = torch.randn(W, device="cuda"), torch.randn(R * D, device="cuda")
    alpha, beta_raw = torch.randn(R, device="cuda"), torch.randn(R, device="cuda")
    conv_w, dt, a = torch.randn(W, KC, device="cuda") * 0.5, torch.randn(R, device="cuda") * 0.1, -torch.rand(R,
                                                                                                          device="cuda")
    gamma = torch.ones(D, device="cuda")
    hists = [torch.zeros(KC - 1, W, device="cuda") for _ in range(96)]
    states = [torch.zeros(R, D, D, device="cuda") for _ in range(96)]
    gact, decay, beta = torch.empty(W, device="cuda"), torch.empty(R, device="cuda"), torch.empty(R, device="cuda")
    gout = torch.empty(R * D, device="cuda")
    timed("gdn_prep", lambda i: K.check(lib.cl_gdn_prep(
        p(qkv), p(alpha), p(beta_raw), p(conv_w), p(hists[i % 96]), p(dt), p(a), G, R, D, KC, ctypes.c_float(1e-6),
        p(gact), p(decay), p(beta), st()), "gdn_prep"), 40, 4 * (W + W * KC + 2 * (KC - 1) * W + W + 4 * R))
    timed("gdn_step", lambda i: K.check(lib.cl_gdn_step(
        p(gact), p(decay), p(beta), p(z), p(gamma), p(states[i % 96]), G, R, D, ctypes.c_float(1e-6), p(gout), st()),
        "gdn_step"), 40, 2 * 4 * R * D * D + 4 * (W + 2 * R * D))
    del hists, states
    # gated attention: q/gate split + per-head norms + partial RoPE + KV append, then decode attention
    mixed = torch.randn(2 * hq * d, device="cuda")
    kr_, vr_ = torch.randn(hkv * d, device="cuda"), torch.randn(hkv * d, device="cuda")
    qn, kn = torch.ones(d, device="cuda"), torch.ones(d, device="cuda")
    table = torch.randn(cap, rot // 2, 2, device="cuda")
    pos = torch.tensor([L - 1], dtype=torch.int32, device="cuda")
    ln = torch.tensor([L], dtype=torch.int32, device="cuda")
    kcs = [torch.randn(cap, hkv * d, device="cuda") for _ in range(64)]
    vcs = [torch.randn(cap, hkv * d, device="cuda") for _ in range(64)]
    q, g = torch.empty(hq * d, device="cuda"), torch.empty(hq * d, device="cuda")
    att = torch.empty(hq * d, device="cuda")
    wsb = int(lib.cl_attn_decode_workspace_bytes(hq, d, cap))
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    timed("attn_gate_prep", lambda i: K.check(lib.cl_attn_gate_prep(
        p(mixed), p(kr_), p(vr_), p(qn), p(kn), hq, hkv, d, rot, p(table), p(pos), ctypes.c_float(1e-6), p(q), p(g),
        p(kcs[i % 64]), p(vcs[i % 64]), st()), "attn_gate_prep"), 40, 4 * (2 * hq * d + 2 * hkv * d + 2 * hq * d))
    timed("attn_decode_512_keys", lambda i: K.check(lib.cl_attn_decode(
        p(q), p(kcs[i % 64]), p(vcs[i % 64]), p(ln), cap, hq, hkv, d, ctypes.c_float(d ** -0.5), p(att), None, p(ws),
        wsb, st()), "attn_decode"), 40, 2 * L * hkv * d * 4 + 8 * hq * d)
    return out


def run_cpu_baseline(path: str, spec=None, prompt: int = 4, decode: int = 2, warmup: int = 0,
                     timeout: int = 900, moe: bool = False):
    """The reference CPULLM sample in a child process (oracle.cpu_baseline),
    so that running out of host memory or time gives an `unavailable` record
    instead of ending the bench.  moe: the reference's qwen35moe kernels run
    on the host instead (the file is mapped, not copied)."""
    if spec is not None and not moe:
        need, avail = reference_host_bytes(spec), mem_available()
        if avail is not None and need > 0.9 * avail:
            return {"value": None, "unavailable": f"the reference CPULLM holds FP32 weights and the file image: "
                                                  f"~{need / 1e9:.0f} GB of host memory, {avail / 1e9:.0f} GB "
                                                  f"available here"}
    cmd = [sys.executable, "-m", "oracle.cpu_baseline", "--model", path, "--prompt", str(prompt),
           "--decode", str(decode), "--warmup", str(warmup)] + (["--moe"] if moe else [])
    try:
        res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired:
        return {"value": None, "unavailable": f"reference CPU sample exceeded {timeout} s"}
    for line in res.stdout.splitlines()[::-1]:
        if line.startswith("{"):
            return json.loads(line)
    tail = (res.stderr or res.stdout).strip().splitlines()[-1:]
    return {"value": None, "unavailable": f"reference CPU sample exited with code {res.returncode}"
                                          + (f": {tail[0]}" if tail else "")}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    return world, rank, local


# The reference's own published decode rates for a workload this bench runs:
# Qwen2.5-14B Q4_K_M batch-1 greedy decode on its Metal backend (Apple M4),
# after its packed-byte Q4_K optimisation (METAL_14B_PROFILE.md:128-132).
# No number is published for the other shapes.
PUBLISHED_DECODE_TOK_S = {"qwen2.5-14b": 5.777}


def vs_published(name, value):
    ref = PUBLISHED_DECODE_TOK_S.get(name)
    return value / ref if ref and value else None


def model_spec(name):
    """(spec, writer) of a synthetic qwen2 or qwen35moe config."""
    from myllm_b200 import synth_gguf as sg
    if name in sg.MOE_CONFIGS:
        return sg.MOE_CONFIGS[name], sg.cached_moe
    if name in sg.CONFIGS:
        return sg.CONFIGS[name], sg.cached_qwen2
    raise SystemExit(f"unknown model {name!r}: one of {sorted(sg.CONFIGS) + sorted(sg.MOE_CONFIGS)}")


def ensure_model(name, rank, world, dist):
    spec, writer = model_spec(name)
    path = os.path.join(MODEL_DIR, f"{spec.name}.gguf")
    if rank == 0 and not os.path.exists(path):
        writer(spec, MODEL_DIR)
    if world > 1:
        dist.barrier()
    return spec, path


def scaling_base(args, device: int):
    """The N > 1 workload (the 14B shape, tensor-parallel there) on this one
    GPU, timed like the main run (CUDA events per decode call, summed over the
    steps): the same-model N = 1 point of the scaling series, since the N = 1
    headline is the 7B shape, whose 4 KV heads do not split 8 ways."""
    from myllm_b200 import CudaLLM
    from myllm_b200 import synth_gguf as sg
    name = model_name(args, 2)
    args = for_model(args, name)
    try:
        spec, path = ensure_model(name, 0, 1, None)
        llm = CudaLLM(path, max_sequence=args.max_sequence, device=device)
        prompt = sg.prompt_ids(spec.seed, args.prompt, spec.vocab)
        llm.prefill(prompt)
        llm.reset()
        tok = llm.prefill(prompt)
        prefill_ms = llm.last_call_ms()
        for _ in range(args.warmup):
            tok = llm.decode(tok)
        dev_ms = 0.0
        for _ in range(args.steps):
            tok = llm.decode(tok)
            dev_ms += llm.last_call_ms()
        llm.close()
    except Exception as e:  # reported in the line; the headline numbers stand
        return {"workload": name, "unavailable": f"{type(e).__name__}: {e}"}
    mid = args.prompt + args.warmup + args.steps // 2
    ms_step = dev_ms / args.steps
    return {"workload": f"{name} Q4_K_M, prompt {args.prompt}, greedy decode, KV capacity {args.max_sequence}",
            "parallelism": "single GPU", "value": args.steps / (dev_ms / 1e3), "unit": "tokens/s",
            "vs_baseline": vs_published(name, args.steps / (dev_ms / 1e3)),
            "ms_per_step": ms_step, "prefill_tokens_per_s": args.prompt / (prefill_ms / 1e3),
            "decode_hbm_gbs": decode_bytes_per_token(spec, mid) / (ms_step * 1e-3) / 1e9}


def time_allreduce(n_floats: int, iters: int, dist) -> float:
    """Device time (µs, max over ranks) of one NCCL all-reduce (sum) of
    n_floats FP32 values: torch.distributed's NCCL group, the calls enqueued
    back to back from the host and bracketed by CUDA events on the current
    stream. Every rank makes the same calls."""
    import torch
    x = torch.ones(n_floats, device="cuda")
    for _ in range(5):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    works = [dist.all_reduce(x, async_op=True) for _ in range(iters)]
    for w in works:
        w.wait()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def tp_collectives_per_token(spec, world: int) -> dict:
    """Collectives of one tensor-parallel decode token: an all-reduce after
    o_proj and after ffn_down in every layer, an all-gather of the attention
    output before o_proj when the shard plan says so, and the LM head's
    (value, index) all-gather."""
    from myllm_b200 import synth_gguf as sg
    from myllm_b200 import tp_plan
    d = spec.hidden // spec.heads
    o_block = max(sg.BLOCK[spec.types(l, "attn_output")][0] for l in range(spec.layers))
    gather = tp_plan(spec.ffn, spec.vocab, spec.heads, spec.kv_heads, d, o_block, world, 0).gather_attn
    return {"all_reduce": 2 * spec.layers, "all_gather": (spec.layers if gather else 0) + 1,
            "all_reduce_bytes": 4 * spec.hidden}


def workload_config(name, spec, args, world) -> dict:
    """The `config` of both arms' lines: the workload of this run."""
    from myllm_b200 import synth_gguf as sg
    moe = isinstance(spec, sg.MoeSpec)
    return {"workload": f"{name} Q4_K_M, prompt {args.prompt}, greedy decode, KV capacity {args.max_sequence}",
            "layers": spec.layers, "hidden": spec.hidden, "ffn": spec.expert_ffn if moe else spec.ffn,
            "vocab": spec.vocab,
            "parallelism": (f"ep{world}" if moe else f"tp{world}") if world > 1 else "single GPU",
            **({"decode_allreduce": os.environ.get("CUDALLM_ALLREDUCE") or "nccl"} if world > 1 and not moe else {}),
            "l2": "no flush: weights (GB) exceed the 126 MB L2 every step"}


def make_line(name, spec, args, world, rank, *, dev_ms, e2e_ms, prefill_ms, prefill_e2e_ms, kern, peak, peak_kind,
              sweep, cpu, base, collectives, clk, fused_ms=0.0) -> dict:
    """The bench's JSON line from the measured numbers (device ms summed over
    the timed decode steps, host ms around them, the prefill's device and host
    ms, the roofline kernel's timing, the peak) and the reports gathered
    beside them."""
    from myllm_b200 import synth_gguf as sg
    moe = isinstance(spec, sg.MoeSpec)
    mid = args.prompt + args.warmup + args.steps // 2
    if moe:
        rep, exp = moe_decode_bytes(spec, mid)
        tok_bytes = rep + exp / world
    else:
        tok_bytes = decode_bytes_per_token(spec, mid) / world
    ms_step = dev_ms / args.steps
    # embed; per layer: QKV GEMV (one launch per run of one format or of a
    # fused format pair), attention split (with RoPE and the KV append) +
    # combine, o, gate/up, down; final head GEMV, argmax, counter
    if moe:
        launches_per_step = moe_launches_per_step(spec, world, rank)
    else:
        qkv = sum(gemv_launches([spec.types(l, t) for t in ("attn_q", "attn_k", "attn_v")])
                  for l in range(spec.layers))
        launches_per_step = 1 + qkv + 5 * spec.layers + 3
        if world > 1 and os.environ.get("CUDALLM_ALLREDUCE") == "p2p":
            launches_per_step += 2 * spec.layers  # the decode all-reduces are this library's kernel then
    if fused_ms > 0:
        launches_per_step = 1  # the whole step is one cooperative launch
    roofline = {"bound": "hbm", "achieved": kern["gbs"], "peak": peak, "unit": "GB/s",
                "frac": kern["gbs"] / peak if kern["gbs"] else None,
                **dict(zip(("traffic", "traffic_source"),
                           profile_traffic("gemv_head" if moe else "gemv_gateup", kern.get("shape"),
                                           kern.get("bytes_per_launch")))),
                "kernel": kern["kernel"], "shape": kern["shape"],
                "bytes_per_launch": kern["bytes_per_launch"], "avg_launch_us": kern["avg_launch_us"],
                "peak_kind": f"{peak_kind} hbm_gbs (STREAM copy)",
                **({"error": kern["error"]} if "error" in kern else {})}
    if fused_ms > 0:
        # the step kernel is the whole decode: its algorithmic bytes are the
        # token's, its duration the CUDA events around it in every timed step
        k_us = fused_ms / args.steps * 1e3
        ach = tok_bytes / (k_us * 1e-6) / 1e9
        roofline = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                    **dict(zip(("traffic", "traffic_source"), profile_traffic(f"decode_fused_{name}"))),
                    "kernel": "decode_fused_kernel (one decode step: every layer, LM head and argmax in one "
                              "cooperative launch)",
                    "shape": f"{name}, position {mid}", "bytes_per_launch": tok_bytes, "avg_launch_us": k_us,
                    "peak_kind": f"{peak_kind} hbm_gbs (STREAM copy)", "per_operator_gemv": kern}
    return {
        "metric": "batch-1 greedy decode tokens/s",
        "value": args.steps / (dev_ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": vs_published(name, args.steps / (dev_ms / 1e3)),
        "dtype": "q4_k_m weights x fp32 activations (int8 limbs, exact integer dots, fp32 scaling)",
        "data": "synthetic (seeded N(0,0.02) weights quantized to GGML blocks; uniform random prompt ids)",
        "config": workload_config(name, spec, args, world),
        "e2e": {"value": args.steps / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "prefill": {"value": args.prompt / (prefill_ms / 1e3), "unit": "tokens/s", "tokens": args.prompt,
                    "e2e_tokens_per_s": args.prompt / (prefill_e2e_ms / 1e3),
                    "roofline": prefill_roofline(spec, args.prompt, prefill_ms, world, moe)},
        "decode_hbm": {"bytes_per_token_per_gpu": tok_bytes, "achieved_gbs": tok_bytes / (ms_step * 1e-3) / 1e9,
                       "peak_gbs": peak, "frac": tok_bytes / (ms_step * 1e-3) / 1e9 / peak,
                       "peak_kind": peak_kind},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "kernel_sweep": sweep,
        "scaling_base": base,
        "collectives": collectives,
        "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
    }


def sharded_parity(path, args, device, prompt, run_tokens, last_logits) -> dict:
    """Tokens and last logits of a sharded (tensor- or expert-parallel) run
    against the same GGUF and prompt on this one GPU, unsharded: the greedy
    token of the prefill and of every decode step (warm-up and timed) must be
    identical, and the last step's logits within 1e-4 of the one-GPU run's
    (max-abs relative), the level every parity test holds.  The one-GPU
    model is itself pinned to the reference CPULLM by the golden tests."""
    import numpy as np
    from myllm_b200 import CudaLLM
    one = CudaLLM(path, max_sequence=args.max_sequence, device=device)
    try:
        toks = [one.prefill(prompt)]
        for t in run_tokens[:-1]:
            toks.append(one.decode(t))  # teacher-forced on the sharded run's own tokens
        ref = one.last_logits()
    finally:
        one.close()
    same = [int(a) == int(b) for a, b in zip(toks, run_tokens)]
    err = float(np.abs(last_logits - ref).max() / np.abs(ref).max())
    ok = all(same) and err <= 1e-4
    return {"status": "ok" if ok else "mismatch",
            "against": "the same GGUF and prompt unsharded on one GPU (CudaLLM, pinned to CPULLM by the goldens)",
            "steps_compared": len(same), "tokens_identical": all(same),
            "first_mismatch": None if all(same) else same.index(False),
            "last_logits_rel_err": err, "tolerance": 1e-4}


def bench_cuda(args):
    import torch
    import torch.distributed as dist
    if args.allreduce:
        os.environ["CUDALLM_ALLREDUCE"] = args.allreduce  # read when the model is created
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    from myllm_b200 import CudaLLM, nccl_unique_id
    from myllm_b200 import synth_gguf as sg
    name = model_name(args, world)
    raw_args, args = args, for_model(args, name)
    spec, path = ensure_model(name, rank, world, dist)
    nid = None
    if world > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    llm = CudaLLM(path, max_sequence=args.max_sequence, device=local, rank=rank, world=world, nccl_id=nid)
    prompt = sg.prompt_ids(spec.seed, args.prompt, spec.vocab)
    if args.prompt + args.warmup + args.steps > args.max_sequence:
        raise SystemExit("prompt + warmup + steps exceed the KV capacity")

    # prefill: one untimed, one timed (host-to-host and device)
    llm.prefill(prompt)
    llm.reset()
    t0 = time.perf_counter()
    tok = llm.prefill(prompt)
    prefill_e2e = time.perf_counter() - t0
    prefill_ms = llm.last_call_ms()
    run_tokens = [tok]

    for _ in range(args.warmup):
        tok = llm.decode(tok)
        run_tokens.append(tok)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    dev_ms = 0.0
    fused_ms = 0.0  # the one-launch step kernel alone (0 on the per-operator graph)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = llm.decode(tok)
        dev_ms += llm.last_call_ms()
        fused_ms += llm.last_kernel_ms()
        run_tokens.append(tok)
    e2e_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    # the last step's full logits (a collective for a sharded model)
    last_logits = llm.last_logits() if world > 1 and not args.no_parity else None
    vals = torch.tensor([dev_ms, e2e_s * 1e3, prefill_ms, prefill_e2e * 1e3], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms, prefill_ms, prefill_e2e_ms = [float(v) for v in vals.cpu()]
    llm.close()
    parity = None
    if world > 1 and not args.no_parity:
        if rank == 0:
            try:
                parity = sharded_parity(path, args, local, prompt, run_tokens, last_logits)
            except Exception as e:  # reported in the line; the measured numbers stand
                parity = {"status": "error", "error": f"{type(e).__name__}: {e}"}
        dist.barrier()
    collectives = None
    if world > 1:
        if isinstance(spec, sg.MoeSpec):  # one all-reduce of the MoE output per layer
            collectives = {"all_reduce": spec.layers, "all_gather": 0, "all_reduce_bytes": 4 * spec.hidden}
        else:
            collectives = tp_collectives_per_token(spec, world)
        us = time_allreduce(spec.hidden, 200, dist)
        ms_all_reduce = us * collectives["all_reduce"] / 1e3
        collectives.update({"all_reduce_us": us, "all_reduce_ms_per_token": ms_all_reduce,
                            "share_of_step": ms_all_reduce / (dev_ms / args.steps),
                            "note": "torch.distributed NCCL all-reduce of the same size, host-launched back to "
                                    "back; the model's own calls run inside its decode CUDA graph"})

    moe = isinstance(spec, sg.MoeSpec)
    peak, peak_kind = measured_peaks()
    # the reports below are each guarded: a failure is recorded in its own
    # field, and the headline numbers already measured still print
    try:
        kern = time_head_kernel(spec, args.kernel_iters) if moe else time_gateup_kernel(spec, args.kernel_iters)
    except Exception as e:
        kern = {"kernel": None, "shape": None, "bytes_per_launch": None, "avg_launch_us": None, "gbs": None,
                "error": f"{type(e).__name__}: {e}"}
    sweep = None
    if world == 1 and not args.no_sweep and not moe:
        try:
            sweep = kernel_sweep(peak, spec.seed)
        except Exception as e:
            sweep = {"error": f"{type(e).__name__}: {e}"}
        try:
            sweep["moe_kernels"] = moe_kernel_times(peak, spec.seed)
        except Exception as e:
            sweep["moe_kernels"] = {"error": f"{type(e).__name__}: {e}"}
    if world > 1:
        dist.barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        # qwen35moe: the reference's own kernels on the host, 2 prompt tokens + 2 decodes
        cpu = run_cpu_baseline(path, spec, prompt=2, moe=True) if moe else run_cpu_baseline(path, spec)
    base = scaling_base(raw_args, local) if world == 1 and not args.no_scaling_base and not args.model else None
    line = make_line(name, spec, args, world, rank, dev_ms=dev_ms, e2e_ms=e2e_ms, prefill_ms=prefill_ms,
                     prefill_e2e_ms=prefill_e2e_ms, kern=kern, peak=peak, peak_kind=peak_kind, sweep=sweep, cpu=cpu,
                     base=base, collectives=collectives, clk=clk, fused_ms=fused_ms)
    if parity is not None:
        line["parity"] = parity
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def bench_reference(args):
    world, rank, local = dist_setup(args)
    if rank != 0:
        return
    name = model_name(args, world)
    args = for_model(args, name)
    from myllm_b200 import synth_gguf as sg
    moe = name in sg.MOE_CONFIGS
    spec, path = ensure_model(name, 0, 1, None)
    steps = min(args.steps, 4)
    warm = min(args.warmup, 1)
    # qwen35moe has no reference CPU path: its own Metal kernels compiled for the host stand in
    res = run_cpu_baseline(path, spec, prompt=2 if moe else 4, decode=steps, warmup=warm, timeout=1800, moe=moe)
    if res.get("value") is None:
        print(json.dumps({"impl": "reference", "unavailable": res.get("unavailable", "reference CPU path failed")}))
        return
    line = {
        "impl": "reference",
        "metric": "batch-1 greedy decode tokens/s",
        "value": res["value"],
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": 1e3 / res["value"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": vs_published(name, res["value"]),
        "dtype": "fp32 (reference kernels decode the blocks per product)" if moe else
                 "fp32 (reference dequantizes to FP32 at load)",
        "data": "synthetic (same seeded GGUF as the cuda arm)",
        "config": workload_config(name, spec, args, world),
        "prefill": {"value": res["prefill_tokens_per_s"], "unit": "tokens/s", "tokens": 2 if moe else 4},
        "cpu_baseline": dict(res, sample=f"{res.get('sample', '')}; a bounded sample of the workload in `config` "
                                         f"(prompt {2 if moe else 4} + {steps} decode tokens), 1 host thread "
                                         f"({'the kernels run one thread at a time' if moe else 'CPULLM has no threading'})"),
        "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        bench_reference(args)
    else:
        bench_cuda(args)


if __name__ == "__main__":
    main()
