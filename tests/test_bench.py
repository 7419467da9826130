"""bench.py's accounting, on the CPU: the algorithmic bytes per decode token
that roofline fractions divide by, and the launch count it reports.

The per-token bytes at position 0 must equal the figures derived from the
synthetic layouts (0.392 / 4.377 / 8.577 GB for the 0.5B / 7B / 14B shapes):
every weight matrix once, one embedding row, norms and biases.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from myllm_b200 import synth_gguf as sg  # noqa: E402


@pytest.mark.parametrize("name,gb", [("qwen2.5-0.5b", 0.392), ("qwen2.5-7b", 4.377), ("qwen2.5-14b", 8.577)])
def test_decode_bytes_per_token_at_position_zero(name, gb):
    spec = sg.CONFIGS[name]
    # the figures are quoted to three decimals of a GB
    assert abs(bench.decode_bytes_per_token(spec, 0) / 1e9 - gb) <= 5e-4


def test_decode_bytes_grow_by_the_kv_rows_read():
    spec = sg.CONFIGS["qwen2.5-7b"]
    kvd = spec.kv_heads * (spec.hidden // spec.heads)
    d = bench.decode_bytes_per_token(spec, 100) - bench.decode_bytes_per_token(spec, 99)
    assert d == spec.layers * 2 * kvd * 4  # one more K row and V row per layer, FP32


def test_gemv_launch_count_groups_formats_and_fused_pairs():
    # a run of one format, or of a fused pair (Q4_K + Q6_K, Q5_0 + Q8_0), is one launch
    assert bench.gemv_launches([sg.Q4_K, sg.Q4_K, sg.Q6_K]) == 1
    assert bench.gemv_launches([sg.Q5_0, sg.Q5_0, sg.Q8_0]) == 1
    assert bench.gemv_launches([sg.Q4_K, sg.Q8_0]) == 2
    assert bench.gemv_launches([sg.Q4_K, sg.Q6_K, sg.Q8_0]) == 2
    # the 7B attention projections: one launch per layer
    spec = sg.CONFIGS["qwen2.5-7b"]
    for layer in range(spec.layers):
        assert bench.gemv_launches([spec.types(layer, t) for t in ("attn_q", "attn_k", "attn_v")]) == 1


def test_sweep_shapes_are_the_config1_shapes():
    assert (18944, 3584) in bench.SWEEP_SHAPES and (3584, 18944) in bench.SWEEP_SHAPES
    # K-quants skip K = 896 (not a multiple of their 256-element blocks)
    assert 896 % sg.BLOCK[sg.Q4_K][0] != 0


class _FakeLLM:
    """Stands in for CudaLLM: every call 'takes' 2 ms of device time."""

    def __init__(self, path, max_sequence=0, device=0, rank=0, world=1, nccl_id=None):
        self.calls = 0

    def prefill(self, ids):
        return 1

    def reset(self):
        pass

    def decode(self, tok):
        self.calls += 1
        return tok

    def last_call_ms(self):
        return 2.0

    def last_kernel_ms(self):
        return 0.0  # the per-operator graph

    def last_logits(self):
        import numpy as np
        return np.linspace(-1.0, 1.0, 64, dtype=np.float32)

    def close(self):
        pass


def _args(**kw):
    import argparse
    base = dict(gpus=1, steps=8, warmup=3, prompt=16, max_sequence=64, model=None, no_scaling_base=False)
    base.update(kw)
    return argparse.Namespace(**base)


def test_scaling_base_times_the_multi_gpu_workload_on_one_gpu(monkeypatch):
    import myllm_b200
    monkeypatch.setattr(myllm_b200, "CudaLLM", _FakeLLM)
    monkeypatch.setattr(bench, "ensure_model", lambda name, r, w, d: (sg.CONFIGS[name], "unused"))
    out = bench.scaling_base(_args(), 0)
    assert out["workload"].startswith("qwen2.5-14b") and out["parallelism"] == "single GPU"
    assert out["value"] == 8 / (8 * 2.0 / 1e3) and out["ms_per_step"] == 2.0
    assert out["prefill_tokens_per_s"] == 16 / 2e-3


def test_scaling_base_failure_is_reported_not_raised(monkeypatch):
    import myllm_b200

    def boom(*a, **k):
        raise RuntimeError("no device")
    monkeypatch.setattr(myllm_b200, "CudaLLM", boom)
    monkeypatch.setattr(bench, "ensure_model", lambda name, r, w, d: (sg.CONFIGS[name], "unused"))
    out = bench.scaling_base(_args(), 0)
    assert out["unavailable"] == "RuntimeError: no device"


def test_prefill_flops_of_the_qwen2_shapes():
    """7B at 512 tokens: 28 layers of q/k/v/o and gate/up/down products over
    512 rows (k and v are 512 wide: 4 KV heads of 128), causal attention over
    28 heads of 128, and the last row's LM head: ~6.74 TFLOP."""
    spec = sg.CONFIGS["qwen2.5-7b"]
    H, F, L = 3584, 18944, 28
    gemm = L * 512 * 2 * (2 * H * H + 2 * 512 * H + 3 * F * H)
    attn = L * 2 * 2 * 28 * 128 * (512 * 513 // 2)
    assert bench.prefill_flops(spec, 512) == gemm + attn + 2 * 152064 * H
    assert 6.7e12 < bench.prefill_flops(spec, 512) < 6.8e12


def test_moe_bytes_per_token():
    spec = sg.MOE_CONFIGS["qwen3.6-35b-a3b"]
    rep, exp = bench.moe_decode_bytes(spec, 0)
    # the active weights of one token: about 2.2 GB for the real file, plus the
    # F32 routers (84 MB) and the DeltaNet state read + write (126 MB) counted here
    assert 2.2e9 < rep + exp < 2.5e9
    # one more position reads one more K and V row in each attention layer
    attn = sum(spec.is_attention(l) for l in range(spec.layers))
    rep1, exp1 = bench.moe_decode_bytes(spec, 1)
    assert rep1 - rep == attn * 2 * spec.kv_heads * spec.head_dim * 4 and exp1 == exp
    # routed experts scale with the number used per token
    half = sg.MoeSpec(**{**spec.__dict__, "experts_used": spec.experts_used // 2})
    shared = exp - 2 * (exp - bench.moe_decode_bytes(half, 0)[1])
    assert 0 < shared < exp / 4


def test_moe_launch_count_per_rank():
    spec = sg.tiny_moe_spec(layers=8, experts=16)
    attn = sum(spec.is_attention(l) for l in range(spec.layers))
    # one GPU: attention layers 5 + the q/k/v GEMV launches (input norm fused),
    # DeltaNet 6 (alpha | beta stacked), MoE 8 (router | shared gate stacked)
    qkv = [bench.gemv_launches([sg.moe_a3b_types(l, t) for t in ("attn_q", "attn_k", "attn_v")])
           for l in range(spec.layers) if spec.is_attention(l)]
    assert bench.moe_launches_per_step(spec, 1, 0) == 1 + sum(5 + q for q in qkv) + 6 * (8 - attn) + 8 * 8 + 3
    # two ranks: the shared expert on every other layer, plus the residual add
    assert bench.moe_launches_per_step(spec, 2, 0) == bench.moe_launches_per_step(spec, 1, 0) - 2 * 4 + 8
    # more ranks than experts: a rank without experts skips the routed GEMVs
    assert bench.moe_launches_per_step(sg.tiny_moe_spec(experts=2, used=2), 4, 3) < \
        bench.moe_launches_per_step(sg.tiny_moe_spec(experts=2, used=2), 4, 1)


def test_tp_collectives_per_token():
    spec = sg.CONFIGS["qwen2.5-14b"]
    # two all-reduces per layer; the attention output is all-gathered only at
    # 8 ranks (5 heads x 128 columns are off the 256-column o_proj grid)
    for world, gathers in ((2, 1), (4, 1), (8, spec.layers + 1)):
        c = bench.tp_collectives_per_token(spec, world)
        assert c == {"all_reduce": 2 * spec.layers, "all_gather": gathers, "all_reduce_bytes": 4 * 5120}


def test_reference_memory_guard(monkeypatch):
    # CPULLM holds FP32 weights plus the file: ~35 GB (7B), ~68 GB (14B)
    assert 34e9 < bench.reference_host_bytes(sg.CONFIGS["qwen2.5-7b"]) < 36e9
    assert 67e9 < bench.reference_host_bytes(sg.CONFIGS["qwen2.5-14b"]) < 69e9
    monkeypatch.setattr(bench, "mem_available", lambda: 16e9)
    out = bench.run_cpu_baseline("unused.gguf", sg.CONFIGS["qwen2.5-14b"])
    assert out["value"] is None and "~68 GB of host memory, 16 GB available" in out["unavailable"]


def test_reference_sample_failure_is_reported(tmp_path):
    # a child that fails (here: no such model) gives an `unavailable` record
    out = bench.run_cpu_baseline(str(tmp_path / "absent.gguf"), timeout=300)
    assert out["value"] is None and out["unavailable"]


def test_vs_baseline_only_where_the_reference_publishes():
    # 14B decode: the reference's Metal figure (5.777 tok/s); nothing for 7B
    assert bench.vs_published("qwen2.5-14b", 57.77) == pytest.approx(10.0)
    assert bench.vs_published("qwen2.5-7b", 466.0) is None


REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "config", "e2e", "roofline", "cpu_baseline", "clocks", "gpu_launches"}


@pytest.mark.parametrize("name,world", [("qwen2.5-7b", 1), ("qwen2.5-14b", 8), ("qwen3.6-35b-a3b", 2)])
def test_json_line_contract(name, world):
    """Every key the driver reads, for the headline, a tensor-parallel and an
    expert-parallel line, built from made-up measurements."""
    import json
    spec, _ = bench.model_spec(name)
    args = _args(steps=128, warmup=4, prompt=512, max_sequence=4096, kernel_iters=40)
    kern = {"kernel": "k", "shape": "s", "bytes_per_launch": 1e8, "avg_launch_us": 20.0, "gbs": 5000.0}
    clk = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    line = bench.make_line(name, spec, args, world, 0, dev_ms=256.0, e2e_ms=260.0, prefill_ms=100.0,
                           prefill_e2e_ms=110.0, kern=kern, peak=6545.0, peak_kind="measured", sweep=None,
                           cpu=None, base=None, collectives=None, clk=clk)
    assert REQUIRED <= set(line)
    json.loads(json.dumps(line))
    assert line["value"] == pytest.approx(500.0) and line["ms_per_step"] == pytest.approx(2.0)
    assert line["n_gpus"] == world and line["higher_is_better"] is True and line["scaling"] == "strong"
    assert set(line["e2e"]) >= {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"}
    assert line["e2e"]["value"] == pytest.approx(128 / 0.26)
    assert set(line["roofline"]) >= {"bound", "achieved", "peak", "unit", "frac", "traffic"}
    assert line["roofline"]["frac"] == pytest.approx(5000 / 6545)
    pr = line["prefill"]["roofline"]
    if "a3b" in name:
        assert "unavailable" in pr
    else:  # useful FLOPs per GPU over the measured bf16 GEMM peak
        sus, burst, _ = bench.measured_tensor_peaks()
        ach = bench.prefill_flops(spec, 512) / world / 0.1 / 1e12
        assert pr["bound"] == "tensor" and pr["unit"] == "TFLOP/s"
        assert pr["achieved"] == pytest.approx(ach) and pr["frac"] == pytest.approx(ach / sus)
    assert "workload" in line["config"] and name in line["config"]["workload"]
    assert line["config"]["parallelism"] == ("single GPU" if world == 1 else
                                             ("ep" if "a3b" in name else "tp") + str(world))
    assert isinstance(line["gpu_launches"], int) and line["gpu_launches"] > 128
    assert (line["vs_baseline"] is None) == (name != "qwen2.5-14b")


def _dry_run(monkeypatch):
    """CPU stand-ins for the GPU side of the bench's sweep code: tensors on
    the host, a library that checks each call's argument count against the C
    signatures, a graph timer that just calls the launches."""
    import numpy as np
    import torch
    from myllm_b200 import _native
    from myllm_b200 import kernels as K

    calls = {}

    class FakeLib:
        def __getattr__(self, name):
            res, args = _native.SIGNATURES[name]

            def f(*a):
                assert len(a) == len(args), name
                calls[name] = calls.get(name, 0) + 1
                if name.endswith("_bytes"):
                    return 4096  # size queries: a small non-zero buffer
                return 0 if res is not None else None
            return f

    for fn in ("randn", "zeros", "ones", "empty", "rand", "arange", "tensor"):
        real = getattr(torch, fn)
        monkeypatch.setattr(torch, fn, lambda *a, _f=real, **k: _f(*a, **{x: v for x, v in k.items() if x != "device"}))
    monkeypatch.setattr(_native, "lib", lambda: FakeLib())
    monkeypatch.setattr(K, "repack", lambda gtype, w, k: torch.from_numpy(w))
    monkeypatch.setattr(K, "_p", lambda t: None if t is None else 1 << 20)
    monkeypatch.setattr(K, "_stream", lambda: None)
    monkeypatch.setattr(sg, "fill", lambda *a, **k: np.zeros((1, 16), dtype=np.uint8))
    monkeypatch.setattr(bench, "graph_time_us", lambda fn, iters: [fn(i) for i in range(iters)] and 5.0)
    return calls


def test_sweep_code_runs(monkeypatch):
    """Config 1's sweep, dry-run: every GEMV entry and the prefill GEMM at
    three batch sizes for every format and shape, without errors."""
    calls = _dry_run(monkeypatch)
    monkeypatch.setattr(bench, "SWEEP_SHAPES", [(896, 896), (256, 512)])
    out = bench.kernel_sweep(6545.0, 1)
    # K-quants skip K = 896: 2 formats x 1 shape + 2 formats x 2 shapes
    assert len(out["gemv"]) == 6 and len(out["gemm"]) == 18
    assert all("error" not in e for e in out["gemm"]), out["gemm"]
    assert calls["cl_gemv"] > 0 and calls["cl_gemm"] > 0
    # K-quant entries also time the packed GEMV; the 7B LM head compares both
    assert all("packed_us" in e for e in out["gemv"] if e["type"] in ("Q4_K", "Q6_K"))
    assert "error" not in out["lm_head_7b"] and calls["cl_gemv_packed"] > 0, out["lm_head_7b"]


def test_moe_kernel_timing_code_runs(monkeypatch):
    """The config-4 kernel timings of the sweep, dry-run on the CPU."""
    calls = _dry_run(monkeypatch)
    out = bench.moe_kernel_times(6545.0, 1)
    assert set(out) == {"router_gemv_f32", "route_topk", "expert_gate_up_swiglu", "expert_down", "gdn_prep",
                        "gdn_step", "attn_gate_prep", "attn_decode_512_keys", "prefill_experts"}
    assert all("error" not in v for v in out.values()), out
    assert calls["cl_moe_expert_gemv"] > 0 and calls["cl_gdn_step"] > 0 and calls["cl_attn_decode"] > 0
    # MoE prefill experts, per route and grouped, at 64- and 512-token chunks
    assert set(out["prefill_experts"]) == {"64", "512"}
    assert all("error" not in v for v in out["prefill_experts"].values()), out["prefill_experts"]
    assert calls["cl_moe_expert_gemv_rows"] > 0 and calls["cl_moe_expert_gemv_grouped"] > 0


class _Event:
    """CUDA event stand-in: every interval is 1 ms."""

    def __init__(self, enable_timing=False):
        pass

    def record(self, stream=None):
        pass

    def elapsed_time(self, other):
        return 1.0


class _Work:
    def wait(self):
        pass


class _Clocks:
    def __init__(self, gpu):
        pass

    def start(self):
        pass

    def stop(self):
        return {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}


def _fake_run(monkeypatch, argv, env):
    """Everything a whole bench run touches, replaced for the CPU: the sweep
    stand-ins of _dry_run, CUDA events and device calls, torch.distributed,
    the model, the model file and the clock sampler; argv and the launcher's
    environment as given."""
    import sys
    import torch
    import torch.distributed as dist
    import myllm_b200
    _dry_run(monkeypatch)
    monkeypatch.setattr(torch.cuda, "Event", _Event)
    for fn in ("synchronize", "set_device", "current_stream"):
        monkeypatch.setattr(torch.cuda, fn, lambda *a: None)
    for fn in ("init_process_group", "barrier", "broadcast_object_list", "destroy_process_group"):
        monkeypatch.setattr(dist, fn, lambda *a, **k: None)
    monkeypatch.setattr(dist, "all_reduce", lambda t, op=None, async_op=False: _Work() if async_op else None)
    monkeypatch.setattr(myllm_b200, "CudaLLM", _FakeLLM)
    monkeypatch.setattr(bench, "ensure_model", lambda name, r, w, d: (bench.model_spec(name)[0], "unused"))
    monkeypatch.setattr(bench, "ClockSampler", _Clocks)
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)


def test_default_run_prints_a_complete_line(monkeypatch, capsys):
    """The N = 1 default run end to end on the CPU: a stand-in model and CUDA
    timer, the sweep and kernel timings dry-run, the reference sample and
    the 14B point stubbed; one JSON line with every key of the contract."""
    import json
    _fake_run(monkeypatch, ["--steps", "8", "--warmup", "3"], {})
    monkeypatch.setattr(bench, "SWEEP_SHAPES", [(256, 512)])
    monkeypatch.setattr(bench, "run_cpu_baseline", lambda *a, **k: {"value": 0.2, "unit": "tokens/s", "cores": 1,
                                                                     "kind": "reference", "sample": "stub"})
    monkeypatch.setattr(bench, "scaling_base", lambda args, dev: {"workload": "qwen2.5-14b", "value": 1.0})
    bench.main()
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert REQUIRED <= set(line) and line["n_gpus"] == 1 and line["steps"] == 8
    assert line["value"] == pytest.approx(8 / (8 * 2.0 / 1e3)) and line["cpu_baseline"]["value"] == 0.2
    assert "moe_kernels" in line["kernel_sweep"] and line["scaling_base"]["value"] == 1.0
    assert line["roofline"]["achieved"] > 0


def test_tensor_parallel_run_prints_a_complete_line(monkeypatch, capsys):
    """Rank 0 of a 2-rank run (the 14B shape, tensor-parallel) on the CPU:
    torch.distributed replaced by stand-ins; the line carries the contract
    keys and the collectives report."""
    import json
    _fake_run(monkeypatch, ["--gpus", "2", "--steps", "8", "--warmup", "3"],
              {"WORLD_SIZE": "2", "RANK": "0", "LOCAL_RANK": "0"})
    bench.main()
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert REQUIRED <= set(line) and line["n_gpus"] == 2 and line["config"]["parallelism"] == "tp2"
    assert line["collectives"]["all_reduce"] == 2 * sg.CONFIGS["qwen2.5-14b"].layers
    assert line["collectives"]["all_reduce_us"] > 0 and line["vs_baseline"] is not None
    assert line["config"]["decode_allreduce"] == "nccl"
    # config 3's prompt, and the sharded run checked against one GPU
    assert "prompt 1024" in line["config"]["workload"]
    assert line["parity"]["status"] == "ok" and line["parity"]["steps_compared"] == 1 + 3 + 8


def test_sharded_parity_reports_a_mismatch(monkeypatch):
    """A one-GPU run that disagrees at the third token is reported, not hidden."""
    import argparse
    import myllm_b200

    class Diverging(_FakeLLM):
        def decode(self, tok):
            self.calls += 1
            return tok + 1 if self.calls == 2 else tok

    monkeypatch.setattr(myllm_b200, "CudaLLM", Diverging)
    out = bench.sharded_parity("unused", argparse.Namespace(max_sequence=64), 0, [1, 2], [1, 1, 1, 1],
                               _FakeLLM("x").last_logits())
    assert out["status"] == "mismatch" and out["first_mismatch"] == 2 and not out["tokens_identical"]


def test_peer_allreduce_switch(monkeypatch, capsys):
    import json
    import os
    # registered with monkeypatch, so the value the bench sets is undone afterwards
    monkeypatch.setenv("CUDALLM_ALLREDUCE", "")
    _fake_run(monkeypatch, ["--gpus", "2", "--steps", "8", "--warmup", "3", "--allreduce", "p2p"],
              {"WORLD_SIZE": "2", "RANK": "0", "LOCAL_RANK": "0"})
    bench.main()
    line = json.loads([l for l in capsys.readouterr().out.splitlines() if l.startswith("{")][0])
    assert os.environ["CUDALLM_ALLREDUCE"] == "p2p" and line["config"]["decode_allreduce"] == "p2p"


@pytest.mark.parametrize("gpus,model,expect", [(1, None, "qwen2.5-7b"), (2, None, "qwen2.5-14b"),
                                               (1, "qwen3.6-35b-a3b", "qwen3.6-35b-a3b")])
def test_reference_arm_prints_its_line(monkeypatch, capsys, gpus, model, expect):
    """`--impl reference`: the CPULLM sample (stubbed) on the cuda arm's
    workload, with the contract keys; rank 0 only; the MoE model times the
    reference's own kernels on the host (stubbed the same way)."""
    import json
    import sys
    seen = {}

    def sample(path, spec=None, **k):
        seen["spec"] = spec.name
        seen["moe"] = k.get("moe", False)
        return {"value": 0.25, "unit": "tokens/s", "cores": 1, "kind": "reference", "sample": "stub",
                "prefill_tokens_per_s": 1.0}
    monkeypatch.setattr(bench, "run_cpu_baseline", sample)
    monkeypatch.setattr(bench, "ensure_model", lambda name, r, w, d: (bench.model_spec(name)[0], "unused"))
    argv = ["bench.py", "--impl", "reference", "--gpus", str(gpus)] + (["--model", model] if model else [])
    monkeypatch.setattr(sys, "argv", argv)
    monkeypatch.setenv("WORLD_SIZE", str(gpus))
    monkeypatch.setenv("RANK", "0")
    bench.main()
    line = json.loads([l for l in capsys.readouterr().out.splitlines() if l.startswith("{")][0])
    assert line["impl"] == "reference"
    if expect is None:
        assert "unavailable" in line
        return
    assert seen["spec"] == expect and seen["moe"] == ("a3b" in expect)
    assert REQUIRED - {"clocks", "gpu_launches", "roofline"} <= set(line) and line["value"] == 0.25
    # the cuda arm's config, so that the driver pairs the two lines
    spec = bench.model_spec(expect)[0]
    assert line["config"] == bench.workload_config(expect, spec, bench.for_model(bench.parse(), expect), gpus)
    assert line["cpu_baseline"]["kind"] == "reference" and "bounded sample" in line["cpu_baseline"]["sample"]
    assert line["e2e"] == {"value": 0.25, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # other ranks print nothing
    monkeypatch.setenv("RANK", "1")
    bench.main()
    assert not capsys.readouterr().out.strip() or gpus == 1


@pytest.mark.parametrize("gpus", [1, 2])
def test_moe_mode_prints_a_complete_line(monkeypatch, capsys, gpus):
    """`--model qwen3.6-35b-a3b`: the expert-parallel workload's line (LM-head
    roofline kernel, replicated + expert bytes; at N = 1 the CPU sample of the
    reference's own kernels on the host, none at N > 1)."""
    import json
    _fake_run(monkeypatch, ["--gpus", str(gpus), "--model", "qwen3.6-35b-a3b", "--prompt", "64", "--steps", "8",
                            "--warmup", "3", "--max-sequence", "1024"],
              {"WORLD_SIZE": str(gpus), "RANK": "0", "LOCAL_RANK": "0"})
    bench.main()
    line = json.loads([l for l in capsys.readouterr().out.splitlines() if l.startswith("{")][0])
    assert REQUIRED <= set(line)
    assert line["config"]["parallelism"] == ("single GPU" if gpus == 1 else "ep2")
    assert line["roofline"]["shape"].endswith("Q6_K")
    assert (line["cpu_baseline"] is None) == (gpus > 1)
    assert (line["collectives"] is None) == (gpus == 1) and line["kernel_sweep"] is None


def test_launch_count_includes_the_peer_allreduce(monkeypatch):
    spec = sg.CONFIGS["qwen2.5-14b"]
    kw = dict(dev_ms=256.0, e2e_ms=260.0, prefill_ms=100.0, prefill_e2e_ms=110.0,
              kern={"kernel": "k", "shape": "s", "bytes_per_launch": 1, "avg_launch_us": 1.0, "gbs": 1.0},
              peak=6545.0, peak_kind="measured", sweep=None, cpu=None, base=None, collectives=None, clk={})
    args = _args(steps=10, warmup=3, prompt=512, max_sequence=4096)
    monkeypatch.delenv("CUDALLM_ALLREDUCE", raising=False)
    nccl = bench.make_line("qwen2.5-14b", spec, args, 2, 0, **kw)["gpu_launches"]
    monkeypatch.setenv("CUDALLM_ALLREDUCE", "p2p")
    p2p = bench.make_line("qwen2.5-14b", spec, args, 2, 0, **kw)["gpu_launches"]
    assert p2p - nccl == 2 * spec.layers * 10


def test_a_failing_report_does_not_lose_the_line(monkeypatch, capsys):
    """The roofline kernel timing and the sweep raising: the line still
    prints, with each failure recorded in its own field."""
    import json

    def boom(*a, **k):
        raise RuntimeError("planted")
    _fake_run(monkeypatch, ["--steps", "8", "--warmup", "3"], {})
    monkeypatch.setattr(bench, "time_gateup_kernel", boom)
    monkeypatch.setattr(bench, "kernel_sweep", boom)
    monkeypatch.setattr(bench, "run_cpu_baseline", lambda *a, **k: {"value": 0.2})
    monkeypatch.setattr(bench, "scaling_base", lambda args, dev: None)
    bench.main()
    line = json.loads([l for l in capsys.readouterr().out.splitlines() if l.startswith("{")][0])
    assert REQUIRED <= set(line) and line["value"] > 0
    assert line["roofline"]["error"] == "RuntimeError: planted" and line["roofline"]["frac"] is None
    assert line["kernel_sweep"]["error"] == "RuntimeError: planted" and "moe_kernels" in line["kernel_sweep"]


def test_traffic_is_measured_or_scaled_per_shape():
    """roofline.traffic: the ncu capture's bytes at the shape it was taken
    at; at another shape of the same kernel its traffic / algorithmic ratio
    times that launch's algorithmic bytes, saying so; None without one."""
    import bench
    t, src = bench.profile_traffic("gemv_gateup", "2x[18944,3584] Q4_K", 76490752)
    assert t == 77935872 and src.startswith("measured")
    algo14 = 2 * 13824 * 5120 * 144 // 256
    t2, src2 = bench.profile_traffic("gemv_gateup", "2x[13824,5120] Q4_K", algo14)
    assert abs(t2 / algo14 - 77935872 / 76490752) < 1e-12 and src2.startswith("scaled")
    assert bench.profile_traffic("gemv_head")[0] is None


def test_moe_reference_sample_runs_the_reference_kernels(tmp_path):
    """qwen35moe's CPU sample: the reference's own kernels on the host
    (oracle/_ref/libref_metal.so) in a child process, on a tiny model."""
    from oracle import metal_ref
    if not metal_ref.available():
        pytest.skip("the reference kernels were not built here")
    path = sg.cached_moe(sg.tiny_moe_spec(seed=5), str(tmp_path))
    out = bench.run_cpu_baseline(path, sg.tiny_moe_spec(seed=5), prompt=2, decode=1, timeout=300, moe=True)
    assert out["value"] > 0 and out["kind"] == "reference" and out["cores"] == 1
    assert "Metal kernels compiled for the host" in out["sample"]
