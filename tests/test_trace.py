"""FlashInfer-Trace loader and evaluation loop (fbmoe_trace).

The trace sets here are synthetic ones written by the tests, in the FlashInfer-Trace
layout: a definition JSON, a workloads JSONL and safetensors blobs. The contest
dataset is not available offline.
"""
import json
import os

import pytest
import torch

H, I, E = 7168, 2048, 256


def _definition(name, E_local, reference):
    axes = {
        "seq_len": {"type": "var"},
        "num_experts": {"type": "const", "value": E},
        "num_local_experts": {"type": "const", "value": E_local},
        "hidden_size": {"type": "const", "value": H},
        "intermediate_size": {"type": "const", "value": I},
        "gemm1_out_size": {"type": "const", "value": 2 * I},
        "num_hidden_blocks": {"type": "const", "value": H // 128},
        "num_intermediate_blocks": {"type": "const", "value": I // 128},
        "num_gemm1_out_blocks": {"type": "const", "value": 2 * I // 128},
    }
    inputs = {
        "routing_logits": {"shape": ["seq_len", "num_experts"], "dtype": "float32"},
        "routing_bias": {"shape": ["num_experts"], "dtype": "bfloat16"},
        "hidden_states": {"shape": ["seq_len", "hidden_size"], "dtype": "float8_e4m3fn"},
        "hidden_states_scale": {"shape": ["num_hidden_blocks", "seq_len"], "dtype": "float32"},
        "gemm1_weights": {"shape": ["num_local_experts", "gemm1_out_size", "hidden_size"], "dtype": "float8_e4m3fn"},
        "gemm1_weights_scale": {"shape": ["num_local_experts", "num_gemm1_out_blocks", "num_hidden_blocks"],
                                "dtype": "float32"},
        "gemm2_weights": {"shape": ["num_local_experts", "hidden_size", "intermediate_size"], "dtype": "float8_e4m3fn"},
        "gemm2_weights_scale": {"shape": ["num_local_experts", "num_hidden_blocks", "num_intermediate_blocks"],
                                "dtype": "float32"},
        "local_expert_offset": {"shape": None, "dtype": "int32"},
        "routed_scaling_factor": {"shape": None, "dtype": "float32"},
    }
    return {"name": name, "op_type": "moe", "axes": axes, "inputs": inputs,
            "outputs": {"output": {"shape": ["seq_len", "hidden_size"], "dtype": "bfloat16"}},
            "reference": reference}


# A cheap stand-in reference: output row t is routing_logits[t, 0] in every column.
CHEAP_REFERENCE = (
    "import torch\n"
    "def run(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,\n"
    "        gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,\n"
    "        routed_scaling_factor):\n"
    "    T = routing_logits.shape[0]\n"
    "    return (routing_logits[:, :1] * routed_scaling_factor).expand(T, 7168).to(torch.bfloat16)\n"
)


def write_trace_set(root, workloads_spec, E_local=2, reference=CHEAP_REFERENCE, name=None):
    """workloads_spec: list of (uuid, T, config, offset, wrapped)."""
    import fbmoe_trace as ft
    import fbmoe_workloads as w
    from safetensors.torch import save_file
    name = name or ft.DEFINITION_NAME
    os.makedirs(os.path.join(root, "definitions", "moe"), exist_ok=True)
    os.makedirs(os.path.join(root, "workloads", "moe"), exist_ok=True)
    os.makedirs(os.path.join(root, "blob", "workloads", "moe"), exist_ok=True)
    with open(os.path.join(root, "definitions", "moe", f"{name}.json"), "w") as f:
        json.dump(_definition(name, E_local, reference), f)
    blobs = {}
    with open(os.path.join(root, "workloads", "moe", f"{name}.jsonl"), "w") as f:
        for i, (uuid, T, config, offset, wrapped) in enumerate(workloads_spec):
            logits, bias, _, _ = w.make_activations(T, 100 + i, config, "cpu", offset, E_local)
            rel = f"./blob/workloads/moe/{uuid}.safetensors"
            save_file({"routing_logits": logits.contiguous(), "routing_bias": bias.contiguous()},
                      os.path.join(root, rel[2:]))
            blobs[uuid] = (logits, bias)
            wl = {"uuid": uuid, "axes": {"seq_len": T}, "inputs": {
                "routing_logits": {"type": "safetensors", "path": rel, "tensor_key": "routing_logits"},
                "routing_bias": {"type": "safetensors", "path": rel},
                "hidden_states": {"type": "random"},
                "hidden_states_scale": {"type": "random"},
                "gemm1_weights": {"type": "random"},
                "gemm1_weights_scale": {"type": "random"},
                "gemm2_weights": {"type": "random"},
                "gemm2_weights_scale": {"type": "random"},
                "local_expert_offset": {"type": "scalar", "value": offset},
                "routed_scaling_factor": {"type": "scalar", "value": 2.5},
            }}
            obj = {"definition": name, "solution": None, "workload": wl, "evaluation": None} if wrapped else wl
            f.write(json.dumps(obj) + "\n")
    return blobs


@pytest.fixture(scope="module")
def trace():
    import fbmoe_trace as ft
    return ft


@pytest.fixture(scope="module")
def small_set(tmp_path_factory):
    root = str(tmp_path_factory.mktemp("traceset"))
    blobs = write_trace_set(root, [("aaaa-1", 1, "standard", 0, True), ("bbbb-7", 7, "group", 0, False),
                                   ("cccc-3", 3, "standard", 0, True)])
    return root, blobs


def test_loader_reads_definition_and_workloads(trace, small_set):
    root, _ = small_set
    dpath, wpath = trace.find_trace_files(root)
    d = trace.load_definition(dpath)
    assert d.name == trace.DEFINITION_NAME and d.var_axes() == ["seq_len"]
    assert [s.name for s in d.inputs][:2] == ["routing_logits", "routing_bias"]
    assert d.const_axes()["hidden_size"] == H
    ws = trace.load_workloads(wpath)
    assert [w.uuid for w in ws] == ["aaaa-1", "bbbb-7", "cccc-3"]  # wrapped and bare lines
    assert ws[1].axes == {"seq_len": 7}
    assert d.resolve(d.inputs[3], ws[1].axes) == (H // 128, 7)
    assert d.resolve(d.inputs[8], ws[1].axes) is None
    with pytest.raises(FileNotFoundError):
        trace.find_trace_files(root, "no_such_definition")


def test_materialize_files_scalars_and_seeded_randoms(trace, small_set):
    root, blobs = small_set
    dpath, wpath = trace.find_trace_files(root)
    d = trace.load_definition(dpath)
    ws = trace.load_workloads(wpath)
    mat = trace.Materializer(d, root, "cpu", seed=3)
    args = mat(ws[1])
    names = [s.name for s in d.inputs]
    a = dict(zip(names, args))
    logits, bias = blobs["bbbb-7"]
    assert torch.equal(a["routing_logits"], logits) and torch.equal(a["routing_bias"], bias)
    assert a["local_expert_offset"] == 0 and isinstance(a["local_expert_offset"], int)
    assert a["routed_scaling_factor"] == 2.5 and isinstance(a["routed_scaling_factor"], float)
    assert a["hidden_states"].shape == (7, H) and a["hidden_states"].dtype == torch.float8_e4m3fn
    assert a["hidden_states_scale"].shape == (H // 128, 7)
    # Scale and values drawn as a pair: every 1x128 block's largest magnitude quantises to 448.
    q = a["hidden_states"].to(torch.float32).reshape(7, H // 128, 128)
    assert torch.all(q.abs().amax(dim=2) == 448.0)
    assert a["gemm1_weights"].shape == (2, 2 * I, H) and a["gemm2_weights_scale"].shape == (2, H // 128, I // 128)
    # Reproducible per (uuid, seed); another workload draws other activations; weights are shared.
    again = dict(zip(names, trace.Materializer(d, root, "cpu", seed=3)(ws[1])))
    assert torch.equal(again["hidden_states"].view(torch.uint8), a["hidden_states"].view(torch.uint8))
    other = dict(zip(names, mat(ws[2])))
    assert not torch.equal(other["hidden_states"][:3].view(torch.uint8), a["hidden_states"][:3].view(torch.uint8))
    assert other["gemm1_weights"] is a["gemm1_weights"]


def test_materialize_rejects_malformed_workloads(trace, small_set, tmp_path):
    root, _ = small_set
    d = trace.load_definition(trace.find_trace_files(root)[0])
    mat = trace.Materializer(d, root, "cpu")
    base = trace.load_workloads(trace.find_trace_files(root)[1])[0]
    with pytest.raises(ValueError, match="var axes"):
        mat(trace.Workload("x", {}, base.inputs))
    bad = dict(base.inputs)
    bad["routing_logits"] = dict(bad["routing_logits"])
    with pytest.raises(ValueError, match="shape"):
        mat(trace.Workload("x", {"seq_len": 5}, bad))  # the file holds T=1
    bad = dict(base.inputs)
    bad["local_expert_offset"] = {"type": "random"}
    with pytest.raises(ValueError, match="cannot be random"):
        mat(trace.Workload("x", {"seq_len": 1}, bad))
    bad = dict(base.inputs)
    bad["hidden_states"] = {"type": "url"}
    with pytest.raises(ValueError, match="unknown type"):
        mat(trace.Workload("x", {"seq_len": 1}, bad))


def test_error_stats_follow_the_reference_rule(trace):
    ref = torch.ones(1000)
    out = ref.clone()
    assert trace.compute_error_stats(out, ref) == (0.0, 0.0, False, 1.0)
    # Unmatched only when abs > atol AND rel > rtol.
    out[:50] += 2.0          # abs 2 > 1, rel 2 > 0.3: unmatched
    out[50:100] += 0.9       # abs below atol: matched
    max_abs, max_rel, exceeds, matched = trace.compute_error_stats(out, ref)
    assert max_abs == pytest.approx(2.0) and max_rel == pytest.approx(2.0)
    assert matched == pytest.approx(0.95) and not exceeds
    out[100:150] += 2.0      # 10 % unmatched: matched 0.90 is still enough
    assert trace.compute_error_stats(out, ref)[2:] == (False, pytest.approx(0.90))
    out[150:151] += 2.0
    assert trace.compute_error_stats(out, ref)[2] is True
    big = torch.full((10,), 100.0)
    assert trace.compute_error_stats(big * 1.2, big)[3] == 1.0  # abs 20 but rel 0.2 <= 0.3
    assert trace.compute_error_stats(torch.empty(0), torch.empty(0)) == (0.0, 0.0, False, 1.0)


def test_evaluate_statuses_and_row_fields(trace, small_set):
    root, _ = small_set
    dpath, wpath = trace.find_trace_files(root)
    d = trace.load_definition(dpath)
    w = trace.load_workloads(wpath)[1]  # T=7
    args = trace.Materializer(d, root, "cpu")(w)
    ref = d.reference_fn()
    cpu = torch.device("cpu")
    kw = dict(warmup=1, iterations=2, trials=1)

    row = trace.evaluate_workload(d, w, args, ref, ref, cpu, **kw)
    ev = row["evaluation"]
    assert ev["status"] == trace.PASSED and row["solution"] == trace.SOLUTION_NAME
    assert row["workload"]["uuid"] == "bbbb-7" and row["definition"] == d.name
    assert ev["correctness"]["max_absolute_error"] == 0.0 and ev["correctness"]["max_relative_error"] == 0.0
    perf = ev["performance"]
    assert perf["latency_ms"] > 0 and perf["reference_latency_ms"] > 0 and perf["speedup_factor"] > 0
    json.dumps(row)

    def shifted(frac):
        def f(*a):
            o = ref(*a).to(torch.float32).clone().reshape(-1)
            n = int(round(frac * o.numel()))
            o[:n] = o[:n] + 1000.0
            return o.reshape(7, H).to(torch.bfloat16)
        return f

    assert trace.evaluate_workload(d, w, args, shifted(0.05), ref, cpu, **kw)["evaluation"]["status"] == trace.PASSED
    bad = trace.evaluate_workload(d, w, args, shifted(0.2), ref, cpu, **kw)["evaluation"]
    assert bad["status"] == trace.INCORRECT_NUMERICAL and bad["performance"] is None
    assert bad["correctness"]["matched_ratio"] == pytest.approx(0.8, abs=1e-3)
    wrong_shape = trace.evaluate_workload(d, w, args, lambda *a: ref(*a)[:3], ref, cpu, **kw)["evaluation"]
    assert wrong_shape["status"] == trace.INCORRECT_SHAPE
    wrong_dtype = trace.evaluate_workload(d, w, args, lambda *a: ref(*a).float(), ref, cpu, **kw)["evaluation"]
    assert wrong_dtype["status"] == trace.INCORRECT_DTYPE

    def boom(*a):
        raise RuntimeError("launch failed")
    err = trace.evaluate_workload(d, w, args, boom, ref, cpu, **kw)["evaluation"]
    assert err["status"] == trace.RUNTIME_ERROR and "launch failed" in err["log"]

    def nan_out(*a):
        o = ref(*a).clone()
        o[0, 0] = float("nan")
        return o
    assert trace.evaluate_workload(d, w, args, nan_out, ref, cpu, **kw)["evaluation"]["status"] == \
        trace.INCORRECT_NUMERICAL


def test_cli_writes_trace_rows(trace, small_set, tmp_path):
    root, _ = small_set
    sol = tmp_path / "sol.py"
    sol.write_text(CHEAP_REFERENCE.replace("def run(", "def solve("))
    out = tmp_path / "traces.jsonl"
    rc = trace.main(["--trace-set", root, "--solution", f"{sol}::solve", "--device", "cpu", "--out", str(out),
                     "--warmup", "1", "--iterations", "2", "--trials", "1", "--uuid", "aaaa-1", "--uuid", "cccc-3"])
    assert rc == 0
    rows = [json.loads(line) for line in out.read_text().splitlines()]
    assert [r["workload"]["uuid"] for r in rows] == ["aaaa-1", "cccc-3"]
    assert all(r["evaluation"]["status"] == "PASSED" for r in rows)
    assert "speedup" in trace.summarize(rows)


def test_entry_point_syntax(trace, tmp_path):
    with pytest.raises(ValueError):
        trace.load_entry_point("main.py")
    f = tmp_path / "m.py"
    f.write_text("def g():\n    return 7\n")
    assert trace.load_entry_point(f"{f}::g")() == 7


ORACLE_REFERENCE = (
    "import oracle\n"
    "def run(*args):\n"
    "    return oracle.run(*args)\n"
)
PLANTED_REFERENCE = (
    "import oracle\n"
    "def run(*args):\n"
    "    return (oracle.run(*args).float() * 1.5).to(oracle.torch.bfloat16)\n"
)


@pytest.mark.gpu
def test_trace_workloads_pass_on_gpu(trace, oracle_mod, fbmoe_lib, tmp_path):
    """The library's fused_moe on a 32-expert trace set, checked against the oracle as the
    definition's reference, at the build's tolerance with every element matched."""
    root = str(tmp_path / "ts")
    write_trace_set(root, [("g-1", 1, "group", 0, True), ("s-7", 7, "standard", 0, True),
                           ("k-24", 24, "skew", 0, False), ("a-5", 5, "away", 224, True)],
                    E_local=32, reference=ORACLE_REFERENCE)
    rows = trace.evaluate(root, device="cuda", atol=1e-2, rtol=2e-2, required_matched_ratio=1.0,
                          warmup=2, iterations=5, trials=1, time_reference=False)
    assert len(rows) == 4
    for r in rows:
        ev = r["evaluation"]
        assert ev["status"] == trace.PASSED, (r["workload"]["uuid"], ev["log"], ev["correctness"])
        assert ev["correctness"]["matched_ratio"] == 1.0
        assert ev["performance"]["latency_ms"] > 0 and ev["performance"]["reference_latency_ms"] is None


@pytest.mark.gpu
def test_trace_detects_a_planted_reference_error(trace, oracle_mod, fbmoe_lib, tmp_path):
    root = str(tmp_path / "ts")
    write_trace_set(root, [("g-3", 3, "group", 0, True)], E_local=32, reference=PLANTED_REFERENCE)
    rows = trace.evaluate(root, device="cuda", atol=1e-2, rtol=2e-2, required_matched_ratio=1.0,
                          warmup=1, iterations=2, trials=1, time_reference=False)
    assert rows[0]["evaluation"]["status"] == trace.INCORRECT_NUMERICAL
