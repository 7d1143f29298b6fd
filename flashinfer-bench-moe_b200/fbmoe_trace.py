"""FlashInfer-Trace workloads in, flashinfer-bench trace rows out, for the fused MoE definition.

The reference is benchmarked by flashinfer-bench on the contest's trace set
(scripts/run_local.py:30-75). That harness loads the definition and its
workloads, materialises each workload's inputs, checks the solution against
the definition's reference ``run`` under a matched-ratio rule, times both, and
dumps one trace per workload. The reference also has its own small loader for
the same files (solution/triton/main.py:2807-2833). This module restates that
loop for the one definition this library implements, so the library can be run
on the real workloads whenever a trace set is present. The contest dataset
(flashinfer-ai/mlsys26-contest) is not part of this repository.

Trace-set layout (FlashInfer-Trace):

* ``definitions/<op_type>/<name>.json``: ``axes`` (``{"type": "const", "value": v}``
  or ``{"type": "var"}``), ``inputs``/``outputs`` (``{"shape": [axis names] | null,
  "dtype": ...}``), and ``reference`` (Python source that defines ``run``);
* ``workloads/<op_type>/<name>.jsonl``: one object per line, either wrapped
  (``{"definition", "workload": {...}}``, as main.py:2818 reads it) or bare, with
  ``uuid``, ``axes`` (values of the var axes) and ``inputs``. Each input is one of
  ``{"type": "safetensors", "path": "./blob/...", "tensor_key": k}``
  (``tensor_key`` defaults to the input's name, as at main.py:2825-2826),
  ``{"type": "scalar", "value": v}``, or ``{"type": "random"}``;
* ``blob/...``: the safetensors files. A relative path is taken from the trace-set
  root (main.py:2822 strips the leading ``.``).

Random inputs are filled the way this library's synthetic workloads are, so
that the numbers are meaningful. Activations are N(0,1) quantised 1x128 with
``scale = amax/448``; weights are N(0,0.02) quantised 128x128. A quantised
tensor and its scale are always drawn as a pair. Logits are N(0,1) and the bias
is N(0,0.1). Activation seeds come from the workload's uuid. Weight seeds come
only from the base seed, so one weight set serves every workload of a run.

Trace rows carry the fields that run_local.py:61-74 reads, under the same names:
``evaluation.status``, ``solution``, ``workload.uuid``,
``evaluation.performance.{latency_ms, reference_latency_ms, speedup_factor}`` and
``evaluation.correctness.{max_absolute_error, max_relative_error}``.

Usage::

    python fbmoe_trace.py --trace-set DIR [--out traces.jsonl] [--solution main.py::fused_moe]
"""
from __future__ import annotations

import argparse
import datetime
import glob
import importlib.util
import json
import os
import sys
import time
import zlib
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence, Tuple

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

import torch  # noqa: E402

import fbmoe_workloads as _wl  # noqa: E402

DEFINITION_NAME = "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"  # config.toml:3
SOLUTION_NAME = "fbmoe-b200"

# BenchmarkConfig of scripts/run_local.py:33.
DEFAULT_WARMUP = 3
DEFAULT_ITERATIONS = 100
DEFAULT_TRIALS = 5
DEFAULT_ATOL = 1.0
DEFAULT_RTOL = 0.3
DEFAULT_MATCHED_RATIO = 0.9

# Status strings of flashinfer-bench's evaluation.
PASSED = "PASSED"
INCORRECT_SHAPE = "INCORRECT_SHAPE"
INCORRECT_DTYPE = "INCORRECT_DTYPE"
INCORRECT_NUMERICAL = "INCORRECT_NUMERICAL"
RUNTIME_ERROR = "RUNTIME_ERROR"

_DTYPES = {
    "float32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "float8_e4m3fn": torch.float8_e4m3fn,
    "float8_e5m2": torch.float8_e5m2,
    "int32": torch.int32,
    "int64": torch.int64,
    "bool": torch.bool,
}

# Quantised tensors drawn as a pair with their scale: value name -> scale name.
_ACT_PAIRS = {"hidden_states": "hidden_states_scale"}
_WEIGHT_NAMES = ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")


def torch_dtype(name: str) -> torch.dtype:
    try:
        return _DTYPES[name]
    except KeyError:
        raise ValueError(f"unsupported dtype {name!r} in the definition") from None


@dataclass
class TensorSpec:
    name: str
    shape: Optional[List[str]]  # axis names; None for a scalar
    dtype: str


@dataclass
class Definition:
    name: str
    op_type: str
    axes: Dict[str, Dict[str, Any]]
    inputs: List[TensorSpec]
    outputs: List[TensorSpec]
    reference: Optional[str]
    path: str = ""

    def const_axes(self) -> Dict[str, int]:
        return {k: int(v["value"]) for k, v in self.axes.items() if v.get("type") == "const"}

    def var_axes(self) -> List[str]:
        return [k for k, v in self.axes.items() if v.get("type") != "const"]

    def resolve(self, spec: TensorSpec, var_values: Dict[str, int]) -> Optional[Tuple[int, ...]]:
        """Concrete shape of ``spec`` under the workload's var-axis values."""
        if spec.shape is None:
            return None
        values = dict(self.const_axes())
        values.update({k: int(v) for k, v in var_values.items()})
        out = []
        for ax in spec.shape:
            if isinstance(ax, int):
                out.append(ax)
            elif ax in values:
                out.append(values[ax])
            else:
                raise ValueError(f"{self.name}: axis {ax!r} of {spec.name!r} has no value in the workload")
        return tuple(out)

    def reference_fn(self) -> Callable:
        """The definition's ``run``, compiled from its ``reference`` source.

        Like the harness, this executes code that the trace set ships, so only
        load trace sets from a trusted source."""
        if not self.reference:
            raise ValueError(f"definition {self.name!r} carries no reference source")
        ns: Dict[str, Any] = {"__name__": f"fbmoe_trace_reference_{self.name}"}
        exec(compile(self.reference, f"<reference of {self.name}>", "exec"), ns)
        if "run" not in ns:
            raise ValueError(f"definition {self.name!r}: reference source defines no run()")
        return ns["run"]


@dataclass
class Workload:
    uuid: str
    axes: Dict[str, int]
    inputs: Dict[str, Dict[str, Any]]
    raw: Dict[str, Any] = field(default_factory=dict)


def _specs(d: Dict[str, Any]) -> List[TensorSpec]:
    return [TensorSpec(k, v.get("shape"), v["dtype"]) for k, v in d.items()]


def load_definition(path: str) -> Definition:
    with open(path, "r", encoding="utf-8") as f:
        d = json.load(f)
    return Definition(
        name=d["name"],
        op_type=d.get("op_type", ""),
        axes=d.get("axes", {}),
        inputs=_specs(d["inputs"]),
        outputs=_specs(d.get("outputs", {})),
        reference=d.get("reference"),
        path=path,
    )


def load_workloads(path: str) -> List[Workload]:
    """Every workload of a JSONL file (wrapped or bare objects), in file order."""
    out = []
    with open(path, "r", encoding="utf-8") as f:
        for n, line in enumerate(f, 1):
            line = line.strip()
            if not line:
                continue
            item = json.loads(line)
            w = item.get("workload", item)
            if "inputs" not in w:
                raise ValueError(f"{path}:{n}: workload has no inputs")
            out.append(Workload(uuid=str(w.get("uuid", f"line{n}")), axes=dict(w.get("axes", {})),
                                inputs=dict(w["inputs"]), raw=w))
    return out


def find_trace_files(root: str, name: str = DEFINITION_NAME) -> Tuple[str, str]:
    """Paths of ``definitions/**/<name>.json`` and ``workloads/**/<name>.jsonl`` under ``root``."""
    defs = sorted(glob.glob(os.path.join(root, "definitions", "**", f"{name}.json"), recursive=True))
    wls = sorted(glob.glob(os.path.join(root, "workloads", "**", f"{name}.jsonl"), recursive=True))
    if not defs:
        raise FileNotFoundError(f"definition {name!r} not found under {root}/definitions")
    if not wls:
        raise FileNotFoundError(f"no workloads for {name!r} under {root}/workloads")
    return defs[0], wls[0]


class _Blobs:
    """Safetensors files read once per run, on the target device."""

    def __init__(self, root: str, device: torch.device):
        self.root = root
        self.device = device
        self.cache: Dict[str, Dict[str, torch.Tensor]] = {}

    def get(self, rel: str, key: str) -> torch.Tensor:
        path = rel if os.path.isabs(rel) else os.path.join(self.root, rel)
        path = os.path.normpath(path)
        if path not in self.cache:
            from safetensors.torch import load_file
            self.cache[path] = load_file(path, device=str(self.device))
        tensors = self.cache[path]
        if key not in tensors:
            raise KeyError(f"{path} holds no tensor {key!r}")
        return tensors[key]


def workload_seed(uuid: str, base_seed: int) -> int:
    return (zlib.crc32(uuid.encode("utf-8")) + 7919 * int(base_seed)) & 0x7FFFFFFF


class Materializer:
    """Turns a workload into the definition's positional arguments on ``device``."""

    def __init__(self, definition: Definition, root: str, device="cpu", seed: int = 0):
        self.defn = definition
        self.root = root
        self.device = torch.device(device)
        self.seed = int(seed)
        self.blobs = _Blobs(root, self.device)
        self._weights: Dict[Tuple, Tuple[torch.Tensor, ...]] = {}

    def _weights_for(self, E_local: int) -> Tuple[torch.Tensor, ...]:
        key = (E_local, str(self.device))
        if key not in self._weights:
            self._weights[key] = _wl.make_weights(E_local, self.seed + 1000, str(self.device))
        return self._weights[key]

    def _random(self, spec: TensorSpec, shape, g: torch.Generator, made: Dict[str, Any],
                specs: Dict[str, TensorSpec], var_values: Dict[str, int]):
        dt = torch_dtype(spec.dtype)
        name = spec.name
        if shape is None:
            raise ValueError(f"scalar input {name!r} cannot be random; the workload must give its value")
        if name in _WEIGHT_NAMES:
            w = self._weights_for(int(shape[0]))
            t = w[_WEIGHT_NAMES.index(name)]
        elif name in _ACT_PAIRS or name in _ACT_PAIRS.values():
            value = name if name in _ACT_PAIRS else next(k for k, v in _ACT_PAIRS.items() if v == name)
            vshape = self.defn.resolve(specs[value], var_values)
            x = torch.randn(vshape, generator=g, device=self.device, dtype=torch.float32)
            q, s = _wl.quantize_act_1x128(x)
            made.setdefault(value, q)
            made.setdefault(_ACT_PAIRS[value], s)
            t = made[name]
        elif name == "routing_bias":
            t = torch.randn(shape, generator=g, device=self.device, dtype=torch.float32) * 0.1
        elif dt.is_floating_point:
            t = torch.randn(shape, generator=g, device=self.device, dtype=torch.float32)
        else:
            t = torch.zeros(shape, dtype=dt, device=self.device)
        t = t.to(dt)
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"random {name!r}: generated shape {tuple(t.shape)} != definition {tuple(shape)}")
        return t

    def __call__(self, w: Workload) -> List[Any]:
        specs = {s.name: s for s in self.defn.inputs}
        missing = [v for v in self.defn.var_axes() if v not in w.axes]
        if missing:
            raise ValueError(f"workload {w.uuid}: no value for var axes {missing}")
        g = torch.Generator(device=self.device)
        g.manual_seed(workload_seed(w.uuid, self.seed))
        made: Dict[str, Any] = {}
        # Files and scalars first, so that a random partner of a given tensor never replaces it.
        order = sorted(self.defn.inputs, key=lambda s: w.inputs.get(s.name, {}).get("type", "random") == "random")
        for spec in order:
            if spec.name in made:
                continue
            desc = w.inputs.get(spec.name, {"type": "random"})
            kind = desc.get("type", "random")
            shape = self.defn.resolve(spec, w.axes)
            if kind == "scalar":
                v = desc["value"]
                made[spec.name] = float(v) if spec.dtype.startswith(("float", "bfloat")) else int(v)
            elif kind == "safetensors":
                t = self.blobs.get(desc["path"], desc.get("tensor_key", spec.name))
                if shape is not None and tuple(t.shape) != shape:
                    raise ValueError(f"workload {w.uuid}: {spec.name} has shape {tuple(t.shape)}, "
                                     f"definition wants {shape}")
                if t.dtype != torch_dtype(spec.dtype):
                    raise ValueError(f"workload {w.uuid}: {spec.name} is {t.dtype}, definition wants {spec.dtype}")
                made[spec.name] = t
            elif kind == "random":
                made[spec.name] = self._random(spec, shape, g, made, specs, w.axes)
            else:
                raise ValueError(f"workload {w.uuid}: input {spec.name!r} has unknown type {kind!r}")
        return [made[s.name] for s in self.defn.inputs]


def compute_error_stats(output: torch.Tensor, reference: torch.Tensor, atol: float = DEFAULT_ATOL,
                        rtol: float = DEFAULT_RTOL,
                        required_matched_ratio: Optional[float] = DEFAULT_MATCHED_RATIO):
    """(max_abs, max_rel, exceeds_tol, matched_ratio) under the reference's rule
    (main.py:2776-2805): an element is unmatched only when its absolute error
    exceeds ``atol`` AND its relative error (against ``|ref| + 1e-8``) exceeds
    ``rtol``; the output fails when the matched fraction is below
    ``required_matched_ratio`` (0.9 when None)."""
    x = output.to(torch.float32)
    y = reference.to(device=x.device, dtype=torch.float32)
    abs_err = (x - y).abs()
    rel_err = abs_err / (y.abs() + 1e-8)
    n = abs_err.numel()
    if n == 0:
        return 0.0, 0.0, False, 1.0
    need = 0.9 if required_matched_ratio is None else float(required_matched_ratio)
    exceeds = float(((abs_err > atol) & (rel_err > rtol)).sum().item())
    matched = max(0.0, min(1.0, 1.0 - exceeds / float(n)))
    return float(abs_err.max().item()), float(rel_err.max().item()), matched < need, matched


def _flush_buffer(device: torch.device) -> Optional[torch.Tensor]:
    if device.type != "cuda":
        return None
    return torch.empty(256 << 20, dtype=torch.uint8, device=device)  # twice the 126 MB L2


def time_call(fn: Callable, args: Sequence[Any], device: torch.device, warmup: int, iterations: int,
              trials: int) -> float:
    """Mean milliseconds per call, the median over ``trials``. On a GPU each call is
    bracketed by CUDA events on the current stream, with L2 flushed before it."""
    for _ in range(warmup):
        fn(*args)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        flush = _flush_buffer(device)
        per_trial = []
        for _ in range(trials):
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
            for i in range(iterations):
                flush.fill_(i & 0xFF)
                starts[i].record()
                fn(*args)
                ends[i].record()
            torch.cuda.synchronize(device)
            per_trial.append(sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / iterations)
        del flush
    else:
        per_trial = []
        for _ in range(trials):
            t0 = time.perf_counter()
            for _ in range(iterations):
                fn(*args)
            per_trial.append((time.perf_counter() - t0) * 1e3 / iterations)
    per_trial.sort()
    return per_trial[len(per_trial) // 2]


def environment(device: torch.device) -> Dict[str, Any]:
    hw = torch.cuda.get_device_name(device) if device.type == "cuda" else "cpu"
    return {"hardware": hw, "libs": {"torch": torch.__version__, "cuda": torch.version.cuda}}


def evaluate_workload(defn: Definition, w: Workload, args: Sequence[Any], solution: Callable,
                      reference: Callable, device: torch.device, *, solution_name: str = SOLUTION_NAME,
                      atol: float = DEFAULT_ATOL, rtol: float = DEFAULT_RTOL,
                      required_matched_ratio: float = DEFAULT_MATCHED_RATIO, warmup: int = DEFAULT_WARMUP,
                      iterations: int = DEFAULT_ITERATIONS, trials: int = DEFAULT_TRIALS,
                      time_reference: bool = True) -> Dict[str, Any]:
    """One trace row: correctness against ``reference``, then timing when it passed."""
    ev: Dict[str, Any] = {"status": None, "log": "", "environment": environment(device),
                          "timestamp": datetime.datetime.now(datetime.timezone.utc).isoformat(),
                          "correctness": None, "performance": None}
    row = {"definition": defn.name, "workload": w.raw or {"uuid": w.uuid, "axes": w.axes, "inputs": w.inputs},
           "solution": solution_name, "evaluation": ev}
    ref = reference(*args)
    if isinstance(ref, (tuple, list)):
        ref = ref[0]
    try:
        out = solution(*args)
        if device.type == "cuda":
            torch.cuda.synchronize(device)
    except Exception as exc:  # the harness records the failure and moves on
        ev["status"], ev["log"] = RUNTIME_ERROR, f"{type(exc).__name__}: {exc}"
        return row
    if isinstance(out, (tuple, list)):
        out = out[0]
    want_shape = defn.resolve(defn.outputs[0], w.axes) if defn.outputs else tuple(ref.shape)
    if tuple(out.shape) != tuple(want_shape):
        ev["status"], ev["log"] = INCORRECT_SHAPE, f"output shape {tuple(out.shape)} != {tuple(want_shape)}"
        return row
    if defn.outputs and out.dtype != torch_dtype(defn.outputs[0].dtype):
        ev["status"], ev["log"] = INCORRECT_DTYPE, f"output dtype {out.dtype} != {defn.outputs[0].dtype}"
        return row
    max_abs, max_rel, exceeds, matched = compute_error_stats(out, ref, atol, rtol, required_matched_ratio)
    finite = bool(torch.isfinite(out.to(torch.float32)).all().item())
    ev["correctness"] = {"max_absolute_error": max_abs, "max_relative_error": max_rel, "matched_ratio": matched}
    if exceeds or not finite:
        ev["status"] = INCORRECT_NUMERICAL
        ev["log"] = f"matched ratio {matched:.6f} < {required_matched_ratio}" if finite else "non-finite output"
        return row
    lat = time_call(solution, args, device, warmup, iterations, trials)
    ref_lat = time_call(reference, args, device, min(warmup, 1), max(1, iterations // 20), 1) if time_reference else None
    ev["performance"] = {"latency_ms": lat, "reference_latency_ms": ref_lat,
                         "speedup_factor": (ref_lat / lat) if (ref_lat and lat > 0) else None}
    ev["status"] = PASSED
    return row


def evaluate(root: str, *, definition: str = DEFINITION_NAME, solution: Optional[Callable] = None,
             reference: Optional[Callable] = None, device=None, seed: int = 0,
             uuids: Optional[Iterable[str]] = None, **kw) -> List[Dict[str, Any]]:
    """Evaluate ``solution`` (default: this library's ``fused_moe``) on every
    workload of ``definition`` in the trace set at ``root``."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    device = torch.device(device)
    dpath, wpath = find_trace_files(root, definition)
    defn = load_definition(dpath)
    if defn.name != definition:
        raise ValueError(f"{dpath} names definition {defn.name!r}, expected {definition!r}")
    if solution is None:
        solution = load_entry_point("main.py::fused_moe")
    if reference is None:
        reference = defn.reference_fn()
    wanted = set(uuids) if uuids is not None else None
    mat = Materializer(defn, root, device, seed)
    rows = []
    for w in load_workloads(wpath):
        if wanted is not None and w.uuid not in wanted:
            continue
        args = mat(w)
        rows.append(evaluate_workload(defn, w, args, solution, reference, device, **kw))
        del args
    return rows


def load_entry_point(spec: str, base: str = _HERE) -> Callable:
    """``"file.py::function"`` (the ``entry_point`` syntax of config.toml:8), the file
    taken relative to ``base`` unless absolute."""
    path, _, fn = spec.partition("::")
    if not fn:
        raise ValueError(f"entry point {spec!r} is not of the form file.py::function")
    path = path if os.path.isabs(path) else os.path.join(base, path)
    mod_name = "fbmoe_entry_" + os.path.splitext(os.path.basename(path))[0]
    s = importlib.util.spec_from_file_location(mod_name, path)
    if s is None or s.loader is None:
        raise ImportError(f"cannot load {path}")
    mod = importlib.util.module_from_spec(s)
    s.loader.exec_module(mod)
    return getattr(mod, fn)


def summarize(rows: Sequence[Dict[str, Any]]) -> str:
    """Console summary in the shape of run_local.py:78-98."""
    lines = []
    for r in rows:
        ev = r["evaluation"]
        uuid = str(r["workload"].get("uuid", "?"))
        s = f"  Workload {uuid[:8]}...: {ev['status']}"
        perf, corr = ev.get("performance"), ev.get("correctness")
        if perf and perf.get("latency_ms") is not None:
            s += f" | {perf['latency_ms']:.3f} ms"
        if perf and perf.get("speedup_factor") is not None:
            s += f" | {perf['speedup_factor']:.2f}x speedup"
        if corr and corr.get("max_absolute_error") is not None:
            s += f" | abs_err={corr['max_absolute_error']:.2e}, rel_err={corr['max_relative_error']:.2e}"
        lines.append(s)
    return "\n".join(lines)


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--trace-set", default=os.environ.get("FIB_DATASET_PATH"),
                    help="trace-set root (default: $FIB_DATASET_PATH, as run_local.py:19-27)")
    ap.add_argument("--definition", default=DEFINITION_NAME)
    ap.add_argument("--solution", default="main.py::fused_moe", help="file.py::function")
    ap.add_argument("--solution-name", default=SOLUTION_NAME)
    ap.add_argument("--out", default=None, help="write the trace rows here as JSONL")
    ap.add_argument("--device", default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--uuid", action="append", default=None, help="only these workloads (repeatable)")
    ap.add_argument("--warmup", type=int, default=DEFAULT_WARMUP)
    ap.add_argument("--iterations", type=int, default=DEFAULT_ITERATIONS)
    ap.add_argument("--trials", type=int, default=DEFAULT_TRIALS)
    ap.add_argument("--atol", type=float, default=DEFAULT_ATOL)
    ap.add_argument("--rtol", type=float, default=DEFAULT_RTOL)
    ap.add_argument("--required-matched-ratio", type=float, default=DEFAULT_MATCHED_RATIO)
    ap.add_argument("--no-reference-timing", action="store_true")
    a = ap.parse_args(argv)
    if not a.trace_set:
        ap.error("--trace-set (or FIB_DATASET_PATH) is required")
    solution = None if a.solution == "main.py::fused_moe" else load_entry_point(a.solution, os.getcwd())
    rows = evaluate(a.trace_set, definition=a.definition, solution=solution, device=a.device, seed=a.seed, uuids=a.uuid,
                    solution_name=a.solution_name, atol=a.atol, rtol=a.rtol,
                    required_matched_ratio=a.required_matched_ratio, warmup=a.warmup, iterations=a.iterations,
                    trials=a.trials, time_reference=not a.no_reference_timing)
    if a.out:
        with open(a.out, "w", encoding="utf-8") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")
    print(f"\n{a.definition}:")
    print(summarize(rows))
    return 0 if all(r["evaluation"]["status"] == PASSED for r in rows) else 1


if __name__ == "__main__":
    sys.exit(main())
