"""Generates the golden fixtures in tests/golden/ from the REFERENCE's own code.

Run in a container where the reference checkout is mounted (read-only):

    python tests/golden/make_golden.py --reference <path-to-flashinfer-bench-moe>

It extracts ``run()`` from ``solution/triton/main.py`` (lines 2430-2609) with
``ast`` -- the module itself cannot be imported without a GPU -- and executes
it on CPU.  Two kinds of fixtures are written:

* ``routing_<case>.npz``: inputs (logits, bias) and the reference routing
  (torch.topk indices in torch's own order and the combination weights), taken
  from the routing statements of ``run()`` (main.py:2522-2553).
* ``moe_<case>.npz``: the seeds/configs used to regenerate the inputs with
  ``fbmoe_workloads.make_inputs(device="cpu")``, input checksums, the reference
  routing, and the reference's bf16 output of ``run()``.

Nothing at test time reads the reference; the fixtures are the pin.
"""
from __future__ import annotations

import argparse
import ast
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "flashinfer-bench-moe_b200"))
import fbmoe_workloads as W  # noqa: E402


def tensor_checksum(t: torch.Tensor) -> str:
    """Order-sensitive 64-bit checksum of a tensor's bytes (fast, numpy-vectorised)."""
    b = t.detach().cpu().reshape(-1).clone().view(torch.uint8).numpy()
    pad = (-b.size) % 8
    if pad:
        b = np.concatenate([b, np.zeros(pad, dtype=np.uint8)])
    v = b.view(np.uint64)
    k = (np.arange(v.size, dtype=np.uint64) % np.uint64(65521)) + np.uint64(1)
    with np.errstate(over="ignore"):
        s = int(np.sum(v * k, dtype=np.uint64))
        s2 = int(np.sum(v ^ (k * np.uint64(0x9E3779B97F4A7C15)), dtype=np.uint64))
    return f"{s:016x}{s2:016x}"


def load_reference(ref_root: str):
    path = os.path.join(ref_root, "solution", "triton", "main.py")
    src = open(path).read()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "run")
    ns = {"torch": torch}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), path, "exec"), ns)
    run = ns["run"]

    # Routing-only function: the statements of run() from the logits cast to the weights.
    body = fn.body
    start = next(i for i, s in enumerate(body) if isinstance(s, ast.Assign)
                 and ast.unparse(s.targets[0]) == "logits")
    end = next(i for i, s in enumerate(body) if isinstance(s, ast.Assign)
               and ast.unparse(s.targets[0]) == "weights"
               and "routed_scaling_factor" in ast.unparse(s.value))
    prelude = ast.parse(
        "T = routing_logits.shape[0]\nE_global = routing_logits.shape[1]\n"
        "TOP_K = 8\nN_GROUP = 8\nTOPK_GROUP = 4\n").body
    ret = ast.parse("return topk_idx, weights, s_with_bias").body
    rfn = ast.FunctionDef(
        name="ref_route",
        args=ast.arguments(posonlyargs=[], args=[ast.arg("routing_logits"), ast.arg("routing_bias"),
                                                  ast.arg("routed_scaling_factor")],
                           kwonlyargs=[], kw_defaults=[], defaults=[]),
        body=prelude + body[start:end + 1] + ret, decorator_list=[], returns=None, type_params=[])
    mod = ast.fix_missing_locations(ast.Module(body=[rfn], type_ignores=[]))
    exec(compile(mod, path, "exec"), ns)
    return run, ns["ref_route"]


def routing_cases():
    g = torch.Generator().manual_seed(7)
    cases = {}
    cases["normal"] = (torch.randn(512, 256, generator=g), torch.randn(256, generator=g) * 0.1)
    # heavy ties: logits on a coarse grid, bias with duplicates
    grid = torch.randint(-3, 4, (512, 256), generator=g).float() * 0.5
    cases["grid"] = (grid, (torch.randint(-2, 3, (256,), generator=g).float() * 0.05))
    cases["zero"] = (torch.zeros(8, 256), torch.randn(256, generator=g) * 0.1)
    cases["zero_zero"] = (torch.zeros(4, 256), torch.zeros(256))
    lg = torch.randn(256, 256, generator=g)
    lg[:, 0:32] += 5.0
    cases["group"] = (lg, torch.randn(256, generator=g) * 0.1)
    la = torch.randn(256, 256, generator=g)
    la[:, 224:256] -= 5.0
    cases["away"] = (la, torch.randn(256, generator=g) * 0.1)
    b = torch.randn(256, generator=g) * 0.1
    b[[0, 9, 18, 27]] += 3.0
    cases["skew"] = (torch.randn(256, 256, generator=g), b)
    out = {}
    for name, (lg_, b_) in cases.items():
        out[name] = (lg_.float().contiguous(), b_.to(torch.bfloat16))
    return out


MOE_CASES = [
    # name, T, config, seed, local_expert_offset, weight_seed, scale
    ("t16_standard", 16, "standard", 0, 0, 1000, 2.5),
    ("t7_offset224_away", 7, "away", 3, 224, 1003, 2.5),
    ("t4_zero", 4, "zero", 5, 0, 1000, 1.11),
    ("t1_group", 1, "group", 9, 0, 1000, 2.5),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="")
    ap.add_argument("--cases", default="", help="comma-separated moe case names (default: all)")
    args = ap.parse_args()
    run, ref_route = load_reference(args.reference)
    torch.set_num_threads(os.cpu_count())

    if args.only in ("", "routing"):
        for name, (lg, b) in routing_cases().items():
            idx, w, sb = ref_route(lg, b, 2.5)
            wsel = torch.gather(w, 1, idx)
            np.savez_compressed(os.path.join(HERE, f"routing_{name}.npz"),
                                logits=lg.numpy(), bias_bits=b.view(torch.int16).numpy(),
                                scale=np.float32(2.5), ref_idx=idx.numpy().astype(np.int32),
                                ref_w=wsel.numpy().astype(np.float32))
            print("routing", name, lg.shape)

    if args.only in ("", "moe"):
        weight_cache = {}
        wanted = set(filter(None, args.cases.split(",")))
        for name, T, cfg, seed, off, wseed, scale in MOE_CASES:
            if wanted and name not in wanted:
                continue
            if wseed not in weight_cache:
                t0 = time.time()
                weight_cache[wseed] = W.make_weights(32, wseed, "cpu")
                print("weights", wseed, f"{time.time() - t0:.1f}s")
            inp = W.make_inputs(T, seed=seed, config=cfg, device="cpu", E_local=32,
                                local_expert_offset=off, routed_scaling_factor=scale,
                                weights=weight_cache[wseed])
            sums = {k: tensor_checksum(v) for k, v in inp.items() if isinstance(v, torch.Tensor)}
            t0 = time.time()
            out = run(*W.as_args(inp))
            dt = time.time() - t0
            idx, w, _ = ref_route(inp["routing_logits"], inp["routing_bias"], scale)
            np.savez_compressed(
                os.path.join(HERE, f"moe_{name}.npz"),
                T=np.int32(T), config=np.array(cfg), seed=np.int32(seed), offset=np.int32(off),
                weight_seed=np.int32(wseed), scale=np.float32(scale),
                checksum_keys=np.array(sorted(sums)), checksum_vals=np.array([sums[k] for k in sorted(sums)]),
                ref_idx=idx.numpy().astype(np.int32), ref_w=torch.gather(w, 1, idx).numpy().astype(np.float32),
                out_bits=out.view(torch.int16).numpy())
            print("moe", name, f"run() {dt:.1f}s", "nonzero rows", int((out.float().abs().sum(1) > 0).sum()))


if __name__ == "__main__":
    main()
