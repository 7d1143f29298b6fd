"""GPU parity of the fused MoE forward (main.py::fused_moe -> fbmoe_forward) against
the reference's golden outputs and against the oracle.

Tolerance (per element, allclose rule): |out - ref| <= 1e-2 + 2e-2 * |ref|; every
element must pass.  Full-size cases are checked on a sample of output rows: each
row depends only on its own token, so the oracle computes just those rows."""
import importlib.util
import os

import numpy as np
import pytest
import torch

from conftest import ATOL, PKG, RTOL, golden_moe_names, rebuild_golden_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def entry():
    spec = importlib.util.spec_from_file_location("fbmoe_main", os.path.join(PKG, "main.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def gpu_weights32(workloads):
    return workloads.make_weights(32, 4242, "cuda")


@pytest.fixture(scope="module")
def cpu_weights32(gpu_weights32):
    return tuple(w.cpu() for w in gpu_weights32)


def _to(inp, device):
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}


def _run(entry, workloads, inp):
    out = entry.fused_moe(*workloads.as_args(inp))
    torch.cuda.synchronize()
    return out


def _check_status(fbmoe_lib, T, E):
    ws = fbmoe_lib.get_workspace(fbmoe_lib.load_library().fbmoe_workspace_size(T, E), torch.device("cuda"),
                                 torch.cuda.current_stream().cuda_stream)
    assert fbmoe_lib.read_status(ws) == 0


@pytest.mark.parametrize("name", golden_moe_names())
def test_forward_matches_reference_golden(oracle_mod, fbmoe_lib, workloads, weights_cache, entry, name):
    inp, ref, z = rebuild_golden_inputs(workloads, name, weights_cache)
    out = _run(entry, workloads, _to(inp, "cuda")).cpu()
    _check_status(fbmoe_lib, int(z["T"]), 32)
    st = oracle_mod.error_stats(out, ref, ATOL, RTOL)
    print(name, st)
    assert st["nonfinite"] == 0
    assert st["frac_pass"] == 1.0, st


CASES = [
    # T, config, offset, n_sample
    (1, "standard", 0, 1),
    (2, "group", 0, 2),
    (7, "away", 224, 7),
    (16, "standard", 0, 16),
    (33, "group", 0, 12),
    (64, "standard", 0, 16),
    (80, "group", 0, 12),
    (901, "standard", 0, 12),
    (1024, "skew", 0, 12),
    (5000, "group", 0, 8),
    (2500, "skew", 0, 12),
    (4097, "standard", 0, 8),
    (4, "zero", 0, 4),
]


@pytest.mark.parametrize("T,config,offset,n_sample", CASES)
def test_forward_matches_oracle(oracle_mod, fbmoe_lib, workloads, entry, gpu_weights32, cpu_weights32,
                                T, config, offset, n_sample):
    inp = workloads.make_inputs(T, seed=100 + T, config=config, device="cuda", local_expert_offset=offset,
                                weights=gpu_weights32)
    out = _run(entry, workloads, inp)
    _check_status(fbmoe_lib, T, 32)
    cpu = _to(inp, "cpu")
    cpu.update(gemm1_weights=cpu_weights32[0], gemm1_weights_scale=cpu_weights32[1],
               gemm2_weights=cpu_weights32[2], gemm2_weights_scale=cpu_weights32[3])
    routing = oracle_mod.route(cpu["routing_logits"], cpu["routing_bias"], cpu["routed_scaling_factor"])
    # sample tokens that have local work first (others must be exactly zero)
    idx = routing[0]
    local = ((idx >= offset) & (idx < offset + 32)).any(1)
    rng = np.random.default_rng(T)
    has = np.nonzero(local)[0]
    pick = rng.choice(has, size=min(n_sample, has.size), replace=False) if has.size else np.array([], int)
    ref = oracle_mod.run(*[cpu[k] for k in workloads.ARG_ORDER], tokens=pick, routing=routing)
    got = out[torch.from_numpy(pick).cuda().long()].cpu() if pick.size else out[:0].cpu()
    st = oracle_mod.error_stats(got, ref, ATOL, RTOL)
    print(T, config, st)
    assert st["nonfinite"] == 0
    assert st["frac_pass"] == 1.0, st
    # tokens without a local expert produce zero rows
    none = np.nonzero(~local)[0]
    if none.size:
        assert out[torch.from_numpy(none).cuda().long()].abs().max().item() == 0.0


def test_forward_is_deterministic(workloads, entry, gpu_weights32):
    inp = workloads.make_inputs(300, seed=5, config="skew", device="cuda", weights=gpu_weights32)
    a = _run(entry, workloads, inp).clone()
    b = _run(entry, workloads, inp)
    assert torch.equal(a, b)


@pytest.mark.parametrize("T", [48, 901, 3000])  # decode-sized kernel; one 1024-token chunk; three chunks
def test_permutation_invariants(oracle_mod, fbmoe_lib, workloads, entry, gpu_weights32, T):
    E = 32
    inp = workloads.make_inputs(T, seed=9, config="standard", device="cuda", weights=gpu_weights32)
    _run(entry, workloads, inp)
    lay = fbmoe_lib.workspace_layout(T, E)
    ws = fbmoe_lib.get_workspace(lay["total"], torch.device("cuda"), torch.cuda.current_stream().cuda_stream)
    def view(name, n, dtype):
        nbytes = n * torch.tensor([], dtype=dtype).element_size()
        return ws[lay[name]:lay[name] + nbytes].view(dtype).cpu()
    cnt = view("expert_cnt", E, torch.int32).numpy()
    poff = view("expert_poff", E + 1, torch.int32).numpy()
    row_token = view("row_token", lay["row_capacity"], torch.int32).numpy()
    token_rows = view("token_rows", T * 8, torch.int32).numpy().reshape(T, 8)
    topk = view("topk_idx", T * 8, torch.int32).numpy().reshape(T, 8)
    ref_idx, _ = oracle_mod.route(inp["routing_logits"].cpu(), inp["routing_bias"].cpu(), 2.5)
    assert np.array_equal(topk, ref_idx)
    local = (topk >= 0) & (topk < E)
    assert cnt.sum() == local.sum()
    assert np.all(poff[:-1] % 16 == 0) and np.all(np.diff(poff) >= cnt)
    for e in range(E):
        seg = row_token[poff[e]:poff[e] + cnt[e]]
        assert np.all(np.diff(seg) > 0)  # token-ascending inside an expert
        toks = np.nonzero((topk == e).any(1))[0]
        assert np.array_equal(seg, toks)
    for t in range(T):
        for k in range(8):
            if local[t, k]:
                r = token_rows[t, k]
                assert row_token[r] == t
            else:
                assert token_rows[t, k] == -1


def test_expert_parallel_shard(oracle_mod, fbmoe_lib, workloads, entry):
    """64 local experts at offset 64 (a world-size-4 shard)."""
    E, off, T = 64, 64, 96
    w = workloads.make_weights(E, 77, "cuda")
    inp = workloads.make_inputs(T, seed=3, config="standard", device="cuda", E_local=E,
                                local_expert_offset=off, weights=w)
    out = _run(entry, workloads, inp)
    _check_status(fbmoe_lib, T, E)
    cpu = _to(inp, "cpu")
    routing = oracle_mod.route(cpu["routing_logits"], cpu["routing_bias"], 2.5)
    local = ((routing[0] >= off) & (routing[0] < off + E)).any(1)
    pick = np.nonzero(local)[0][:10]
    ref = oracle_mod.run(*[cpu[k] for k in workloads.ARG_ORDER], tokens=pick, routing=routing)
    st = oracle_mod.error_stats(out[torch.from_numpy(pick).cuda().long()].cpu(), ref, ATOL, RTOL)
    print(st)
    assert st["frac_pass"] == 1.0, st


@pytest.mark.parametrize("T,config", [(40, "standard"), (64, "group")])
def test_decode_all_256_experts(oracle_mod, fbmoe_lib, workloads, entry, T, config):
    """Decode path (T <= 64) with all 256 experts local (the N=1 expert-parallel layout): many blocks, so the
    decode kernel's balanced ranges cut GEMM1 units into several segments and GEMM2 units into two planes."""
    E = 256
    w = workloads.make_weights(E, 91, "cuda")
    inp = workloads.make_inputs(T, seed=17 + T, config=config, device="cuda", E_local=E, weights=w)
    out = _run(entry, workloads, inp)
    _check_status(fbmoe_lib, T, E)
    cpu = _to(inp, "cpu")
    routing = oracle_mod.route(cpu["routing_logits"], cpu["routing_bias"], 2.5)
    pick = np.random.default_rng(T).choice(T, size=4, replace=False)
    ref = oracle_mod.run(*[cpu[k] for k in workloads.ARG_ORDER], tokens=pick, routing=routing)
    st = oracle_mod.error_stats(out[torch.from_numpy(pick).cuda().long()].cpu(), ref, ATOL, RTOL)
    print(T, config, st)
    assert st["nonfinite"] == 0
    assert st["frac_pass"] == 1.0, st
    del w
    torch.cuda.empty_cache()
