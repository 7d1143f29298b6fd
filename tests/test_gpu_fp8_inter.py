"""GPU tests of the fp8-intermediate mode (fbmoe_forward_fp8_intermediate, forward(intermediate="fp8")): the
reference solution's numerics, where the SwiGLU output is re-quantised with the 1x128 rule
(solution/triton/main.py:1476-1488) and GEMM2 multiplies fp8 by fp8 (main.py:433-600).

Two comparisons per case, on sampled token rows:
* against the oracle with the same re-quantisation (oracle.run(requant=True)): the operator's tolerance
  (atol 1e-2, rtol 2e-2) must hold on at least 99.9 % of the elements -- the GPU's fp32 sums differ from
  the CPU's in the last bits, which moves an intermediate element across an e4m3 rounding boundary now and
  then;
* against the definition's fp32 intermediate (oracle.run): the fraction within tolerance is the cost of the
  mode.  It is printed and bounded from below only loosely; the f16 default path passes on every element.
T <= 64 runs the decode kernel, which has no fp8 mode: its output must equal fbmoe_forward's bit for bit.
"""
import numpy as np
import pytest
import torch

from conftest import ATOL, RTOL
from test_gpu_parity_bench import local_mask, pick_tokens, weights

pytestmark = pytest.mark.gpu

# name, T, E_local, offset, config, input seed, weight seed, sampled rows
CASES = [
    ("T256_standard", 256, 32, 0, "standard", 11, 4242, 12),
    ("T1024_skew", 1024, 32, 0, "skew", 1024, 4242, 10),
    ("T4096_group", 4096, 32, 0, "group", 4097, 4242, 8),
    ("config3_T8192_E256", 8192, 256, 0, "standard", 0, 1000, 4),
]


@pytest.mark.parametrize("name,T,E,offset,config,seed,wseed,n_sample", CASES, ids=[c[0] for c in CASES])
def test_fp8_intermediate_matches_requant_oracle(oracle_mod, fbmoe_lib, workloads, name, T, E, offset, config, seed,
                                                 wseed, n_sample):
    w = weights(workloads, E, wseed)
    inp = workloads.make_inputs(T, seed=seed, config=config, device="cuda", E_local=E, local_expert_offset=offset,
                                weights=w)
    args = workloads.as_args(inp)
    out = fbmoe_lib.forward(*args, intermediate="fp8", sync_status=True)
    routing = oracle_mod.route(inp["routing_logits"].cpu(), inp["routing_bias"].cpu(), inp["routed_scaling_factor"])
    pick = pick_tokens(routing[0], offset, E, n_sample, seed)
    assert pick.size > 0
    got = out[torch.from_numpy(pick).to(out.device).long()].cpu()
    ref_rq = oracle_mod.run(*args, tokens=pick, routing=routing, requant=True)
    ref = oracle_mod.run(*args, tokens=pick, routing=routing)
    st_rq = oracle_mod.error_stats(got, ref_rq, ATOL, RTOL)
    st = oracle_mod.error_stats(got, ref, ATOL, RTOL)
    print(name, "vs requant oracle", st_rq, "vs fp32 oracle", st)
    assert st_rq["nonfinite"] == 0
    assert st_rq["frac_pass"] >= 0.999, st_rq
    assert st["frac_pass"] >= 0.5, st
    none = np.nonzero(~local_mask(routing[0], offset, E))[0]
    if none.size:
        assert out[torch.from_numpy(none).to(out.device).long()].abs().max().item() == 0.0


def test_fp8_intermediate_is_faster_path_only_for_prefill(fbmoe_lib, workloads):
    """T <= 64 takes the decode kernel in both modes: identical outputs."""
    w = weights(workloads, 32, 4242)
    for T in (1, 16, 64):
        inp = workloads.make_inputs(T, seed=T + 5, config="standard", device="cuda", E_local=32, weights=w)
        a = fbmoe_lib.forward(*workloads.as_args(inp), sync_status=True)
        b = fbmoe_lib.forward(*workloads.as_args(inp), intermediate="fp8", sync_status=True)
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), T


def test_fp8_intermediate_argument_checks(fbmoe_lib, workloads):
    w = weights(workloads, 32, 4242)
    inp = workloads.make_inputs(128, seed=3, config="standard", device="cuda", E_local=32, weights=w)
    with pytest.raises(RuntimeError):
        fbmoe_lib.forward(*workloads.as_args(inp), intermediate="fp8", partial_f32=True)
    with pytest.raises(RuntimeError):
        fbmoe_lib.forward(*workloads.as_args(inp), intermediate="bf16")
