"""CPU tests: the oracle is pinned to the reference before it is trusted.

* the tie-exact selection equals std::nth_element and torch.topk(sorted=False);
* routing equals the reference's own routing code (golden fixtures made by
  tests/golden/make_golden.py from solution/triton/main.py:2522-2553);
* the full oracle equals the reference's run() outputs (golden fixtures).
"""
import os
import subprocess

import numpy as np
import pytest
import torch

from conftest import ATOL, ORACLE, RTOL, golden_moe_names, golden_routing_names, rebuild_golden_inputs


def test_nth_element_matches_libstdcxx(oracle_mod):
    exe = os.path.join(ORACLE, "_build", "nth_check")
    r = subprocess.run([exe, "100000"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mismatches=0" in r.stdout


@pytest.mark.parametrize("n,k", [(256, 8), (32, 2), (8, 4), (128, 8), (20, 3)])
def test_topk_nth_matches_torch_topk(oracle_mod, n, k):
    g = torch.Generator().manual_seed(n * 131 + k)
    for trial in range(300):
        nuniq = [1, 2, 3, 7, 1000][trial % 5]
        v = torch.randint(0, nuniq, (n,), generator=g).float()
        if trial % 7 == 0:
            v = torch.randn(n, generator=g)
        ref = torch.topk(v, k, sorted=False).indices.numpy().astype(np.int32)
        got = oracle_mod.topk_nth(v.numpy(), k)
        assert np.array_equal(ref, got), (v.tolist(), ref, got)


@pytest.mark.parametrize("name", golden_routing_names())
def test_routing_matches_reference_fixture(oracle_mod, name):
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", f"routing_{name}.npz"))
    logits = torch.from_numpy(z["logits"])
    bias = torch.from_numpy(z["bias_bits"]).view(torch.bfloat16)
    idx, w = oracle_mod.route(logits, bias, float(z["scale"]))
    ref_idx = z["ref_idx"]
    ref_w = z["ref_w"]
    # same set of experts per token
    assert np.array_equal(np.sort(idx, 1), np.sort(ref_idx, 1))
    # same weight per expert (weights are normalised sums: a few ulp of fp32)
    order_ref = np.argsort(ref_idx, 1)
    order_got = np.argsort(idx, 1)
    wr = np.take_along_axis(ref_w, order_ref, 1)
    wg = np.take_along_axis(w, order_got, 1)
    np.testing.assert_allclose(wg, wr, rtol=2e-6, atol=1e-7)


def test_routing_tie_flags_cover_fixture_ties(oracle_mod):
    """The all-zero-logit fixtures really exercise boundary ties."""
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "routing_zero_zero.npz"))
    idx, w, sb, tie = oracle_mod.route(torch.from_numpy(z["logits"]),
                                       torch.from_numpy(z["bias_bits"]).view(torch.bfloat16), 2.5,
                                       with_details=True)
    assert (tie & 3).all()  # every group and every expert ties when all scores are equal
    assert np.array_equal(np.sort(idx, 1), np.sort(z["ref_idx"], 1))


def test_routing_random_matches_torch_reference_formula(oracle_mod):
    """Large random batch: the oracle's sets equal a torch restatement of main.py:2522-2553
    except where the 8th/9th values are within 1 ulp (torch's CPU exp differs from the
    correctly rounded exp in the last bit for ~1% of inputs)."""
    g = torch.Generator().manual_seed(11)
    T = 4096
    logits = torch.randn(T, 256, generator=g)
    bias = (torch.randn(256, generator=g) * 0.1).to(torch.bfloat16)
    idx, w, sb, tie = oracle_mod.route(logits, bias, 2.5, with_details=True)
    s = 1.0 / (1.0 + torch.exp(-logits))
    swb = s + bias.float()
    top2 = torch.topk(swb.view(T, 8, 32), 2, dim=2, sorted=False).values.sum(2)
    gidx = torch.topk(top2, 4, dim=1, sorted=False).indices
    gmask = torch.zeros(T, 8).scatter_(1, gidx, 1.0).unsqueeze(2).expand(T, 8, 32).reshape(T, 256)
    pruned = swb.masked_fill(gmask == 0, torch.finfo(torch.float32).min)
    ref = torch.topk(pruned, 8, dim=1, sorted=False).indices.numpy()
    same = (np.sort(ref, 1) == np.sort(idx, 1)).all(1)
    assert same.mean() >= 0.999, same.mean()


@pytest.mark.slow
@pytest.mark.parametrize("name", golden_moe_names())
def test_oracle_matches_reference_run(oracle_mod, workloads, weights_cache, name):
    inp, ref, z = rebuild_golden_inputs(workloads, name, weights_cache)
    idx, w = oracle_mod.route(inp["routing_logits"], inp["routing_bias"], inp["routed_scaling_factor"])
    assert np.array_equal(np.sort(idx, 1), np.sort(z["ref_idx"], 1))
    out = oracle_mod.run(*[inp[k] for k in workloads.ARG_ORDER])
    st = oracle_mod.error_stats(out, ref, ATOL, RTOL)
    # same fp32 math in a different summation order: bf16 outputs agree to an ulp
    assert st["frac_pass"] == 1.0, st
    assert st["max_abs"] <= 2e-2, st
    nz = ref.float().abs().sum(1) > 0
    assert torch.equal(out.float().abs().sum(1) > 0, nz)


def test_act_quantiser_restatement_matches_the_input_generator(oracle_mod, workloads):
    """The oracle's 1x128 activation quantiser (reference main.py:1476-1488) and the synthetic-input generator
    apply the same rule: identical bytes and scales (fp32 input, zero block, large block)."""
    g = torch.Generator().manual_seed(11)
    x = torch.randn((6, 7168), generator=g) * 5
    x[0, :128] = 0
    x[1, 128:256] *= 1e6
    q1, s1 = oracle_mod.quantize_act_1x128(x)
    q2, s2 = workloads.quantize_act_1x128(x)
    assert torch.equal(s1, s2)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8))
    assert torch.all(s1[0, 0] == 1.0)
