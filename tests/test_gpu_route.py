"""GPU parity of the router kernel (fbmoe_route through the C ABI) against the oracle.

Expert indices must be bit-exact (same set, same canonical order) including the
tie cases, where the kernel replays torch.topk's CPU selection."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_routing_names

pytestmark = pytest.mark.gpu


def _route_gpu(fbmoe_lib, logits, bias, scale):
    idx, w = fbmoe_lib.route(logits.cuda().contiguous(), bias.cuda().contiguous(), scale)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy()


def _assert_same(oracle_mod, fbmoe_lib, logits, bias, scale):
    ref_idx, ref_w = oracle_mod.route(logits, bias, scale)
    idx, w = _route_gpu(fbmoe_lib, logits, bias, scale)
    bad = np.nonzero((idx != ref_idx).any(1))[0]
    assert bad.size == 0, f"{bad.size} tokens differ, first {bad[:5]}: gpu {idx[bad[:2]]} oracle {ref_idx[bad[:2]]}"
    np.testing.assert_allclose(w, ref_w, rtol=1e-6, atol=0)
    return float((w == ref_w).mean())


@pytest.mark.parametrize("name", golden_routing_names())
def test_route_golden_fixtures(oracle_mod, fbmoe_lib, name):
    z = np.load(os.path.join(GOLDEN, f"routing_{name}.npz"))
    logits = torch.from_numpy(z["logits"])
    bias = torch.from_numpy(z["bias_bits"]).view(torch.bfloat16)
    _assert_same(oracle_mod, fbmoe_lib, logits, bias, float(z["scale"]))
    idx, _ = _route_gpu(fbmoe_lib, logits, bias, float(z["scale"]))
    assert np.array_equal(np.sort(idx, 1), np.sort(z["ref_idx"], 1))  # the reference's own selection


@pytest.mark.parametrize("config", ["standard", "group", "away", "skew", "zero"])
def test_route_full_size(oracle_mod, fbmoe_lib, workloads, config):
    T = 14107
    off = 224 if config == "away" else 0
    logits, bias, _, _ = workloads.make_activations(T, seed=21, config=config, device="cpu",
                                                    local_expert_offset=off)
    exact = _assert_same(oracle_mod, fbmoe_lib, logits, bias, 2.5)
    assert exact >= 0.99


def test_route_heavy_ties(oracle_mod, fbmoe_lib):
    g = torch.Generator().manual_seed(5)
    T = 4096
    logits = torch.randint(-2, 3, (T, 256), generator=g).float() * 0.25
    bias = (torch.randint(-1, 2, (256,), generator=g).float() * 0.125).to(torch.bfloat16)
    _assert_same(oracle_mod, fbmoe_lib, logits, bias, 1.0)
