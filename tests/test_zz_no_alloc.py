"""fbmoe_forward_noalloc against fbmoe_forward (GPU, through the C ABI).

fbmoe_forward_noalloc serves callers that cannot allocate device memory: it
keeps its workspace in a fixed device array inside the library instead of
taking one from the caller.  This file is named to be collected last, so that a
run stopping at the first failure has already run every other test; it passes
alone in a fresh process and after the other tests.  Two calls in a row (with
different inputs) must each match the workspace-taking entry point within the
tolerance the other parity tests use; the second call also shows that the
array's leftover contents from the first call do not leak into the result.
"""
import ctypes

import pytest
import torch

from conftest import ATOL, RTOL

pytestmark = pytest.mark.gpu

ARGS = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
        "gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")


def _bind(lib):
    vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.fbmoe_forward_noalloc.argtypes = [vp] * 8 + [i32, i32, i32, f32, vp, vp]
    lib.fbmoe_forward_noalloc.restype = i32
    return lib


def _noalloc(lib, inp, out):
    T, E = inp["hidden_states"].size(0), inp["gemm1_weights"].size(0)
    stream = torch.cuda.current_stream().cuda_stream
    return lib.fbmoe_forward_noalloc(*[inp[k].data_ptr() for k in ARGS], T, E, inp["local_expert_offset"],
                                     inp["routed_scaling_factor"], out.data_ptr(), stream)


def test_noalloc_matches_forward_twice(fbmoe_lib, workloads, oracle_mod):
    """Calls in a row of different sizes (down, then back up) and a call whose tokens route to no
    local expert (offset 224, logits pushed away from experts 224..255: the output must be all
    zeros).  Each must match the workspace-taking entry point, and the array's status word must
    read clean after each."""
    lib = _bind(fbmoe_lib.load_library())
    weights = workloads.make_weights(32, 606, "cuda")
    calls = [(16, "group", 0), (5, "standard", 0), (16, "standard", 0), (7, "away", 224)]
    for call, (T, config, offset) in enumerate(calls):
        inp = workloads.make_inputs(T, seed=40 + call, config=config, device="cuda", local_expert_offset=offset,
                                    weights=weights)
        ref = fbmoe_lib.forward(*[inp[k] for k in ARGS], inp["local_expert_offset"], inp["routed_scaling_factor"])
        out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = _noalloc(lib, inp, out)
        assert rc == 0, lib.fbmoe_error_string(rc)
        torch.cuda.synchronize()
        assert fbmoe_lib.noalloc_read_status() == 0, call
        st = oracle_mod.error_stats(out.cpu(), ref.cpu(), ATOL, RTOL)
        assert st["nonfinite"] == 0 and st["frac_pass"] == 1.0, (call, st)
        if config == "away":
            idx, _ = oracle_mod.route(inp["routing_logits"].cpu(), inp["routing_bias"].cpu(), 2.5)
            if not ((idx >= offset) & (idx < offset + 32)).any():
                assert out.abs().max().item() == 0.0


def test_noalloc_zero_tokens_is_a_no_op(fbmoe_lib):
    lib = _bind(fbmoe_lib.load_library())
    nul = None
    assert lib.fbmoe_forward_noalloc(*([nul] * 8), 0, 32, 0, 2.5, nul, nul) == 0


def test_noalloc_rejects_sizes_beyond_its_limit(fbmoe_lib, workloads):
    lib = _bind(fbmoe_lib.load_library())
    weights = workloads.make_weights(1, 7, "cuda")
    inp = workloads.make_inputs(17, seed=1, device="cuda", E_local=1, weights=weights)
    out = torch.empty((17, 7168), dtype=torch.bfloat16, device="cuda")
    assert _noalloc(lib, inp, out) == -7  # FBMOE_ERR_NOALLOC_LIMIT
    assert b"T <= 16" in lib.fbmoe_error_string(-7)
