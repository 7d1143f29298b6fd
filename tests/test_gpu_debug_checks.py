"""The debug-check build (lib/libfbmoe_debug.so, built from the same sources with
-DFBMOE_DEBUG_CHECKS) on valid inputs, through the C ABI.

In that build every index a kernel reads back from the workspace (the token of a
permuted row, the permuted row of a (token, slot), a GEMM block's expert and row
range) is range-checked before it addresses memory; a bad one sets status bit 9
and the access is skipped.  It stands in for a device memory checker on hardware
where none runs.  On the parity cases the debug build must report status 0 and
produce the normal library's output bit for bit, and so it must when its workspace
starts filled with 0x7F or 0xFF bytes (f16 NaN, fp32 3.4e38 or NaN, int32 2139062143
or -1): any read of a workspace byte that the call did not write first would change
the output or trip a check.
"""
import ctypes
import os

import pytest
import torch

from conftest import PKG

pytestmark = pytest.mark.gpu

ARGS = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
        "gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")


@pytest.fixture(scope="module")
def dbg(fbmoe_lib):
    lib = ctypes.CDLL(os.path.join(PKG, "lib", "libfbmoe_debug.so"))
    vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    lib.fbmoe_forward.argtypes = [vp] * 8 + [i32, i32, i32, f32, vp, vp, sz, vp]
    lib.fbmoe_forward.restype = i32
    lib.fbmoe_workspace_size.argtypes = [i32, i32]
    lib.fbmoe_workspace_size.restype = sz
    lib.fbmoe_read_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint32), vp]
    lib.fbmoe_read_status.restype = i32
    return lib


_W = {}


def weights(workloads, E, seed):
    if (E, seed) not in _W:
        _W.clear()
        torch.cuda.empty_cache()
        _W[(E, seed)] = workloads.make_weights(E, seed, "cuda")
    return _W[(E, seed)]


def run_debug(lib, inp, fill):
    T, E = inp["hidden_states"].size(0), inp["gemm1_weights"].size(0)
    ws = torch.full((int(lib.fbmoe_workspace_size(T, E)),), fill, dtype=torch.uint8, device="cuda")
    out = torch.empty((T, 7168), dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.fbmoe_forward(*[inp[k].data_ptr() for k in ARGS], T, E, inp["local_expert_offset"],
                           inp["routed_scaling_factor"], out.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    assert rc == 0, rc
    st = ctypes.c_uint32(0)
    lib.fbmoe_read_status(ws.data_ptr(), ctypes.byref(st), stream)
    return out, int(st.value)


# T, E_local, offset, config, seed, weight seed (decode, prefill and the benchmark sizes)
CASES = [
    (1, 32, 0, "standard", 1, 4242),
    (16, 32, 0, "group", 16, 4242),
    (64, 32, 0, "standard", 64, 4242),
    (7, 32, 224, "away", 7, 4242),
    (901, 32, 0, "standard", 901, 4242),
    (8192, 32, 0, "skew", 8192, 4242),
    (14107, 32, 0, "group", 14108, 4242),
    (5000, 32, 224, "away", 5000, 4242),
    (5000, 32, 0, "zero", 5001, 4242),
    (64, 256, 0, "group", 81, 1000),
    (8192, 256, 0, "standard", 0, 1000),
]


@pytest.mark.parametrize("T,E,offset,config,seed,wseed", CASES)
def test_debug_build_matches_and_reads_only_what_it_wrote(fbmoe_lib, workloads, dbg, T, E, offset, config, seed,
                                                          wseed):
    inp = workloads.make_inputs(T, seed=seed, config=config, device="cuda", E_local=E, local_expert_offset=offset,
                                weights=weights(workloads, E, wseed))
    ref = fbmoe_lib.forward(*workloads.as_args(inp), sync_status=True)
    for fill in (0x00, 0x7F, 0xFF):
        out, status = run_debug(dbg, inp, fill)
        assert status == 0, (fill, hex(status))
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), fill
