"""Offline W1 pre-pack (fbmoe_prepack_w1 + fbmoe_forward_prepacked): the packed layout is
the documented permutation of W1's rows, and the forward on packed weights is bit-identical
to the forward on raw weights on the decode kernel (T <= 64) and the prefill kernels."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def w32(workloads):
    return workloads.make_weights(32, 4242, "cuda")


def test_prepack_layout(fbmoe_lib, w32):
    w1 = w32[0][:3]
    packed = fbmoe_lib.prepack_w1(w1.contiguous())
    torch.cuda.synchronize()
    a = w1.view(torch.uint8).view(3, 2, 32, 64, 7168)          # [e, half, slice, row, k]
    b = packed.view(torch.uint8).view(3, 32, 2, 64, 7168)      # [e, slice, half, row, k]
    assert torch.equal(a.permute(0, 2, 1, 3, 4), b)


@pytest.mark.parametrize("T,E,config,seed", [(1, 32, "standard", 1), (16, 32, "group", 16), (64, 32, "standard", 64),
                                             (901, 32, "standard", 901), (4096, 32, "skew", 4096),
                                             (64, 256, "group", 3), (8192, 256, "standard", 0)])
def test_prepacked_forward_is_bit_identical(fbmoe_lib, workloads, w32, T, E, config, seed):
    w = w32 if E == 32 else workloads.make_weights(E, 1000, "cuda")
    inp = workloads.make_inputs(T, seed=seed, config=config, device="cuda", E_local=E, weights=w)
    ref = fbmoe_lib.forward(*workloads.as_args(inp), sync_status=True)
    packed = fbmoe_lib.prepack_w1(inp["gemm1_weights"])
    args = list(workloads.as_args(inp))
    args[4] = packed
    out = fbmoe_lib.forward(*args, sync_status=True, w1_packed=True)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    del packed, w
    torch.cuda.empty_cache()
