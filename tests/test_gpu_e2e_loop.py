"""The pipelined host-buffer loop behind bench.py's `e2e` (bench.E2ELoop, N = 1): uploads on one copy stream,
downloads on another, two device buffer sets.  Every step's downloaded rows must equal fused_moe's output on the
same inputs bit for bit, whatever the order in which the streams ran, so no step reads a buffer still being
written or downloads one still being computed."""
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("T,config", [(64, "standard"), (512, "skew")])
def test_e2e_loop_downloads_the_operator_output(fbmoe_lib, workloads, T, config):
    sys.path.insert(0, REPO)
    import bench
    w = workloads.make_weights(32, 4242, "cuda")
    inp = workloads.make_inputs(T, seed=T + 1, config=config, device="cuda", E_local=32, weights=w)
    ref = fbmoe_lib.forward(*workloads.as_args(inp), sync_status=True).cpu()
    loop = bench.E2ELoop(1, 0, inp, None, "single")
    assert loop.h2d == sum(inp[k].numel() * inp[k].element_size() for k in loop.names)
    for i in range(5):
        loop.step(i)
    loop.flush()
    torch.cuda.synchronize()
    for b in range(2):
        assert torch.equal(loop.out_host[b].view(torch.int16), ref.view(torch.int16)), b
