"""Device-side errors reach the caller (GPU, no fault involved).

The decode kernel's CTAs meet at a grid-wide arrival before the combine; the test hook
fbmoe_test_expire_grid_wait makes that bounded wait wait for one arrival that never comes,
with a 2 ms budget.  Every CTA's wait then expires: it sets status bit 2 and returns without
combining, exactly as a real timeout would.  fused_moe must raise RuntimeError for such a
call -- at once with sync_status, or at the next call on the same workspace by default -- and
the context must stay usable: the next clean call gives the same output as before.
"""
import importlib.util
import os

import pytest
import torch

from conftest import PKG

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def entry():
    spec = importlib.util.spec_from_file_location("fbmoe_main_status", os.path.join(PKG, "main.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def case(workloads):
    w = workloads.make_weights(32, 5150, "cuda")
    return workloads.make_inputs(4, seed=8, config="group", device="cuda", weights=w)


@pytest.fixture
def expire(fbmoe_lib):
    lib = fbmoe_lib.load_library()

    def set_(on):
        assert lib.fbmoe_test_expire_grid_wait(1 if on else 0) == 0
    yield set_
    set_(False)


def test_decode_kernel_launch_mode(fbmoe_lib, workloads, entry, case):
    entry.fused_moe(*workloads.as_args(case))
    torch.cuda.synchronize()
    mode = fbmoe_lib.decode_launch_mode()
    print("decode launch mode", mode)
    want = (1, 2) if os.environ.get("FBMOE_DECODE_COOPERATIVE") == "1" else (3,)
    assert mode in want


def test_decode_kernel_cooperative_launch_in_a_child_process():
    """FBMOE_DECODE_COOPERATIVE=1: the decode kernel is launched cooperatively (the launch guarantees that all its
    CTAs are resident together) and gives the same output bits as the default launch."""
    code = r"""
import os, sys, torch
sys.path.insert(0, os.path.join(os.environ["FBMOE_REPO"], "flashinfer-bench-moe_b200"))
import fbmoe_lib as L, fbmoe_workloads as W
w = W.make_weights(32, 5150, "cuda")
inp = W.make_inputs(4, seed=8, config="group", device="cuda", weights=w)
out = L.forward(*W.as_args(inp), sync_status=True)
torch.save(out.cpu(), sys.argv[1])
print("mode", L.decode_launch_mode())
"""
    import subprocess
    import sys
    import tempfile
    from conftest import REPO
    outs, modes = [], []
    for coop in ("0", "1"):
        with tempfile.NamedTemporaryFile(suffix=".pt") as f:
            env = dict(os.environ, FBMOE_DECODE_COOPERATIVE=coop, FBMOE_REPO=REPO)
            r = subprocess.run([sys.executable, "-c", code, f.name], env=env, capture_output=True, text=True,
                               timeout=600)
            assert r.returncode == 0, r.stderr[-2000:]
            modes.append(int(r.stdout.strip().split()[-1]))
            outs.append(torch.load(f.name))
    assert modes[0] == 3 and modes[1] in (1, 2), modes
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))


def test_expired_wait_raises_with_sync_status(fbmoe_lib, workloads, entry, case, expire):
    good = entry.fused_moe(*workloads.as_args(case)).clone()
    fbmoe_lib.check_status()
    expire(True)
    with pytest.raises(RuntimeError) as ei:
        fbmoe_lib.forward(*workloads.as_args(case), sync_status=True)
    assert isinstance(ei.value, fbmoe_lib.DeviceStatusError)
    assert ei.value.word & 0x4, hex(ei.value.word)
    expire(False)
    again = fbmoe_lib.forward(*workloads.as_args(case), sync_status=True)
    assert torch.equal(again, good)


def test_expired_wait_raises_at_the_next_call(fbmoe_lib, workloads, entry, case, expire):
    good = entry.fused_moe(*workloads.as_args(case)).clone()
    fbmoe_lib.check_status()
    expire(True)
    entry.fused_moe(*workloads.as_args(case))  # returns; its status word reaches the sink
    expire(False)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError):
        entry.fused_moe(*workloads.as_args(case))
    out = entry.fused_moe(*workloads.as_args(case))  # the sink was cleared by the raise
    fbmoe_lib.check_status()
    assert torch.equal(out, good)


def test_check_status_reports_a_failed_call(fbmoe_lib, workloads, entry, case, expire):
    expire(True)
    entry.fused_moe(*workloads.as_args(case))
    expire(False)
    with pytest.raises(fbmoe_lib.DeviceStatusError):
        fbmoe_lib.check_status()
    fbmoe_lib.check_status()  # cleared
