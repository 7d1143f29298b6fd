"""CPU tests of the C ABI surface (no kernel is launched): the library loads,
exports every entry point include/fbmoe.h declares, and validates arguments."""
import ctypes
import os
import re

import pytest

from conftest import REPO


def header_functions():
    src = open(os.path.join(REPO, "include", "fbmoe.h")).read()
    return re.findall(r"FBMOE_API\s+[\w\s\*]+?\b(fbmoe_\w+)\s*\(", src)


def test_header_declares_entry_points():
    names = header_functions()
    assert "fbmoe_forward" in names and "fbmoe_route" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol(fbmoe_lib):
    lib = fbmoe_lib.load_library()
    for name in header_functions():
        assert hasattr(lib, name), name


def test_workspace_layout_consistent(fbmoe_lib):
    lib = fbmoe_lib.load_library()
    for T in (1, 7, 16, 64, 901, 14107):
        for E in (32, 64, 128, 256):
            lay = fbmoe_lib.workspace_layout(T, E)
            assert lay["total"] == lib.fbmoe_workspace_size(T, E)
            offs = [lay[k] for k in fbmoe_lib.LAYOUT_FIELDS[:12]]
            assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)
            pcap = lay["row_capacity"]
            assert pcap >= 8 * T + 16 * E and pcap % 128 == 0
            assert lay["pair_out"] + pcap * 7168 * 2 <= lay["total"]


def test_invalid_arguments_are_rejected_without_launching(fbmoe_lib):
    lib = fbmoe_lib.load_library()
    nul = None
    # E_local out of range
    rc = lib.fbmoe_forward(nul, nul, nul, nul, nul, nul, nul, nul, 4, 0, 0, 2.5, nul, nul, 0, nul)
    assert rc == -1
    rc = lib.fbmoe_forward(nul, nul, nul, nul, nul, nul, nul, nul, 4, 257, 0, 2.5, nul, nul, 0, nul)
    assert rc == -1
    # negative T
    assert lib.fbmoe_forward(nul, nul, nul, nul, nul, nul, nul, nul, -1, 32, 0, 2.5, nul, nul, 0, nul) == -1
    # T == 0 is a no-op
    assert lib.fbmoe_forward(nul, nul, nul, nul, nul, nul, nul, nul, 0, 32, 0, 2.5, nul, nul, 0, nul) == 0
    # null pointers
    assert lib.fbmoe_forward(nul, nul, nul, nul, nul, nul, nul, nul, 4, 32, 0, 2.5, nul, nul, 0, nul) == -3
    assert lib.fbmoe_workspace_size(-1, 32) == 0
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert lib.fbmoe_error_string(code)
    assert lib.fbmoe_block_rows(1, 32) in (16, 32, 64, 128)
    assert lib.fbmoe_version() >= 100


def test_host_checks_reject_cpu_tensors(fbmoe_lib, workloads):
    import torch
    inp = workloads.make_activations(2, 0)
    with pytest.raises(RuntimeError, match="CUDA"):
        fbmoe_lib.check_inputs(inp[0], inp[1], inp[2], inp[3], torch.empty(1), torch.empty(1),
                               torch.empty(1), torch.empty(1), 0)


def test_quantizers_roundtrip(workloads):
    import torch
    g = torch.Generator().manual_seed(0)
    x = torch.randn(8, 7168, generator=g)
    q, s = workloads.quantize_act_1x128(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (56, 8)
    deq = q.float() * s.t().repeat_interleave(128, 1)
    assert torch.allclose(deq, x, rtol=0.07, atol=1e-3)
    w = torch.randn(256, 384, generator=g) * 0.02
    qw, sw = workloads.quantize_weight_128x128(w)
    assert sw.shape == (2, 3)
    deqw = qw.float() * sw.repeat_interleave(128, 0).repeat_interleave(128, 1)
    assert torch.allclose(deqw, w, rtol=0.07, atol=1e-5)
    z, zs = workloads.quantize_act_1x128(torch.zeros(2, 7168))
    assert (zs == 1.0).all() and (z.float() == 0).all()


def test_expert_parallel_entry_points_validate_without_launching(fbmoe_lib):
    lib = fbmoe_lib.load_library()
    nul = None
    assert fbmoe_lib.ep_recv_bytes(8192, 8) == 256 + 2 * 1024 * 8 * 7168 * 2
    assert fbmoe_lib.ep_recv_bytes(100, 3) == 0 and fbmoe_lib.ep_recv_bytes(8, 9) == 0
    assert fbmoe_lib.ep_workspace_size(8, 32) == lib.fbmoe_ep_workspace_size(8, 32) > 0
    # the expert-parallel workspace is the row-major chain's at every T (no split-K buffers)
    assert fbmoe_lib.ep_workspace_size(8192, 32) == fbmoe_lib.workspace_layout(8192, 32)["total"]
    assert 0 < fbmoe_lib.ep_workspace_size(8, 128)

    def send(T, E, offset, rank, world, peers, epoch=1):
        return lib.fbmoe_forward_ep_send(nul, nul, nul, nul, nul, nul, nul, nul, T, E, offset, 2.5, rank, world,
                                         peers, epoch, nul, 0, nul)

    two = fbmoe_lib._ptr_array([16, 32])
    assert send(64, 128, 0, 0, 3, two) == -1          # 256 experts do not split over 3 ranks
    assert send(64, 64, 0, 0, 2, two) == -1           # E_local * world != 256
    assert send(63, 128, 0, 0, 2, two) == -1          # T not a multiple of the world size
    assert send(64, 128, 0, 1, 2, two) == -1          # offset != rank * E_local
    assert send(64, 128, 128, 2, 2, two) == -1        # rank outside the world
    assert send(64, 128, 0, 0, 2, two, epoch=0) == -1  # epoch 0 is reserved
    assert send(64, 128, 0, 0, 2, None) == -3         # no peer table
    assert send(64, 128, 0, 0, 2, fbmoe_lib._ptr_array([16, 0])) == -3
    assert send(64, 128, 0, 0, 2, fbmoe_lib._ptr_array([16, 40])) == -4  # misaligned peer buffer
    assert send(0, 128, 0, 0, 2, two) == 0            # T == 0 is a no-op
    assert lib.fbmoe_forward_ep_recv(nul, 64, 0, 2, 0, nul, nul, nul) == -1
    assert lib.fbmoe_forward_ep_recv(nul, 64, 0, 2, 1, nul, nul, nul) == -3
    assert lib.fbmoe_forward_ep_recv(nul, 0, 0, 2, 1, nul, nul, nul) == 0
    assert lib.fbmoe_ipc_alloc(0, None) == -3
    assert lib.fbmoe_ipc_handle(None, None) == -3 and lib.fbmoe_ipc_open(None, None) == -3
    assert lib.fbmoe_ipc_free(None) == 0 and lib.fbmoe_ipc_close(None) == 0


def test_expert_parallel_token_ownership():
    import fbmoe_ep
    assert [fbmoe_ep.owner_of(t, 16, 4) for t in range(16)] == [t // 4 for t in range(16)]
    assert fbmoe_ep.row_range(3, 4, 16) == (12, 16)
    with pytest.raises(ValueError):
        fbmoe_ep.owner_of(0, 10, 4)
