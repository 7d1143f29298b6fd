"""Expert parallelism with the combine fused into GEMM2 (pair rows stored into the owner
rank's receive buffer).

Ranks are emulated on one GPU: each rank has its expert shard, its own receive
buffer and workspace, and every rank's send is enqueued before any receive, so no
kernel ever waits on a kernel that has not been launched.  The result must equal
the single-GPU operator with all 256 experts bit for bit (same pair rows, summed
in the same slot order).  The multi-process path over CUDA IPC is
tests/test_gpu_ep_multiproc.py.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

E_ALL = 256


@pytest.fixture(scope="module")
def weights256(workloads):
    return workloads.make_weights(E_ALL, 777, "cuda")


def _inputs(workloads, weights, T, seed, config="standard"):
    return workloads.make_inputs(T, seed=seed, config=config, device="cuda", E_local=E_ALL, weights=weights)


class EmulatedRanks:
    """world ranks on one GPU: receive buffers, workspaces, shards."""

    def __init__(self, lib, T, world):
        self.lib, self.T, self.world = lib, T, world
        self.E = E_ALL // world
        self.bufs = [lib.ipc_alloc(lib.ep_recv_bytes(T, world)) for _ in range(world)]
        self.ws = [torch.empty(lib.ep_workspace_size(T, self.E), dtype=torch.uint8, device="cuda")
                   for _ in range(world)]

    def shard_inputs(self, inp, r):
        lo, hi = r * self.E, (r + 1) * self.E
        return (inp["routing_logits"], inp["routing_bias"], inp["hidden_states"], inp["hidden_states_scale"],
                inp["gemm1_weights"][lo:hi], inp["gemm1_weights_scale"][lo:hi], inp["gemm2_weights"][lo:hi],
                inp["gemm2_weights_scale"][lo:hi], lo, inp["routed_scaling_factor"])

    def send(self, inp, r, epoch):
        self.lib.ep_send(self.shard_inputs(inp, r), r, self.world, self.bufs, epoch, self.ws[r])

    def recv(self, r, epoch):
        out = torch.empty((self.T // self.world, 7168), dtype=torch.bfloat16, device="cuda")
        return self.lib.ep_recv(self.bufs[r], self.T, r, self.world, epoch, out, self.ws[r])

    def forward(self, inp, epoch):
        for r in range(self.world):
            self.send(inp, r, epoch)
        return torch.cat([self.recv(r, epoch) for r in range(self.world)], dim=0)

    def statuses(self):
        return [self.lib.read_status(w) for w in self.ws]

    def close(self):
        torch.cuda.synchronize()
        for b in self.bufs:
            self.lib.ipc_free(b)


def _single_gpu(fbmoe_lib, workloads, inp):
    return fbmoe_lib.forward(*workloads.as_args(inp))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ep_scatter_equals_single_gpu_bit_for_bit(fbmoe_lib, workloads, weights256, world):
    T = 256
    inp = _inputs(workloads, weights256, T, seed=11)
    ref = _single_gpu(fbmoe_lib, workloads, inp)
    ranks = EmulatedRanks(fbmoe_lib, T, world)
    try:
        out = ranks.forward(inp, epoch=1)
        assert ranks.statuses() == [0] * world
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    finally:
        ranks.close()


def test_ep_scatter_alternating_epochs_and_skewed_routing(fbmoe_lib, workloads, weights256):
    """Consecutive epochs use alternate receive regions; each must match its own input."""
    T, world = 384, 2
    ranks = EmulatedRanks(fbmoe_lib, T, world)
    try:
        for epoch, (seed, config) in enumerate([(1, "standard"), (2, "group"), (3, "skew"), (4, "zero")], start=1):
            inp = _inputs(workloads, weights256, T, seed=seed, config=config)
            ref = _single_gpu(fbmoe_lib, workloads, inp)
            out = ranks.forward(inp, epoch=epoch)
            assert ranks.statuses() == [0] * world, (epoch, config)
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (epoch, config)
    finally:
        ranks.close()


def test_ep_scatter_small_T_within_tolerance(fbmoe_lib, workloads, weights256):
    """At T <= 64 the single-GPU operator takes the decode kernel (another K order);
    the expert-parallel path always takes the row-major one."""
    T, world = 8, 2
    inp = _inputs(workloads, weights256, T, seed=5)
    ref = _single_gpu(fbmoe_lib, workloads, inp).float()
    ranks = EmulatedRanks(fbmoe_lib, T, world)
    try:
        out = ranks.forward(inp, epoch=7).float()
        assert ranks.statuses() == [0] * world
        assert torch.allclose(out, ref, atol=1e-2, rtol=2e-2)
    finally:
        ranks.close()


def test_ep_recv_times_out_when_a_peer_never_sends(fbmoe_lib, workloads, weights256):
    """Rank 1 never sends: rank 0's bounded wait expires (about 4 s), sets status bit 7
    and returns; the context stays usable."""
    T, world = 128, 2
    inp = _inputs(workloads, weights256, T, seed=3)
    ranks = EmulatedRanks(fbmoe_lib, T, world)
    try:
        ranks.send(inp, 0, epoch=1)
        ranks.recv(0, epoch=1)
        assert ranks.statuses()[0] & (1 << 7)
        # the next epoch runs normally once both ranks send
        ref = _single_gpu(fbmoe_lib, workloads, inp)
        out = ranks.forward(inp, epoch=2)
        assert ranks.statuses() == [0] * world
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    finally:
        ranks.close()


class EmulatedDispatch(EmulatedRanks):
    """Token-dispatch ranks on one GPU: rank r passes only tokens [r*T/N, (r+1)*T/N).
    All dispatches, then all computes, then all receives."""

    def __init__(self, lib, T, world):
        super().__init__(lib, T, world)
        self.dbufs = [lib.ipc_alloc(lib.ep_dispatch_bytes(T, world)) for _ in range(world)]

    def local_inputs(self, inp, r):
        n = self.T // self.world
        lo, hi = r * n, (r + 1) * n
        return (inp["routing_logits"][lo:hi].contiguous(), inp["routing_bias"], inp["hidden_states"][lo:hi].contiguous(),
                inp["hidden_states_scale"][:, lo:hi].contiguous())

    def forward(self, inp, epoch):
        for r in range(self.world):
            logits, bias, hs, hss = self.local_inputs(inp, r)
            self.lib.ep_dispatch_send(logits, bias, hs, hss, self.T, self.E, inp["routed_scaling_factor"], r,
                                      self.world, self.dbufs, epoch, self.ws[r])
        for r in range(self.world):
            lo, hi = r * self.E, (r + 1) * self.E
            self.lib.ep_dispatch_compute(inp["gemm1_weights"][lo:hi], inp["gemm1_weights_scale"][lo:hi],
                                         inp["gemm2_weights"][lo:hi], inp["gemm2_weights_scale"][lo:hi], self.T, r,
                                         self.world, self.dbufs[r], self.bufs, epoch, self.ws[r])
        return torch.cat([self.recv(r, epoch) for r in range(self.world)], dim=0)

    def close(self):
        super().close()
        for b in self.dbufs:
            self.lib.ipc_free(b)


@pytest.mark.parametrize("world", [1, 2, 8])
def test_token_dispatch_equals_single_gpu_bit_for_bit(fbmoe_lib, workloads, weights256, world):
    T = 256
    ranks = EmulatedDispatch(fbmoe_lib, T, world)
    try:
        for epoch, (seed, config) in enumerate([(21, "standard"), (22, "group"), (23, "skew")], start=1):
            inp = _inputs(workloads, weights256, T, seed=seed, config=config)
            ref = _single_gpu(fbmoe_lib, workloads, inp)
            out = ranks.forward(inp, epoch=epoch)
            assert ranks.statuses() == [0] * world, (world, config)
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (world, config)
    finally:
        ranks.close()
