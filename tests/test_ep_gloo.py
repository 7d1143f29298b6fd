"""Expert-parallel host logic on CPU ranks (gloo, world size 2).

The GPU path runs the same code over NCCL (bench.py --gpus N); here the
shard assignment, the fp32 combine and the equivalence of sharded and
unsharded computation are checked without a GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ATOL, ORACLE, PKG, RTOL


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_cover_all_experts_once():
    import fbmoe_ep
    for world in (1, 2, 4, 8):
        owned = []
        for r in range(world):
            e_local, off = fbmoe_ep.shard(r, world)
            assert e_local == 256 // world
            owned.extend(range(off, off + e_local))
        assert sorted(owned) == list(range(256))
    with pytest.raises(ValueError):
        fbmoe_ep.shard(0, 3)
    with pytest.raises(ValueError):
        fbmoe_ep.row_range(0, 3, 8)


class LazyExperts:
    """W1/W2 of global experts [offset, offset+n), generated per expert on demand."""

    def __init__(self, offset, n, which, seed=5):
        import fbmoe_workloads as W
        self.W, self.offset, self.n, self.which, self.seed = W, offset, n, which, seed
        self.shape = {"w1": (n, 4096, 7168), "s1": (n, 32, 56), "w2": (n, 7168, 2048), "s2": (n, 56, 16)}[which]

    def __getitem__(self, le):
        w1, s1, w2, s2 = self.W.make_weights(1, self.seed * 1000 + self.offset + le, "cpu")
        return {"w1": w1, "s1": s1, "w2": w2, "s2": s2}[self.which][0]


def _rank_main(rank, world, port, T, q):
    import sys
    for p in (PKG, ORACLE):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import fbmoe_ep
        import fbmoe_workloads as W
        import oracle
        # (1) combine of random partials
        g = torch.Generator().manual_seed(100 + rank)
        part = torch.randn(T, 7168, generator=g)
        mine = fbmoe_ep.combine(part.clone())
        # (2) the operator on this rank's expert shard
        e_local, off = fbmoe_ep.shard(rank, world)
        logits, bias, hs, hs_scale = W.make_activations(T, seed=7, config="standard", device="cpu")
        partial = oracle.run(logits, bias, hs, hs_scale, LazyExperts(off, e_local, "w1"),
                             LazyExperts(off, e_local, "s1"), LazyExperts(off, e_local, "w2"),
                             LazyExperts(off, e_local, "s2"), off, 2.5, return_fp32=True)
        rows = fbmoe_ep.combine(partial)
        q.put((rank, mine.view(torch.int16).numpy(), rows.view(torch.int16).numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.slow
def test_ep_combine_and_shard_equivalence_gloo(oracle_mod):
    world, T = 2, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, T, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict()
    for _ in range(world):
        r, mine, rows = q.get(timeout=600)
        got[r] = (torch.from_numpy(mine).view(torch.bfloat16), torch.from_numpy(rows).view(torch.bfloat16))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # (1) rank r holds rows [r*T/2, (r+1)*T/2) of the fp32 sum, rounded once
    parts = [torch.randn(T, 7168, generator=torch.Generator().manual_seed(100 + r)) for r in range(world)]
    total = (parts[0] + parts[1]).to(torch.bfloat16)
    for r in range(world):
        lo, hi = r * T // world, (r + 1) * T // world
        assert torch.equal(got[r][0], total[lo:hi])
    # (2) the combined shards equal the unsharded operator over all 256 experts
    import fbmoe_workloads as W
    logits, bias, hs, hs_scale = W.make_activations(T, seed=7, config="standard", device="cpu")
    full = oracle_mod.run(logits, bias, hs, hs_scale, LazyExperts(0, 256, "w1"), LazyExperts(0, 256, "s1"),
                          LazyExperts(0, 256, "w2"), LazyExperts(0, 256, "s2"), 0, 2.5)
    combined = torch.cat([got[r][1] for r in range(world)])
    st = oracle_mod.error_stats(combined, full, ATOL, RTOL)
    assert st["frac_pass"] == 1.0 and st["max_abs"] <= 1e-2, st


def _exchange_rank(rank, world, port, q):
    import sys
    sys.path.insert(0, PKG)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import fbmoe_ep
        import fbmoe_lib
        fbmoe_lib.load_library()
        try:
            fbmoe_ep.PeerExchange(8, device=torch.device("cpu"))
            q.put((rank, "constructed"))
        except RuntimeError as e:
            q.put((rank, str(e)))
        dist.barrier()  # the ranks are still in step after the failure
    finally:
        dist.destroy_process_group()


def test_peer_exchange_setup_fails_on_every_rank_alike(fbmoe_lib):
    """Without a GPU the receive buffers cannot be allocated: every rank must raise the same error
    (none may be left waiting in a collective), so a caller can fall back on all ranks together."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1] and got[0].startswith("peer exchange unavailable")
    assert "rank 0" in got[0] and "rank 1" in got[0]


def _replicate_rank(rank, world, port, T, q):
    import sys
    sys.path.insert(0, PKG)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import fbmoe_ep
        import fbmoe_workloads as W
        logits, _, hs, hs_scale = W.make_activations(T, seed=11, config="standard", device="cpu")
        lo, hi = fbmoe_ep.row_range(rank, world, T)
        rep = fbmoe_ep.TokenReplicator(T, device=torch.device("cpu"))
        out_l = torch.full_like(logits, float("nan"))
        out_h = torch.zeros_like(hs)
        out_s = torch.full_like(hs_scale, float("nan"))
        rep.gather(logits[lo:hi].contiguous(), hs[lo:hi].contiguous(), hs_scale[:, lo:hi].contiguous(),
                   out_l, out_h, out_s)
        ok = (torch.equal(out_l, logits) and torch.equal(out_h.view(torch.uint8), hs.view(torch.uint8))
              and torch.equal(out_s, hs_scale))
        try:
            rep.gather(logits[lo:hi], hs[lo:hi], hs_scale[:, lo:hi], out_l[:1], out_h, out_s)
            bad_shape = "accepted"
        except RuntimeError:
            bad_shape = "rejected"
        q.put((rank, ok, bad_shape))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T", [(2, 64), (4, 96)])
def test_token_replicator_rebuilds_the_replicated_inputs(world, T):
    """Each rank holds T/N tokens (rows of logits and fp8 hidden states, columns of the [56, T] scales);
    after the gather every rank holds all T tokens bit for bit (gloo ranks on CPU)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_replicate_rank, args=(r, world, port, T, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    assert sorted(r for r, _, _ in got) == list(range(world))
    assert all(ok for _, ok, _ in got), got
    assert all(b == "rejected" for _, _, b in got), got
