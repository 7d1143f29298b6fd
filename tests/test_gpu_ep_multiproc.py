"""Expert parallelism over CUDA-IPC peer memory, one process per GPU (2 or 4 ranks when
the box has that many GPUs; on one GPU a single rank still runs the whole host path).  Each rank checks its token rows against the single-GPU
operator with all 256 experts, bit for bit, over three consecutive calls of the
replicated-input layer and three of the token-dispatch layer."""
import os
import socket
import sys
from datetime import timedelta

import pytest
import torch

from conftest import PKG

pytestmark = pytest.mark.gpu

T = 512


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    try:
        sys.path.insert(0, PKG)
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        import fbmoe_ep
        import fbmoe_lib as L
        import fbmoe_workloads as W
        L.load_library()
        w1, s1, w2, s2 = W.make_weights(256, 777, "cuda")
        ex = fbmoe_ep.PeerExchange(T, dispatch=True)
        E, off = ex.E_local, ex.offset
        lo, hi = fbmoe_ep.row_range(rank, world, T)
        ok, msg = True, ""
        for seed, config in ((1, "standard"), (2, "group"), (3, "skew")):
            inp = W.make_inputs(T, seed=seed, config=config, device="cuda", E_local=256, weights=(w1, s1, w2, s2))
            ref = L.forward(*W.as_args(inp))
            out = ex.forward(inp["routing_logits"], inp["routing_bias"], inp["hidden_states"],
                             inp["hidden_states_scale"], w1[off:off + E], s1[off:off + E], w2[off:off + E],
                             s2[off:off + E], inp["routed_scaling_factor"])
            st = ex.status()
            same = torch.equal(out.view(torch.int16), ref[lo:hi].view(torch.int16))
            if st != 0 or not same:
                ok, msg = False, f"{config}: status {st}, equal {same}"
            out = ex.forward_dispatch(inp["routing_logits"][lo:hi].contiguous(), inp["routing_bias"],
                                      inp["hidden_states"][lo:hi].contiguous(),
                                      inp["hidden_states_scale"][:, lo:hi].contiguous(), w1[off:off + E],
                                      s1[off:off + E], w2[off:off + E], s2[off:off + E], inp["routed_scaling_factor"])
            st = ex.status()
            same = torch.equal(out.view(torch.int16), ref[lo:hi].view(torch.int16))
            if st != 0 or not same:
                ok, msg = False, f"dispatch {config}: status {st}, equal {same}"
        # bench.py's pipelined e2e loop on the token-dispatch layer: every downloaded row block equals the
        # single-GPU operator's rows of this rank (copies ordered behind each step's dispatch send)
        sys.path.insert(0, os.path.dirname(PKG))
        import bench
        shard = dict(inp, gemm1_weights=w1[off:off + E], gemm1_weights_scale=s1[off:off + E],
                     gemm2_weights=w2[off:off + E], gemm2_weights_scale=s2[off:off + E], local_expert_offset=off)
        loop = bench.E2ELoop(world, rank, shard, ex, "dispatch")
        for i in range(4):
            loop.step(i)
        loop.flush()
        torch.cuda.synchronize()
        for b in range(2):
            if not torch.equal(loop.out_host[b].view(torch.int16), ref[lo:hi].cpu().view(torch.int16)):
                ok, msg = False, f"e2e loop slot {b} differs"
        if ex.status() != 0:
            ok, msg = False, f"e2e loop status {ex.status()}"
        ex.close()
        dist.destroy_process_group()
        q.put((rank, ok, msg))
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))


def test_ep_over_peer_memory_matches_single_gpu():
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    world = 4 if n >= 4 else (2 if n >= 2 else 1)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=600))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert sorted(r for r, _, _ in results) == list(range(world))
    for rank, ok, msg in results:
        assert ok, f"rank {rank}: {msg}"
