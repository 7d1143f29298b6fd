"""Expert parallelism across the GPUs of one node.

The 256 experts shard by contiguous ranges: rank r of N owns experts
[r*256/N, (r+1)*256/N) and passes that range to the operator through
``local_expert_offset`` (the reference operator's only expert-parallel knob,
solution/triton/main.py:2558-2564).  Every rank routes all tokens (routing is
replicated and cheap) and produces the un-rounded fp32 sum over its experts;
the partials are summed across ranks and rounded to bf16 once.

Two ways to sum the ranks' contributions; rank r ends with rows
[r*T/N, (r+1)*T/N) of the layer output either way:

* ``PeerExchange`` (the fast path): GEMM2's epilogue stores every (token, slot)
  pair row straight into the receive buffer of the token's owner over NVLink
  peer memory (CUDA IPC), overlapping the GEMM; each owner then sums its tokens'
  8 slots in slot order.  Same values, same order as the single-GPU operator, so
  the rows equal its output bit for bit.
* ``combine`` (the NCCL baseline): each rank's un-rounded fp32 partial over its
  experts, then one ``reduce_scatter_tensor``; on backends without it (gloo, used
  by the CPU tests) an all-reduce followed by taking the rank's rows.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

E_TOTAL = 256
H = 7168


def shard(rank: int, world: int, e_total: int = E_TOTAL) -> Tuple[int, int]:
    """(E_local, local_expert_offset) of `rank` among `world` ranks."""
    if world < 1 or e_total % world != 0:
        raise ValueError(f"{e_total} experts do not divide over {world} ranks")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside 0..{world - 1}")
    e_local = e_total // world
    return e_local, rank * e_local


def row_range(rank: int, world: int, T: int) -> Tuple[int, int]:
    """Token rows [lo, hi) that `rank` owns after the combine."""
    if T % world != 0:
        raise ValueError(f"T={T} must be a multiple of the world size {world}")
    n = T // world
    return rank * n, (rank + 1) * n


def combine(partial_f32: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
            out: Optional[torch.Tensor] = None, scratch: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sum the ranks' fp32 partials [T, H]; return this rank's rows [T/N, H] in bf16."""
    if partial_f32.dtype != torch.float32 or partial_f32.dim() != 2:
        raise RuntimeError("partial must be a 2-D float32 tensor")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T = partial_f32.size(0)
    lo, hi = row_range(rank, world, T)
    if dist.get_backend(group) == "nccl":
        shard_f32 = scratch if scratch is not None else torch.empty((hi - lo, partial_f32.size(1)),
                                                                    dtype=torch.float32, device=partial_f32.device)
        dist.reduce_scatter_tensor(shard_f32, partial_f32, group=group)
    else:
        dist.all_reduce(partial_f32, group=group)
        shard_f32 = partial_f32[lo:hi]
    if out is None:
        return shard_f32.to(torch.bfloat16)
    out.copy_(shard_f32)
    return out


class TokenReplicator:
    """Builds the replicated inputs of ``PeerExchange.forward`` from token-sharded ones: rank r holds rows
    [r*T/N, (r+1)*T/N) of routing_logits [T, 256] and hidden_states [T, 7168] and the same columns of
    hidden_states_scale [56, T]; after ``gather`` every rank holds all T tokens.

    A host that feeds the layer uploads each token once (to the rank that holds it) and the ranks exchange
    the slices over NVLink (one all-gather per tensor) instead of every rank uploading all T tokens over
    PCIe.  Issue it on the stream that runs the layer: the collective then never shares the SMs with the
    layer's persistent kernels.  Collective: every rank calls ``gather`` in the same order."""

    def __init__(self, T: int, group: Optional[dist.ProcessGroup] = None, device: Optional[torch.device] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T = int(T)
        row_range(self.rank, self.world, self.T)  # validates T % world
        self.rows = self.T // self.world
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
                else torch.device("cpu")
        self.device = device
        # all_gather_into_tensor stacks slices along dim 0: the scale columns come back as [world, 56, T/N]
        self._scale_stack = torch.empty((self.world, H // 128, self.rows), dtype=torch.float32, device=device)

    def _gather(self, out: torch.Tensor, local: torch.Tensor) -> None:
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(out, local, group=self.group)
        else:  # gloo has no all_gather_into_tensor
            dist.all_gather(list(out.view((self.world,) + tuple(local.shape)).unbind(0)), local, group=self.group)

    def gather(self, logits_local: torch.Tensor, hs_local: torch.Tensor, hs_scale_local: torch.Tensor,
               logits: torch.Tensor, hs: torch.Tensor, hs_scale: torch.Tensor) -> None:
        """Fill logits [T, 256], hs [T, 7168] and hs_scale [56, T] from every rank's slices."""
        n, W = self.rows, self.world
        if (tuple(logits_local.shape) != (n, E_TOTAL) or tuple(hs_local.shape) != (n, H)
                or tuple(hs_scale_local.shape) != (H // 128, n)):
            raise RuntimeError(f"slices must be [{n}, 256], [{n}, 7168] and [56, {n}]")
        if (tuple(logits.shape) != (self.T, E_TOTAL) or tuple(hs.shape) != (self.T, H)
                or tuple(hs_scale.shape) != (H // 128, self.T)):
            raise RuntimeError(f"outputs must be [{self.T}, 256], [{self.T}, 7168] and [56, {self.T}]")
        for t in (logits_local, hs_local, hs_scale_local, logits, hs, hs_scale):
            if not t.is_contiguous():
                raise RuntimeError("slices and outputs must be contiguous")
        self._gather(logits, logits_local)
        # fp8 rows travel as bytes (collectives of float8 types are not available on every backend)
        self._gather(hs.view(torch.uint8), hs_local.view(torch.uint8))
        self._gather(self._scale_stack, hs_scale_local)
        hs_scale.view(H // 128, W, n).copy_(self._scale_stack.permute(1, 0, 2))


def fused_moe_ep(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                 gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset: int,
                 routed_scaling_factor: float, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """One MoE layer across the ranks of `group`: this rank's weights are its expert
    shard; returns this rank's token rows of the bf16 output."""
    import fbmoe_lib
    partial = fbmoe_lib.forward(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                                routed_scaling_factor, partial_f32=True)
    return combine(partial, group)


def owner_of(t: int, T: int, world: int) -> int:
    """Rank that owns output token t (rows_per_rank consecutive tokens per rank)."""
    row_range(0, world, T)  # validates T % world
    return t // (T // world)


class PeerExchange:
    """Receive buffers of every rank for the fused GEMM2 scatter, mapped into this process.

    Collective: every rank of ``group`` constructs it with the same T (token count per
    call, a multiple of the world size) and E_local = 256 / world.  Buffers are
    exchanged once (CUDA IPC handles over ``all_gather_object``); each ``forward``
    is one expert-parallel MoE layer with no NCCL call in the data path."""

    def __init__(self, T: int, group: Optional[dist.ProcessGroup] = None, device: Optional[torch.device] = None,
                 dispatch: bool = False):
        import fbmoe_lib
        self.lib = fbmoe_lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T = int(T)
        self.E_local, self.offset = shard(self.rank, self.world)
        row_range(self.rank, self.world, self.T)  # validates T % world
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        nbytes = fbmoe_lib.ep_recv_bytes(self.T, self.world)
        if nbytes == 0:
            raise ValueError(f"no receive buffer for T={T}, world={self.world}")
        self.opened: List[int] = []
        self.local, self.dispatch_local, self.dispatch_ptrs = 0, 0, None
        # Set-up succeeds on every rank or fails on every rank with the same error: local steps
        # are caught, the collectives always run, and the ranks exchange their errors.
        self.local, self.ptrs, err = self._share(nbytes, None)
        if dispatch:
            self.dispatch_local, self.dispatch_ptrs, err = self._share(
                fbmoe_lib.ep_dispatch_bytes(self.T, self.world), err)
        self.workspace = None
        if err is None:
            try:
                self.workspace = torch.empty(fbmoe_lib.ep_workspace_size(self.T, self.E_local), dtype=torch.uint8,
                                             device=self.device)
            except Exception as e:  # reported collectively below
                err = f"workspace: {e!r}"
        errors: List[Optional[str]] = [None] * self.world
        dist.all_gather_object(errors, err, group=group)
        failed = [(r, e) for r, e in enumerate(errors) if e is not None]
        if failed:
            self._release()
            raise RuntimeError("peer exchange unavailable: " + "; ".join(f"rank {r}: {e}" for r, e in failed))
        self.epoch = 0
        dist.barrier(group=group)  # every rank's buffer exists and is mapped before the first send

    def _share(self, nbytes: int, err: Optional[str]):
        """Allocate this rank's buffer and map every peer's: (own address, addresses by rank, error or None).
        The handle exchange runs on every rank whatever happened locally."""
        local, handle, ptrs = 0, None, []
        if err is None:
            try:
                local = self.lib.ipc_alloc(nbytes)
                handle = self.lib.ipc_handle(local)
            except Exception as e:
                err = f"allocation: {e!r}"
        handles: List[Optional[bytes]] = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        if err is None:
            try:
                for o in range(self.world):
                    if o == self.rank:
                        ptrs.append(local)
                    elif handles[o] is None:
                        raise RuntimeError(f"rank {o} has no buffer")
                    else:
                        p = self.lib.ipc_open(handles[o])
                        self.opened.append(p)
                        ptrs.append(p)
            except Exception as e:
                err = f"mapping: {e!r}"
        return local, ptrs, err

    def _release(self) -> None:
        for p in self.opened:
            try:
                self.lib.ipc_close(p)
            except Exception:
                pass
        self.opened = []
        for attr in ("local", "dispatch_local"):
            if getattr(self, attr, 0):
                try:
                    self.lib.ipc_free(getattr(self, attr))
                except Exception:
                    pass
                setattr(self, attr, 0)

    def _next_epoch(self) -> int:
        self.epoch = self.epoch + 1 if self.epoch < 0xFFFFFFF0 else 1
        return self.epoch

    def forward_dispatch(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                         gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor,
                         out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Token-dispatch layer: this rank passes only its own tokens (routing_logits [T/N, 256], hidden_states
        [T/N, 7168], hidden_states_scale [56, T/N]) and its expert shard; returns its tokens' output rows."""
        if self.dispatch_ptrs is None:
            raise RuntimeError("PeerExchange was created without dispatch=True")
        epoch = self._next_epoch()
        if out is None:
            out = torch.empty((self.T // self.world, H), dtype=torch.bfloat16, device=self.device)
        self.lib.ep_dispatch_send(routing_logits, routing_bias, hidden_states, hidden_states_scale, self.T,
                                  self.E_local, routed_scaling_factor, self.rank, self.world, self.dispatch_ptrs,
                                  epoch, self.workspace)
        self.lib.ep_dispatch_compute(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, self.T,
                                     self.rank, self.world, self.dispatch_local, self.ptrs, epoch, self.workspace)
        return self.lib.ep_recv(self.local, self.T, self.rank, self.world, epoch, out, self.workspace)

    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor,
                out: Optional[torch.Tensor] = None, check: bool = True) -> torch.Tensor:
        """This rank's token rows [T/world, 7168] bf16 of the layer output (its expert shard's weights); every
        rank passes all T tokens' inputs (replicated)."""
        self._next_epoch()
        if out is None:
            out = torch.empty((self.T // self.world, H), dtype=torch.bfloat16, device=self.device)
        inputs = (routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                  gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, self.offset, routed_scaling_factor)
        self.lib.ep_send(inputs, self.rank, self.world, self.ptrs, self.epoch, self.workspace, check=check)
        return self.lib.ep_recv(self.local, self.T, self.rank, self.world, self.epoch, out, self.workspace)

    def status(self) -> int:
        """Device status word of the last forward (synchronises the current stream)."""
        return self.lib.read_status(self.workspace)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: call on every rank)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no peer still writes into this rank's buffer
        self._release()
