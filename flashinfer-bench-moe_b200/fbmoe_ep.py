"""Expert parallelism across the GPUs of one node.

The 256 experts shard by contiguous ranges: rank r of N owns experts
[r*256/N, (r+1)*256/N) and passes that range to the operator through
``local_expert_offset`` (the reference operator's only expert-parallel knob,
solution/triton/main.py:2558-2564).  Every rank routes all tokens (routing is
replicated and cheap) and produces the un-rounded fp32 sum over its experts;
the partials are summed across ranks and rounded to bf16 once.

``combine`` reduce-scatters over token rows: rank r ends with rows
[r*T/N, (r+1)*T/N) of the layer output.  On NCCL this is one
``reduce_scatter_tensor``; on backends without it (gloo, used by the CPU tests)
an all-reduce followed by taking the rank's rows gives the same result.
"""
from __future__ import annotations

from typing import Optional, Tuple

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
