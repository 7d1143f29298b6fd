"""Entry point of the solution: ``main.py::fused_moe`` (value-returning, no destination argument).

Drop-in for weichengz0616/flashinfer-bench-moe ``solution/triton/main.py::fused_moe``
(main.py:2668-2774; config.toml: entry_point = "main.py::fused_moe",
destination_passing_style = false) for the definition
``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``.

Differences from the reference, by design:
* the result is a fresh bf16 tensor, not a view into a module-global workspace
  that the next call overwrites (main.py:2774);
* no 15000-token cap (main.py:2657): the workspace grows with T;
* any number of local experts 1..256 (expert-parallel shards), where the
  reference hard-codes 32;
* every kernel is hand-written sm_100a CUDA behind the C ABI of include/fbmoe.h;
  there is no Triton and no CPU or eager-PyTorch fallback.
"""
from __future__ import annotations

import os
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

import torch  # noqa: E402

import fbmoe_lib as _fbmoe  # noqa: E402


@torch.no_grad()
def fused_moe(
    routing_logits: torch.Tensor,
    routing_bias: torch.Tensor,
    hidden_states: torch.Tensor,
    hidden_states_scale: torch.Tensor,
    gemm1_weights: torch.Tensor,
    gemm1_weights_scale: torch.Tensor,
    gemm2_weights: torch.Tensor,
    gemm2_weights_scale: torch.Tensor,
    local_expert_offset: int,
    routed_scaling_factor: float,
):
    """DeepSeek-V3 FP8 block-scale MoE over the local experts
    ``[local_expert_offset, local_expert_offset + E_local)``; returns bf16 ``[T, 7168]``."""
    return _fbmoe.forward(
        routing_logits,
        routing_bias,
        hidden_states,
        hidden_states_scale,
        gemm1_weights,
        gemm1_weights_scale,
        gemm2_weights,
        gemm2_weights_scale,
        int(local_expert_offset),
        float(routed_scaling_factor),
    )
