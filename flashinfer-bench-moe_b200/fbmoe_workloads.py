"""Synthetic workloads and the FP8 block-scale quantisers that produce the operator's inputs.

The contest dataset (flashinfer-ai/mlsys26-contest) is not available offline, so
seeded synthetic inputs with its shapes and value distributions stand in for it:

* ``routing_logits`` fp32 ~N(0,1) ``[T, 256]``; ``routing_bias`` bf16 ~N(0,0.1) ``[256]``;
* ``hidden_states``: fp32 ~N(0,1) quantised per 1x128 block to e4m3 with
  ``scale = amax/448`` (1.0 for an all-zero block); the scale is stored
  transposed ``[H/128, T]`` as the operator expects (reference main.py:2485);
* ``gemm1_weights [E,4096,7168]`` / ``gemm2_weights [E,7168,2048]``: fp32
  ~N(0,0.02) quantised per 128x128 block, scales ``[E,32,56]`` / ``[E,56,16]``.

Configs follow the benchmark definitions: ``standard`` (N(0,1) logits),
``skew`` (+3.0 bias on four local experts), ``group`` (+5.0 logits on the local
group), ``away`` (-5.0 logits on the local experts, used with offset 224),
``zero`` (all-zero logits: exact ties).

Generation on ``cpu`` uses ``torch.Generator().manual_seed(seed)`` and is
reproducible across hosts running the same torch build; generation on
``cuda`` is fast and used for benchmarking.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

H = 7168
I = 2048
E_GLOBAL = 256
BLOCK = 128
FP8_MAX = 448.0


def quantize_act_1x128(x: torch.Tensor):
    """fp32 [T, H] -> (e4m3 [T, H], fp32 scale [H/128, T]) with scale = amax/448."""
    T, K = x.shape
    xb = x.reshape(T, K // BLOCK, BLOCK)
    amax = xb.abs().amax(dim=2)
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (xb / scale.unsqueeze(2)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(T, K), scale.t().contiguous()


def quantize_weight_128x128(w: torch.Tensor):
    """fp32 [N, K] -> (e4m3 [N, K], fp32 scale [N/128, K/128]) with scale = amax/448."""
    N, K = w.shape
    wb = w.reshape(N // BLOCK, BLOCK, K // BLOCK, BLOCK)
    amax = wb.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (wb / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(N, K), scale.contiguous()


def make_weights(E_local: int, seed: int, device: str = "cpu", std: float = 0.02):
    """Per-expert seeded weights; experts are drawn one after another so host memory stays small."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w1 = torch.empty((E_local, 2 * I, H), dtype=torch.float8_e4m3fn, device=dev)
    s1 = torch.empty((E_local, 2 * I // BLOCK, H // BLOCK), dtype=torch.float32, device=dev)
    w2 = torch.empty((E_local, H, I), dtype=torch.float8_e4m3fn, device=dev)
    s2 = torch.empty((E_local, H // BLOCK, I // BLOCK), dtype=torch.float32, device=dev)
    for e in range(E_local):
        a = torch.randn((2 * I, H), generator=g, device=dev, dtype=torch.float32) * std
        w1[e], s1[e] = quantize_weight_128x128(a)
        del a
        b = torch.randn((H, I), generator=g, device=dev, dtype=torch.float32) * std
        w2[e], s2[e] = quantize_weight_128x128(b)
        del b
    return w1, s1, w2, s2


def make_activations(T: int, seed: int, config: str = "standard", device: str = "cpu",
                     local_expert_offset: int = 0, E_local: int = 32):
    """Routing logits/bias and the quantised hidden states for one call."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    logits = torch.randn((T, E_GLOBAL), generator=g, device=dev, dtype=torch.float32)
    bias = (torch.randn((E_GLOBAL,), generator=g, device=dev, dtype=torch.float32) * 0.1)
    x = torch.randn((T, H), generator=g, device=dev, dtype=torch.float32)
    if config == "skew":
        hot = [local_expert_offset + e for e in (0, 9, 18, 27) if e < E_local]
        bias[hot] += 3.0
    elif config == "group":
        g0 = (local_expert_offset // 32) * 32
        logits[:, g0:g0 + 32] += 5.0
    elif config == "away":
        lo = local_expert_offset
        logits[:, lo:lo + E_local] -= 5.0
    elif config == "zero":
        logits.zero_()
    elif config != "standard":
        raise ValueError(f"unknown config {config!r}")
    hs, hs_scale = quantize_act_1x128(x)
    return logits, bias.to(torch.bfloat16), hs, hs_scale


def make_inputs(T: int, seed: int = 0, config: str = "standard", device: str = "cpu",
                E_local: int = 32, local_expert_offset: int = 0, routed_scaling_factor: float = 2.5,
                weights: Optional[tuple] = None, weight_seed: Optional[int] = None) -> Dict[str, object]:
    """All ten ``fused_moe`` arguments as a dict (keyword names of the entry point)."""
    logits, bias, hs, hs_scale = make_activations(T, seed, config, device, local_expert_offset, E_local)
    if weights is None:
        weights = make_weights(E_local, seed + 1000 if weight_seed is None else weight_seed, device)
    w1, s1, w2, s2 = weights
    return dict(
        routing_logits=logits,
        routing_bias=bias,
        hidden_states=hs,
        hidden_states_scale=hs_scale,
        gemm1_weights=w1,
        gemm1_weights_scale=s1,
        gemm2_weights=w2,
        gemm2_weights_scale=s2,
        local_expert_offset=int(local_expert_offset),
        routed_scaling_factor=float(routed_scaling_factor),
    )


ARG_ORDER = (
    "routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
    "gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale",
    "local_expert_offset", "routed_scaling_factor",
)


def as_args(inputs: Dict[str, object]):
    return tuple(inputs[k] for k in ARG_ORDER)
