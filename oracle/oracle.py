"""TEST INFRASTRUCTURE ONLY -- the parity oracle for the fused MoE operator.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module; the product path never does.

CPU restatement of the reference operator ``run()`` of
weichengz0616/flashinfer-bench-moe (solution/triton/main.py:2430-2609):

* FP8 block-scale dequantisation (main.py:2496-2519): ``A = fp8 * scale`` with
  1x128 per-token scales stored transposed ``[H/128, T]``; W13/W2 with 128x128
  block scales.  Here each expert is dequantised lazily, only when it has a
  routed token; the arithmetic (one fp32 multiply per element) is identical.
* DeepSeek-V3 no-aux routing (main.py:2522-2553), in C (oracle/routing.c):
  tie-exact restatement of torch.topk(sorted=False) on CPU.
* Per local expert (main.py:2561-2605): ``G1 = A_e @ W13_e^T``;
  ``C = silu(G1[:, I:]) * G1[:, :I]`` with ``silu(x) = x / (1 + exp(-x))``;
  ``O = C @ W2_e^T``; ``output.index_add_(0, tok, O * w)`` in fp32; bf16 cast
  (main.py:2609).  The intermediate is NOT requantised.
* ``assert E_local == 32`` (main.py:2471) is dropped so that expert-parallel
  shards of 64/128/256 local experts can be checked.

``error_stats`` restates the reference's matching rule (main.py:2776-2803) and
also reports the stricter per-element allclose rule the build is held to.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, Optional, Sequence

import numpy as np
import torch

H = 7168
I = 2048
E_GLOBAL = 256
TOP_K = 8
BLOCK = 128

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compile oracle/routing.c (and its std::nth_element checker)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        i32p = ctypes.POINTER(ctypes.c_int32)
        lib.route_tokens.argtypes = [f32p, f32p, ctypes.c_int, ctypes.c_float, i32p, f32p, f32p, i32p]
        lib.route_tokens.restype = None
        lib.topk_nth.argtypes = [f32p, ctypes.c_int, ctypes.c_int, i32p]
        lib.topk_nth.restype = None
        _lib = lib
    return _lib


def _fp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _ip(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def topk_nth(values: np.ndarray, k: int) -> np.ndarray:
    """torch.topk(values, k, sorted=False).indices for a 1-D fp32 array (order included)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(k, dtype=np.int32)
    _load().topk_nth(_fp(v), int(v.shape[0]), int(k), _ip(out))
    return out


def route(routing_logits, routing_bias, routed_scaling_factor: float, with_details: bool = False):
    """Routing of main.py:2522-2553.  Returns (topk_idx int32 [T,8] global ids in
    canonical order, topk_w fp32 [T,8]) and optionally (s_with_bias, tie_flags)."""
    logits = np.ascontiguousarray(_to_numpy(routing_logits).astype(np.float32))
    bias = np.ascontiguousarray(_to_numpy_f32(routing_bias).reshape(-1))
    T = logits.shape[0]
    assert logits.shape == (T, E_GLOBAL) and bias.shape == (E_GLOBAL,)
    idx = np.empty((T, TOP_K), dtype=np.int32)
    w = np.empty((T, TOP_K), dtype=np.float32)
    sb = np.empty((T, E_GLOBAL), dtype=np.float32) if with_details else None
    tie = np.empty((T,), dtype=np.int32) if with_details else None
    _load().route_tokens(
        _fp(logits), _fp(bias), int(T), ctypes.c_float(float(routed_scaling_factor)),
        _ip(idx), _fp(w),
        _fp(sb) if sb is not None else ctypes.POINTER(ctypes.c_float)(),
        _ip(tie) if tie is not None else ctypes.POINTER(ctypes.c_int32)(),
    )
    if with_details:
        return idx, w, sb, tie
    return idx, w


def _to_numpy(t):
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().numpy()
    return np.asarray(t)


def _to_numpy_f32(t):
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().to(torch.float32).numpy()
    return np.asarray(t, dtype=np.float32)


def quantize_act_1x128(x: torch.Tensor):
    """Activation quantiser restated on the CPU: per row and 128-column block, scale = amax / 448 (1 for an
    all-zero block), q = e4m3(clamp(x / scale, -448, 448)) in fp32 with round-to-nearest-even -- the
    reference's 1x128 rule, solution/triton/main.py:1476-1488.  x: [T, 7168] (any float dtype, evaluated in
    fp32).  Returns (q e4m3 [T, 7168], scale fp32 [56, T])."""
    xf = x.float().reshape(x.size(0), -1, 128)
    amax = xf.abs().amax(dim=2)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (xf / scale.unsqueeze(2)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.reshape(x.size(0), -1), scale.t().contiguous()


def dequant_act(hidden_states: torch.Tensor, hidden_states_scale: torch.Tensor, rows=None) -> torch.Tensor:
    """A = fp8 * scale with the transposed [H/128, T] scale layout (main.py:2496-2505)."""
    hs = hidden_states.cpu()
    sc = hidden_states_scale.cpu().to(torch.float32)
    if rows is not None:
        rows_t = torch.as_tensor(rows, dtype=torch.long)
        hs = hs.index_select(0, rows_t)
        sc = sc.index_select(1, rows_t)
    a = hs.to(torch.float32)
    s = sc.t().contiguous().repeat_interleave(BLOCK, dim=1)
    return a * s


def dequant_block(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp8 [N, K] with 128x128 block scales [N/128, K/128] -> fp32 [N, K] (main.py:2507-2519)."""
    wf = w.cpu().to(torch.float32)
    sf = s.cpu().to(torch.float32).repeat_interleave(BLOCK, dim=0).repeat_interleave(BLOCK, dim=1)
    return wf * sf


@torch.no_grad()
def run(
    routing_logits,
    routing_bias,
    hidden_states,
    hidden_states_scale,
    gemm1_weights,
    gemm1_weights_scale,
    gemm2_weights,
    gemm2_weights_scale,
    local_expert_offset: int,
    routed_scaling_factor: float,
    tokens: Optional[Sequence[int]] = None,
    routing=None,
    return_fp32: bool = False,
    requant: bool = False,
) -> torch.Tensor:
    """The reference operator on CPU.  With ``tokens`` only those output rows are
    computed (each output row depends only on its own token), returned in the
    given order as bf16 ``[len(tokens), H]``.

    ``requant``: the reference solution's intermediate numerics instead of the
    definition's fp32 -- the SwiGLU output re-quantised with the 1x128 rule
    (act_quant_kernel, solution/triton/main.py:1476-1488) before GEMM2 (its fp8
    gemm2_kernel, main.py:433-600), for checking the fp8-intermediate mode."""
    T = routing_logits.shape[0]
    E_local = gemm1_weights.shape[0]
    assert hidden_states.shape == (T, H)
    assert hidden_states_scale.shape == (H // BLOCK, T)
    assert gemm1_weights.shape == (E_local, 2 * I, H)
    assert gemm1_weights_scale.shape == (E_local, 2 * I // BLOCK, H // BLOCK)
    assert gemm2_weights.shape == (E_local, H, I)
    assert gemm2_weights_scale.shape == (E_local, H // BLOCK, I // BLOCK)

    if routing is None:
        routing = route(routing_logits, routing_bias, routed_scaling_factor)
    idx, w = routing
    rows = np.arange(T) if tokens is None else np.asarray(tokens, dtype=np.int64)
    sub_idx = idx[rows]
    sub_w = w[rows]
    out = torch.zeros((len(rows), H), dtype=torch.float32)
    if len(rows) == 0:
        return out if return_fp32 else out.to(torch.bfloat16)

    A = dequant_act(hidden_states, hidden_states_scale, rows)
    start = int(local_expert_offset)
    for le in range(E_local):
        ge = start + le
        if ge < 0 or ge >= E_GLOBAL:
            continue
        hit = sub_idx == ge
        sel = np.nonzero(hit.any(axis=1))[0]
        if sel.size == 0:
            continue
        w_tok = torch.from_numpy(sub_w[hit]).to(torch.float32)  # one hit per selected row
        sel_t = torch.from_numpy(sel.astype(np.int64))
        W13 = dequant_block(gemm1_weights[le], gemm1_weights_scale[le])
        W2 = dequant_block(gemm2_weights[le], gemm2_weights_scale[le])
        A_e = A.index_select(0, sel_t)
        G1 = A_e.matmul(W13.t())
        X1 = G1[:, :I]
        X2 = G1[:, I:]
        C = (X2 / (1.0 + torch.exp(-X2))) * X1
        if requant:
            q, sc = quantize_act_1x128(C)
            C = q.to(torch.float32) * sc.t().repeat_interleave(BLOCK, dim=1)
        O = C.matmul(W2.t())
        out.index_add_(0, sel_t, O * w_tok.unsqueeze(1))
    return out if return_fp32 else out.to(torch.bfloat16)


def error_stats(out: torch.Tensor, ref: torch.Tensor, atol: float = 1e-2, rtol: float = 2e-2) -> Dict[str, float]:
    """Per-element comparison.

    ``frac_pass``: fraction with |out-ref| <= atol + rtol*|ref| (the allclose rule).
    ``matched_ratio``: the reference's rule (main.py:2793-2798): an element fails only
    if abs_err > atol AND rel_err > rtol.
    """
    x = out.detach().cpu().to(torch.float32)
    y = ref.detach().cpu().to(torch.float32)
    n = x.numel()
    if n == 0:
        return {"n": 0, "max_abs": 0.0, "max_rel": 0.0, "frac_pass": 1.0, "matched_ratio": 1.0, "nonfinite": 0}
    d = (x - y).abs()
    rel = d / (y.abs() + 1e-8)
    ok = d <= atol + rtol * y.abs()
    fail_ref = (d > atol) & (rel > rtol)
    return {
        "n": n,
        "max_abs": float(d.max()),
        "max_rel": float(rel.max()),
        "frac_pass": float(ok.float().mean()),
        "matched_ratio": 1.0 - float(fail_ref.float().sum()) / n,
        "nonfinite": int((~torch.isfinite(x)).sum()),
    }
