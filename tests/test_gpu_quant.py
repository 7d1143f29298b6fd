"""GPU parity of the activation quantiser (fbmoe_quantize_act, the producer of fused_moe's hidden_states
and hidden_states_scale) against the oracle's restatement of the reference's 1x128 rule: bit-exact e4m3
bytes and fp32 scales, including all-zero blocks, a saturating block and bf16 extremes."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, 7168), generator=g) * torch.exp(torch.randn((T, 1), generator=g) * 3)
    if T >= 3:
        x[0, :128] = 0.0                      # all-zero block: scale 1
        x[1, 128:256] = 3.0e38                # bf16 near-max values in one block
        x[2, 256:384] = torch.linspace(-1e-30, 1e-30, 128)  # tiny values
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("T,seed", [(1, 1), (5, 2), (64, 3), (1000, 4), (8192, 5)])
def test_quantize_act_bit_exact(oracle_mod, fbmoe_lib, T, seed):
    x = _case(T, seed)
    q, s = fbmoe_lib.quantize_act(x.cuda())
    torch.cuda.synchronize()
    q_ref, s_ref = oracle_mod.quantize_act_1x128(x)
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))


def test_quantize_act_rejects_bad_input(fbmoe_lib):
    with pytest.raises(RuntimeError):
        fbmoe_lib.quantize_act(torch.zeros((4, 7168), dtype=torch.float32, device="cuda"))


def test_quantize_act_bit_exact_on_rounding_midpoints(oracle_mod, fbmoe_lib):
    """Blocks built so that many x / scale land on (or next to) e4m3 rounding midpoints: x = amax * k / 64 and
    amax * k / 56 with amax a power of two or 7 * 2^j.  The kernel's reciprocal path must hand these to the
    exact division and still match the oracle's IEEE division bit for bit."""
    g = torch.Generator().manual_seed(99)
    T = 512
    k = torch.randint(-64, 65, (T, 7168), generator=g).float()
    amax = torch.tensor([1.0, 8.0, 7.0, 0.875, 3.5, 1.75e-3, 2.0 ** 20, 5.0])[torch.arange(T * 56) % 8]
    amax = amax.view(T, 56).repeat_interleave(128, dim=1)
    denom = torch.where(torch.arange(7168) % 2 == 0, torch.tensor(64.0), torch.tensor(56.0))
    x = (amax * k / denom)
    x[:, ::128] = amax[:, ::128]          # every block reaches its amax exactly
    x = x.to(torch.bfloat16)
    q, s = fbmoe_lib.quantize_act(x.cuda())
    torch.cuda.synchronize()
    q_ref, s_ref = oracle_mod.quantize_act_1x128(x)
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))


def _sweep_chunk(a0, a1):
    """Blocks for every amax bit pattern a in [a0, a1) (finite positive bf16): each block holds +amax at element 0
    and 127 of the 2(a+1) bf16 values with |x| <= amax (both signs of every magnitude, zeros padding the last
    block), 56 blocks per row."""
    a = torch.arange(a0, a1, dtype=torch.int32, device="cuda")
    cnt = 2 * (a + 1)
    nblk = (cnt + 126) // 127
    blk_a = torch.repeat_interleave(a, nblk)
    first = torch.cumsum(nblk, 0) - nblk
    k0 = (torch.arange(blk_a.numel(), device="cuda", dtype=torch.int32)
          - torch.repeat_interleave(first.to(torch.int32), nblk)) * 127
    idx = k0[:, None] + torch.arange(127, device="cuda", dtype=torch.int32)[None, :]
    bits = torch.where(idx < torch.repeat_interleave(cnt, nblk)[:, None], (idx >> 1) | ((idx & 1) << 15), 0)
    blocks = torch.cat([blk_a[:, None], bits], dim=1)
    pad = (-blocks.size(0)) % 56
    if pad:
        blocks = torch.cat([blocks, torch.zeros((pad, 128), dtype=torch.int32, device="cuda")])
    return blocks.to(torch.int16).view(torch.bfloat16).reshape(-1, 7168)


def _rule_on_device(x):
    """The oracle's 1x128 rule (oracle.quantize_act_1x128) evaluated by torch on x's device.  Both divisions take
    tensor divisors: torch's CUDA division by a host scalar multiplies by the scalar's reciprocal, which is not
    the IEEE quotient."""
    xf = x.float().reshape(x.size(0), -1, 128)
    amax = xf.abs().amax(dim=2)
    scale = torch.where(amax > 0, amax / torch.full_like(amax, 448.0), torch.ones_like(amax))
    q = (xf / scale.unsqueeze(2)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.reshape(x.size(0), -1), scale.t().contiguous()


def test_quantize_act_exhaustive_bf16(oracle_mod, fbmoe_lib):
    """Every finite positive bf16 amax, and for each every bf16 x with |x| <= amax (about 1.07e9 elements in 16
    chunks): bit-exact against the oracle's rule evaluated on the same device (_rule_on_device, itself checked
    against the CPU oracle on a sample of each chunk).  This pins the kernel's FMA-based scale, reciprocal and
    quotient (and the exact division it falls back to for tiny scales) on the whole bf16 input domain."""
    edges = torch.linspace(1, 0x7F80, 17).long().tolist()
    for a0, a1 in zip(edges[:-1], edges[1:]):
        x = _sweep_chunk(a0, a1)
        q, s = fbmoe_lib.quantize_act(x)
        q_ref, s_ref = _rule_on_device(x)
        rows = torch.linspace(0, x.size(0) - 1, 8).long()
        q_cpu, s_cpu = oracle_mod.quantize_act_1x128(x[rows].cpu())
        assert torch.equal(q_ref[rows].cpu().view(torch.uint8), q_cpu.view(torch.uint8))
        assert torch.equal(s_ref[:, rows].cpu().view(torch.int32), s_cpu.view(torch.int32))
        assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32)), (a0, a1)
        assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8)), (a0, a1)
        del x, q, s, q_ref, s_ref


def test_quantize_act_nonfinite(oracle_mod, fbmoe_lib):
    """A block holding an infinity takes the exact path (scale inf: finite x -> signed zero, inf -> NaN), as in
    the oracle.  A NaN element becomes an e4m3 NaN (either sign) and does not enter its block's amax, so the rest
    of its block matches the oracle run on the same input with that element set to zero."""
    x = torch.randn((2, 7168), generator=torch.Generator().manual_seed(5)) * 5
    x[0, 3] = float("inf")
    x[0, 200] = float("-inf")
    x[1, 7] = float("nan")
    xb = x.to(torch.bfloat16)
    q, s = fbmoe_lib.quantize_act(xb.cuda())
    q, s = q.cpu().view(torch.uint8), s.cpu()
    q_ref, s_ref = oracle_mod.quantize_act_1x128(torch.where(torch.isnan(xb), torch.zeros_like(xb), xb))
    q_ref = q_ref.view(torch.uint8)
    expect_nan = (q_ref & 0x7F) == 0x7F
    expect_nan[1, 7] = True
    assert torch.equal((q & 0x7F) == 0x7F, expect_nan)
    assert torch.equal(q[~expect_nan], q_ref[~expect_nan])
    assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
    assert s[0, 0].item() == float("inf") and s[1, 0].item() == float("inf")
