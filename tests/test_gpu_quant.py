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
