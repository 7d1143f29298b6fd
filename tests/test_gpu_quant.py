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
