"""The Flash V2 operator surface (echo/stau_opus_flash_v2.py:403-583):
STauOpusFlashV2Function, STauOpusFlashV2Module, get_best_stau_function and
_HAS_TRITON, served by the same fused B200 operator."""
import pytest
import torch

from tau_dxb_b200 import attention as A
from tau_dxb_b200 import stau_opus_flash_v2 as FV2


def test_names_and_selection():
    assert FV2.STauOpusFlashV2Function is A.STauOpusAttentionFunction
    assert FV2.get_best_stau_function() is FV2.STauOpusFlashV2Function
    # the library loads without a GPU, so the fused path counts as available
    assert FV2._HAS_TRITON is True
    assert FV2._SIGMA_NAME_TO_ID == {"softplus": 0, "sigmoid": 1, "exp": 2, "relu": 3}


def test_module_parameters_and_state_dict_keys():
    m = FV2.STauOpusFlashV2Module(12, "sigmoid")
    assert [n for n, _ in m.named_parameters()] == ["log_tau", "log_alpha"]
    assert list(m.state_dict()) == ["log_tau", "log_alpha"]
    assert m.log_tau.shape == (12,) and m.sigma_name == "sigmoid"
    # a checkpoint of the reference's module loads as is
    m.load_state_dict({"log_tau": torch.full((12,), 0.3), "log_alpha": torch.zeros(12)})


def test_cpu_inputs_raise():
    m = FV2.STauOpusFlashV2Module(2)
    Q = torch.randn(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(Q, Q, Q)


@pytest.mark.gpu
def test_module_matches_fused_function_on_gpu():
    """Forward and backward of the module are the fused operator's, bit for bit,
    with a mask tensor and a scale, as echo/patch_whisper_stau.py:237-259 calls it."""
    g = torch.Generator().manual_seed(3)
    B, H, L = 2, 4, 200
    Q, K, V, dO = (torch.randn(B, H, L, 64, generator=g).to(torch.bfloat16).cuda() for _ in range(4))
    mask = torch.zeros(B, 1, L, L)
    mask[:, :, :, 150:] = torch.finfo(torch.float32).min
    mask = mask.cuda()
    m = FV2.STauOpusFlashV2Module(H, "softplus").cuda()
    with torch.no_grad():
        m.log_tau.copy_(torch.randn(H, generator=g).cuda() * 0.5)
    q1, k1, v1 = (t.clone().requires_grad_() for t in (Q, K, V))
    out1 = m(q1, k1, v1, attn_mask=mask, scale=0.125)
    out1.backward(dO)
    lt = m.log_tau.detach().clone().requires_grad_()
    la = m.log_alpha.detach().clone().requires_grad_()
    q2, k2, v2 = (t.clone().requires_grad_() for t in (Q, K, V))
    fn = FV2.get_best_stau_function()
    out2, none = fn.apply(q2, k2, v2, lt, la, "softplus", mask, 0.125)
    assert none is None
    out2.backward(dO)
    torch.cuda.synchronize()
    assert torch.equal(out1, out2) and torch.equal(v1.grad, v2.grad)
    # dQ, dK and the per-head sums accumulate in fp32 with atomics, whose order
    # varies: equal up to that, i.e. one bf16 rounding step for dQ and dK
    for a, b in [(q1.grad, q2.grad), (k1.grad, k2.grad)]:
        assert torch.allclose(a.float(), b.float(), rtol=2 ** -7, atol=1e-6)
    assert torch.allclose(m.log_tau.grad, lt.grad, rtol=1e-5, atol=1e-7)
