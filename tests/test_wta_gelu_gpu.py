"""GELU fused into the WTA kernels (TAU_DXB_WTA_GELU_INPUT, wta_bwd_gelu)
against torch's bf16 GELU followed by the unfused WTA: the same y, mask and
win counts bit for bit, and the same bf16 gradient, at the encoder size
[24000, 3072] and other fast-path widths; and a patched model's step with and
without the fusion."""
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,d,k", [(24000, 3072, 306), (513, 1024, 100), (64, 768, 1), (7, 4096, 4096)])
def test_gelu_wta_matches_gelu_then_wta(n, d, k):
    from tau_dxb_b200 import _capi as C
    from tau_dxb_b200 import wta as W
    g = torch.Generator(device="cuda").manual_seed(n + d)
    x = (torch.randn(n, d, device="cuda", generator=g) * 1.7 - 0.3).to(torch.bfloat16)
    dy = torch.randn(n, d, device="cuda", generator=g).to(torch.bfloat16)
    a = torch.nn.functional.gelu(x)
    win0 = torch.zeros(d, dtype=torch.int32, device="cuda")
    y0, bits0 = W.wta_select(a, k, W.THRESHOLD, write_y=True, win_counts=win0)
    win1 = torch.zeros(d, dtype=torch.int32, device="cuda")
    y1, bits1 = W.wta_select(x, k, W.THRESHOLD | C.WTA_GELU_INPUT, write_y=True, win_counts=win1)
    assert torch.equal(bits1, bits0)
    assert torch.equal(y1.view(torch.int16), y0.view(torch.int16))
    assert torch.equal(win1, win0)
    # backward: the WTA mask on dy, then torch's GELU backward, both in bf16
    xr = x.clone().requires_grad_()
    ar = torch.nn.functional.gelu(xr)
    ar.backward(W.wta_backward(dy, bits0))
    dx = W.wta_backward_gelu(dy, x, bits1)
    same = (dx.view(torch.int16) == xr.grad.view(torch.int16)).float().mean().item()
    assert rel_err(dx.float().cpu().numpy(), xr.grad.float().cpu().numpy()) < 1e-2
    assert same > 0.999, same


def test_gelu_wta_unsupported_forms_raise():
    from tau_dxb_b200 import _capi as C
    from tau_dxb_b200 import wta as W
    x = torch.randn(8, 3072, device="cuda")
    with pytest.raises(C.TauDxbError):
        W.wta_select(x, 10, W.THRESHOLD | C.WTA_GELU_INPUT)                 # fp32
    with pytest.raises(C.TauDxbError):
        W.wta_select(x.to(torch.bfloat16), 10, W.EXACT_K | C.WTA_GELU_INPUT)  # exact-k


def test_model_step_with_and_without_gelu_fusion():
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import train as T
    from test_model_gpu import tiny_cfg
    cfg = tiny_cfg(batch=2, ffn=768)                # an MLP width with a fused kernel
    mel, labels = T.synthetic_batch(cfg, "cuda", torch.Generator().manual_seed(31))
    model = T.build_model(cfg, "cuda")
    assert sum(getattr(m.fc2, "_tau_dxb_gelu_in", False) for m in model.modules()
               if m.__class__.__name__ == "WhisperEncoderLayer") == cfg.encoder_layers

    def run():
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(input_features=mel, labels=labels)
        out.loss.backward()
        return float(out.loss), {n: p.grad.detach().float().cpu() for n, p in model.named_parameters()
                                 if p.grad is not None}

    lf, gf = run()
    SG.unfuse_gelu_from_wta(model)
    ls, gs = run()
    assert abs(lf - ls) <= 1e-5 * abs(ls), (lf, ls)
    for n in gs:
        assert rel_err(gf[n], gs[n]) < 1e-2, (n, rel_err(gf[n], gs[n]))
    model.eval()
    with torch.no_grad():                              # inference keeps the GELU when fused
        SG.fuse_gelu_into_wta(model)
        a = model(input_features=mel, labels=labels).loss
        SG.unfuse_gelu_from_wta(model)
        b = model(input_features=mel, labels=labels).loss
    assert abs(float(a) - float(b)) <= 1e-5 * abs(float(b))
