"""fp32 LayerNorm kernels (tau_layer_norm_fwd / _bwd) against torch's fp32
layer_norm: outputs, dx, dgamma and dbeta at the train step's sizes (encoder
24000 x 768, decoder 7168 x 768) and ragged ones, every supported width class,
deterministic parameter gradients, and the autocast contract (fp32 out)."""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _ref(x, w, b, dy, eps):
    xr = x.detach().clone().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    br = b.detach().clone().requires_grad_()
    y = torch.nn.functional.layer_norm(xr, (x.shape[-1],), wr, br, eps)
    y.backward(dy)
    return y.detach(), xr.grad, wr.grad, br.grad


@pytest.mark.parametrize("M,d", [(24000, 768), (7168, 768), (1, 128), (37, 384), (1000, 1024), (517, 640),
                                 (3, 896), (2049, 256)])
def test_layer_norm_matches_torch(M, d):
    from tau_dxb_b200 import layernorm as LN
    g = torch.Generator(device="cuda").manual_seed(M + d)
    x = torch.randn(M, d, device="cuda", generator=g) * 3.0 + 1.5
    w = torch.randn(d, device="cuda", generator=g)
    b = torch.randn(d, device="cuda", generator=g)
    dy = torch.randn(M, d, device="cuda", generator=g)
    ry, rdx, rdw, rdb = _ref(x, w, b, dy, 1e-5)
    xs = x.clone().requires_grad_()
    ws = w.clone().requires_grad_()
    bs = b.clone().requires_grad_()
    y = LN.fused_layer_norm(xs, ws, bs, 1e-5)
    y.backward(dy)
    f = lambda t: t.detach().cpu().numpy()
    assert rel_err(f(y), f(ry)) < 2e-6, rel_err(f(y), f(ry))
    assert rel_err(f(xs.grad), f(rdx)) < 2e-5, rel_err(f(xs.grad), f(rdx))
    # dgamma / dbeta sum M rows: fp32 summation order differs from torch's
    assert rel_err(f(ws.grad), f(rdw)) < 2e-5, rel_err(f(ws.grad), f(rdw))
    assert rel_err(f(bs.grad), f(rdb)) < 2e-5, rel_err(f(bs.grad), f(rdb))


def test_layer_norm_backward_is_deterministic_and_batched_shapes():
    from tau_dxb_b200 import layernorm as LN
    x = torch.randn(4, 1500, 768, device="cuda")
    w = torch.randn(768, device="cuda")
    b = torch.randn(768, device="cuda")
    dy = torch.randn(4, 1500, 768, device="cuda")
    grads = []
    for _ in range(2):
        ws = w.clone().requires_grad_()
        bs = b.clone().requires_grad_()
        y = LN.fused_layer_norm(x, ws, bs, 1e-5)
        assert y.shape == x.shape and y.dtype == torch.float32
        y.backward(dy)
        grads.append((ws.grad.clone(), bs.grad.clone()))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])


def test_patched_norm_under_autocast_returns_fp32_like_torch():
    from tau_dxb_b200 import layernorm as LN
    ln = torch.nn.LayerNorm(768).cuda()
    torch.nn.init.normal_(ln.weight)
    x = torch.randn(64, 768, device="cuda").to(torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref = ln(x)
    assert LN.patch_layer_norms(ln) == 1
    with torch.autocast("cuda", dtype=torch.bfloat16):
        got = ln(x)
    assert got.dtype == ref.dtype == torch.float32
    assert rel_err(got.detach().cpu().numpy(), ref.detach().cpu().numpy()) < 2e-6
    # outside autocast an fp32 input takes the kernels too
    xf = x.float()
    assert rel_err(ln(xf).detach().cpu().numpy(), ref.detach().cpu().numpy()) < 2e-6
    LN.unpatch_layer_norms(ln)
    assert "forward" not in ln.__dict__


@pytest.mark.parametrize("M,d", [(24000, 768), (37, 384)])
def test_layer_norm_bf16_output_and_gradient(M, d):
    """bf16 y is torch's fp32 norm rounded to bf16 (to 1 ulp where the two
    fp32 results straddle a rounding boundary, in under 0.1% of elements); a
    bf16 dy gives torch's dx,
    dgamma, dbeta for that dy in fp32."""
    from tau_dxb_b200 import layernorm as LN
    g = torch.Generator(device="cuda").manual_seed(7 * M + d)
    x = torch.randn(M, d, device="cuda", generator=g) * 2.0 - 0.5
    w = torch.randn(d, device="cuda", generator=g)
    b = torch.randn(d, device="cuda", generator=g)
    dy = torch.randn(M, d, device="cuda", generator=g).to(torch.bfloat16)
    ry, rdx, rdw, rdb = _ref(x, w, b, dy.float(), 1e-5)
    xs = x.clone().requires_grad_()
    ws = w.clone().requires_grad_()
    bs = b.clone().requires_grad_()
    y = LN.fused_layer_norm(xs, ws, bs, 1e-5, out_bf16=True)
    assert y.dtype == torch.bfloat16
    ref_b = ry.to(torch.bfloat16)
    diff = (y.float() - ref_b.float()).abs()
    # one bf16 ulp, plus 1e-5 absolute where y = xhat gamma + beta cancels to
    # near zero and the two fp32 results differ by ~1e-7 before rounding
    ulp = ref_b.float().abs() * 2.0 ** -7 + 1e-5
    assert bool((diff <= ulp).all()), float((diff / ulp).max())
    assert float((diff > 0).float().mean()) < 1e-3
    y.backward(dy)
    f = lambda t: t.detach().cpu().numpy()
    assert rel_err(f(xs.grad), f(rdx)) < 2e-5
    assert rel_err(f(ws.grad), f(rdw)) < 2e-5
    assert rel_err(f(bs.grad), f(rdb)) < 2e-5

