"""Column sums (tau_column_sum) against torch's sum, and the Linear function
of the train step against F.linear under bf16 autocast: same output, same
dX / dW GEMMs, bias gradient summed in fp32 in another order."""
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,dt", [(24000, 3072, torch.bfloat16), (24000, 768, torch.bfloat16),
                                    (7168, 2304, torch.bfloat16), (1, 8, torch.bfloat16), (37, 1536, torch.float32),
                                    (4099, 51904, torch.bfloat16), (300, 264, torch.float32)])
def test_column_sum_matches_torch(M, N, dt):
    from tau_dxb_b200 import linear as L
    g = torch.Generator(device="cuda").manual_seed(M + N)
    x = (torch.randn(M, N, device="cuda", generator=g) * 3.0 + 0.5).to(dt)
    ref = x.double().sum(0)
    got32 = L.column_sum(x, torch.float32)
    assert rel_err(got32.double().cpu().numpy(), ref.cpu().numpy()) < 2e-6 * max(1.0, M ** 0.5)
    got = L.column_sum(x)
    assert got.dtype == dt
    assert rel_err(got.double().cpu().numpy(), ref.cpu().numpy()) < (1e-2 if dt == torch.bfloat16 else 1e-5)
    assert torch.equal(L.column_sum(x, torch.float32), got32)        # fixed summation order


def test_linear_function_matches_f_linear_under_autocast():
    from tau_dxb_b200 import linear as L
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(16, 1500, 768, device="cuda", generator=g)
    w = torch.randn(3072, 768, device="cuda", generator=g) * 0.02
    b = torch.randn(3072, device="cuda", generator=g)
    dy = torch.randn(16, 1500, 3072, device="cuda", generator=g).to(torch.bfloat16)
    outs = []
    for fn in (torch.nn.functional.linear, L.linear):
        xs, ws, bs = (t.clone().requires_grad_() for t in (x, w, b))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = fn(xs, ws, bs)
        y.backward(dy)
        outs.append((y.detach(), xs.grad, ws.grad, bs.grad))
    (y0, dx0, dw0, db0), (y1, dx1, dw1, db1) = outs
    assert y1.dtype == y0.dtype == torch.bfloat16 and torch.equal(y1, y0)
    f = lambda t: t.detach().float().cpu().numpy()
    assert rel_err(f(dx1), f(dx0)) < 1e-2
    assert rel_err(f(dw1), f(dw0)) < 1e-2
    assert db1.dtype == db0.dtype == torch.float32
    assert rel_err(f(db1), f(db0)) < 1e-2


@pytest.mark.parametrize("M,V", [(7168, 51904), (37, 1000), (1, 8)])
def test_cross_entropy_matches_autocast_f_cross_entropy(M, V):
    """Loss and bf16 logit gradient of the fused cross-entropy against
    F.cross_entropy of the same bf16 logits under autocast (fp32 math):
    -inf pad columns, ignored rows, a row of all ignored labels."""
    from tau_dxb_b200 import linear as L
    g = torch.Generator(device="cuda").manual_seed(M)
    logits = (torch.randn(M, V, device="cuda", generator=g) * 4.0).to(torch.bfloat16)
    if V > 64:
        logits[:, V - 39:] = float("-inf")                 # padded vocabulary
    labels = torch.randint(0, V - 39 if V > 64 else V, (M,), device="cuda", generator=g)
    if M > 3:
        labels[::3] = -100
    outs = []
    for fn in (torch.nn.functional.cross_entropy, L.cross_entropy):
        x = logits.clone().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = fn(x, labels)
        (loss * 2.5).backward()
        outs.append((loss.detach().float(), x.grad))
    (l0, g0), (l1, g1) = outs
    assert g1.dtype == g0.dtype == torch.bfloat16
    # both are fp32 log-sum-exps over up to 52k terms in different orders: the
    # fused loss must be as close to the fp64 loss as autocast's fp32 one is
    ref = float(torch.nn.functional.cross_entropy(logits.double(), labels))
    e0, e1 = abs(float(l0) - ref), abs(float(l1) - ref)
    assert e1 <= max(2.0 * e0, 2e-6 * abs(ref)), (float(l1), float(l0), ref)
    f = lambda t: t.detach().float().cpu().numpy()
    assert rel_err(f(g1), f(g0)) < 1e-2, rel_err(f(g1), f(g0))
    if M > 3:
        assert bool((g1[::3] == 0).all())
