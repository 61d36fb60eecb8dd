"""tau-opus attention on the tensor-core path at the sizes the benchmark times,
against the fp32 oracle (2e-2 max relative error, the bf16 bar).

Workloads (Q, K, V, dO ~ N(0,1) bf16, log_tau ~ N(0, 0.5), log_alpha = 0,
head_dim 64, 12 heads):
  encoder_self   softplus, B=16, Lq=Lk=1500, scale 1/8
  decoder_self   sigmoid, B=16, 448 x 448, causal (additive finfo.min mask
                 tensor, and the built-in causal flag)
  decoder_cross  exp, B=16, 448 x 1500; and tau = 1 against softmax attention
  long context   softplus, B=4, Lq=Lk=6000 (two heads checked over the batch)

At these sizes some rows have their two largest scores within fp32
accumulation rounding of each other, and the kernel (which sums QK^T in
another order) can pick the second of the two as the argmax. The argmax
decides where the backward puts the shift correction of the row, so the
oracle is given the kernel's argmax for exactly those rows, after the test
has checked, in float64, that the kernel's choice is a maximum within
rounding. Every other row keeps the oracle's own argmax.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err
from oracle import stau_attention as OA

from test_attn_gpu import DEV, NAMES, TOL_BF16, fwd_direct, make_inputs

pytestmark = pytest.mark.gpu

# fp32 accumulation of 64 products of N(0,1) bf16 values, times the scale:
# the two summation orders differ by well under this
TIE_EPS = 1e-4


@pytest.fixture(scope="module")
def A():
    from tau_dxb_b200 import attention
    return attention


def gpu_fwd_bwd(A, Q, K, V, lt, la, sigma, dO, mask=None, scale=0.125, causal_fn=False):
    """Forward + backward through the autograd Functions on the auto path."""
    from tau_dxb_b200 import _capi as C
    q, k, v = (t.to(DEV).requires_grad_() for t in (Q, K, V))
    ltd, lad = lt.to(DEV).requires_grad_(), la.to(DEV).requires_grad_()
    if causal_fn:
        out = A.STauOpusCausalFunction.apply(q, k, v, ltd, lad, sigma, scale)
    else:
        out, none = A.STauOpusAttentionFunction.apply(
            q, k, v, ltd, lad, sigma, None if mask is None else mask.to(DEV), scale)
        assert none is None
    out.backward(dO.to(DEV))
    torch.cuda.synchronize()
    assert C.lib().tau_dxb_device_error(1) == 0
    f = lambda t: t.detach().float().cpu().numpy()
    res = [f(out), f(q.grad), f(k.grad), f(v.grad), f(ltd.grad), f(lad.grad)]
    del q, k, v, out
    torch.cuda.empty_cache()
    return res


def checked_argmax(Qb, Kb, scale, mask_b, kernel_amax):
    """The kernel's argmax where it is a maximum within TIE_EPS of the float64
    row max (asserted for every row), as an index array for the oracle; also
    the number of rows where it differs from the first float64 argmax."""
    s = np.matmul(Qb.astype(np.float64), np.swapaxes(Kb.astype(np.float64), -1, -2)) * scale
    if mask_b is not None:
        s = s + mask_b.astype(np.float64)
    smax = s.max(axis=-1)
    picked = np.take_along_axis(s, kernel_amax[..., None].astype(np.int64), axis=-1)[..., 0]
    live = smax > -1e30            # fully masked rows: every score rounds alike
    bad = live & (picked < smax - TIE_EPS)
    assert not bad.any(), f"kernel argmax is not a row maximum in {int(bad.sum())} rows"
    differs = int((kernel_amax != s.argmax(axis=-1)).sum())
    return kernel_amax, differs


def oracle_by_item(Q, K, V, lt, la, sigma, dO, mask, scale, amax, heads=None):
    """Oracle over the batch one item at a time (bounded host memory); the
    per-head parameter gradients are summed over the items. heads: optional
    subset of heads (every head is independent of the others)."""
    f = lambda t: t.float().numpy()
    B = Q.shape[0]
    hs = slice(None) if heads is None else list(heads)
    outs, dqs, dks, dvs = [], [], [], []
    dlt = dla = 0.0
    differs = 0
    for b in range(B):
        Qb, Kb, Vb, dOb = (f(t[b:b + 1][:, hs]) for t in (Q, K, V, dO))
        mb = None
        if mask is not None:
            mb = f(mask[b:b + 1] if mask.shape[0] > 1 else mask)
        a, d = checked_argmax(Qb, Kb, scale, mb, amax[b:b + 1][:, hs])
        differs += d
        out, (dq, dk, dv, gt, ga), _ = OA.forward_backward(
            Qb, Kb, Vb, f(lt[hs]), f(la[hs]), sigma, dOb, mb, scale, argmax=a)
        outs.append(out); dqs.append(dq); dks.append(dk); dvs.append(dv)
        dlt = dlt + gt
        dla = dla + ga
    cat = lambda xs: np.concatenate(xs, axis=0)
    return [cat(outs), cat(dqs), cat(dks), cat(dvs), np.asarray(dlt), np.asarray(dla)], differs


def assert_close_all(mine, ref, label, tol=TOL_BF16):
    errs = {n: rel_err(a, b) for n, a, b in zip(NAMES, mine, ref)}
    print(label, {n: f"{e:.2e}" for n, e in errs.items()})
    for n, e in errs.items():
        assert e < tol, f"{label} {n}: rel err {e:.3e} >= {tol}"


def kernel_argmax(Q, K, V, lt, la, sigma, scale, mask=None, causal=False):
    """Row argmax the tensor-core forward records (deterministic: the same
    kernel on the same inputs picks the same index every time)."""
    return fwd_direct(Q, K, V, lt, la, sigma, scale, "auto", mask=mask, causal=causal)[3]


def test_encoder_self_b16_l1500(A):
    Q, K, V, lt, la, dO = make_inputs(16, 12, 1500, 1500, seed=1500, dtype=torch.bfloat16)
    mine = gpu_fwd_bwd(A, Q, K, V, lt, la, "softplus", dO)
    amax = kernel_argmax(Q, K, V, lt, la, "softplus", 0.125)
    ref, differs = oracle_by_item(Q, K, V, lt, la, "softplus", dO, None, 0.125, amax)
    assert differs <= 16 * 12 * 1500 // 1000, differs
    assert_close_all(mine, ref, f"encoder_self B16 L1500 (argmax ties taken: {differs})")


@pytest.mark.parametrize("causal_fn", [False, True], ids=["mask_tensor", "causal_flag"])
def test_decoder_self_b16_l448_causal(A, causal_fn):
    L = 448
    Q, K, V, lt, la, dO = make_inputs(16, 12, L, L, seed=448, dtype=torch.bfloat16)
    mask = torch.from_numpy(OA.causal_mask(L, L))
    mine = gpu_fwd_bwd(A, Q, K, V, lt, la, "sigmoid", dO, None if causal_fn else mask, 0.125,
                       causal_fn=causal_fn)
    amax = kernel_argmax(Q, K, V, lt, la, "sigmoid", 0.125, causal=True)
    ref, differs = oracle_by_item(Q, K, V, lt, la, "sigmoid", dO, mask, 0.125, amax)
    assert_close_all(mine, ref, f"decoder_self B16 448 causal (argmax ties taken: {differs})")


def test_decoder_cross_b16_448x1500(A):
    Q, K, V, lt, la, dO = make_inputs(16, 12, 448, 1500, seed=4481500, dtype=torch.bfloat16)
    mine = gpu_fwd_bwd(A, Q, K, V, lt, la, "exp", dO)
    amax = kernel_argmax(Q, K, V, lt, la, "exp", 0.125)
    ref, differs = oracle_by_item(Q, K, V, lt, la, "exp", dO, None, 0.125, amax)
    assert_close_all(mine, ref, f"decoder_cross B16 448x1500 (argmax ties taken: {differs})")


def test_decoder_cross_tau1_is_softmax_attention(A):
    """sigma = exp at tau = 1 (log_tau = -inf) and alpha = 1 is softmax
    attention; out and dQ, dK, dV against torch's fp32 softmax attention on the
    host (the shift correction sums to zero there: softmax is shift invariant)."""
    Q, K, V, _, la, dO = make_inputs(16, 12, 448, 1500, seed=7, dtype=torch.bfloat16)
    lt = torch.full((12,), -float("inf"))
    mine = gpu_fwd_bwd(A, Q, K, V, lt, la, "exp", dO)
    q, k, v = (t.float().requires_grad_() for t in (Q, K, V))
    out = torch.softmax((q @ k.transpose(-1, -2)) * 0.125, dim=-1) @ v
    out.backward(dO.float())
    ref = [out.detach().numpy(), q.grad.numpy(), k.grad.numpy(), v.grad.numpy()]
    for n, a, b in zip(NAMES[:4], mine[:4], ref):
        e = rel_err(a, b)
        assert e < TOL_BF16, f"tau=1 {n}: {e:.3e}"
    # d log_tau = dtau * sigmoid(-inf) = 0 exactly
    assert np.all(mine[4] == 0.0)


def test_long_context_b4_l6000(A):
    """Encoder self-attention at 6000 keys; the whole batch runs on the GPU and
    heads 0 and 7 (every item) are checked against the oracle, including their
    batch-summed dlog_tau / dlog_alpha."""
    L = 6000
    heads = [0, 7]
    Q, K, V, lt, la, dO = make_inputs(4, 12, L, L, seed=6000, dtype=torch.bfloat16)
    mine = gpu_fwd_bwd(A, Q, K, V, lt, la, "softplus", dO)
    amax = kernel_argmax(Q, K, V, lt, la, "softplus", 0.125)
    ref, differs = oracle_by_item(Q, K, V, lt, la, "softplus", dO, None, 0.125, amax, heads=heads)
    sub = [m[:, heads] for m in mine[:4]] + [mine[4][heads], mine[5][heads]]
    assert_close_all(sub, ref, f"long context B4 L6000 heads {heads} (argmax ties taken: {differs})")
