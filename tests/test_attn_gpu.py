"""tau-opus attention kernels against the oracle and the reference's golden
vectors. fp32 inputs: 1e-4 max relative error; bf16 inputs: 2e-2."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_err
from oracle import stau_attention as OA

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL_FP32 = 1e-4
TOL_BF16 = 2e-2
NAMES = ["out", "dQ", "dK", "dV", "dlog_tau", "dlog_alpha"]


@pytest.fixture(scope="module")
def A():
    from tau_dxb_b200 import attention
    return attention


def run_op(A, Q, K, V, log_tau, log_alpha, sigma, dO, mask=None, scale=None, path="auto",
           causal_fn=False):
    """Run forward+backward through the autograd Function; numpy fp32 results."""
    q, k, v = (t.detach().clone().to(DEV).requires_grad_() for t in (Q, K, V))
    lt = log_tau.detach().clone().to(DEV).requires_grad_()
    la = log_alpha.detach().clone().to(DEV).requires_grad_()
    with A.attention_path(path):
        if causal_fn:
            out = A.STauOpusCausalFunction.apply(q, k, v, lt, la, sigma, scale)
        else:
            out, none = A.STauOpusAttentionFunction.apply(
                q, k, v, lt, la, sigma, None if mask is None else mask.to(DEV), scale)
            assert none is None
        out.backward(dO.to(DEV).to(out.dtype))
    torch.cuda.synchronize()
    f = lambda t: t.detach().float().cpu().numpy()
    return [f(out), f(q.grad), f(k.grad), f(v.grad), f(lt.grad), f(la.grad)]


def oracle(Q, K, V, log_tau, log_alpha, sigma, dO, mask=None, scale=None):
    f = lambda t: None if t is None else t.detach().float().cpu().numpy()
    out, grads, _ = OA.forward_backward(f(Q), f(K), f(V), f(log_tau), f(log_alpha), sigma,
                                        f(dO), f(mask), scale)
    return [out, *grads]


def assert_close(mine, ref, tol, label="", zero_params=False):
    """zero_params: dlog_tau is exactly 0 in exact arithmetic (relu: every
    sigma is clamped to the same 1e-8, so log sigma is constant and
    sum P (dP - D) = 0), so both sides are rounding noise. Check it against
    an absolute bound scaled like the other per-head gradient instead: the
    bf16 paths take D = rowsum(dO * O) from the bf16 output, which leaves
    a residue of order tol * |dlog_alpha|."""
    for n, a, b in zip(NAMES, mine, ref):
        if zero_params and n == "dlog_tau":
            bound = max(1e-3, tol * float(np.abs(ref[5]).max()))
            assert np.abs(a).max() < bound and np.abs(b).max() < 1e-3, (label, n, np.abs(a).max())
            continue
        e = rel_err(a, b)
        assert e < tol, f"{label} {n}: rel err {e:.3e} >= {tol}"


def make_inputs(B, H, Lq, Lk, D=64, seed=0, dtype=torch.float32, lt_std=0.5, la_std=0.0):
    g = torch.Generator().manual_seed(seed)
    Q = torch.randn(B, H, Lq, D, generator=g).to(dtype)
    K = torch.randn(B, H, Lk, D, generator=g).to(dtype)
    V = torch.randn(B, H, Lk, D, generator=g).to(dtype)
    dO = torch.randn(B, H, Lq, D, generator=g).to(dtype)
    lt = torch.randn(H, generator=g) * lt_std
    la = torch.randn(H, generator=g) * la_std
    return Q, K, V, lt, la, dO


def assert_no_near_ties(Q, K, scale, mask=None, min_gap=1e-5):
    gap = OA.row_top2_gap(Q.float().numpy(), K.float().numpy(), scale,
                          None if mask is None else mask.numpy())
    assert gap > min_gap, f"seeded inputs have a near-tied row max (gap {gap})"


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p)[:-4])
def test_precise_path_matches_reference_golden(A, path):
    z = np.load(path)
    t = lambda n: torch.from_numpy(z[n])
    scale = float(z["scale"])
    scale = None if np.isnan(scale) else scale
    mask = t("mask") if "mask" in z.files else None
    mine = run_op(A, t("Q"), t("K"), t("V"), t("log_tau"), t("log_alpha"), str(z["sigma"]),
                  t("dO"), mask, scale, path="precise")
    ref = [z[n] for n in NAMES]
    assert_close(mine, ref, TOL_FP32, os.path.basename(path))


@pytest.mark.parametrize("sigma,causal", [("softplus", False), ("sigmoid", True), ("exp", False),
                                          ("relu", False)])
@pytest.mark.parametrize("Lq,Lk", [(1, 1), (63, 63), (65, 129), (127, 64), (200, 200)])
def test_precise_fp32_shapes(A, sigma, causal, Lq, Lk):
    Q, K, V, lt, la, dO = make_inputs(2, 3, Lq, Lk, seed=Lq * 1000 + Lk, la_std=0.2)
    mask = torch.from_numpy(OA.causal_mask(Lq, Lk)) if causal else None
    assert_no_near_ties(Q, K, 0.125, mask)
    mine = run_op(A, Q, K, V, lt, la, sigma, dO, mask, None, path="precise")
    ref = oracle(Q, K, V, lt, la, sigma, dO, mask, None)
    assert_close(mine, ref, TOL_FP32, f"{sigma} {Lq}x{Lk}", zero_params=sigma == "relu")


def test_causal_function_equals_mask_tensor(A):
    Q, K, V, lt, la, dO = make_inputs(2, 4, 70, 70, seed=9)
    mask = torch.from_numpy(OA.causal_mask(70, 70))
    a = run_op(A, Q, K, V, lt, la, "sigmoid", dO, mask, 1.0, path="precise")
    b = run_op(A, Q, K, V, lt, la, "sigmoid", dO, None, 1.0, path="precise", causal_fn=True)
    for x, y in zip(a, b):
        assert rel_err(x, y) < 1e-6


@pytest.mark.parametrize("sigma,causal,Lq,Lk", [("softplus", False, 300, 300),
                                                ("sigmoid", True, 200, 200),
                                                ("exp", False, 96, 300)])
def test_bf16_auto_path_vs_fp32_oracle(A, sigma, causal, Lq, Lk):
    Q, K, V, lt, la, dO = make_inputs(2, 4, Lq, Lk, seed=Lq + Lk, dtype=torch.bfloat16)
    mask = torch.from_numpy(OA.causal_mask(Lq, Lk)) if causal else None
    scale = 0.125 if sigma == "softplus" else 1.0 / 8
    assert_no_near_ties(Q, K, scale, mask)
    mine = run_op(A, Q, K, V, lt, la, sigma, dO, mask, scale, path="auto")
    ref = oracle(Q, K, V, lt, la, sigma, dO, mask, scale)
    assert_close(mine, ref, TOL_BF16, f"bf16 {sigma}")


@pytest.mark.parametrize("sigma", ["softplus", "sigmoid", "exp"])
def test_bf16_tensor_path_clamped_and_clean_chunks(A, sigma):
    """Large alpha and tau and a wide score range: some 16-column chunks of the
    backward have sigma, sigma^tau below 1e-8 or the +-30 clip active (every
    clamp of the reference applied), others none (the clamp-free path)."""
    g = torch.Generator().manual_seed(11)
    B, H, L = 2, 4, 260
    Q = (torch.randn(B, H, L, 64, generator=g) * 1.6).to(torch.bfloat16)
    K = (torch.randn(B, H, L, 64, generator=g) * 1.6).to(torch.bfloat16)
    V = torch.randn(B, H, L, 64, generator=g).to(torch.bfloat16)
    dO = torch.randn(B, H, L, 64, generator=g).to(torch.bfloat16)
    lt = torch.tensor([-1.0, 0.5, 2.0, 3.5])
    la = torch.tensor([0.0, 1.0, 1.5, -0.4])
    assert_no_near_ties(Q, K, 0.125)
    mine = run_op(A, Q, K, V, lt, la, sigma, dO, None, 0.125, path="tensor")
    ref = oracle(Q, K, V, lt, la, sigma, dO, None, 0.125)
    assert_close(mine, ref, TOL_BF16, f"clamped/clean {sigma}")


def test_tau1_exp_equals_softmax_on_gpu(A):
    Q, K, V, _, la, dO = make_inputs(2, 4, 100, 150, seed=4)
    lt = torch.full((4,), -30.0)
    out = run_op(A, Q, K, V, lt, la, "exp", dO, None, None, path="precise")[0]
    s = (Q @ K.transpose(-1, -2)) * 0.125
    ref = (torch.softmax(s, -1) @ V).numpy()
    assert rel_err(out, ref) < 1e-5


def test_noncontiguous_inputs(A):
    # q/k/v as transposed views of [B, L, H, D] buffers, like the Whisper projections
    g = torch.Generator().manual_seed(6)
    Qb, Kb, Vb, dOb = (torch.randn(2, 90, 3, 64, generator=g) for _ in range(4))
    Q, K, V, dO = (t.transpose(1, 2) for t in (Qb, Kb, Vb, dOb))
    lt = torch.randn(3, generator=g) * 0.5
    la = torch.zeros(3)
    q, k, v = (t.to(DEV).detach().requires_grad_() for t in (Qb, Kb, Vb))
    lt_d, la_d = lt.to(DEV).requires_grad_(), la.to(DEV).requires_grad_()
    with A.attention_path("precise"):
        out, _ = A.STauOpusAttentionFunction.apply(q.transpose(1, 2), k.transpose(1, 2),
                                                   v.transpose(1, 2), lt_d, la_d, "softplus")
        out.backward(dO.to(DEV))
    ref = oracle(Q, K, V, lt, la, "softplus", dO)
    mine = [out.detach().cpu().numpy(), q.grad.transpose(1, 2).cpu().numpy(),
            k.grad.transpose(1, 2).cpu().numpy(), v.grad.transpose(1, 2).cpu().numpy(),
            lt_d.grad.cpu().numpy(), la_d.grad.cpu().numpy()]
    assert_close(mine, ref, TOL_FP32, "strided")


def test_errors(A):
    Q, K, V, lt, la, dO = make_inputs(1, 2, 8, 8)
    with pytest.raises(KeyError):
        A.STauOpusAttentionFunction.apply(Q.to(DEV), K.to(DEV), V.to(DEV), lt.to(DEV),
                                          la.to(DEV), "nope")
    with pytest.raises(RuntimeError):
        A.STauOpusAttentionFunction.apply(Q, K, V, lt, la, "softplus")


def test_module_api(A):
    m = A.STauOpusAttentionModule(4, "softplus").to(DEV)
    assert [n for n, _ in m.named_parameters()] == ["log_tau", "log_alpha"]
    Q, K, V, *_ = make_inputs(1, 4, 16, 16)
    out = m(Q.to(DEV), K.to(DEV), V.to(DEV))
    assert out.shape == (1, 4, 16, 64)


# ------------------------------------------------------------ tensor-core forward

def fwd_direct(Q, K, V, lt, la, sigma, scale, path, mask=None, causal=False, layout="blhd"):
    """Forward through the C ABI only; returns out, row_max, row_z, row_argmax (CPU)."""
    import torch.nn.functional as F
    from tau_dxb_b200 import _capi as C
    B, H, Lq, D = Q.shape
    Lk = K.shape[2]

    def dev(t):
        if layout == "blhd":   # [B,H,L,D] view of a [B,L,H,D] buffer, like the Whisper projections
            return t.transpose(1, 2).contiguous().to(DEV).transpose(1, 2)
        return t.contiguous().to(DEV)
    q, k, v = dev(Q), dev(K), dev(V)
    tau = (F.softplus(lt) + 1).float().to(DEV)
    alpha = torch.exp(la).float().to(DEV)
    out = torch.empty(B, Lq, H, D, dtype=Q.dtype, device=DEV).transpose(1, 2)
    m = torch.empty(B, H, Lq, device=DEV)
    z = torch.empty_like(m)
    a = torch.empty(B, H, Lq, dtype=torch.int32, device=DEV)
    md = None
    if mask is not None:
        md = mask.to(DEV).expand(B, H, Lq, Lk)
    rc = C.lib().tau_attn_fwd(
        q.data_ptr(), C.strides4(q), k.data_ptr(), C.strides4(k), v.data_ptr(), C.strides4(v),
        C.dtype_code(Q.dtype), B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(),
        C.SIGMA_IDS[sigma], float(scale), md.data_ptr() if md is not None else None,
        C.F32 if md is not None else 0, C.strides4(md) if md is not None else None, int(causal),
        out.data_ptr(), C.strides4(out), m.data_ptr(), z.data_ptr(), a.data_ptr(),
        {"tensor": C.PATH_TENSOR, "precise": C.PATH_PRECISE, "auto": C.PATH_AUTO}[path], C.stream_ptr())
    C.check("tau_attn_fwd", rc)
    torch.cuda.synchronize()
    assert C.lib().tau_dxb_device_error(1) == 0
    return out.float().cpu().numpy(), m.cpu().numpy(), z.cpu().numpy(), a.cpu().numpy()


@pytest.mark.parametrize("sigma,causal,B,H,Lq,Lk", [
    ("softplus", False, 2, 3, 300, 300), ("softplus", False, 1, 2, 1, 1),
    ("softplus", False, 1, 2, 128, 128), ("softplus", False, 1, 2, 256, 384),
    ("sigmoid", True, 2, 2, 200, 200), ("exp", False, 2, 3, 96, 300),
    ("exp", False, 1, 2, 520, 77), ("relu", False, 1, 2, 64, 64)])
def test_tensor_forward_vs_oracle(sigma, causal, B, H, Lq, Lk):
    Q, K, V, lt, la, _ = make_inputs(B, H, Lq, Lk, seed=Lq * 7 + Lk, dtype=torch.bfloat16, la_std=0.2)
    scale = 0.125
    mask = torch.from_numpy(OA.causal_mask(Lq, Lk)) if causal else None
    assert_no_near_ties(Q, K, scale, mask)
    out, m, z, a = fwd_direct(Q, K, V, lt, la, sigma, scale, "tensor", causal=causal)
    f = lambda t: t.float().numpy()
    ref_out, ctx = OA.forward(f(Q), f(K), f(V), f(lt), f(la), sigma,
                              None if mask is None else mask.numpy(), scale)
    assert rel_err(out, ref_out) < TOL_BF16, rel_err(out, ref_out)
    assert np.abs(m - ctx["m"]).max() < 1e-4
    assert np.array_equal(a, ctx["argmax"])
    assert rel_err(z, ctx["Z"]) < 1e-3


def test_tensor_forward_mask_tensor_and_layouts():
    Q, K, V, lt, la, _ = make_inputs(2, 2, 150, 150, seed=77, dtype=torch.bfloat16)
    mask = torch.from_numpy(OA.causal_mask(150, 150))
    a1 = fwd_direct(Q, K, V, lt, la, "sigmoid", 0.125, "tensor", mask=mask)
    a2 = fwd_direct(Q, K, V, lt, la, "sigmoid", 0.125, "tensor", causal=True, layout="bhld")
    for x, y in zip(a1, a2):
        assert rel_err(x, y) < 1e-6


@pytest.mark.parametrize("sigma,causal,B,H,Lq,Lk", [
    ("softplus", False, 2, 3, 300, 300), ("softplus", False, 1, 2, 1, 1),
    ("softplus", False, 1, 2, 128, 256), ("softplus", False, 2, 2, 257, 130),
    ("sigmoid", True, 2, 2, 200, 200), ("exp", False, 2, 3, 96, 300),
    ("exp", False, 1, 2, 520, 77), ("relu", False, 1, 2, 64, 64)])
def test_tensor_fwd_bwd_vs_oracle(A, sigma, causal, B, H, Lq, Lk):
    Q, K, V, lt, la, dO = make_inputs(B, H, Lq, Lk, seed=Lq * 11 + Lk, dtype=torch.bfloat16, la_std=0.2)
    mask = torch.from_numpy(OA.causal_mask(Lq, Lk)) if causal else None
    assert_no_near_ties(Q, K, 0.125, mask)
    mine = run_op(A, Q, K, V, lt, la, sigma, dO, mask, 0.125, path="tensor")
    from tau_dxb_b200 import _capi as C
    assert C.lib().tau_dxb_device_error(1) == 0
    ref = oracle(Q, K, V, lt, la, sigma, dO, mask, 0.125)
    assert_close(mine, ref, TOL_BF16, f"tensor {sigma} {Lq}x{Lk}", zero_params=sigma == "relu")


@pytest.mark.parametrize("sigma", ["sigmoid", "softplus"])
@pytest.mark.parametrize("causal_fn", [False, True], ids=["mask_tensor", "causal_flag"])
def test_tensor_causal_row_with_negative_max(A, sigma, causal_fn):
    """Causal query row 0 sees key 0 only; with its score far below zero the
    padded key rows of the last key tile (past Lk) must still contribute
    nothing (they once turned dQ/dK row 0 and dlog_tau into NaN)."""
    Q, K, V, lt, la, dO = make_inputs(2, 3, 200, 200, seed=17, dtype=torch.bfloat16)
    K[:, :, 0] = (-0.6 * Q[:, :, 0].float()).to(torch.bfloat16)     # s00 = -0.6 |q0|^2 / 8, about -5
    mask = torch.from_numpy(OA.causal_mask(200, 200))
    assert_no_near_ties(Q, K, 0.125, mask)
    mine = run_op(A, Q, K, V, lt, la, sigma, dO, None if causal_fn else mask, 0.125, path="tensor",
                  causal_fn=causal_fn)
    ref = oracle(Q, K, V, lt, la, sigma, dO, mask, 0.125)
    for a in mine:
        assert np.isfinite(a).all()
    assert_close(mine, ref, TOL_BF16, f"negative row max {sigma}")


def test_tensor_causal_flag_equals_mask(A):
    Q, K, V, lt, la, dO = make_inputs(2, 2, 190, 190, seed=5, dtype=torch.bfloat16)
    mask = torch.from_numpy(OA.causal_mask(190, 190))
    a = run_op(A, Q, K, V, lt, la, "sigmoid", dO, mask, 0.125, path="tensor")
    b = run_op(A, Q, K, V, lt, la, "sigmoid", dO, None, 0.125, path="tensor", causal_fn=True)
    for x, y in zip(a, b):
        assert rel_err(x, y) < 2e-3


# ------------------------------------------------------------ decode forward (Lq <= 8)

@pytest.mark.parametrize("sigma,causal,B,H,Lq,Lk", [
    ("sigmoid", True, 2, 12, 1, 37),        # decoder self-attention, one new token
    ("sigmoid", True, 2, 3, 1, 448),
    ("exp", False, 2, 12, 1, 1500),         # cross-attention over the encoder frames
    ("softplus", False, 1, 4, 3, 700),
    ("softplus", False, 2, 2, 8, 64),
    ("relu", False, 1, 2, 2, 50)])
def test_decode_forward_vs_oracle(sigma, causal, B, H, Lq, Lk):
    """A few query rows (KV-cached decoding) take the one-pass decode kernel on
    the auto path; fp32 math, so the row state is held to the precise path's
    tolerance and the bf16 output to its rounding."""
    Q, K, V, lt, la, _ = make_inputs(B, H, Lq, Lk, seed=Lq * 31 + Lk, dtype=torch.bfloat16, la_std=0.3)
    scale = 0.125
    mask = torch.from_numpy(OA.causal_mask(Lq, Lk)) if causal else None
    assert_no_near_ties(Q, K, scale, mask)
    out, m, z, a = fwd_direct(Q, K, V, lt, la, sigma, scale, "auto", causal=causal)
    f = lambda t: t.float().numpy()
    ref_out, ctx = OA.forward(f(Q), f(K), f(V), f(lt), f(la), sigma,
                              None if mask is None else mask.numpy(), scale)
    assert rel_err(out, ref_out) < 8e-3, rel_err(out, ref_out)
    assert np.abs(m - ctx["m"]).max() < 1e-5
    assert np.array_equal(a, ctx["argmax"])
    assert rel_err(z, ctx["Z"]) < TOL_FP32


def test_decode_forward_mask_tensor_and_fallback():
    """An explicit additive mask on the decode kernel; fp32 inputs (no 16-byte
    rows of 8 halves) take the tiled precise kernel on the auto path."""
    Q, K, V, lt, la, _ = make_inputs(2, 3, 2, 90, seed=5, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(5)
    mask = torch.where(torch.rand(1, 1, 2, 90, generator=g) < 0.3, -1e9, 0.0)
    out, m, z, a = fwd_direct(Q, K, V, lt, la, "softplus", 0.125, "auto", mask=mask)
    f = lambda t: t.float().numpy()
    ref_out, ctx = OA.forward(f(Q), f(K), f(V), f(lt), f(la), "softplus", mask.numpy(), 0.125)
    assert rel_err(out, ref_out) < 8e-3
    assert np.array_equal(a, ctx["argmax"]) and rel_err(z, ctx["Z"]) < TOL_FP32
    Qf, Kf, Vf = Q.float(), K.float(), V.float()
    out, m, z, a = fwd_direct(Qf, Kf, Vf, lt, la, "softplus", 0.125, "auto", layout="bhld")
    ref_out, ctx = OA.forward(f(Qf), f(Kf), f(Vf), f(lt), f(la), "softplus", None, 0.125)
    assert rel_err(out, ref_out) < TOL_FP32 and np.array_equal(a, ctx["argmax"])


def test_decode_rows_through_autograd_fwd_bwd(A):
    """One-row calls through STauOpusAttentionFunction: the decode forward's row
    state feeds the backward."""
    Q, K, V, lt, la, dO = make_inputs(2, 4, 1, 300, seed=8, dtype=torch.bfloat16, la_std=0.2)
    assert_no_near_ties(Q, K, 0.125)
    mine = run_op(A, Q, K, V, lt, la, "softplus", dO, None, 0.125, path="auto")
    ref = oracle(Q, K, V, lt, la, "softplus", dO, None, 0.125)
    assert_close(mine, ref, TOL_BF16, "decode fwd + bwd")
