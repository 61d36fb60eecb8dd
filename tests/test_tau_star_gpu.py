"""GPU tau* solver (tau_star_solve) against the reference's own outputs
(tests/golden/tau_star.npz, made by tau_star/tau_star_solver.py:60-128) and
against the numpy oracle on seeded scores: every transfer function, ragged and
long rows (register and shared-memory kernels), padding, -inf masks, strided
input, per-head means as compute_tau_star_echo.py:116-136 reports them, and
the full encoder-layer size through the Newton fixed-point property."""
import os

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(ROOT, "tests", "golden")


def _check(tau, kl, ref_tau, ref_kl, T, what, scores=None, sigma=None):
    """tau within tolerance except on rows where log sigma is constant: there
    p_tau is uniform for every tau, the KL does not depend on tau, and the
    Newton step is one ulp of E_p - e_ref divided by eps, so tau is rounding
    noise in the reference as well; those rows check the KL only."""
    from oracle import tau_star as OT
    T = int(T)
    tau, kl = tau.cpu().numpy().reshape(-1), kl.cpu().numpy().reshape(-1)
    ref_tau, ref_kl = np.asarray(ref_tau).reshape(-1), np.asarray(ref_kl).reshape(-1)
    free = np.zeros(tau.shape, bool)
    cond = np.zeros(tau.shape)
    if scores is not None:
        with np.errstate(all="ignore"):
            ls = OT.log_sigma(sigma, np.asarray(scores, np.float32).reshape(-1, T))
            free = ls.max(-1) == ls.min(-1)
            # the fixed point E_p[ls] = e_ref moves by (rounding of E_p - e_ref) /
            # Var_p: fp32 sums of T terms of size max|ls|, at the reference's tau
            l64 = ls.astype(np.float64)
            x = ref_tau[:, None].astype(np.float64) * l64
            p = np.exp(x - x.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            e_p = (p * l64).sum(-1)
            var = (p * (l64 - e_p[:, None]) ** 2).sum(-1)
            cond = 2.0 ** -23 * np.abs(l64).max(-1) * np.sqrt(T) / var
        cond = np.nan_to_num(cond, nan=0.0, posinf=0.0)
    # two keys: the KL is flat in tau near its minimum, so fp32 rounding moves
    # tau by ~1e-3 while the KL agrees to 2e-7; otherwise the Newton fixed point
    # agrees to a few fp32 ulps of the accumulated sums, scaled by its condition
    rtol = 2e-3 if T <= 2 else 1e-4
    d = ~free
    err = np.abs(tau - ref_tau)
    assert np.all((err <= 2e-5 + rtol * np.abs(ref_tau) + cond)[d]), (what, err[d].max())
    assert np.allclose(kl[d], ref_kl[d], rtol=1e-3, atol=2e-6), (what, np.abs(kl[d] - ref_kl[d]).max())
    if free.any():
        # the KL is tau-free only in exact arithmetic: exp(tau ls - logsumexp)
        # rounds its exponent at the scale of tau |ls| (up to 10 x 69 for relu),
        # and each side does so at its own tau
        scale = np.maximum(np.abs(tau), np.abs(ref_tau))[free] * np.abs(ls[free]).max(-1)
        err = np.abs(kl[free] - ref_kl[free])
        assert np.all(err <= 2e-6 + 1e-3 * np.abs(ref_kl[free]) + 4.8e-7 * scale), (what, err.max())


def test_tau_star_matches_reference_golden():
    from tau_dxb_b200 import tau_star as TS
    z = np.load(os.path.join(GOLDEN, "tau_star.npz"))
    for ci in range(6):
        k = f"c{ci}"
        T, n_iter, tau_init = z[k + "_meta"]
        s = torch.from_numpy(z[k + "_scores"]).cuda()
        tau, kl = TS.solve_tau_star(s, str(z[k + "_sigma"]), int(n_iter), float(tau_init))
        _check(tau, kl, z[k + "_tau"], z[k + "_kl"], T, k, z[k + "_scores"], str(z[k + "_sigma"]))


def _scores(seed, rows, T, scale=2.0):
    g = np.random.default_rng(seed)
    return (g.standard_normal((rows, T)) * scale + g.standard_normal((rows, 1))).astype(np.float32)


@pytest.mark.parametrize("sigma", ["softplus", "sigmoid", "exp", "relu"])
@pytest.mark.parametrize("T", [2, 3, 31, 33, 100, 448, 1500, 2048, 2049, 4000])
def test_tau_star_matches_oracle(sigma, T):
    from oracle import tau_star as OT
    from tau_dxb_b200 import tau_star as TS
    rows = 37 if T <= 2048 else 9
    s = _scores(T * 7 + len(sigma), rows, T)
    s[3, T // 2:] = -1e9                     # padded keys
    ref_tau, ref_kl = OT.solve_tau_star(s, sigma, n_iter=40)
    tau, kl = TS.solve_tau_star(torch.from_numpy(s).cuda(), sigma, n_iter=40)
    _check(tau, kl, ref_tau, ref_kl, T, (sigma, T), s, sigma)


def test_tau_star_edge_rows():
    """-inf keys (NaN path -> tau_init, 0 in the reference for sigmoid/exp),
    constant rows (zero variance, eps damping), clamping at both bounds, n_iter
    0, one key, no rows, strided and batched input."""
    from oracle import tau_star as OT
    from tau_dxb_b200 import tau_star as TS
    T = 80
    s = _scores(5, 16, T)
    s[0, 40:] = -np.inf
    s[1] = 0.5
    s[2] *= 40.0
    s[3] *= 0.01
    for sigma in ("softplus", "sigmoid", "exp", "relu"):
        for n_iter, kw in ((30, {}), (0, {}), (15, dict(tau_init=0.5, tau_min=0.2, tau_max=3.0, eps=1e-3))):
            ref_tau, ref_kl = OT.solve_tau_star(s, sigma, n_iter=n_iter, **kw)
            tau, kl = TS.solve_tau_star(torch.from_numpy(s).cuda(), sigma, n_iter=n_iter, **kw)
            _check(tau, kl, ref_tau, ref_kl, T, (sigma, n_iter), s, sigma)
    # strided rows: every other row of a wider buffer, [..., T] batch shape
    big = torch.from_numpy(_scores(6, 2 * 3 * 5, 2 * T)).cuda().view(2, 3, 5, 2 * T)[..., 7:7 + T]
    tau, kl = TS.solve_tau_star(big, "softplus")
    assert tau.shape == (2, 3, 5)
    ref_tau, ref_kl = OT.solve_tau_star(big.cpu().numpy(), "softplus")
    _check(tau, kl, ref_tau, ref_kl, T, "strided")
    tau, kl = TS.solve_tau_star(torch.randn(4, 6, 1, device="cuda"), "exp", tau_init=1.5)
    assert torch.all(tau == 1.5) and torch.all(kl == 0)
    tau, kl = TS.solve_tau_star(torch.randn(0, 50, device="cuda"))
    assert tau.shape == (0,) and kl.shape == (0,)
    with pytest.raises(TypeError):
        TS.solve_tau_star(torch.randn(2, 8, device="cuda"), sigma=lambda x: x)


def test_estimate_tau_per_head_matches_oracle():
    from oracle import tau_star as OT
    from tau_dxb_b200 import tau_star as TS
    B, H, Lq, Lk = 2, 3, 24, 60
    s = np.random.default_rng(11).standard_normal((B, H, Lq, Lk)).astype(np.float32) * 3.0
    taus, kls = TS.estimate_tau_per_head(torch.from_numpy(s).cuda(), None, "sigmoid")
    for h in range(H):
        rt, rk = OT.solve_tau_star(s[:, h].reshape(-1, Lk), "sigmoid", n_iter=100)
        assert abs(taus[h] - round(float(rt.mean()), 4)) <= 2e-4, (h, taus[h], rt.mean())
        assert abs(kls[h] - round(float(rk.mean()), 6)) <= 2e-6, (h, kls[h], rk.mean())


def test_tau_star_encoder_layer_fixed_point():
    """One Whisper-small encoder self-attention call (12 heads x 1500 x 1500,
    n_iter 100): sampled rows equal the oracle's, and every row not at a clamp
    bound sits at the Newton fixed point E_p[log sigma] = E_ref[log sigma]
    (checked in fp64)."""
    from oracle import tau_star as OT
    from tau_dxb_b200 import tau_star as TS
    g = torch.Generator(device="cuda").manual_seed(3)
    s = torch.randn(1, 12, 1500, 1500, device="cuda", generator=g) * 2.5
    tau, kl = TS.solve_tau_star(s, "softplus", n_iter=100)
    torch.cuda.synchronize()
    assert torch.isfinite(tau).all() and torch.isfinite(kl).all() and (kl >= -1e-6).all()
    flat = s.view(-1, 1500)
    pick = torch.arange(0, flat.shape[0], 997, device="cuda")
    sample = flat[pick].cpu().numpy()
    rt, rk = OT.solve_tau_star(sample, "softplus", n_iter=100)
    _check(tau.view(-1)[pick], kl.view(-1)[pick], rt, rk, 1500, "encoder sample")
    x = flat[:2048].double()
    ls = torch.log(torch.nn.functional.softplus(x).clamp_min(1e-30))
    e_ref = (torch.softmax(x, -1) * ls).sum(-1)
    t = tau.view(-1)[:2048].double()
    e_p = (torch.softmax(t[:, None] * ls, -1) * ls).sum(-1)
    inside = (t > 0.1 + 1e-4) & (t < 10.0 - 1e-4)
    assert inside.any()
    assert (e_p - e_ref)[inside].abs().max().item() < 2e-4


def test_analytic_matches_reference_and_oracle():
    from oracle import tau_star as OT
    from tau_dxb_b200 import tau_star as TS
    z = np.load(os.path.join(GOLDEN, "tau_star.npz"))
    for ci in range(6):
        k = f"c{ci}"
        a = TS.solve_tau_star_analytic(torch.from_numpy(z[k + "_scores"]).cuda(), str(z[k + "_sigma"]))
        assert np.allclose(a.cpu().numpy(), z[k + "_analytic"], rtol=1e-4, atol=2e-6), k
    for sigma in ("softplus", "sigmoid", "exp", "relu"):
        s = _scores(77, 40, 1500)
        s[5, 700:] = -1e9
        a = TS.solve_tau_star_analytic(torch.from_numpy(s).cuda().view(4, 10, 1500), sigma)
        assert a.shape == (4, 10)
        ref = OT.solve_tau_star_analytic(s, sigma)
        assert np.allclose(a.cpu().numpy().reshape(-1), ref, rtol=1e-4, atol=2e-6), sigma


def test_estimator_on_gpu_matches_reference():
    from tau_dxb_b200 import tau_star as TS
    z = np.load(os.path.join(GOLDEN, "tau_star.npz"))
    est = TS.TauStarEstimator(n_iter=25)
    for ci in range(4):
        est.collect(str(z[f"e{ci}_name"]), torch.from_numpy(z[f"e{ci}_scores"]))
    for mi, r in enumerate(est.aggregate()):
        assert r.module_name == str(z[f"m{mi}_name"])
        assert np.allclose(r.tau_per_head, z[f"m{mi}_tau"], atol=2e-4)
        assert np.allclose(r.kl_per_head, z[f"m{mi}_kl"], atol=2e-6)

