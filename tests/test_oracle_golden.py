"""Pin the oracle: it must reproduce the reference's own outputs.

The golden files were produced by running the reference's eager operators
(tests/golden/make_golden.py). Everything here runs on CPU.
"""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, rel_err
from oracle import stau_attention as OA
from oracle import wta as OW

ATTN_FILES = sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz")))


def _load(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("path", ATTN_FILES, ids=lambda p: os.path.basename(p)[:-4])
def test_attention_oracle_matches_reference(path):
    g = _load(path)
    scale = float(g["scale"])
    scale = None if np.isnan(scale) else scale
    out, grads, _ = OA.forward_backward(g["Q"], g["K"], g["V"], g["log_tau"], g["log_alpha"],
                                        str(g["sigma"]), g["dO"], g.get("mask"), scale)
    names = ["dQ", "dK", "dV", "dlog_tau", "dlog_alpha"]
    assert rel_err(out, g["out"]) < 2e-6
    for n, a in zip(names, grads):
        tol = 5e-5 if n.startswith("dlog") else 2e-5
        assert rel_err(a, g[n]) < tol, (n, rel_err(a, g[n]))


@pytest.mark.parametrize("path", ATTN_FILES, ids=lambda p: os.path.basename(p)[:-4])
def test_torch_host_oracle_matches_reference(path):
    """The torch restatement bench.py times as the reference's eager CPU path."""
    from oracle import stau_attention_torch as OT
    g = _load(path)
    scale = float(g["scale"])
    scale = None if np.isnan(scale) else scale
    out, grads = OT.forward_backward(g["Q"], g["K"], g["V"], g["log_tau"], g["log_alpha"],
                                     str(g["sigma"]), g["dO"], g.get("mask"), scale)
    assert rel_err(out.numpy(), g["out"]) < 2e-6
    for n, a in zip(["dQ", "dK", "dV", "dlog_tau", "dlog_alpha"], grads):
        tol = 5e-5 if n.startswith("dlog") else 2e-5
        assert rel_err(a.numpy(), g[n]) < tol, (n, rel_err(a.numpy(), g[n]))


def test_attention_oracle_fp64_agrees():
    g = _load(os.path.join(GOLDEN, "attn_softplus_l65.npz"))
    out32, gr32, _ = OA.forward_backward(g["Q"], g["K"], g["V"], g["log_tau"], g["log_alpha"],
                                         "softplus", g["dO"])
    out64, gr64, _ = OA.forward_backward(g["Q"], g["K"], g["V"], g["log_tau"], g["log_alpha"],
                                         "softplus", g["dO"], dtype=np.float64)
    assert rel_err(out32, out64) < 1e-5
    for a, b in zip(gr32, gr64):
        assert rel_err(a, b) < 1e-4


def test_tau1_exp_is_softmax():
    g = _load(os.path.join(GOLDEN, "attn_exp_tau1_softmax.npz"))
    out, _ = OA.forward(g["Q"], g["K"], g["V"], g["log_tau"], g["log_alpha"], "exp")
    assert rel_err(out, g["softmax_out"]) < 1e-5
    assert rel_err(g["out"], g["softmax_out"]) < 1e-5


def test_causal_mask_matches_golden():
    g = _load(os.path.join(GOLDEN, "attn_sigmoid_causal_l70.npz"))
    m = OA.causal_mask(70, 70)
    assert np.array_equal(m, g["mask"])


def test_bad_sigma_name_raises():
    with pytest.raises(KeyError):
        OA.sigma("nope", np.zeros(3, np.float32))


# ---------------------------------------------------------------- WTA

@pytest.fixture(scope="module")
def wta_golden():
    return _load(os.path.join(GOLDEN, "wta_gelu_48x3072.npz"))


def test_wta_threshold_masks_bit_exact(wta_golden):
    g = wta_golden
    x = OW.bf16_bits_to_f32(g["x_bits"])
    for k in g["ks"]:
        m = OW.pack_mask_bits(OW.threshold_mask(x, int(k)))
        assert np.array_equal(m, g[f"thr_mask_k{k}"]), k
        assert bool(g[f"sg_out_is_x_k{k}"])


def test_wta_exact_k_masks_on_tie_free_rows(wta_golden):
    g = wta_golden
    x = OW.bf16_bits_to_f32(g["x_bits"])
    for k in g["ks"]:
        k = int(k)
        mine = OW.exact_k_mask(x, k)
        ref = np.unpackbits(g[f"exact_mask_k{k}"], axis=-1, bitorder="little")[:, :x.shape[1]].astype(bool)
        ties = OW.tie_rows(x, k)
        assert np.array_equal(mine[~ties], ref[~ties]), k
        # tie rows: same count, strict winners kept, chosen ties drawn from the tie set
        assert (ref.sum(-1) == k).all()
        thr = OW.threshold_values(x, k)[:, None]
        assert (ref[x > thr]).all()
        assert not (ref & (x < thr)).any()


def test_wta_y_and_dx_bits(wta_golden):
    g = wta_golden
    x = OW.bf16_bits_to_f32(g["x_bits"])
    dy = OW.bf16_bits_to_f32(g["dy_bits"])
    m_exact = np.unpackbits(g["exact_mask_k306"], axis=-1, bitorder="little").astype(bool)
    y = np.where(m_exact, x, np.float32(0))
    ref_y = OW.bf16_bits_to_f32(g["exact_y_bits_k306"])
    assert np.array_equal(y, ref_y)
    m_thr = OW.threshold_mask(x, 306)
    dx = OW.wta_backward(dy, m_thr)
    assert np.array_equal(dx, OW.bf16_bits_to_f32(g["sg_dx_bits_k306"]))


def test_k_rounding_table():
    g = _load(os.path.join(GOLDEN, "k_table.npz"))
    for lg, d, k in zip(g["logit"], g["d_ff"], g["k"]):
        assert OW.k_from_logit(float(lg), int(d)) == int(k), (lg, d, k)
    assert OW.k_from_logit(-2.2, 3072) == 306
    for r, lg in zip(g["init_ratio"], g["init_logit"]):
        assert OW.logit_for_ratio(float(r)) == pytest.approx(float(lg), abs=1e-6)


def test_bf16_roundtrip():
    rng = np.random.default_rng(0)
    v = rng.standard_normal(1000).astype(np.float32)
    bits = OW.f32_to_bf16_bits(v)
    back = OW.bf16_bits_to_f32(bits)
    assert np.abs(back - v).max() <= np.abs(v).max() * 2 ** -8
    assert np.array_equal(OW.f32_to_bf16_bits(back), bits)


def test_tau_star_oracle_matches_reference_golden():
    from oracle import tau_star as OT
    z = np.load(os.path.join(GOLDEN, "tau_star.npz"))
    for ci in range(6):
        k = f"c{ci}"
        T, n_iter, tau_init = z[k + "_meta"]
        tau, kl = OT.solve_tau_star(z[k + "_scores"], str(z[k + "_sigma"]), int(n_iter), float(tau_init))
        # two keys: the KL is flat in tau near its minimum, so fp32 rounding moves
        # tau by ~1e-3 while the KL agrees to 2e-7
        rtol = 2e-3 if T <= 2 else 2e-5
        assert np.allclose(tau, z[k + "_tau"], rtol=rtol, atol=2e-5), (ci, np.abs(tau - z[k + "_tau"]).max())
        assert np.allclose(kl, z[k + "_kl"], rtol=1e-3, atol=2e-6), (ci, np.abs(kl - z[k + "_kl"]).max())


def test_fixed_tau_oracle_matches_reference():
    """oracle.stau_fixed against STauOpusMaxStableFn's own outputs
    (echo/patch_whisper_stau.py:74-112): every sigma, per-head and scalar tau."""
    from oracle import stau_fixed as OF
    g = _load(os.path.join(GOLDEN, "maxstable.npz"))
    for ci in range(int(g["n_cases"])):
        sg = str(g[f"c{ci}_sigma"])
        sc, tau, dO = g[f"c{ci}_scores"], g[f"c{ci}_tau"], g[f"c{ci}_dO"]
        attn = OF.forward(sc, tau, sg)
        assert rel_err(attn, g[f"c{ci}_attn"]) < 2e-6, (ci, sg)
        ds = OF.backward(sc, tau, sg, dO)
        assert rel_err(ds, g[f"c{ci}_dscores"]) < 2e-5, (ci, sg, rel_err(ds, g[f"c{ci}_dscores"]))
