"""Host logic of the tau* estimator (collect, flatten to (N, H, T), -1e9
padding to the longest key length, sigma by module name, per-entry means and
rounding, to_dict) against the reference's own TauStarEstimator output
(tests/golden/tau_star.npz, tau_star/tau_star_solver.py:154-281). The solver
itself is the oracle here: this file needs no GPU."""
import json
import os

import numpy as np
import torch

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")


def test_estimator_host_logic_matches_reference(monkeypatch):
    from oracle import tau_star as OT
    from tau_dxb_b200 import tau_star as TS

    def oracle_solve(scores, sigma="softplus", n_iter=30, tau_init=2.0, tau_min=0.1, tau_max=10.0, eps=1e-6):
        t, k = OT.solve_tau_star(scores.numpy(), sigma, n_iter, tau_init, tau_min, tau_max, eps)
        return torch.from_numpy(np.asarray(t)), torch.from_numpy(np.asarray(k))

    monkeypatch.setattr(TS, "solve_tau_star", oracle_solve)
    z = np.load(os.path.join(GOLDEN, "tau_star.npz"))
    est = TS.TauStarEstimator(n_iter=25)
    est.collect("empty", torch.zeros(0, 4, 3))           # ignored, as in the reference
    for ci in range(4):
        est.collect(str(z[f"e{ci}_name"]), torch.from_numpy(z[f"e{ci}_scores"]))
    res = est.aggregate(device="cpu")
    assert [r.module_name for r in res] == [str(z["m0_name"]), str(z["m1_name"])]
    # substring match on the map's keys: names that contain a key take its
    # sigma; HF module names ("decoder.layers.1.encoder_attn") contain none of
    # them, so they take softplus, as in the reference
    assert est._resolve_sigma("whisper.decoder.encoder_attn") == "exp"
    assert est._resolve_sigma("m.decoder.self_attn.k") == "sigmoid"
    assert est._resolve_sigma("model.decoder.layers.1.encoder_attn") == "softplus"
    assert est._resolve_sigma("something.else") == "softplus"
    for mi, r in enumerate(res):
        assert r.num_heads == 4
        assert np.allclose(r.tau_per_head, z[f"m{mi}_tau"], atol=2e-4), (r.tau_per_head, z[f"m{mi}_tau"])
        assert np.allclose(r.kl_per_head, z[f"m{mi}_kl"], atol=2e-6)
        d, ref = r.to_dict(), json.loads(str(z[f"m{mi}_dict"]))
        assert set(d) == set(ref)
        assert abs(d["tau_mean"] - ref["tau_mean"]) < 2e-4 and abs(d["tau_std"] - ref["tau_std"]) < 2e-4
    assert TS._std([]) == 0.0 and TS.ModuleResult("x", 2).to_dict()["tau_mean"] == 0.0


def test_analytic_oracle_matches_reference_golden():
    from oracle import tau_star as OT
    z = np.load(os.path.join(GOLDEN, "tau_star.npz"))
    for ci in range(6):
        k = f"c{ci}"
        a = OT.solve_tau_star_analytic(z[k + "_scores"], str(z[k + "_sigma"]))
        assert np.allclose(a, z[k + "_analytic"], rtol=1e-5, atol=2e-6), (ci, np.abs(a - z[k + "_analytic"]).max())
