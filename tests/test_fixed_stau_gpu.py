"""The fixed-tau path: STauOpusMaxStableFn on tau_opus_fixed_fwd / _bwd against
the reference's own outputs (tests/golden/maxstable.npz) and the oracle, and
apply_fixed_stau on a small Whisper (echo/patch_whisper_stau.py:74-112,
190-214, 279-322). fp32 throughout with accurate math functions: 3e-5 on the
weights (tanhf / powf rounding grows with tau up to 3), 1e-4 on the score
gradient (max relative error)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_err
from oracle import stau_fixed as OF

DEV = "cuda"


@pytest.fixture(scope="module")
def P():
    from tau_dxb_b200 import patch_whisper_stau
    return patch_whisper_stau


def _run(P, scores, tau, sigma, dO):
    s = torch.from_numpy(scores).to(DEV).requires_grad_()
    t = torch.from_numpy(tau).to(DEV).view(1, -1, 1, 1) if tau.size > 1 else float(tau[0])
    attn = P.STauOpusMaxStableFn.apply(s, t, sigma)
    attn.backward(torch.from_numpy(dO).to(DEV))
    torch.cuda.synchronize()
    return attn.detach().cpu().numpy(), s.grad.cpu().numpy()


@pytest.mark.gpu
def test_fixed_weights_match_reference_golden(P):
    g = np.load(os.path.join(GOLDEN, "maxstable.npz"))
    for ci in range(int(g["n_cases"])):
        sg = str(g[f"c{ci}_sigma"])
        attn, ds = _run(P, g[f"c{ci}_scores"], g[f"c{ci}_tau"], sg, g[f"c{ci}_dO"])
        assert rel_err(attn, g[f"c{ci}_attn"]) < 3e-5, (ci, sg, rel_err(attn, g[f"c{ci}_attn"]))
        assert rel_err(ds, g[f"c{ci}_dscores"]) < 1e-4, (ci, sg, rel_err(ds, g[f"c{ci}_dscores"]))


@pytest.mark.gpu
@pytest.mark.parametrize("sigma", OF.SIGMAS)
def test_fixed_weights_match_oracle_decoder_cross_size(P, sigma):
    """B=2, H=12, 448 x 1500 (the cross-attention shape), per-head tau."""
    rng = np.random.default_rng(7)
    scores = (rng.standard_normal((2, 12, 448, 1500)) * 2.5).astype(np.float32)
    tau = (1.0 + rng.random(12) * 2.0).astype(np.float32)
    dO = rng.standard_normal(scores.shape).astype(np.float32)
    attn, ds = _run(P, scores, tau, sigma, dO)
    assert rel_err(attn, OF.forward(scores, tau, sigma)) < 3e-5
    ref = OF.backward(scores, tau, sigma, dO)
    if sigma == "relu":       # sigma' = 0 for every x <= 0: the gradient is exactly zero
        assert np.abs(ds).max() == 0 and np.abs(ref).max() == 0
    else:
        assert rel_err(ds, ref) < 1e-4


@pytest.mark.gpu
def test_fixed_weights_edges(P):
    """Masked rows (finfo.min and -inf), a single key, a scalar tau below 1."""
    rng = np.random.default_rng(3)
    scores = rng.standard_normal((1, 2, 5, 9)).astype(np.float32)
    scores[0, 0, 1, 3:] = np.finfo(np.float32).min
    scores[0, 1, 2, :7] = -np.inf
    dO = rng.standard_normal(scores.shape).astype(np.float32)
    for tau in (np.array([0.6], np.float32), np.array([1.3, 2.2], np.float32)):
        attn, ds = _run(P, scores, tau, "softplus", dO)
        assert rel_err(attn, OF.forward(scores, tau, "softplus")) < 3e-5
        assert rel_err(ds, OF.backward(scores, tau, "softplus", dO)) < 1e-4
    one = rng.standard_normal((3, 1)).astype(np.float32)
    attn, ds = _run(P, one, np.array([2.0], np.float32), "sigmoid", np.ones_like(one))
    assert np.allclose(attn, 1.0) and np.allclose(ds, OF.backward(one, 2.0, "sigmoid", np.ones_like(one)), atol=1e-6)


def _torch_fixed_weights(scores, tau, sigma_name):
    """The same weights written with differentiable torch ops (autograd gives
    the reference's gradient up to the clamped entries, whose share is ~1e-8)."""
    import torch.nn.functional as F
    x = scores - scores.max(dim=-1, keepdim=True).values
    sig = {"softplus": F.softplus, "sigmoid": torch.sigmoid, "exp": lambda v: torch.exp(v.clamp(max=20)),
           "relu": F.relu, "tanh_shift": lambda v: torch.tanh(v) + 1}[sigma_name](x).clamp(min=1e-8)
    q = sig.pow(tau)
    return q / q.sum(dim=-1, keepdim=True).clamp(min=1e-8)


@pytest.mark.gpu
def test_apply_fixed_stau_on_whisper(P, monkeypatch):
    from tau_dxb_b200 import train as T
    from transformers import WhisperForConditionalGeneration
    cfg = T.StepConfig(batch=2, frames=200, label_len=24, min_label=8, encoder_layers=2, decoder_layers=2,
                       d_model=128, heads=2, ffn=256, vocab=300)
    g = torch.Generator().manual_seed(2)
    mel, labels = T.synthetic_batch(cfg, DEV, g)
    taus = {"encoder_self": {0: [1.5, 2.0], 1: [1.2, 1.1]}, "decoder_self": {0: [3.0, 1.0]},
            "decoder_cross": {1: [1.4, 1.6]}}
    sig = {"encoder_self": "softplus", "decoder_self": "sigmoid", "decoder_cross": "tanh_shift"}

    def run():
        torch.manual_seed(0)
        model = WhisperForConditionalGeneration(T.whisper_config(cfg)).to(DEV)
        P.apply_fixed_stau(model, taus, sig)
        loss = model(input_features=mel, labels=labels).loss
        loss.backward()
        grads = {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}
        P.remove_stau(model)
        return loss.detach(), grads, model

    loss, grads, model = run()
    attn = model.model.encoder.layers[0].self_attn
    assert attn._stau_tau is None     # cleared by remove_stau
    monkeypatch.setattr(P.STauOpusMaxStableFn, "apply", staticmethod(_torch_fixed_weights))
    loss_ref, grads_ref, _ = run()
    assert torch.isfinite(loss) and abs(float(loss) - float(loss_ref)) < 1e-5 * abs(float(loss_ref))
    for n, v in grads_ref.items():
        assert rel_err(grads[n].cpu().numpy(), v.cpu().numpy()) < 1e-4, n


def test_apply_fixed_stau_sets_site_taus_and_sigmas(P):
    """Host-side bookkeeping (no kernel runs): per-site tau tensors and sigmas,
    the eager-attention swap, unknown tau_source types rejected."""
    from tau_dxb_b200 import train as T
    from transformers import WhisperForConditionalGeneration
    from transformers.models.whisper import modeling_whisper as W
    cfg = T.StepConfig(batch=1, frames=200, label_len=16, min_label=6, encoder_layers=2, decoder_layers=1,
                       d_model=128, heads=2, ffn=256, vocab=300)
    model = WhisperForConditionalGeneration(T.whisper_config(cfg))
    P.apply_fixed_stau(model, {"encoder_self": {1: [1.5, 2.5]}}, {"decoder_cross": "exp"})
    enc1 = model.model.encoder.layers[1].self_attn
    enc0 = model.model.encoder.layers[0].self_attn
    cross = model.model.decoder.layers[0].encoder_attn
    assert enc1._stau_tau.shape == (1, 2, 1, 1) and enc1._stau_tau.flatten().tolist() == [1.5, 2.5]
    assert enc0._stau_tau.flatten().tolist() == [1.0, 1.0]
    assert enc1._stau_sigma == "softplus" and cross._stau_sigma == "exp"
    assert W.eager_attention_forward is not P._ORIGINAL_EAGER_FORWARD
    P.apply_fixed_stau(model, 2.0)
    assert cross._stau_tau.flatten().tolist() == [2.0, 2.0]
    with pytest.raises(TypeError):
        P.apply_fixed_stau(model, [1.0, 2.0])
    with pytest.raises(RuntimeError, match="CUDA"):
        P.STauOpusMaxStableFn.apply(torch.zeros(1, 2, 3, 4), 1.5, "softplus")
    with pytest.raises(KeyError):
        P.STauOpusMaxStableFn.apply(torch.zeros(1, 2, 3, 4), 1.5, "nope")
    P.remove_stau(model)
    assert W.eager_attention_forward is P._ORIGINAL_EAGER_FORWARD
