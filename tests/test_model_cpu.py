"""Host logic of the Whisper patches and the train step, on CPU.

The tau-opus / WTA operators are routed to the oracle here (the CUDA kernels
need a GPU); everything else -- module attachment, parameter names, tau
initialisation, hooks, learnable k, sparsity loss, win tracking, pruning,
removal -- is the product code."""
import json
import math

import pytest
import numpy as np
import torch

from oracle_ops import use_oracle_ops
from oracle import wta as OW


def tiny_cfg(**kw):
    from tau_dxb_b200.train import StepConfig
    c = dict(batch=2, frames=200, label_len=24, min_label=8, encoder_layers=1, decoder_layers=1,
             d_model=128, heads=2, ffn=512, vocab=500)
    c.update(kw)
    return StepConfig(**c)


@pytest.fixture()
def patched(monkeypatch):
    use_oracle_ops(monkeypatch)
    from tau_dxb_b200 import train as T
    cfg = tiny_cfg()
    model = T.build_model(cfg, "cpu")
    yield cfg, model
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import patch_whisper_stau as ST
    ST.remove_stau(model)
    SG.remove_sparse_grad(model)


def test_attachment_names_and_sigmas(patched):
    cfg, model = patched
    names = [n for n, _ in model.named_parameters()]
    taus = [n for n in names if n.endswith("_stau_opus.log_tau")]
    alphas = [n for n in names if n.endswith("_stau_opus.log_alpha")]
    ks = [n for n in names if n.endswith("_learnable_k.logit_k")]
    assert len(taus) == 3 and len(alphas) == 3 and len(ks) == 2
    sig = {}
    for n, m in model.named_modules():
        if hasattr(m, "_stau_opus") and m._stau_opus is not None:
            sig[n] = m._stau_opus.sigma_name
    assert sig["model.encoder.layers.0.self_attn"] == "softplus"
    assert sig["model.decoder.layers.0.self_attn"] == "sigmoid"
    assert sig["model.decoder.layers.0.encoder_attn"] == "exp"
    dec = dict(model.named_modules())["model.decoder.layers.0.self_attn"]._stau_opus
    assert dec.assume_causal
    enc = dict(model.named_modules())["model.encoder.layers.0.self_attn"]._stau_opus
    assert not enc.assume_causal


def test_tau_init_and_log_tau_mapping():
    from tau_dxb_b200 import patch_whisper_stau as ST
    for t in (1.0, 1.0005, 1.2, 2.5, 4.6):
        lt = ST._log_tau_for_init(t)
        back = math.log1p(math.exp(lt)) + 1
        if t <= 1.001:
            assert lt == -8.0
        else:
            assert back == pytest.approx(t, abs=1e-9)


def test_load_tau_dict_formats(tmp_path):
    from tau_dxb_b200 import patch_whisper_stau as ST
    a = [{"module_name": "model.encoder.layers.3.self_attn", "tau_per_head": [1.5, 1.2]},
         {"module_name": "model.decoder.layers.1.encoder_attn", "tau_per_head": [1.0, 1.0]},
         {"module_name": "model.decoder.layers.2.self_attn", "tau_per_head": [2.0, 3.0]}]
    b = [{"attention_type": "decoder_self", "layer_idx": 4, "tau_per_head": [1.1, 1.3]},
         {"is_decoder": True, "cross_attention": True, "layer_idx": 0, "tau_per_head": [1.0, 1.0]},
         {"is_decoder": False, "tau_per_head": [1.7, 1.8]}]
    pa, pb = tmp_path / "a.json", tmp_path / "b.json"
    pa.write_text(json.dumps(a))
    pb.write_text(json.dumps(b))
    da, db = ST.load_tau_dict(pa), ST.load_tau_dict(pb)
    assert da["encoder_self"][3] == [1.5, 1.2] and da["decoder_cross"][1] == [1.0, 1.0]
    assert da["decoder_self"][2] == [2.0, 3.0]
    assert db["decoder_self"][4] == [1.1, 1.3] and db["decoder_cross"][0] == [1.0, 1.0]
    assert db["encoder_self"][0] == [1.7, 1.8]


def test_learnable_k_rounding_and_sparsity_loss(patched):
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    lk = SG.LearnableKRatio(0.4)
    assert lk.get_k(3072) == OW.k_from_logit(float(lk.logit_k), 3072)
    torch.nn.init.constant_(lk.logit_k, -2.2)
    assert lk.get_k(3072) == 306
    assert float(lk.logit_k) == pytest.approx(-2.2)
    sp = SG.get_sparsity_loss()
    assert float(sp) == pytest.approx(0.4, abs=1e-6)
    for r in (0.05, 0.5, 0.95):
        assert float(SG.LearnableKRatio(r).logit_k) == pytest.approx(OW.logit_for_ratio(r), abs=1e-6)


def test_forward_backward_reaches_every_added_parameter(patched):
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import train as T
    cfg, model = patched
    g = torch.Generator().manual_seed(0)
    mel, labels = T.synthetic_batch(cfg, "cpu", g)
    out = model(input_features=mel, labels=labels)
    loss = out.loss + cfg.sparsity_lambda * SG.get_sparsity_loss()
    assert torch.isfinite(loss)
    loss.backward()
    for n, p in model.named_parameters():
        if "log_tau" in n or "log_alpha" in n or "logit_k" in n:
            assert p.grad is not None and torch.isfinite(p.grad).all(), n
    tr = SG.get_win_tracker()
    w = tr.win_counts["model.encoder.layers.0"]
    k = dict(model.named_modules())["model.encoder.layers.0"]._learnable_k.get_k(cfg.ffn)
    assert int(w.sum()) >= k * cfg.batch * (cfg.frames // 2)   # >= k wins per encoder token


def test_hooks_inert_without_grad_and_removal(patched, monkeypatch):
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import patch_whisper_stau as ST
    cfg, model = patched
    calls = []
    monkeypatch.setattr(SG, "_WTAFusedCounting", type("Spy", (), {"apply": staticmethod(
        lambda x, k, w: calls.append(1) or x)}))
    with torch.no_grad():
        model(input_features=torch.randn(1, 80, 200), decoder_input_ids=torch.zeros(1, 4, dtype=torch.long))
    assert calls == []
    ST.remove_stau(model)
    SG.remove_sparse_grad(model)
    from transformers.models.whisper import modeling_whisper as W
    assert W.eager_attention_forward is ST._ORIGINAL_EAGER_FORWARD
    assert SG._HOOK_HANDLES == []


def test_prune_low_winners_masks_gradients(patched):
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    cfg, model = patched
    tr = SG.get_win_tracker()
    buf = tr.buffer("model.encoder.layers.0", cfg.ffn, "cpu")
    buf.fill_(10)
    buf[:7] = 0
    n = SG.prune_low_winners(model, threshold=0.05)
    assert n == 7
    fc1 = dict(model.named_modules())["model.encoder.layers.0"].fc1
    g = torch.ones_like(fc1.weight)
    hooked = SG._make_fc1_weight_grad_hook("model.encoder.layers.0")(g)
    assert float(hooked[:7].abs().sum()) == 0 and float(hooked[7:].abs().min()) == 1
    SG.unfreeze_all()
    assert SG._GRAD_MASKS == {}


def test_step_flops_formula():
    from tau_dxb_b200.train import StepConfig, model_flops_per_step
    assert model_flops_per_step(StepConfig()) / 1e12 == pytest.approx(26.79, abs=0.01)


def test_padded_head_loss_equals_the_plain_head():
    """The train step's LM head over a vocabulary padded to a multiple of 64
    (zero weight rows, -inf bias) gives HF Whisper's own loss and gradients."""
    from tau_dxb_b200 import train as T
    cfg = T.StepConfig(batch=2, frames=200, label_len=16, min_label=6, encoder_layers=1,
                       decoder_layers=1, d_model=64, heads=2, ffn=128, vocab=300)
    torch.manual_seed(0)
    from transformers import WhisperForConditionalGeneration
    model = WhisperForConditionalGeneration(T.whisper_config(cfg)).double()
    mel, labels = T.synthetic_batch(cfg, "cpu", torch.Generator().manual_seed(3))
    mel = mel.double()
    ref = model(input_features=mel, labels=labels).loss
    ref.backward()
    g_ref = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    model.zero_grad(set_to_none=True)
    head = T.PaddedHeadLoss(model)
    assert head.pad == 20
    loss = head(mel, labels)
    loss.backward()
    assert torch.allclose(loss, ref, rtol=1e-12, atol=1e-12)
    for n, p in model.named_parameters():
        if n in g_ref:
            assert torch.allclose(p.grad, g_ref[n], rtol=1e-10, atol=1e-12), n


def test_lr_schedule_matches_reference_table():
    """Warmup + cosine warm restarts, against the reference's own lambda."""
    import os
    from conftest import GOLDEN
    from tau_dxb_b200 import train as T
    z = np.load(os.path.join(GOLDEN, "lr_table.npz"))
    for w, t0, tm, step, f in zip(z["warmup"], z["t0"], z["t_mult"], z["step"], z["factor"]):
        assert abs(T.lr_lambda(int(w), int(t0), int(tm))(int(step)) - float(f)) < 1e-12, (w, t0, tm, step)


def test_train_step_ema_schedule_and_accumulation(monkeypatch):
    """grad_accum micro-batches make one optimiser step; the LR schedule steps
    with it and the EMA shadow moves by (1 - decay) toward the new weights."""
    from tau_dxb_b200 import train as T
    use_oracle_ops(monkeypatch)
    cfg = T.StepConfig(batch=1, frames=200, label_len=16, min_label=6, encoder_layers=1,
                       decoder_layers=1, d_model=64, heads=2, ffn=128, vocab=300, grad_accum=2,
                       ema_decay=0.9, warmup_steps=4, t0_steps=8, lr=1e-3)
    step = T.TrainStep(cfg, "cpu")
    g = torch.Generator().manual_seed(4)
    b = [T.synthetic_batch(cfg, "cpu", g) for _ in range(2)]
    w0 = [p.detach().clone() for p in step.model.parameters()]
    step.step(*b[0])
    assert all(torch.equal(a, p.detach()) for a, p in zip(w0, step.model.parameters()))
    assert step.sched.last_epoch == 0 and step.micro == 1
    step.step(*b[1])
    assert step.sched.last_epoch == 1 and step.micro == 0
    # the first optimiser step runs at warmup factor 0 (as in the reference)
    assert all(torch.equal(a, p.detach()) for a, p in zip(w0, step.model.parameters()))
    assert step.opt.param_groups[0]["lr"] == pytest.approx(1e-3 * T.lr_lambda(4, 8, 2)(1))
    shadow1 = [t.clone() for t in step.ema.shadow]
    step.step(*b[0])
    step.step(*b[1])
    params = [p for p in step.model.parameters() if p.requires_grad]
    moved = 0
    for p, s0, s1 in zip(params, shadow1, step.ema.shadow):
        assert torch.allclose(s1, s0 + 0.1 * (p.detach() - s0), atol=1e-7)
        moved += int(not torch.equal(s1, s0))
    assert moved > 0
