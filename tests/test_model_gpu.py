"""Model-level parity: a small Whisper patched with the B200 kernels (CUDA)
against the same model patched with the oracle (CPU), one step of loss and
gradients; plus the bf16 autocast step on the tensor-core path."""
import pytest
import torch

from conftest import rel_err
from oracle_ops import use_oracle_ops

pytestmark = pytest.mark.gpu


def tiny_cfg(**kw):
    from tau_dxb_b200.train import StepConfig
    c = dict(batch=2, frames=400, label_len=40, min_label=10, encoder_layers=2, decoder_layers=2,
             d_model=128, heads=2, ffn=512, vocab=700)
    c.update(kw)
    return StepConfig(**c)


def _run(cfg, device, mel, labels):
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import train as T
    model = T.build_model(cfg, device)
    out = model(input_features=mel.to(device), labels=labels.to(device))
    loss = out.loss + cfg.sparsity_lambda * SG.get_sparsity_loss().to(out.loss.device)
    loss.backward()
    grads = {n: p.grad.detach().float().cpu() for n, p in model.named_parameters()
             if p.grad is not None}
    return float(loss), grads


def test_fp32_step_matches_oracle_model(monkeypatch):
    from tau_dxb_b200 import train as T
    # full fp32 everywhere else in the model (cuDNN convolutions default to TF32)
    monkeypatch.setattr(torch.backends.cudnn, "allow_tf32", False)
    monkeypatch.setattr(torch.backends.cuda.matmul, "allow_tf32", False)
    cfg = tiny_cfg()
    mel, labels = T.synthetic_batch(cfg, "cpu", torch.Generator().manual_seed(7))
    with monkeypatch.context() as m:
        use_oracle_ops(m)
        ref_loss, ref = _run(cfg, "cpu", mel, labels)
    loss, got = _run(cfg, "cuda", mel, labels)
    assert abs(loss - ref_loss) < 1e-4 * max(1.0, abs(ref_loss))
    assert set(got) == set(ref)
    for n in got:
        tol = 2e-3 if ("log_tau" in n or "log_alpha" in n) else 1e-3
        assert rel_err(got[n], ref[n]) < tol, (n, rel_err(got[n], ref[n]))


def test_bf16_autocast_train_step_runs_on_tensor_cores():
    from tau_dxb_b200 import _capi as C
    from tau_dxb_b200 import train as T
    cfg = tiny_cfg(batch=4)
    step = T.TrainStep(cfg, "cuda")
    g = torch.Generator().manual_seed(3)
    losses = []
    for _ in range(3):
        mel, labels = T.synthetic_batch(cfg, "cuda", g)
        losses.append(float(step.step(mel, labels)))
    torch.cuda.synchronize()
    assert all(torch.isfinite(torch.tensor(losses)))
    assert step.skipped == 0
    assert C.lib().tau_dxb_device_error(1) == 0
    for n, p in step.model.named_parameters():
        assert torch.isfinite(p).all(), n


def test_strided_attention_forward_matches_transformers_path():
    """The patched WhisperAttention forward (q/k/v as strided views, the
    1/sqrt(d) scale given to the kernel) and the row-major encoder stream give
    the values of transformers' own forward (contiguous copies, q * scaling in
    bf16) followed by the operator: the same loss, and gradients equal up to
    the order of the backward's fp32 reductions."""
    from tau_dxb_b200 import train as T
    cfg = tiny_cfg(batch=2)
    mel, labels = T.synthetic_batch(cfg, "cuda", torch.Generator().manual_seed(11))
    model = T.build_model(cfg, "cuda")

    def run():
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(input_features=mel, labels=labels)
        out.loss.backward()
        return float(out.loss), {n: p.grad.detach().float().cpu() for n, p in model.named_parameters()
                                 if p.grad is not None}

    for m in model.modules():                      # the layout change alone: exact
        if hasattr(m, "_stau_fused_qkv"):
            m._stau_fused_qkv = False
    loss_a, ga = run()
    n_patched = 0
    for m in model.modules():
        if hasattr(m, "_stau_opus") and "forward" in m.__dict__:
            del m.__dict__["forward"]
            n_patched += 1
    model._tau_dxb_encoder_hook.remove()
    loss_b, gb = run()
    assert n_patched == 3 * cfg.encoder_layers     # encoder self + decoder self + cross per layer pair
    assert abs(loss_a - loss_b) <= 1e-6 * abs(loss_b), (loss_a, loss_b)
    assert set(ga) == set(gb)
    for n in ga:
        assert rel_err(ga[n], gb[n]) < 1e-2, (n, rel_err(ga[n], gb[n]))


def test_fused_qkv_projection_matches_separate_projections():
    """fuse_qkv (one GEMM over [Wq; Wk; Wv], [Wk; Wv] for cross-attention)
    against the three projections: bf16 autocast step, same loss and
    gradients up to bf16 rounding."""
    from tau_dxb_b200 import train as T
    cfg = tiny_cfg(batch=2)
    mel, labels = T.synthetic_batch(cfg, "cuda", torch.Generator().manual_seed(12))
    model = T.build_model(cfg, "cuda")

    def run(fused):
        for m in model.modules():
            if hasattr(m, "_stau_fused_qkv"):
                m._stau_fused_qkv = fused
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(input_features=mel, labels=labels)
        out.loss.backward()
        return float(out.loss), {n: p.grad.detach().float().cpu() for n, p in model.named_parameters()
                                 if p.grad is not None}

    loss_f, gf = run(True)
    loss_s, gs = run(False)
    assert abs(loss_f - loss_s) <= 2e-3 * abs(loss_s), (loss_f, loss_s)
    assert set(gf) == set(gs)
    for n in gf:
        assert rel_err(gf[n], gs[n]) < 3e-2, (n, rel_err(gf[n], gs[n]))


def test_lagged_and_graphed_steps_match_synchronous_step():
    """Three forms of the train step over good x4, NaN, good batches: the
    synchronous check, the step that reads its non-finite flag one step late
    (fused AdamW skipping on the device), and that step replayed from CUDA
    graphs (two eager warm-up steps, capture on the third). All skip exactly
    one step, leave the LR schedule and the EMA at the same point, and end at
    the same weights (up to the attention backward's reduction order)."""
    from tau_dxb_b200 import train as T
    cfg = tiny_cfg(batch=2, warmup_steps=2)
    g = torch.Generator().manual_seed(21)
    batches = [T.synthetic_batch(cfg, "cuda", g) for _ in range(6)]
    bad_mel = batches[4][0].clone()
    bad_mel[0, 0, 0] = float("nan")
    batches[4] = (bad_mel, batches[4][1])
    runs = {}
    for mode in ("sync", "lagged", "graph"):
        step = T.TrainStep(cfg, "cuda", cuda_graph=(mode == "graph"))
        assert step.lagged and step.graphed == (mode == "graph")
        step.lagged = mode != "sync"
        losses = [float(step.step(m, l)) for m, l in batches]
        if mode == "graph":
            assert step._gA is not None
        # the win tracker's step counts advance on replayed steps too
        from tau_dxb_b200 import patch_whisper_sparse_grad as SG
        counts = SG._TRACKER.total_steps
        assert counts and all(v == len(batches) for v in counts.values()), dict(counts)
        runs[mode] = (step.skipped, step.sched.last_epoch, losses,
                      {n: p.detach().float().cpu() for n, p in step.model.named_parameters()},
                      [t.float().cpu() for t in step.ema.shadow],
                      [float(gr["lr"]) for gr in step.opt.param_groups])
    sk, ep, lo, pr, em, lr = runs["sync"]
    assert sk == 1 and ep == 5
    assert not torch.isfinite(torch.tensor(lo[4]))
    for mode in ("lagged", "graph"):
        sk2, ep2, lo2, pr2, em2, lr2 = runs[mode]
        assert (sk2, ep2) == (sk, ep), mode
        assert lr2 == pytest.approx(lr, rel=1e-6), mode
        for i in (0, 1, 2, 3, 5):
            assert abs(lo2[i] - lo[i]) <= 1e-3 * abs(lo[i]), (mode, i, lo2[i], lo[i])
        for n in pr:
            assert rel_err(pr2[n], pr[n]) < 1e-3, (mode, n, rel_err(pr2[n], pr[n]))
        for a, b in zip(em2, em):
            assert rel_err(a, b) < 1e-3, mode
