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
