"""Soft prune on the GPU: win counts -> prune_low_winners -> gradient masks on
fc1.weight rows, fc1.bias and fc2.weight columns
(echo/patch_whisper_sparse_grad.py:167-194, 352-395), the masks applied by
the tau_grad_mask kernel."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape,axis", [((3072, 768), 0), ((768, 3072), 1), ((3072,), 1), ((37, 21), 0),
                                         ((21, 37), 1)])
def test_grad_mask_kernel_matches_torch_multiply(dtype, shape, axis):
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    g = torch.Generator(device=DEV).manual_seed(sum(shape) + axis)
    grad = torch.randn(*shape, device=DEV, generator=g).to(dtype)
    flat = grad.view(-1)
    flat[::97] = float("inf")
    flat[5::89] = float("nan")
    flat[7::61] = -flat[7::61].abs()        # negative values: x * 0 keeps the sign (-0)
    n = shape[axis] if len(shape) > 1 else shape[0]
    keep = torch.rand(n, device=DEV, generator=g) > 0.4
    mine = SG.masked_grad(grad, keep, axis)
    m = keep.to(dtype)
    ref = grad * (m.unsqueeze(-1) if (len(shape) > 1 and axis == 0) else m)
    assert torch.equal(mine.isnan(), ref.isnan())
    ok = ~ref.isnan()
    bits = torch.int32 if dtype == torch.float32 else torch.int16
    assert torch.equal(mine[ok].view(bits), ref[ok].view(bits))


def _tiny_model():
    from tau_dxb_b200 import train as T
    cfg = T.StepConfig(batch=2, frames=400, label_len=40, min_label=10, encoder_layers=2, decoder_layers=2,
                       d_model=128, heads=2, ffn=512, vocab=700)
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import patch_whisper_stau as ST
    from transformers import WhisperForConditionalGeneration
    torch.manual_seed(0)
    model = WhisperForConditionalGeneration(T.whisper_config(cfg)).to(DEV)
    ST.apply_learnable_stau(model, tau_init=1.5, sigma_name=T.SIGMA_MAP)
    SG.apply_sparse_grad_wta(model, encoder_mode="wta_activation", decoder_mode="sparse_grad",
                             encoder_k_ratio=0.25, decoder_k_ratio=0.25, track_wins=True)
    model.train()
    return cfg, model


def _loss(model, mel, labels):
    with torch.autocast("cuda", dtype=torch.bfloat16):
        return model(input_features=mel, labels=labels).loss


def test_prune_low_winners_masks_gradients():
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import train as T
    cfg, model = _tiny_model()
    g = torch.Generator().manual_seed(5)
    batches = [T.synthetic_batch(cfg, DEV, g) for _ in range(3)]
    for mel, labels in batches:
        _loss(model, mel, labels).backward()
    model.zero_grad(set_to_none=True)
    tracker = SG.get_win_tracker()
    enc = [n for n, m in model.named_modules() if m.__class__.__name__ == "WhisperEncoderLayer"]
    for name in enc:
        counts = tracker.win_counts[name].cpu().numpy().astype(np.float64)
        assert tracker.total_steps[name] == 3 and counts.sum() > 0
        # win_rate = counts / max(mean, 1) (echo/patch_whisper_sparse_grad.py:108-113)
        np.testing.assert_allclose(tracker.win_rate(name).cpu().numpy(), counts / max(counts.mean(), 1.0),
                                   rtol=1e-6)
    # threshold 1.0: the neurons that win less often than average are frozen
    n_pruned = SG.prune_low_winners(model, threshold=1.0)
    assert 0 < n_pruned < 2 * 512
    mel, labels = batches[0]
    _loss(model, mel, labels).backward()
    masked = {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}
    model.zero_grad(set_to_none=True)
    masks = dict(SG._GRAD_MASKS)
    SG.unfreeze_all()
    _loss(model, mel, labels).backward()
    full = {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}
    model.zero_grad(set_to_none=True)
    assert set(masks) == set(enc)      # the decoder layers collect no wins (sparse_grad mode)
    for name in enc:
        keep = masks[name]
        w1, b1, w2 = (f"{name}.fc1.weight", f"{name}.fc1.bias", f"{name}.fc2.weight")
        assert torch.all(masked[w1][~keep] == 0) and torch.all(masked[b1][~keep] == 0)
        assert torch.all(masked[w2][:, ~keep] == 0)
        # the kept neurons' gradients are the unmasked ones (the attention
        # backward sums with atomics, so equal up to summation order)
        torch.testing.assert_close(masked[w1][keep], full[w1][keep], rtol=1e-3, atol=1e-6)
        torch.testing.assert_close(masked[w2][:, keep], full[w2][:, keep], rtol=1e-3, atol=1e-6)
    SG.remove_sparse_grad(model)
