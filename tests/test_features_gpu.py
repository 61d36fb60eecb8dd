"""GPU log-mel front end against transformers' WhisperFeatureExtractor (the
host call of the reference's dataset, echo/train_echo_opus1.py:126)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _audio(seed, n):
    g = np.random.default_rng(seed)
    t = np.arange(n) / 16000.0
    x = 0.05 * g.standard_normal(n)
    for f, a in ((220.0, 0.3), (1330.0, 0.1), (5200.0, 0.05)):
        x += a * np.sin(2 * np.pi * f * t + g.uniform(0, 6.28))
    x[: n // 7] *= 0.01                      # a quiet stretch
    return x.astype(np.float32)


@pytest.fixture(scope="module")
def fe():
    from transformers import WhisperFeatureExtractor
    return WhisperFeatureExtractor()


@pytest.mark.parametrize("lengths", [(480000,), (480000, 480000, 480000, 480000), (20800,), (512000, 3000)])
def test_log_mel_matches_feature_extractor(fe, lengths):
    from tau_dxb_b200 import features as Fe
    audios = [_audio(i + len(lengths), n) for i, n in enumerate(lengths)]
    ref = np.stack([fe(a, sampling_rate=16000, return_tensors="np").input_features[0] for a in audios])
    padded = np.zeros((len(audios), max(lengths)), np.float32)
    for i, a in enumerate(audios):
        padded[i, :len(a)] = a
    mine = Fe.log_mel_spectrogram(torch.from_numpy(padded).cuda()) if len(set(lengths)) == 1 else \
        torch.stack([Fe.log_mel_spectrogram(torch.from_numpy(a).cuda()) for a in audios])
    mine = mine.cpu().numpy()
    assert mine.shape == ref.shape == (len(lengths), 80, 3000)
    assert np.abs(mine - ref).max() < 2e-4, np.abs(mine - ref).max()


def test_log_mel_silence_and_batch_independence():
    from tau_dxb_b200 import features as Fe
    x = torch.zeros(3, 480000, device="cuda")
    x[1] = torch.from_numpy(_audio(9, 480000)).cuda()
    out = Fe.log_mel_spectrogram(x)
    # silence: log10(1e-10) everywhere, then max - 8 clamp and scaling
    assert torch.allclose(out[0], torch.full_like(out[0], (-10.0 + 4.0) / 4.0))
    alone = Fe.log_mel_spectrogram(x[1])
    assert torch.equal(out[1], alone)
