"""The mel filter bank of the GPU log-mel front end against transformers'
(the one WhisperFeatureExtractor uses), and argument checks of the C entry."""
import numpy as np
import pytest


def test_mel_filters_match_transformers():
    from transformers.audio_utils import mel_filter_bank
    from tau_dxb_b200 import features as Fe
    ref = mel_filter_bank(num_frequency_bins=201, num_mel_filters=80, min_frequency=0.0,
                          max_frequency=8000.0, sampling_rate=16000, norm="slaney", mel_scale="slaney")
    mine = Fe.mel_filters()
    assert mine.shape == ref.shape == (201, 80)
    assert np.allclose(mine, ref, rtol=1e-12, atol=1e-15)


def test_log_mel_argument_checks_without_gpu():
    from tau_dxb_b200 import _capi as C
    lib = C.lib()
    assert lib.whisper_log_mel_workspace_bytes(16) >= 16 * 4 + 80 * 201 * 4
    rc = lib.whisper_log_mel(None, 2, 480001, None, None, None, 0, None)   # not a multiple of 160
    assert rc == C.ERR_INVALID_ARGUMENT
    assert "multiple of 160" in C.last_error()
    assert lib.whisper_log_mel(None, 0, 480000, None, None, None, 0, None) == C.OK


def test_cpu_tensor_raises():
    import torch
    from tau_dxb_b200 import features as Fe
    with pytest.raises(RuntimeError):
        Fe.log_mel_spectrogram(torch.zeros(480000))
