"""The Python-level drop-in: the reference's unmodified patch modules bind this
package's operators once tau_dxb_b200.install_reference_aliases() has run.

The reference is not part of this repository. These tests run when
TAU_DXB_REFERENCE names a checkout of it (the directory holding echo/), and
are skipped otherwise. Each case runs in a fresh interpreter, because the
reference's modules patch transformers' module globals and sys.path when
they are imported.

The block the first test runs is the one INTEGRATION.md shows (the fenced
block tagged `python dropin`), read from that file, so the documented recipe
is the tested one.
"""
import json
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("TAU_DXB_REFERENCE", "")
pytestmark = pytest.mark.skipif(
    not (REF and os.path.isfile(os.path.join(REF, "echo", "patch_whisper_stau.py"))),
    reason="set TAU_DXB_REFERENCE to a checkout of the reference to run the drop-in tests")

TINY_WHISPER = """
import torch
from transformers import WhisperConfig, WhisperForConditionalGeneration
torch.manual_seed(0)
cfg = WhisperConfig(vocab_size=100, d_model=64, encoder_layers=1, decoder_layers=1,
                    encoder_attention_heads=2, decoder_attention_heads=2,
                    encoder_ffn_dim=128, decoder_ffn_dim=128, num_mel_bins=8,
                    max_source_positions=16, max_target_positions=16,
                    decoder_start_token_id=1, pad_token_id=0, attn_implementation="eager")
model = WhisperForConditionalGeneration(cfg)
"""


def documented_block() -> str:
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    m = re.search(r"```python dropin\n(.*?)```", text, re.S)
    assert m, "INTEGRATION.md has no ```python dropin block"
    return m.group(1)


def run_child(body: str) -> dict:
    """Run `body` in a fresh interpreter from the repository root; it prints one
    JSON object as its last line."""
    prelude = f"import sys\nsys.path.insert(0, {ROOT!r})\nREFERENCE_CHECKOUT = {REF!r}\n"
    r = subprocess.run([sys.executable, "-c", prelude + body], cwd=ROOT, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_documented_recipe_binds_b200_operators():
    body = documented_block() + TINY_WHISPER + """
import json
import patch_whisper_stau as ref_stau
import patch_whisper_sparse_grad as ref_sg
import tau_dxb_b200.attention as A
import tau_dxb_b200.stau_opus_flash_v2 as FV2
import tau_dxb_b200.wta as W
res = {
    "stau_file": ref_stau.__file__,
    "sg_file": ref_sg.__file__,
    "attn_fn": ref_stau.STauOpusAttentionFunction is A.STauOpusAttentionFunction,
    "flash_module": ref_stau.STauOpusFlashV2Module is FV2.STauOpusFlashV2Module,
    "flash_flag": bool(ref_stau._HAS_FLASH_V2),
    "wta_fn": ref_sg._triton_wta_forward is W.wta_fused_forward,
    "wta_flag": bool(ref_sg._HAS_TRITON_WTA),
}
apply_learnable_stau(model, tau_init=2.0, sigma_name={"encoder_self": "softplus",
                     "decoder_self": "sigmoid", "decoder_cross": "exp"})
apply_sparse_grad_wta(model, encoder_mode="wta_activation", decoder_mode="sparse_grad")
res["state_keys"] = sorted(k for k in model.state_dict() if "_stau_opus" in k)[:2]
# a CPU forward reaches the fused operator, which runs on CUDA tensors only
feats = torch.randn(1, 8, 32)
try:
    model(input_features=feats, decoder_input_ids=torch.tensor([[1, 2, 3]]))
    res["cpu_forward"] = "ran"
except RuntimeError as e:
    res["cpu_forward"] = str(e)
print(json.dumps(res))
"""
    res = run_child(body)
    echo = os.path.join(os.path.realpath(REF), "echo")
    assert os.path.realpath(res["stau_file"]).startswith(echo), res["stau_file"]
    assert os.path.realpath(res["sg_file"]).startswith(echo), res["sg_file"]
    for key in ("attn_fn", "flash_module", "flash_flag", "wta_fn", "wta_flag"):
        assert res[key] is True, (key, res)
    assert res["state_keys"] == ["model.decoder.layers.0.encoder_attn._stau_opus.log_alpha",
                                 "model.decoder.layers.0.encoder_attn._stau_opus.log_tau"], res
    assert "tau_dxb_b200" in res["cpu_forward"] and "CUDA" in res["cpu_forward"], res["cpu_forward"]


def test_patch_module_aliases_win_over_the_reference_path():
    """patch_modules=True: with the reference's echo/ first on sys.path, the
    training script's imports (echo/train_echo_opus1.py:39-43) still bind this
    package's patch modules."""
    body = """
import json, os, sys
import tau_dxb_b200
tau_dxb_b200.install_reference_aliases(patch_modules=True)
sys.path.insert(0, os.path.join(REFERENCE_CHECKOUT, "echo"))
from patch_whisper_stau import apply_learnable_stau
from patch_whisper_sparse_grad import apply_sparse_grad_wta, get_sparsity_loss
from triton_wta import has_triton
import tau_dxb_b200.patch_whisper_stau as PS
import tau_dxb_b200.patch_whisper_sparse_grad as PG
print(json.dumps({"stau": apply_learnable_stau is PS.apply_learnable_stau,
                  "sg": apply_sparse_grad_wta is PG.apply_sparse_grad_wta,
                  "loss": get_sparsity_loss is PG.get_sparsity_loss,
                  "has_triton": has_triton()}))
"""
    res = run_child(body)
    assert res == {"stau": True, "sg": True, "loss": True, "has_triton": True}, res


def test_alias_after_reference_import_raises():
    """The reference's own operator module imported first: the aliases would
    not reach the objects its callers already bound, so installing them fails."""
    body = """
import json, os, sys
sys.path.insert(0, os.path.join(REFERENCE_CHECKOUT, "echo"))
import stau_opus_operator
import tau_dxb_b200
try:
    tau_dxb_b200.install_reference_aliases()
    print(json.dumps({"raised": False}))
except RuntimeError as e:
    print(json.dumps({"raised": True, "msg": str(e)}))
"""
    res = run_child(body)
    assert res["raised"] and "stau_opus_operator" in res["msg"], res
