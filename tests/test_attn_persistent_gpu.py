"""The persistent backward at moderate sizes, where a CTA takes several work
items of different lengths (more items than SMs, a number that is not a
multiple of the SM count): the per-tile barrier phases, the K/V double
buffer and the cross-item MMA stream run across item boundaries. Checked
against the fp32 oracle at the bf16 tolerance, under the built-in causal flag
with Lq < Lk (items of 1 to 3 query tiles, longest first), an additive mask
tensor with padded keys, and partial query and key tiles without a mask."""
import numpy as np
import pytest
import torch

from test_attn_gpu import A, TOL_BF16, assert_close, assert_no_near_ties, make_inputs, oracle, run_op  # noqa: F401
from oracle import stau_attention as OA

pytestmark = pytest.mark.gpu


def _check(A, label, sigma, Q, K, V, lt, la, dO, mask=None, causal_fn=False, ref_mask=None):
    from tau_dxb_b200 import _capi as C
    assert_no_near_ties(Q, K, 0.125, ref_mask if ref_mask is not None else mask)
    C.lib().tau_dxb_device_error(1)
    mine = run_op(A, Q, K, V, lt, la, sigma, dO, mask, 0.125, path="tensor", causal_fn=causal_fn)
    assert C.lib().tau_dxb_device_error(1) == 0, label
    ref = oracle(Q, K, V, lt, la, sigma, dO, ref_mask if ref_mask is not None else mask, 0.125)
    assert_close(mine, ref, TOL_BF16, label)


def test_causal_flag_items_of_several_lengths(A):
    """B=2, H=30, 300 queries x 700 keys: 360 backward items of 1-3 query tiles."""
    Q, K, V, lt, la, dO = make_inputs(2, 30, 300, 700, seed=21, dtype=torch.bfloat16, la_std=0.2)
    _check(A, "causal flag 300x700", "sigmoid", Q, K, V, lt, la, dO, causal_fn=True,
           ref_mask=torch.from_numpy(OA.causal_mask(300, 700)))


def test_mask_tensor_with_padded_keys(A):
    """B=2, H=40, 200 x 300 with an additive [B, 1, Lq, Lk] mask: batch item 1
    has its last 37 keys padded; 240 backward items."""
    Q, K, V, lt, la, dO = make_inputs(2, 40, 200, 300, seed=22, dtype=torch.bfloat16, la_std=0.2)
    mask = torch.zeros(2, 1, 200, 300)
    mask[1, :, :, 263:] = torch.finfo(torch.float32).min
    _check(A, "mask tensor 200x300", "softplus", Q, K, V, lt, la, dO, mask=mask)


def test_partial_tiles_without_mask(A):
    """B=3, H=20, 260 x 390 (partial query and key tiles): 240 items."""
    Q, K, V, lt, la, dO = make_inputs(3, 20, 260, 390, seed=34, dtype=torch.bfloat16, la_std=0.2)
    _check(A, "no mask 260x390", "exp", Q, K, V, lt, la, dO)
