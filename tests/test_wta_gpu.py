"""WTA kernels (K4 forward, K5 backward) against the oracle and the reference's
golden vectors. Masks, outputs and gradients must be bit-exact."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import wta as OW

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bits_to_bf16(bits_u16):
    t = torch.from_numpy(bits_u16.astype(np.int16)).view(torch.bfloat16)
    return t


def _bf16_to_bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def golden():
    z = np.load(os.path.join(GOLDEN, "wta_gelu_48x3072.npz"))
    return {k: z[k] for k in z.files}


@pytest.fixture(scope="module")
def W():
    from tau_dxb_b200 import wta
    return wta


def test_threshold_masks_match_reference_golden(golden, W):
    x = _bits_to_bf16(golden["x_bits"]).to(DEV)
    xf = OW.bf16_bits_to_f32(golden["x_bits"])
    for k in golden["ks"]:
        k = int(k)
        y, bits = W.wta_select(x, k, W.THRESHOLD)
        assert np.array_equal(bits.cpu().numpy(), golden[f"thr_mask_k{k}"]), k
        ref_y, _ = OW.wta_forward(xf, k, "threshold")
        assert np.array_equal(_bf16_to_bits(y), OW.f32_to_bf16_bits(ref_y)), k


def test_sparse_grad_backward_bits_match_golden(golden, W):
    x = _bits_to_bf16(golden["x_bits"]).to(DEV).requires_grad_()
    dy = _bits_to_bf16(golden["dy_bits"]).to(DEV)
    out = W.SparseGradWTA_Function.apply(x, 306)
    assert torch.equal(out.detach(), x.detach())
    out.backward(dy)
    assert np.array_equal(_bf16_to_bits(x.grad), golden["sg_dx_bits_k306"])


def test_exact_k_against_reference_cpu_semantics(golden, W):
    x = _bits_to_bf16(golden["x_bits"]).to(DEV)
    xf = OW.bf16_bits_to_f32(golden["x_bits"])
    for k in golden["ks"]:
        k = int(k)
        y, bits = W.wta_select(x, k, W.EXACT_K)
        mine = W.unpack_mask(bits, 3072).cpu().numpy()
        assert np.array_equal(mine, OW.exact_k_mask(xf, k)), k        # lowest-index ties
        ref = np.unpackbits(golden[f"exact_mask_k{k}"], axis=-1, bitorder="little").astype(bool)
        ties = OW.tie_rows(xf, k)
        assert np.array_equal(mine[~ties], ref[~ties]), k
        assert (mine.sum(-1) == k).all()
    y, _ = W.wta_select(x, 306, W.EXACT_K)
    # the reference's y on tie-free rows
    ties = OW.tie_rows(xf, 306)
    assert np.array_equal(_bf16_to_bits(y)[~ties], golden["exact_y_bits_k306"][~ties])


def test_exact_k_tie_order_vs_torch_topk_cuda(W):
    """exact_k keeps the lowest-index ties at the threshold. On CUDA tensors the
    reference's exact path is x.topk(k) (echo/triton_wta.py:117-123), whose CUDA
    kernel takes the values above the k-th largest and then the ties in index
    order: every row, tied or not, must select the same set."""
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.nn.functional.gelu(torch.randn(512, 3072, device=DEV, generator=g)).to(torch.bfloat16)
    for k in (154, 306):
        _, bits = W.wta_select(x, k, W.EXACT_K)
        mine = W.unpack_mask(bits, 3072)
        idx = x.topk(k, dim=-1).indices
        ref = torch.zeros_like(mine).scatter_(-1, idx, True)
        thr = x.float().kthvalue(3072 - k + 1, dim=-1, keepdim=True).values
        tie_rows = (x.float() >= thr).sum(-1) > k
        assert int(tie_rows.sum()) > 0, k          # bf16 rows of 3072: ties at the threshold are common
        same_rows = (mine == ref).all(-1)
        assert bool(same_rows.all()), (k, int((~same_rows).sum()), int(tie_rows.sum()))


@pytest.mark.parametrize("rows,k", [(24000, 154), (24000, 306), (24000, 307), (24000, 768), (24000, 1536),
                                    (7168, 306), (7168, 1536)])
def test_full_size_encoder_threshold_vs_torch(W, rows, k):
    """Encoder [24000, 3072] and decoder [7168, 3072] sizes (the decoder's takes
    the kernel variant without row prefetch)."""
    g = torch.Generator(device=DEV).manual_seed(k)
    x = torch.nn.functional.gelu(torch.randn(rows, 3072, device=DEV, generator=g)).to(torch.bfloat16)
    y, bits = W.wta_select(x, k, W.THRESHOLD)
    thr = x.float().kthvalue(3072 - k + 1, dim=-1, keepdim=True).values
    keep = x.float() >= thr
    assert torch.equal(W.unpack_mask(bits, 3072), keep)
    assert torch.equal(y, torch.where(keep, x, torch.zeros_like(x)))
    # oracle on a sample of rows
    sample = slice(0, 256)
    ref = OW.threshold_mask(x[sample].float().cpu().numpy(), k)
    assert np.array_equal(W.unpack_mask(bits[sample], 3072).cpu().numpy(), ref)
    dy = torch.randn(rows, 3072, device=DEV, generator=g).to(torch.bfloat16)
    dx = W.wta_backward(dy, bits)
    assert torch.equal(dx, dy * keep.to(dy.dtype))


@pytest.mark.parametrize("d,dtype,stride_pad", [
    (3072, torch.float32, 0), (3072, torch.float16, 0), (1000, torch.bfloat16, 0),
    (100, torch.bfloat16, 3), (768, torch.bfloat16, 16), (2048, torch.float32, 5), (5, torch.float32, 0)])
def test_generic_paths_vs_oracle(W, d, dtype, stride_pad):
    g = torch.Generator(device=DEV).manual_seed(d)
    base = torch.randn(300, d + stride_pad, device=DEV, generator=g).to(dtype)
    x = base[:, :d]
    xf = x.float().cpu().numpy()
    for k in (1, 7, d // 3 + 1, d):
        for mode, ref_fn in ((W.THRESHOLD, OW.threshold_mask), (W.EXACT_K, OW.exact_k_mask)):
            y, bits = W.wta_select(x, k, mode)
            mine = W.unpack_mask(bits, d).cpu().numpy()
            assert np.array_equal(mine, ref_fn(xf, k)), (d, dtype, k, mode)
            yr, _ = OW.wta_forward(xf, k, "threshold" if mode == W.THRESHOLD else "exact")
            yf = y.float().cpu().numpy()
            assert np.array_equal(yf, yr) and np.array_equal(np.signbit(yf), np.signbit(yr))


def test_ties_zeros_and_clamping(W):
    d = 3072
    x = torch.zeros(8, d, dtype=torch.bfloat16, device=DEV)
    x[1] = 1.0                                        # all tied
    x[2, ::2] = -0.0                                  # +0 / -0 mix
    x[2, 1::4] = 2.0
    x[3] = torch.linspace(-5, 5, d)
    x[4, 100] = float("inf")
    x[5] = -1.0
    x[5, :10] = -0.5
    xf = x.float().cpu().numpy()
    for k in (0, 1, 5, 306, d, d + 50):
        kk = max(1, min(d, k))
        y, bits = W.wta_select(x, k, W.THRESHOLD)
        assert np.array_equal(W.unpack_mask(bits, d).cpu().numpy(), OW.threshold_mask(xf, kk)), k
        y, bits = W.wta_select(x, k, W.EXACT_K)
        assert np.array_equal(W.unpack_mask(bits, d).cpu().numpy(), OW.exact_k_mask(xf, kk)), k


def test_empty_and_device_k(W):
    x = torch.empty(0, 3072, dtype=torch.bfloat16, device=DEV)
    y, bits = W.wta_select(x, 10)
    assert bits.shape == (0, 384)
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(4, 250, 3072, device=DEV, generator=g).to(torch.bfloat16)
    kd = torch.tensor([306], dtype=torch.int32, device=DEV)
    y1, b1 = W.wta_select(x, kd)
    y2, b2 = W.wta_select(x, 306)
    assert torch.equal(b1, b2) and torch.equal(y1, y2)
    assert b1.shape == (4, 250, 384)


def test_win_counts_are_column_sums(W):
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.nn.functional.gelu(torch.randn(1000, 3072, device=DEV, generator=g)).to(torch.bfloat16)
    win = torch.zeros(3072, dtype=torch.int32, device=DEV)
    _, bits = W.wta_select(x, 306, W.THRESHOLD, win_counts=win)
    assert torch.equal(win, W.unpack_mask(bits, 3072).sum(0).to(torch.int32))
    win2 = torch.zeros(3072, dtype=torch.int32, device=DEV)
    W.wta_select(x, 306, W.THRESHOLD, write_y=False, win_counts=win2)
    assert torch.equal(win, win2)


def test_k_from_logits_matches_reference_table(W):
    z = np.load(os.path.join(GOLDEN, "k_table.npz"))
    for d_ff in np.unique(z["d_ff"]):
        sel = z["d_ff"] == d_ff
        lg = torch.from_numpy(z["logit"][sel]).to(DEV)
        k = W.k_from_logits(lg, int(d_ff)).cpu().numpy()
        assert np.array_equal(k, z["k"][sel]), d_ff


def test_autograd_ste_and_exact_function(W):
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.nn.functional.gelu(torch.randn(64, 3072, device=DEV, generator=g)).to(torch.bfloat16)
    x.requires_grad_()
    dy = torch.randn(64, 3072, device=DEV, generator=g).to(torch.bfloat16)
    y = W.wta_fused_forward(x, 306)
    y.backward(dy)
    keep = W.wta_fused_forward_with_mask(x.detach(), 306)[1]
    assert torch.equal(x.grad, dy * keep.to(dy.dtype))
    x.grad = None
    y = W.WTA_Activation_Function.apply(x, 306)
    y.backward(dy)
    assert int((y != 0).sum(-1).max()) <= 306
    assert torch.equal(x.grad != 0, (y != 0) & (dy != 0))


def test_cpu_tensor_raises(W):
    with pytest.raises(RuntimeError):
        W.wta_fused_forward(torch.randn(2, 3072), 10)


@pytest.mark.parametrize("d,dtype", [(3072, torch.bfloat16), (3072, torch.float16), (1000, torch.bfloat16),
                                     (3072, torch.float32)])
def test_nan_rows_follow_reference_semantics(W, d, dtype):
    """NaN sorts largest in the reference's topk / kthvalue and then fails
    x >= thr: the threshold is the (k - #NaN)-th largest non-NaN value, NaN is
    never kept, and a row with #NaN >= k keeps nothing. The fast and generic
    paths agree with the oracle on such rows."""
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(64, d, device=DEV, generator=g).to(dtype)
    x[0, ::7] = float("nan")
    x[1] = float("nan")
    x[1, :5] = 1.0
    x[2, :20] = float("nan")
    x[2, 20:] = -float("inf")
    x[3, 100] = float("nan")
    x[3, 200] = float("inf")
    x[4] = torch.randn(d, device=DEV, generator=g).to(dtype) * 1e-39 if dtype != torch.float16 else x[4]
    xf = x.float().cpu().numpy()
    for k in (1, 5, 19, 21, 306, d):
        kk = min(k, d)
        for mode, ref_fn in ((W.THRESHOLD, OW.threshold_mask), (W.EXACT_K, OW.exact_k_mask)):
            y, bits = W.wta_select(x, kk, mode)
            mine = W.unpack_mask(bits, d).cpu().numpy()
            assert np.array_equal(mine, ref_fn(xf, kk)), (d, dtype, k, mode)


def test_threshold_search_rows_of_mixed_scale(W):
    """Consecutive rows with very different thresholds (the fast path starts
    each search at the previous row's threshold of its warp)."""
    g = torch.Generator(device=DEV).manual_seed(6)
    base = torch.randn(4096, 3072, device=DEV, generator=g)
    scale = torch.logspace(-20, 20, 4096, device=DEV)[torch.randperm(4096, device=DEV, generator=g)]
    x = (base * scale[:, None]).to(torch.bfloat16)
    x[::3] = x[::3].abs()
    x[1::5] = -x[1::5].abs()
    for k in (1, 306, 1536, 3072):
        y, bits = W.wta_select(x, k, W.THRESHOLD)
        thr = x.float().kthvalue(3072 - k + 1, dim=-1, keepdim=True).values
        keep = x.float() >= thr
        assert torch.equal(W.unpack_mask(bits, 3072), keep), k
        assert torch.equal(y, torch.where(keep, x, torch.zeros_like(x))), k
