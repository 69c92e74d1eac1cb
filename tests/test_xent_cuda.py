"""GPU parity of the fused cross-entropy (``spikegpt_b200.fused.cross_entropy``)
against F.cross_entropy(logits.float(), targets) on bf16 logits, as the model
computes its loss under autocast: the loss to 1e-5 relative; the bf16
gradient to one bf16 rounding (the same float32 quantity, its softmax sums
taken in another order, rounded once). Covers a vocabulary that is not a
multiple of 8 read from a padded row pitch (the pitch's tail gets zero
gradient), ignored targets (-100), a NaN logit, and the model's use."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from spikegpt_b200 import _capi, fused

pytestmark = pytest.mark.gpu


def _case(rows, v, ld, seed, cuda):
    g = torch.Generator(device="cpu").manual_seed(seed)
    full = (torch.randn(rows, ld, generator=g) * 3).to(torch.bfloat16).to(cuda)
    t = torch.randint(0, v, (rows,), generator=g).to(cuda)
    return full, t


@pytest.mark.parametrize("rows,v,ld", [(64, 256, 256), (37, 50257, 50304), (5, 13, 16), (1, 1, 8)])
def test_matches_eager(cuda, rows, v, ld):
    full, t = _case(rows, v, ld, rows + v, cuda)
    if rows > 3:
        t[1] = -100
        t[3] = -100
    a = full.clone().requires_grad_()
    loss = fused.cross_entropy(a, t, v)
    loss.backward()
    b = full[:, :v].clone().requires_grad_()
    ref = F.cross_entropy(b.float(), t)
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 1e-5 * max(1.0, abs(ref.item()))
    got, want = a.grad[:, :v].float(), b.grad.float()
    assert float((got - want).abs().max()) <= 2 ** -7 * float(want.abs().max()) + 1e-7
    assert torch.count_nonzero(a.grad[:, v:]) == 0
    if rows > 3:
        assert torch.count_nonzero(a.grad[1]) == 0


def test_nan_logit_makes_its_row_nan(cuda):
    full, t = _case(4, 40, 40, 3, cuda)
    full[2, 7] = float("nan")
    rows, _ = torch.ops.spikegpt_b200.cross_entropy_rows(full, t, 40)
    assert torch.isnan(rows[2]) and torch.isfinite(rows[[0, 1, 3]]).all()


def test_errors_and_launch_counts(cuda):
    full, t = _case(4, 40, 40, 4, cuda)
    with pytest.raises(ValueError):
        fused.cross_entropy(full.float(), t)
    with pytest.raises(ValueError):
        fused.cross_entropy(full[:, :36], t, 40)
    lib = _capi.lib()
    assert lib.cross_entropy_forward(full.data_ptr(), 36, t.data_ptr(), 4, 40, None, None, None) == \
        _capi.WKV_ERR_INVALID_ARGUMENT
    before = _capi.launch_counts()
    x = full.clone().requires_grad_()
    fused.cross_entropy(x, t).backward()
    after = _capi.launch_counts()
    assert after["xent_fwd_kernel"] - before["xent_fwd_kernel"] == 1
    assert after["xent_bwd_kernel"] - before["xent_bwd_kernel"] == 1


@pytest.mark.parametrize("bad", [-1, 40, 1000])
def test_out_of_range_target_makes_the_loss_nan_and_sets_the_flag(cuda, bad):
    """PyTorch rejects a target outside [0, V) other than ignore_index -100;
    the fused loss makes that row (so the mean) NaN and its gradient row NaN,
    and records WKV_DEVERR_BAD_TARGET, instead of silently lowering the mean."""
    full, t = _case(4, 40, 40, 5, cuda)
    t[2] = bad
    t[0] = -100
    assert _capi.device_error_flags(clear=True) == 0
    x = full.clone().requires_grad_()
    loss = fused.cross_entropy(x, t)
    loss.backward()
    assert torch.isnan(loss)
    assert torch.isnan(x.grad[2].float()).all()
    assert torch.count_nonzero(x.grad[0]) == 0 and torch.isfinite(x.grad[[1, 3]].float()).all()
    assert _capi.device_error_flags(clear=True) == _capi.WKV_DEVERR_BAD_TARGET
