"""The reference's own model code, unmodified, on this package's ops (GPU).

``spikegpt_b200.dropin.install()`` makes the reference's ``spikegpt.wkv_triton``
and ``spikegpt.wkv_bf16`` imports (src/spikegpt/language.py:37-38) resolve to
this package, and ``tests/_reference.route_fused_paths`` makes the reference's
CUDA branches run (``has_triton()`` true; its fused LIF calls, language.py:
862-906, go to this package's LIF op). A ``SpikeGPTBlock`` (language.py:
1223-1360) built by the reference is then run forward and backward:

* against the same block on the same GPU taking the reference's own PyTorch
  paths (``weighted_key_value``, the associative scan of language.py:452-527,
  and the per-step LIF loop of language.py:907-918), in float32 and under
  bf16 autocast;
* compiled per block with ``torch.compile(block, fullgraph=True)``, which is
  what the reference's regional compile does
  (examples/train_tiny_spikegpt.py:69-89), against eager.

The reference code comes from ``baseline/_ref`` (``baseline/install_ref.py``).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import _reference
from spikegpt_b200 import _capi

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not _reference.available(), reason="baseline/_ref has no reference install"),
]

B, T, C = 3, 96, 128


@pytest.fixture(scope="module")
def language():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return _reference.import_language(dropin=True)


def _block(language, layer_id: int, spiking: bool, device):
    cfg = language.SpikeGPTConfig(vocab_size=256, context_length=T, n_layer=4, n_embd=C, dropout=0.0,
                                  spiking=spiking)
    torch.manual_seed(1234 + layer_id)
    block = language.SpikeGPTBlock(cfg, layer_id)
    with torch.no_grad():  # spread the decays / bonuses beyond the init profile
        block.att.time_decay.uniform_(-5.0, 1.0)
        block.att.time_first.uniform_(-1.0, 1.0)
    return block.to(device)


def _run(block, x, gy, *, autocast: bool):
    x = x.detach().clone().requires_grad_()
    block.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        out = block(x)
    out.float().backward(gy)
    # (a compiled block names its parameters "_orig_mod.<name>")
    grads = {n.removeprefix("_orig_mod."): p.grad.detach().float().cpu().numpy()
             for n, p in block.named_parameters() if p.grad is not None}
    grads["input"] = x.grad.detach().float().cpu().numpy()
    return out.detach().float().cpu().numpy(), grads


def _scaled(a, b) -> float:
    return float(np.abs(a - b).max() / max(1.0, float(np.abs(b).max())))


def _inputs(device, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, C, generator=g).to(device)
    gy = torch.randn(B, T, C, generator=g).to(device)
    return x, gy


def _wkv_launches():
    n = _capi.launch_counts()
    return n["wkv_fwd_kernel<y>"], n["wkv_bwd_kernel<grad>"]


@pytest.mark.parametrize("layer_id", [0, 1])
@pytest.mark.parametrize("autocast", [False, True])
def test_block_matches_the_reference_pytorch_path(cuda, language, layer_id, autocast):
    """Continuous twin (spiking=False): only the WKV differs between the runs."""
    block = _block(language, layer_id, spiking=False, device=cuda)
    x, gy = _inputs(cuda, seed=layer_id)
    _reference.unroute(language)
    ref_out, ref_grads = _run(block, x, gy, autocast=autocast)
    _reference.route_fused_paths(language)
    before = _wkv_launches()
    out, grads = _run(block, x, gy, autocast=autocast)
    after = _wkv_launches()
    _reference.unroute(language)
    assert after[0] > before[0] and after[1] > before[1], "the drop-in ops did not run"
    tol = 2e-2 if autocast else 1e-4
    assert _scaled(out, ref_out) <= tol
    assert set(grads) == set(ref_grads)
    for name in grads:
        assert _scaled(grads[name], ref_grads[name]) <= tol, name


def test_spiking_block_runs_on_the_package_ops(cuda, language):
    """Spiking block in float32: the reference's LIF loop and this package's LIF
    op give the same spikes (up to membranes that sit within rounding of the
    threshold), and the gradients agree."""
    block = _block(language, 1, spiking=True, device=cuda)
    x, gy = _inputs(cuda, seed=7)
    _reference.unroute(language)
    ref_out, ref_grads = _run(block, x, gy, autocast=False)
    _reference.route_fused_paths(language)
    lif_before = _capi.launch_counts()["lif_fwd_kernel"]
    out, grads = _run(block, x, gy, autocast=False)
    _reference.unroute(language)
    assert _capi.launch_counts()["lif_fwd_kernel"] >= lif_before + 2
    mismatch = np.count_nonzero(np.abs(out - ref_out) > 1e-3) / out.size
    assert mismatch <= 1e-3
    if mismatch == 0:
        for name in grads:
            assert _scaled(grads[name], ref_grads[name]) <= 1e-3, name


@pytest.mark.parametrize("spiking,autocast", [(False, False), (True, True)])
def test_regional_compile_fullgraph(cuda, language, spiking, autocast):
    """torch.compile(block, fullgraph=True), the reference's regional compile,
    traces the drop-in ops without a graph break; the compiled backward uses the
    saved state (no state sweep) and matches eager."""
    block = _block(language, 2, spiking=spiking, device=cuda)
    x, gy = _inputs(cuda, seed=11)
    _reference.route_fused_paths(language)
    try:
        eager_out, eager_grads = _run(block, x, gy, autocast=autocast)
        torch._dynamo.reset()
        compiled = torch.compile(block, fullgraph=True)
        _run(compiled, x, gy, autocast=autocast)  # compile
        before = _capi.launch_counts()
        out, grads = _run(compiled, x, gy, autocast=autocast)
        after = _capi.launch_counts()
    finally:
        _reference.unroute(language)
        torch._dynamo.reset()
    assert after["wkv_fwd_kernel<y>"] == before["wkv_fwd_kernel<y>"] + 1
    assert after["wkv_bwd_kernel<grad>"] == before["wkv_bwd_kernel<grad>"] + 1
    assert after["wkv_fwd_kernel<state>"] == before["wkv_fwd_kernel<state>"]
    if spiking:
        assert after["lif_fwd_kernel"] == before["lif_fwd_kernel"] + 2
    tol = 2e-2 if autocast else 1e-4
    if spiking:  # the fused kernels' roundings can flip a spike near threshold
        assert np.count_nonzero(out != eager_out) / out.size <= 1e-3
        return
    assert _scaled(out, eager_out) <= tol
    for name in grads:
        assert _scaled(grads[name], eager_grads[name]) <= tol, name
