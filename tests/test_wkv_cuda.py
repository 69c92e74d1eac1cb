"""GPU parity of the sm_100a WKV ops against the CPU oracle and the reference's
golden vectors. Every call goes through the registered custom ops, i.e. through
the C ABI of libspikegpt_wkv.so.

Tolerances (the parity contract): max|x - ref| / max(1, max|ref|) <= 1e-5 for
float32 I/O and <= 2e-2 for bf16/fp16 I/O, on y, grad_key, grad_value,
grad_time_decay and grad_time_first. The oracle is float64.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from _wkvtest import TOL_16BIT, TOL_FP32, config_inputs, golden_inputs, load_golden, scaled_err
from make_golden import CFG0_STRIDE

import spikegpt_b200  # noqa: F401
from oracle import oracle
from spikegpt_b200 import _capi, weighted_key_value_cuda, weighted_key_value_cuda_bf16io

pytestmark = pytest.mark.gpu

CASES = load_golden()
NAMES = sorted(CASES)
FIELDS = ("y", "gk", "gv", "gtd", "gtf")


@pytest.fixture(autouse=True)
def _reset_overrides():
    yield
    _capi.set_debug_overrides()
    spikegpt_b200.set_state_saving(True)


def _run(fn, k, v, td, tf, gy, *, dtype, device):
    """Forward + backward through autograd, like the reference's
    tests/test_wkv_triton.py:21-32 helper."""
    tens = [torch.as_tensor(np.asarray(x)).to(device=device, dtype=dtype) for x in (k, v)]
    tens += [torch.as_tensor(np.asarray(x)).to(device=device, dtype=torch.float32) for x in (td, tf)]
    leaves = [x.clone().requires_grad_(True) for x in tens]
    y = fn(*leaves)
    y.backward(torch.as_tensor(np.asarray(gy)).to(device=device, dtype=dtype))

    def z(g, ref):  # an unused input (time_decay at T=1) yields None
        return torch.zeros_like(ref) if g is None else g

    out = [y] + [z(x.grad, x) for x in leaves]
    return [o.detach().double().cpu().numpy() for o in out]


def _oracle(k, v, td, tf, gy, *, round_to=None):
    if round_to is not None:  # the op sees inputs rounded to its I/O dtype
        k, v, gy = (torch.as_tensor(np.asarray(x, np.float32)).to(round_to).double().numpy() for x in (k, v, gy))
    return oracle.forward_backward(k, v, td, tf, gy)


def _assert_close(got, ref, tol, what=""):
    for g, r, name in zip(got, ref, FIELDS, strict=True):
        err = scaled_err(g, r)
        assert err <= tol, f"{what} {name}: scaled error {err:.3e} > {tol:.0e}"


# ------------------------------------------------------------ golden vectors


def _fp32_tol(k, v, td, tf, gy) -> float:
    """1e-5, or, where the reference's own algorithm run in float32 cannot reach
    it (keys of magnitude ~80 in kscale20), twice that algorithm's error."""
    ref = oracle.forward_backward(k, v, td, tf, gy)
    f32 = oracle.forward_backward(k, v, td, tf, gy, dtype=np.float32)
    return max(TOL_FP32, 2.0 * max(scaled_err(a, b) for a, b in zip(f32, ref, strict=True)))


@pytest.mark.parametrize("name", NAMES)
def test_golden_cases_float32(cuda, name):
    """Every reference-generated golden case, float32 I/O through myelin::wkv_forward."""
    k, v, td, tf, gy = golden_inputs(name, CASES)
    got = _run(weighted_key_value_cuda, k, v, td, tf, gy, dtype=torch.float32, device=cuda)
    g = CASES[name]
    if name == "cfg0":
        got[:3] = [a.reshape(-1)[::CFG0_STRIDE] for a in got[:3]]
    _assert_close(got, [g[f] for f in FIELDS], _fp32_tol(k, v, td, tf, gy), name)


@pytest.mark.parametrize("name", ["triton_t7", "triton_t64", "channels70", "kscale4", "kscale20", "decay_extremes", "bf16_rounded"])
@pytest.mark.parametrize("path", ["generic", "seg2", "seg3", "slow", "slow_seg2", "nostate", "nostate_seg2", "nostate_slow"])
def test_golden_cases_on_every_execution_path(cuda, name, path):
    """Every execution path: TMA or generic tiles, one sequential sweep or time
    segments, fast or exact arithmetic, with and without the saved-state hand-off."""
    k, v, td, tf, gy = golden_inputs(name, CASES)
    seg = {"seg2": 2, "seg3": 3, "slow_seg2": 2, "nostate_seg2": 2}.get(path, 0)
    _capi.set_debug_overrides(force_segments=seg, force_generic=path == "generic", force_slow="slow" in path)
    spikegpt_b200.set_state_saving(not path.startswith("nostate"))
    got = _run(weighted_key_value_cuda, k, v, td, tf, gy, dtype=torch.float32, device=cuda)
    _assert_close(got, [CASES[name][f] for f in FIELDS], _fp32_tol(k, v, td, tf, gy), f"{name}/{path}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("op", ["bf16io", "fp32io"])
def test_16bit_io_matches_oracle(cuda, dtype, op):
    k, v, td, tf, gy = golden_inputs("bf16_rounded", CASES)
    fn = weighted_key_value_cuda_bf16io if op == "bf16io" else weighted_key_value_cuda
    got = _run(fn, k, v, td, tf, gy, dtype=dtype, device=cuda)
    ref = _oracle(k, v, td, tf, gy, round_to=dtype)
    _assert_close(got, ref, TOL_16BIT, f"{op}/{dtype}")


# --------------------------------------------------- reference test shapes


@pytest.mark.parametrize("t", [1, 7, 64])
def test_reference_triton_shapes(cuda, t):
    """tests/test_wkv_triton.py:35-54 of the reference: B=3, C=96, seed=t."""
    torch.manual_seed(t)
    b, c = 3, 96
    k, v = torch.randn(b, t, c), torch.randn(b, t, c)
    td, tf = torch.randn(c), torch.randn(c)
    gy = torch.randn(b, t, c)
    args = [x.numpy() for x in (k, v, td, tf, gy)]
    got = _run(weighted_key_value_cuda, *args, dtype=torch.float32, device=cuda)
    _assert_close(got, _oracle(*args), TOL_FP32)


@pytest.mark.parametrize("c", [1, 7, 8, 36, 40, 70, 96, 100, 520])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_channel_counts_and_tails(cuda, c, dtype):
    """C not a multiple of the 32-lane CTA (reference test_wkv_triton.py:57-68),
    TMA-eligible and not, with a T tail that is not a multiple of 16 or 32."""
    k, v, td, tf, gy = config_inputs(2, 45, c, seed=c)
    got = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=dtype, device=cuda)
    tol = TOL_FP32 if dtype == torch.float32 else TOL_16BIT
    _assert_close(got, _oracle(k, v, td, tf, gy, round_to=dtype), tol, f"C={c}")


@pytest.mark.parametrize("t", [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 200])
def test_time_lengths(cuda, t):
    k, v, td, tf, gy = config_inputs(3, t, 64, seed=t, kscale=2.0)
    got = _run(weighted_key_value_cuda, k, v, td, tf, gy, dtype=torch.float32, device=cuda)
    _assert_close(got, _oracle(k, v, td, tf, gy), TOL_FP32, f"T={t}")


@pytest.mark.parametrize("b", [1, 2, 4, 8])
def test_long_context_small_batch_uses_segments(cuda, b):
    """Config 2b: B=1..8 at T=3072 runs the chunked (segmented) scan."""
    tma, seg = _capi.plan(_capi.DTYPE_BF16, b, 3072, 512)
    assert tma and seg > 1
    k, v, td, tf, gy = config_inputs(b, 3072, 512, seed=20 + b, kscale=4.0)
    got = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=torch.bfloat16, device=cuda)
    _assert_close(got, _oracle(k, v, td, tf, gy, round_to=torch.bfloat16), TOL_16BIT, f"B={b}")


# ------------------------------------------------------- full-size configs


def test_config0_float32_full(cuda):
    """Config 0 (B=2, T=256, C=512, fp32): every element against the oracle."""
    k, v, td, tf, gy = config_inputs(2, 256, 512)
    got = _run(weighted_key_value_cuda, k, v, td, tf, gy, dtype=torch.float32, device=cuda)
    _assert_close(got, _oracle(k, v, td, tf, gy), TOL_FP32, "cfg0")


def test_config1_bf16_full(cuda):
    """Config 1 (B=64, T=1024, C=512, bf16, k/v x4): every element of y and the
    gradients against the float64 oracle on the same bf16 inputs."""
    k, v, td, tf, gy = config_inputs(64, 1024, 512, kscale=4.0)
    got = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=torch.bfloat16, device=cuda)
    _assert_close(got, _oracle(k, v, td, tf, gy, round_to=torch.bfloat16), TOL_16BIT, "cfg1")


def test_config2_bf16_full(cuda):
    """Config 2 (B=24, T=3072, C=512, bf16, k/v x4) against the oracle."""
    k, v, td, tf, gy = config_inputs(24, 3072, 512, seed=2, kscale=4.0)
    got = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=torch.bfloat16, device=cuda)
    _assert_close(got, _oracle(k, v, td, tf, gy, round_to=torch.bfloat16), TOL_16BIT, "cfg2")


def test_config1_float32_matches_oracle(cuda):
    """Config 1 shape with float32 I/O, where the 1e-5 bound applies."""
    k, v, td, tf, gy = config_inputs(64, 1024, 512, seed=3, kscale=4.0)
    got = _run(weighted_key_value_cuda, k, v, td, tf, gy, dtype=torch.float32, device=cuda)
    _assert_close(got, _oracle(k, v, td, tf, gy), TOL_FP32, "cfg1-fp32")


# ------------------------------------------- size-independent properties


def test_known_answer_first_step_is_value(cuda):
    """reference tests/test_language.py:31-46: y[:, 0] == v[:, 0]."""
    key = torch.randn(2, 4, 3, device=cuda)
    value = torch.randn(2, 4, 3, device=cuda)
    out = weighted_key_value_cuda(key, value, torch.zeros(3, device=cuda), torch.zeros(3, device=cuda))
    assert torch.allclose(out[:, 0], value[:, 0])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_shift_invariance_in_key_at_full_size(cuda, dtype):
    """Adding a constant to every key scales every weight by the same factor, so
    y is unchanged (checked at config-1 size, both execution regimes)."""
    k, v, td, tf, _ = config_inputs(64, 1024, 512, seed=9, kscale=4.0)
    k = np.clip(np.round(k * 4.0) / 4.0, -48.0, 48.0)  # k and k + 8 exact in bf16
    kt = torch.as_tensor(k).to(cuda, dtype)
    vt = torch.as_tensor(v).to(cuda, dtype)
    tdt, tft = torch.as_tensor(td).to(cuda), torch.as_tensor(tf).to(cuda)
    y0 = weighted_key_value_cuda_bf16io(kt, vt, tdt, tft).float()
    y1 = weighted_key_value_cuda_bf16io((kt.float() + 8.0).to(dtype), vt, tdt, tft).float()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert (y1 - y0).abs().max().item() / max(1.0, y0.abs().max().item()) < tol


def test_affine_equivariance_in_value(cuda):
    """y(a v + b) = a y(v) + b: y is a convex combination of values."""
    k, v, td, tf, _ = config_inputs(8, 512, 256, seed=4)
    kt, vt = torch.as_tensor(k).cuda(), torch.as_tensor(v).cuda()
    tdt, tft = torch.as_tensor(td).cuda(), torch.as_tensor(tf).cuda()
    y = weighted_key_value_cuda(kt, vt, tdt, tft)
    y2 = weighted_key_value_cuda(kt, 3.0 * vt - 2.0, tdt, tft)
    assert torch.allclose(y2, 3.0 * y - 2.0, atol=1e-4, rtol=1e-5)


def test_gradient_of_sum_over_batch_is_sum_of_shards(cuda):
    """Data-parallel invariant: the per-channel gradients of a batch equal the
    sum over batch shards (reference tests/test_grad_accum.py:35-48)."""
    k, v, td, tf, gy = config_inputs(8, 256, 128, seed=6)
    full = _run(weighted_key_value_cuda, k, v, td, tf, gy, dtype=torch.float32, device=cuda)
    parts = [_run(weighted_key_value_cuda, k[i : i + 2], v[i : i + 2], td, tf, gy[i : i + 2], dtype=torch.float32, device=cuda) for i in range(0, 8, 2)]
    for idx in (3, 4):
        summed = sum(p[idx] for p in parts)
        assert scaled_err(summed, full[idx]) < 1e-5


@pytest.mark.parametrize("segments", [1, 3])
def test_state_handoff_matches_self_contained_backward(cuda, segments):
    """The saved-state backward agrees with the self-contained one: bit for bit
    on the sequential plan (both sweep the same checkpoints from t=0), within
    tolerance when time is split into segments (the self-contained backward then
    builds segment-local checkpoints, rounded differently)."""
    _capi.set_debug_overrides(force_segments=segments)
    k, v, td, tf, gy = config_inputs(8, 512, 256, seed=31, kscale=4.0)
    spikegpt_b200.set_state_saving(True)
    before = _capi.launch_counts()["wkv_fwd_kernel<state>"]
    a = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=torch.bfloat16, device=cuda)
    # with the hand-off the only state-only launch is the forward's segment summary
    assert _capi.launch_counts()["wkv_fwd_kernel<state>"] == before + (1 if segments > 1 else 0)
    spikegpt_b200.set_state_saving(False)
    b = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=torch.bfloat16, device=cuda)
    for x, y in zip(a, b, strict=True):
        if segments == 1:
            np.testing.assert_array_equal(x, y)
        else:
            assert scaled_err(x, y) <= TOL_16BIT


def test_no_state_is_saved_without_grad(cuda):
    k, v, td, tf, _ = config_inputs(2, 64, 64, seed=32)
    kt, vt = torch.as_tensor(k).cuda().requires_grad_(), torch.as_tensor(v).cuda()
    before = _capi.launch_counts()
    with torch.no_grad():
        weighted_key_value_cuda_bf16io(kt, vt, torch.as_tensor(td).cuda(), torch.as_tensor(tf).cuda())
    after = _capi.launch_counts()
    assert after["wkv_fwd_kernel<y>"] == before["wkv_fwd_kernel<y>"] + 1
    assert after["wkv_fwd_kernel<state>"] == before["wkv_fwd_kernel<state>"]


def test_results_are_deterministic(cuda):
    k, v, td, tf, gy = config_inputs(16, 512, 256, seed=8, kscale=4.0)
    a = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=torch.bfloat16, device=cuda)
    b = _run(weighted_key_value_cuda_bf16io, k, v, td, tf, gy, dtype=torch.bfloat16, device=cuda)
    for x, y in zip(a, b, strict=True):
        np.testing.assert_array_equal(x, y)


# --------------------------------------------------------------- contract


def test_direct_backward_op_contract(cuda):
    """myelin::wkv_backward(grad_y, w, u, k, v) -> [gk, gv, g_td (x w), g_tf]
    (reference wkv_triton.py:164-198) called directly."""
    k, v, td, tf, gy = config_inputs(3, 33, 40, seed=12)
    kt, vt, gyt = (torch.as_tensor(x).cuda() for x in (k, v, gy))
    w = -torch.exp(torch.as_tensor(td).cuda())
    u = torch.as_tensor(tf).cuda()
    gk, gv, gtd, gtf = torch.ops.myelin.wkv_backward(gyt, w, u, kt, vt)
    assert gk.dtype == gv.dtype == torch.float32 and gtd.shape == gtf.shape == (40,)
    _, rgk, rgv, rgtd, rgtf = _oracle(k, v, td, tf, gy)
    for got, ref in zip((gk, gv, gtd, gtf), (rgk, rgv, rgtd, rgtf), strict=True):
        assert scaled_err(got.double().cpu().numpy(), ref) <= TOL_FP32


def test_float64_inputs_round_trip_dtype(cuda):
    k, v, td, tf, gy = golden_inputs("variants_square", CASES)
    got = _run(weighted_key_value_cuda, k, v, td, tf, gy, dtype=torch.float64, device=cuda)
    _assert_close(got, [CASES["variants_square"][f] for f in FIELDS], TOL_FP32, "f64")


def test_misaligned_pointers_use_the_generic_path(cuda):
    """A contiguous view starting 2 bytes into its buffer cannot be TMA-staged."""
    b, t, c = 2, 40, 64
    k, v, td, tf, gy = config_inputs(b, t, c, seed=13)
    n = b * t * c
    buf = torch.zeros(3 * n + 8, dtype=torch.bfloat16, device=cuda)
    kt = buf[1 : 1 + n].view(b, t, c)
    vt = buf[2 + n : 2 + 2 * n].view(b, t, c)
    kt.copy_(torch.as_tensor(k))
    vt.copy_(torch.as_tensor(v))
    assert kt.data_ptr() % 16 != 0
    y = weighted_key_value_cuda_bf16io(kt, vt, torch.as_tensor(td).cuda(), torch.as_tensor(tf).cuda())
    ref = _oracle(k, v, td, tf, gy, round_to=torch.bfloat16)[0]
    assert scaled_err(y.double().cpu().numpy(), ref) <= TOL_16BIT


def test_bad_shapes_raise_value_error(cuda):
    key = torch.randn(2, 4, 3, device=cuda)
    with pytest.raises(ValueError, match="same shape"):
        weighted_key_value_cuda(key, torch.randn(2, 4, 2, device=cuda), torch.zeros(3, device=cuda), torch.zeros(3, device=cuda))
    with pytest.raises(ValueError, match="time_decay must have shape"):
        weighted_key_value_cuda(key, key, torch.zeros(4, device=cuda), torch.zeros(3, device=cuda))


@pytest.mark.parametrize("shape", [(0, 4, 8), (2, 0, 8), (2, 4, 0)])
def test_empty_inputs(cuda, shape):
    c = shape[2]
    k = torch.randn(*shape, device=cuda, requires_grad=True)
    v = torch.randn(*shape, device=cuda, requires_grad=True)
    td = torch.randn(c, device=cuda, requires_grad=True)
    tf = torch.randn(c, device=cuda, requires_grad=True)
    y = weighted_key_value_cuda(k, v, td, tf)
    assert y.shape == shape
    y.sum().backward()
    assert torch.count_nonzero(td.grad) == 0 and torch.count_nonzero(tf.grad) == 0


def test_opcheck_forward_and_backward(cuda):
    k, v, td, tf, _ = config_inputs(2, 20, 16, seed=14)
    args = [torch.as_tensor(x).cuda().requires_grad_() for x in (k, v, td, tf)]
    torch.library.opcheck(torch.ops.myelin.wkv_forward.default, args)
    torch.library.opcheck(torch.ops.myelin.wkv_forward_bf16io.default, args)


def test_torch_compile_fullgraph_matches_eager(cuda):
    k, v, td, tf, gy = config_inputs(4, 128, 64, seed=15)

    def block(k, v, td, tf):
        return (weighted_key_value_cuda_bf16io(k * 1.0, v, td, tf) * 2.0).sum(-1)

    compiled = torch.compile(block, fullgraph=True)
    outs = []
    for fn in (block, compiled):
        leaves = [torch.as_tensor(x).cuda().requires_grad_() for x in (k, v, td, tf)]
        out = fn(*leaves).sum()
        torch.cuda.synchronize()
        before = _capi.launch_counts()
        out.backward()
        torch.cuda.synchronize()
        after = _capi.launch_counts()
        # both take the saved-state backward: no state sweep, one gradient launch
        assert after["wkv_fwd_kernel<state>"] == before["wkv_fwd_kernel<state>"]
        assert after["wkv_bwd_kernel<grad>"] == before["wkv_bwd_kernel<grad>"] + 1
        outs.append([leaves[0].grad, leaves[1].grad, leaves[2].grad, leaves[3].grad])
    for a, b in zip(*outs, strict=True):
        assert scaled_err(a.cpu().numpy(), b.cpu().numpy()) <= TOL_FP32


def test_torch_compile_without_state_saving_uses_the_schema_backward(cuda):
    """With the hand-off disabled the compiled graph calls the reference's
    self-contained backward op, which runs its own state sweep."""
    k, v, td, tf, gy = config_inputs(4, 128, 64, seed=16)
    spikegpt_b200.set_state_saving(False)
    try:
        torch._dynamo.reset()
        compiled = torch.compile(lambda *a: weighted_key_value_cuda_bf16io(*a).sum(), fullgraph=True)
        leaves = [torch.as_tensor(x).cuda().requires_grad_() for x in (k, v, td, tf)]
        out = compiled(*leaves)
        before = _capi.launch_counts()
        out.backward()
        torch.cuda.synchronize()
        assert _capi.launch_counts()["wkv_fwd_kernel<state>"] > before["wkv_fwd_kernel<state>"]
    finally:
        spikegpt_b200.set_state_saving(True)
        torch._dynamo.reset()


def test_no_device_side_errors_were_raised(cuda):
    torch.cuda.synchronize()
    assert _capi.device_error_flags(clear=True) == 0
