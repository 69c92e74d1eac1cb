"""GPU parity of the recurrent WKV step (wkv_step through the registered op
spikegpt_b200::wkv_step_) against the reference's own SpikeTimeMix.step golden
vectors and the CPU oracle. Tolerances as for the sequence op:
max|x - ref| / max(1, max|ref|) <= 1e-5 (float32 I/O), <= 2e-2 (bf16/fp16)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
from _wkvtest import TOL_16BIT, TOL_FP32, config_inputs, scaled_err

import spikegpt_b200
from oracle import oracle
from spikegpt_b200 import (
    _capi,
    initial_step_state,
    weighted_key_value_cuda,
    weighted_key_value_cuda_bf16io,
    weighted_key_value_step,
    weighted_key_value_step_,
)

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "wkv_step_golden.npz")
SINGLE = ["random_state", "initial_state", "large_keys", "decay_extremes"]
FIELDS = ("y", "num", "den", "ls")


def _case(name):
    return {f.split("/")[1]: GOLDEN[f] for f in GOLDEN.files if f.startswith(name + "/")}


def _dev(x, dtype, device):
    return torch.as_tensor(np.asarray(x, np.float64)).to(device=device, dtype=dtype)


def _run_step(g, dtype, device):
    fmin = torch.finfo(dtype).min
    k, v, num, den = (_dev(g[f], dtype, device) for f in ("k", "v", "num", "den"))
    ls = _dev(np.maximum(g["ls"], fmin), dtype, device)
    td, tf = (torch.as_tensor(g[f]).to(device) for f in ("td", "tf"))
    out = weighted_key_value_step(k, v, td, tf, num, den, ls)
    return [o.double().cpu().numpy() for o in out], (k, v, num, den, ls, td, tf)


@pytest.mark.parametrize("name", SINGLE)
def test_float32_step_matches_reference(cuda, name):
    g = _case(name)
    got, _ = _run_step(g, torch.float32, cuda)
    for field, x in zip(FIELDS, got, strict=True):
        err = scaled_err(x, g[f"{field}_f64"])
        assert err <= TOL_FP32, f"{name} {field}: {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name", SINGLE)
def test_16bit_step_matches_oracle_on_rounded_inputs(cuda, name, dtype):
    g = _case(name)
    got, ins = _run_step(g, dtype, cuda)
    k, v, num, den, ls, td, tf = (x.double().cpu().numpy() for x in ins)
    ref = oracle.step(k, v, td, tf, num, den, ls)
    for field, x, r in zip(FIELDS, got, ref, strict=True):
        err = scaled_err(x, r)
        assert err <= TOL_16BIT, f"{name} {field}: {err:.3e}"
    if dtype == torch.bfloat16:  # and the reference's own bf16 arithmetic
        for field, x in zip(FIELDS, got, strict=True):
            err = scaled_err(x, g[f"{field}_bf16"])
            assert err <= TOL_16BIT, f"{name} {field} vs reference bf16: {err:.3e}"


def test_first_step_from_initial_state_is_value(cuda):
    g = _case("initial_state")
    k, v = (_dev(g[f], torch.float32, cuda) for f in ("k", "v"))
    state = initial_step_state(*k.shape, device=cuda, dtype=torch.float32)
    y = weighted_key_value_step_(k, v, torch.as_tensor(g["td"]).to(cuda), torch.as_tensor(g["tf"]).to(cuda), *state)
    assert torch.equal(y, v)


def test_sequence_of_steps_matches_reference_loop(cuda):
    g = _case("sequence")
    b, t, c = g["k"].shape
    td, tf = (torch.as_tensor(g[f]).to(cuda) for f in ("td", "tf"))
    state = initial_step_state(b, c, device=cuda, dtype=torch.float32)
    ys = []
    for i in range(t):
        ys.append(weighted_key_value_step_(_dev(g["k"][:, i], torch.float32, cuda),
                                           _dev(g["v"][:, i], torch.float32, cuda), td, tf, *state))
    ys = torch.stack(ys, 1).double().cpu().numpy()
    assert scaled_err(ys, g["y_loop"]) <= TOL_FP32
    for field, x in zip(("num", "den", "ls"), state, strict=True):
        assert scaled_err(x.double().cpu().numpy(), g[f"{field}_f64"]) <= TOL_FP32


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_steps_agree_with_the_sequence_op_at_config_scale(cuda, dtype):
    """Decoding T tokens one step at a time with a float32 state (the autocast
    case for 16-bit keys) gives the sequence op's y."""
    b, t, c = 64, 48, 512
    k, v, td, tf, _ = config_inputs(b, t, c, seed=21, kscale=4.0)
    kd, vd = (torch.as_tensor(x).to(cuda, dtype) for x in (k, v))
    tdd, tfd = (torch.as_tensor(x).to(cuda) for x in (td, tf))
    seq_op = weighted_key_value_cuda if dtype == torch.float32 else weighted_key_value_cuda_bf16io
    with torch.no_grad():
        y_seq = seq_op(kd, vd, tdd, tfd).double().cpu().numpy()
    state = initial_step_state(b, c, device=cuda, dtype=torch.float32)
    ys = torch.stack([weighted_key_value_step_(kd[:, i].contiguous(), vd[:, i].contiguous(), tdd, tfd, *state)
                      for i in range(t)], 1)
    assert ys.dtype == torch.float32
    ys = ys.double().cpu().numpy()
    tol = TOL_FP32 if dtype == torch.float32 else TOL_16BIT
    assert scaled_err(ys, y_seq) <= tol
    ref = oracle.forward(kd.double().cpu().numpy(), vd.double().cpu().numpy(), td, tf)
    assert scaled_err(ys, ref) <= tol


def test_16bit_state_decoding_matches_the_oracle_step_by_step(cuda):
    """With the state kept in bf16 (a module run entirely in bf16, as the
    reference's initial_state gives), each step agrees with the oracle fed the
    same stored state. (The stored log-scale is rounded every step, so a bf16
    state drifts from the float32 sequence; that is the reference's design.)"""
    b, t, c = 16, 24, 512
    k, v, td, tf, _ = config_inputs(b, t, c, seed=22, kscale=4.0)
    kd, vd = (torch.as_tensor(x).to(cuda, torch.bfloat16) for x in (k, v))
    tdd, tfd = (torch.as_tensor(x).to(cuda) for x in (td, tf))
    state = initial_step_state(b, c, device=cuda, dtype=torch.bfloat16)
    for i in range(t):
        before = [x.double().cpu().numpy() for x in state]
        ki, vi = kd[:, i].contiguous(), vd[:, i].contiguous()
        y = weighted_key_value_step_(ki, vi, tdd, tfd, *state)
        assert y.dtype == torch.bfloat16
        ref = oracle.step(ki.double().cpu().numpy(), vi.double().cpu().numpy(), td, tf, *before)
        for x, r in zip((y, *state), ref, strict=True):
            assert scaled_err(x.double().cpu().numpy(), r) <= TOL_16BIT, i


@pytest.mark.parametrize("c", [1, 7, 70, 96, 520])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_channel_counts_vector_and_scalar_paths(cuda, c, dtype):
    rng = np.random.default_rng(c)
    b = 5
    k, v = rng.standard_normal((2, b, c)) * 3
    td, tf = rng.uniform(-5, 1, c).astype(np.float32), rng.uniform(-1, 1, c).astype(np.float32)
    den = rng.uniform(0.5, 3, (b, c))
    num, ls = den * rng.uniform(-1, 1, (b, c)), rng.standard_normal((b, c))
    got, ins = _run_step({"k": k, "v": v, "td": td, "tf": tf, "num": num, "den": den, "ls": ls}, dtype, cuda)
    ref = oracle.step(*(x.double().cpu().numpy() for x in ins[:2]), td, tf,
                      *(x.double().cpu().numpy() for x in ins[2:5]))
    tol = TOL_FP32 if dtype == torch.float32 else TOL_16BIT
    for field, x, r in zip(FIELDS, got, ref, strict=True):
        assert scaled_err(x, r) <= tol, field


def test_misaligned_tensors_use_the_scalar_path(cuda):
    b, c = 4, 64
    base = torch.randn(b * c + 1, device=cuda)
    k = base[1:].view(b, c)  # 4-byte offset: not 16-byte aligned
    v = torch.randn(b, c, device=cuda)
    td, tf = torch.rand(c, device=cuda) * 6 - 5, torch.rand(c, device=cuda) * 2 - 1
    num, den, ls = torch.zeros(b, c, device=cuda), torch.ones(b, c, device=cuda), torch.zeros(b, c, device=cuda)
    y, *_ = weighted_key_value_step(k, v, td, tf, num, den, ls)
    ref = oracle.step(k.double().cpu().numpy(), v.double().cpu().numpy(), td.cpu().numpy(), tf.cpu().numpy(),
                      num.double().cpu().numpy(), den.double().cpu().numpy(), ls.double().cpu().numpy())
    assert scaled_err(y.double().cpu().numpy(), ref[0]) <= TOL_FP32


def test_functional_form_leaves_the_state_untouched_in_place_form_updates_it(cuda):
    b, c = 3, 32
    k, v = torch.randn(2, b, c, device=cuda)
    td, tf = torch.zeros(c, device=cuda), torch.zeros(c, device=cuda)
    state = initial_step_state(b, c, device=cuda, dtype=torch.float32)
    before = [s.clone() for s in state]
    _, n2, d2, l2 = weighted_key_value_step(k, v, td, tf, *state)
    for s, s0 in zip(state, before, strict=True):
        assert torch.equal(s, s0)
    weighted_key_value_step_(k, v, td, tf, *state)
    for s, s2 in zip(state, (n2, d2, l2), strict=True):
        assert torch.equal(s, s2)


def test_empty_batch_and_bad_shapes(cuda):
    z = torch.empty(0, 8, device=cuda)
    y, *_ = weighted_key_value_step(z, z, torch.zeros(8, device=cuda), torch.zeros(8, device=cuda), z, z, z)
    assert y.shape == (0, 8)
    k = torch.zeros(2, 8, device=cuda)
    with pytest.raises(ValueError):
        weighted_key_value_step(k, k, torch.zeros(7, device=cuda), torch.zeros(8, device=cuda), k, k, k)
    with pytest.raises(ValueError):
        weighted_key_value_step(k, k.double(), torch.zeros(8, device=cuda), torch.zeros(8, device=cuda), k, k, k)


def test_decode_step_compiles_fullgraph(cuda):
    b, c = 8, 64
    td, tf = torch.rand(c, device=cuda) * 6 - 5, torch.rand(c, device=cuda) * 2 - 1

    def decode(k, v, num, den, ls):
        return weighted_key_value_step_(k, v, td, tf, num, den, ls) * 2.0

    fn = torch.compile(decode, fullgraph=True)
    k, v = torch.randn(2, b, c, device=cuda)
    s1 = initial_step_state(b, c, device=cuda, dtype=torch.float32)
    s2 = [s.clone() for s in s1]
    for _ in range(3):
        a = fn(k, v, *s1)
        e = decode(k, v, *s2)
        assert torch.equal(a, e)
    for x, y in zip(s1, s2, strict=True):
        assert torch.equal(x, y)


def test_step_kernel_launches_are_counted(cuda):
    before = _capi.launch_counts()["wkv_step_kernel"]
    k = torch.randn(2, 16, device=cuda)
    weighted_key_value_step(k, k, torch.zeros(16, device=cuda), torch.zeros(16, device=cuda),
                            *initial_step_state(2, 16, device=cuda, dtype=torch.float32))
    assert _capi.launch_counts()["wkv_step_kernel"] == before + 1
    assert spikegpt_b200.weighted_key_value_step is weighted_key_value_step
