"""The RWKV-7 DPLR oracle (numpy float64) on CPU. The reference ships no code
for this op, so parity is unpinned; what is checked here are the published
recurrence's special cases: with a = b = 0 and w = 1 it is causal linear
attention, y_t = sum_{s<=t} v_s (k_s . r_t); with w = 0 and a = b = 0 the
state is the last outer product; and chunking T with the state carried over
gives the same result as one pass."""

from __future__ import annotations

import numpy as np

from oracle import oracle


def _rand(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape)


def test_linear_attention_special_case():
    b, t, h, n = 2, 9, 3, 8
    r, k, v = (_rand((b, t, h, n), s) for s in (1, 2, 3))
    zero, one = np.zeros((b, t, h, n)), np.ones((b, t, h, n))
    y, s = oracle.rwkv7_forward_numpy(r, one, k, v, zero, zero)
    ref = np.zeros_like(r)
    for tt in range(t):
        ref[:, tt] = np.einsum("bshi,bshj,bhj->bhi", v[:, : tt + 1], k[:, : tt + 1], r[:, tt])
    np.testing.assert_allclose(y, ref, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(s, np.einsum("bshi,bshj->bhij", v, k), rtol=1e-12, atol=1e-12)


def test_zero_decay_keeps_last_outer_product():
    b, t, h, n = 1, 5, 2, 4
    r, k, v = (_rand((b, t, h, n), s) for s in (4, 5, 6))
    zero = np.zeros((b, t, h, n))
    y, s = oracle.rwkv7_forward_numpy(r, zero, k, v, zero, zero)
    np.testing.assert_allclose(y[:, -1], v[:, -1] * np.einsum("bhj,bhj->bh", k[:, -1], r[:, -1])[..., None])
    np.testing.assert_allclose(s, np.einsum("bhi,bhj->bhij", v[:, -1], k[:, -1]))


def test_state_carry_equals_one_pass():
    b, t, h, n = 2, 12, 2, 8
    ins = [_rand((b, t, h, n), s) * 0.3 for s in range(6)]
    ins[1] = 1 / (1 + np.exp(-ins[1]))  # decay in (0, 1)
    y, s = oracle.rwkv7_forward_numpy(*ins)
    y1, s1 = oracle.rwkv7_forward_numpy(*(x[:, :5] for x in ins))
    y2, s2 = oracle.rwkv7_forward_numpy(*(x[:, 5:] for x in ins), s0=s1)
    np.testing.assert_allclose(np.concatenate([y1, y2], 1), y, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(s2, s, rtol=1e-12, atol=1e-12)
