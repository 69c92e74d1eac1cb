"""Generate golden vectors for the recurrent WKV step from the reference itself.

Run in a container that has the reference checkout (not needed at test time;
the output ``wkv_step_golden.npz`` is committed):

    python tests/golden/make_golden_step.py --reference /path/to/spikegpt-myelin

The reference has no standalone step function: the WKV arithmetic of a step
lives inside ``SpikeTimeMix.step`` (src/spikegpt/language.py:977-1013). This
script calls that method on a ``SpikeTimeMix`` whose projections are set so the
WKV part is observed directly:

* ``key`` and ``value`` are identity maps, ``time_mix_k = 1`` and
  ``time_mix_v = 0``, so the step's key is the token input and its value is the
  state's ``previous`` entry (chosen freely by the caller);
* ``receptance`` has zero weights, so the gate is sigmoid(0) = 0.5 exactly, and
  ``output`` is 2 * identity, so the module output is the WKV value exactly.

Cases: a random state (B=3, C=96), the initial state (known answer y = v), a
16-step sequence from the initial state (B=2, C=70) whose outputs are compared
with ``weighted_key_value_loop`` on the same sequence, large keys, and decay
extremes. Each case is evaluated in float64, float32 and bfloat16 (the
reference computes the step in the model's dtype). Inputs are stored exactly.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference", help="reference checkout root")
    ap.add_argument("--out", default=str(HERE / "wkv_step_golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, str(HERE / "_myelin_shim"))
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch
    from spikegpt.language import SpikeTimeMix, SpikeTimeMixState, weighted_key_value_loop

    torch.manual_seed(0)

    def module(c, td, tf, dtype):
        m = SpikeTimeMix(n_embd=c, n_layer=2, layer_id=0)
        with torch.no_grad():
            m.time_decay.copy_(torch.as_tensor(td))
            m.time_first.copy_(torch.as_tensor(tf))
            m.time_mix_k.fill_(1.0)
            m.time_mix_v.fill_(0.0)
            m.time_mix_r.fill_(1.0)
            m.key.weight.copy_(torch.eye(c))
            m.value.weight.copy_(torch.eye(c))
            m.receptance.weight.zero_()
            m.output.weight.copy_(2.0 * torch.eye(c))
        return m.to(dtype)

    def step(m, k, v, num, den, ls, dtype):
        state = SpikeTimeMixState(
            previous=torch.as_tensor(v).to(dtype),
            numerator=torch.as_tensor(num).to(dtype),
            denominator=torch.as_tensor(den).to(dtype),
            log_scale=torch.as_tensor(ls).to(dtype),
        )
        with torch.no_grad():
            y, nxt = m.step(torch.as_tensor(k).to(dtype), state)
        return [x.to(torch.float64).numpy() for x in (y, nxt.numerator, nxt.denominator, nxt.log_scale)]

    out: dict[str, np.ndarray] = {}
    dtypes = {"f64": torch.float64, "f32": torch.float32, "bf16": torch.bfloat16}

    def add_single(name, k, v, td, tf, num, den, ls):
        c = k.shape[1]
        for key in ("k", "v", "td", "tf", "num", "den", "ls"):
            out[f"{name}/{key}"] = np.asarray(locals()[key])
        for dn, dt in dtypes.items():
            m = module(c, td, tf, dt)
            state_ls = ls if dn == "f64" else np.maximum(ls, float(torch.finfo(dt).min))
            y, n2, d2, l2 = step(m, k, v, num, den, state_ls, dt)
            out[f"{name}/y_{dn}"], out[f"{name}/num_{dn}"] = y, n2
            out[f"{name}/den_{dn}"], out[f"{name}/ls_{dn}"] = d2, l2

    rng = np.random.default_rng(7)
    b, c = 3, 96
    td = rng.uniform(-5, 1, c).astype(np.float32)
    tf = rng.uniform(-1, 1, c).astype(np.float32)
    k = rng.standard_normal((b, c)).astype(np.float32)
    v = rng.standard_normal((b, c)).astype(np.float32)
    ls = (rng.standard_normal((b, c)) * 3).astype(np.float32)
    den = rng.uniform(0.5, 4.0, (b, c)).astype(np.float32)
    num = (den * rng.uniform(-2, 2, (b, c))).astype(np.float32)
    add_single("random_state", k, v, td, tf, num, den, ls)
    add_single("initial_state", k, v, td, tf, np.zeros((b, c), np.float32), np.zeros((b, c), np.float32),
               np.full((b, c), np.finfo(np.float64).min))
    add_single("large_keys", (k * 20).astype(np.float32), v, td, tf, num, den, ls)
    td_ext = np.where(np.arange(c) % 2 == 0, -9.0, 4.0).astype(np.float32)
    add_single("decay_extremes", k, v, td_ext, tf, num, den, ls)

    # a 16-step sequence from the initial state, float64, against the loop oracle
    b, c, t = 2, 70, 16
    td = rng.uniform(-5, 1, c).astype(np.float32)
    tf = rng.uniform(-1, 1, c).astype(np.float32)
    ks = (rng.standard_normal((b, t, c)) * 4).astype(np.float32)
    vs = rng.standard_normal((b, t, c)).astype(np.float32)
    m = module(c, td, tf, torch.float64)
    num, den = np.zeros((b, c)), np.zeros((b, c))
    ls = np.full((b, c), np.finfo(np.float64).min)
    ys = []
    for i in range(t):
        y, num, den, ls = step(m, ks[:, i], vs[:, i], num, den, ls, torch.float64)
        ys.append(y)
    loop = weighted_key_value_loop(*(torch.as_tensor(x, dtype=torch.float64) for x in (ks, vs, td, tf)))
    out.update({"sequence/k": ks, "sequence/v": vs, "sequence/td": td, "sequence/tf": tf,
                "sequence/y_f64": np.stack(ys, 1), "sequence/y_loop": loop.numpy(),
                "sequence/num_f64": num, "sequence/den_f64": den, "sequence/ls_f64": ls})
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays")


if __name__ == "__main__":
    main()
