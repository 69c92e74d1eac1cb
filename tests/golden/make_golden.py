"""Generate the golden WKV vectors from the reference implementation itself.

Run in a container that has the reference checkout (it is NOT needed at test
time; the output ``wkv_golden.npz`` is committed):

    python tests/golden/make_golden.py --reference /path/to/spikegpt-myelin

It imports the reference's ``spikegpt.language`` (with the test-only ``myelin``
stand-in in ``_myelin_shim/``, because the real dependency is not installable
offline) and evaluates, in float64 with autograd:

* ``weighted_key_value_loop`` (reference ``src/spikegpt/language.py:399-449``),
  the reference's own correctness oracle, forward and backward;
* ``weighted_key_value`` (``language.py:452-527``, the reference's CPU path,
  an ``associative_scan``) forward, as a cross-check of the loop.

Cases mirror the reference's own WKV tests:
``tests/test_wkv_triton.py:35-68`` (T in {1, 7, 64}, B=3, C=96, seed=t; C=70),
``tests/test_wkv_variants.py:24-56`` (B=3, C=8, T in {1,4,16,17,40}; backward of
``out.square().sum()`` at B=2, T=24, seed 1), plus config 0 of the benchmark
(B=2, T=256, C=512; outputs stored subsampled), large-magnitude keys that
stress the log-space max path, fast/slow decay extremes, and bf16-rounded
inputs. Inputs are stored exactly (float32 or float64 as generated), outputs
in float64.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CFG0_STRIDE = 97  # cfg0 outputs are stored at flat indices 0, 97, 194, ...


def cfg0_inputs(b: int = 2, t: int = 256, c: int = 512, *, seed: int = 0, kscale: float = 1.0):
    """Config-0 distributions (seeded numpy PCG64): k, v, gy ~ N(0,1) [B,T,C];
    time_decay ~ U(-5, 1), time_first ~ U(-1, 1) [C]; all float32."""
    rng = np.random.default_rng(seed)
    k = (rng.standard_normal((b, t, c)) * kscale).astype(np.float32)
    v = (rng.standard_normal((b, t, c)) * kscale).astype(np.float32)
    td = rng.uniform(-5.0, 1.0, c).astype(np.float32)
    tf = rng.uniform(-1.0, 1.0, c).astype(np.float32)
    gy = rng.standard_normal((b, t, c)).astype(np.float32)
    return k, v, td, tf, gy


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference", help="reference checkout root")
    ap.add_argument("--out", default=str(HERE / "wkv_golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, str(HERE / "_myelin_shim"))
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch
    from spikegpt.language import weighted_key_value, weighted_key_value_loop

    out: dict[str, np.ndarray] = {}

    def run(name, k, v, td, tf, gy, *, store_inputs=True, stride=None):
        tensors = [torch.tensor(np.asarray(x), dtype=torch.float64) for x in (k, v, td, tf)]
        leaves = [x.clone().requires_grad_(True) for x in tensors]
        y = weighted_key_value_loop(*leaves)
        y.backward(torch.tensor(np.asarray(gy), dtype=torch.float64))
        grads = [
            torch.zeros_like(x) if x.grad is None else x.grad for x in leaves
        ]  # T=1 leaves time_decay without a gradient (reference test_wkv_triton.py:29-30)
        y_assoc = weighted_key_value(*tensors)
        res = {
            "y": y.detach().numpy(),
            "gk": grads[0].numpy(),
            "gv": grads[1].numpy(),
            "gtd": grads[2].numpy(),
            "gtf": grads[3].numpy(),
            "y_assoc": y_assoc.numpy(),
        }
        if stride:
            for key in ("y", "gk", "gv", "y_assoc"):
                res[key] = res[key].reshape(-1)[::stride].copy()
        elif res["y"].size > 4096:  # keep the fixture small: only the loop-vs-scan gap
            res["y_assoc_maxdiff"] = np.array([np.abs(res.pop("y_assoc") - res["y"]).max()])
        if store_inputs:
            for key, x in zip(("k", "v", "td", "tf", "gy"), (k, v, td, tf, gy), strict=True):
                out[f"{name}/{key}"] = np.asarray(x)
        for key, val in res.items():
            out[f"{name}/{key}"] = val
        print(f"{name}: y[0]={float(res['y'].reshape(-1)[0]):.6f}")

    # reference tests/test_wkv_triton.py:35-54 (generated on CPU in float32)
    for t in (1, 7, 64):
        torch.manual_seed(t)
        b, c = 3, 96
        k, v = torch.randn(b, t, c), torch.randn(b, t, c)
        td, tf = torch.randn(c), torch.randn(c)
        gy = torch.randn(b, t, c)
        run(f"triton_t{t}", *(x.numpy() for x in (k, v, td, tf, gy)))
    # reference tests/test_wkv_triton.py:57-68 (C not a multiple of the block)
    torch.manual_seed(0)
    b, t, c = 2, 16, 70
    k, v = torch.randn(b, t, c), torch.randn(b, t, c)
    td, tf = torch.randn(c), torch.randn(c)
    gy = torch.randn(b, t, c)
    run("channels70", *(x.numpy() for x in (k, v, td, tf, gy)))
    # reference tests/test_wkv_variants.py:24-40 (float64 inputs, B=3, C=8)
    for t in (1, 4, 16, 17, 40):
        g = torch.Generator().manual_seed(0)
        k = torch.randn(3, t, 8, generator=g, dtype=torch.float64)
        v = torch.randn(3, t, 8, generator=g, dtype=torch.float64)
        td = torch.randn(8, generator=g, dtype=torch.float64)
        tf = torch.randn(8, generator=g, dtype=torch.float64)
        gy = torch.zeros_like(k)  # forward-only case in the reference; gy=0 here
        run(f"variants_t{t}", *(x.numpy() for x in (k, v, td, tf, gy)))
    # reference tests/test_wkv_variants.py:43-56: grads of out.square().sum()
    g = torch.Generator().manual_seed(1)
    k = torch.randn(2, 24, 8, generator=g, dtype=torch.float64)
    v = torch.randn(2, 24, 8, generator=g, dtype=torch.float64)
    td = torch.randn(8, generator=g, dtype=torch.float64)
    tf = torch.randn(8, generator=g, dtype=torch.float64)
    y0 = weighted_key_value_loop(k, v, td, tf)
    run("variants_square", *(x.numpy() for x in (k, v, td, tf, 2.0 * y0)))
    # config 0 of the benchmark, outputs subsampled (inputs regenerate from seed 0)
    k, v, td, tf, gy = cfg0_inputs()
    out["cfg0/input_sums"] = np.array(
        [float(np.sum(x, dtype=np.float64)) for x in (k, v, td, tf, gy)]
    )
    run("cfg0", k, v, td, tf, gy, store_inputs=False, stride=CFG0_STRIDE)
    # large-magnitude keys (x4 and x20): the running log-scale max path
    for scale in (4.0, 20.0):
        k, v, td, tf, gy = cfg0_inputs(2, 96, 16, seed=7, kscale=scale)
        run(f"kscale{int(scale)}", k, v, td, tf, gy)
    # decay extremes: very slow (td=-8 -> w~-3e-4) and very fast (td=3 -> w~-20)
    k, v, _, tf, gy = cfg0_inputs(2, 80, 8, seed=11)
    td = np.array([-8.0, -8.0, -3.0, 0.0, 1.0, 2.0, 3.0, 3.0], dtype=np.float32)
    run("decay_extremes", k, v, td, tf, gy)
    # bf16-rounded inputs (config 1 distributions at a small size)
    k, v, td, tf, gy = cfg0_inputs(2, 64, 32, seed=3, kscale=4.0)
    to_bf16 = lambda x: torch.tensor(x).to(torch.bfloat16).float().numpy()  # noqa: E731
    run("bf16_rounded", to_bf16(k), to_bf16(v), td, tf, to_bf16(gy))

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out} ({Path(args.out).stat().st_size / 1024:.1f} KiB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
