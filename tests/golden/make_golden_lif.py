"""Generate golden vectors for the LIF sequence op from the reference's own
SpikingSequenceLIF (src/spikegpt/language.py:766-918).

Run in a container with the reference checkout (not needed at test time; the
output ``lif_golden.npz`` is committed):

    python tests/golden/make_golden_lif.py --reference /path/to/spikegpt-myelin

On CPU the reference's forward takes its per-step loop (language.py:907-918,
the loop the reference keeps as the correctness oracle for its fused kernels),
so the membrane update, threshold, reset and every gradient path come from the
reference's code under torch autograd. The spike function and its surrogate
gradient come from ``tests/golden/_myelin_shim/myelin/surrogates.py``, a
restatement of the published arc-tangent surrogate, because the reference's
dependency myelin@68b8ebb is absent: the surrogate itself is unpinned.

Cases: B=3 T=40 C=96 (default parameters tau=2, threshold=1, reset=0, slope=2);
ragged C=70; custom parameters (tau=3, threshold=0.5, reset=-0.2, slope=4);
large currents (frequent spikes). Evaluated in float64 (spikes, d loss / d
input for a random upstream gradient).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--out", default=str(HERE / "lif_golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, str(HERE / "_myelin_shim"))
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch
    from spikegpt.language import SpikingSequenceLIF

    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(11)

    def run(name, b, t, c, *, scale=1.0, tau=2.0, threshold=1.0, reset=0.0, slope=2.0):
        x = (rng.standard_normal((b, t, c)) * scale + 0.4).astype(np.float32)
        gs = rng.standard_normal((b, t, c)).astype(np.float32)
        lif = SpikingSequenceLIF(tau=tau, threshold=threshold, reset=reset, surrogate_slope=slope)
        xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
        spikes = lif(xt)
        spikes.backward(torch.tensor(gs, dtype=torch.float64))
        out[f"{name}/x"] = x
        out[f"{name}/gs"] = gs
        out[f"{name}/params"] = np.array([tau, threshold, reset, slope])
        out[f"{name}/spikes"] = spikes.detach().numpy()
        out[f"{name}/gx"] = xt.grad.numpy()

    run("default", 3, 40, 96)
    run("channels70", 2, 33, 70)
    run("custom_params", 2, 48, 64, tau=3.0, threshold=0.5, reset=-0.2, slope=4.0)
    run("large_currents", 2, 32, 64, scale=4.0)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays")


if __name__ == "__main__":
    main()
