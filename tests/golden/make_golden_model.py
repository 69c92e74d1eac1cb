"""Generate golden vectors for the SpikeGPT model from the reference itself.

Run in a container with the reference checkout (not needed at test time; the
output ``model_golden.npz`` is committed):

    python tests/golden/make_golden_model.py --reference /path/to/spikegpt-myelin

Builds the reference's ``SpikeLanguageModel`` (src/spikegpt/language.py:1361)
at a small configuration with its defaults (spiking embedding, RWKV time and
channel mixing, LIF activations; dropout 0), seeded, and runs it on the CPU in
float32: its WKV takes the associative-scan path (language.py:452-527) and its
LIF the per-step loop (language.py:907-918), with the spike function and its
arc-tangent surrogate from the test-only stand-in for the absent myelin
(``tests/golden/_myelin_shim``). Saved: every parameter (the state dict, whose
names this package's ``SpikeGPT`` shares), the token ids and targets, the
loss, the logits and every parameter's gradient.
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
    ap.add_argument("--out", default=str(HERE / "model_golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, str(HERE / "_myelin_shim"))
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch
    from spikegpt.language import SpikeGPTConfig, SpikeLanguageModel

    torch.manual_seed(3)
    cfg = SpikeGPTConfig(vocab_size=64, context_length=48, n_layer=2, n_embd=64, dropout=0.0)
    model = SpikeLanguageModel(cfg)
    # larger weights than the reference's init so that spikes fire in every layer
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith(".weight") and p.ndim == 2:
                p.normal_(0.0, 0.2 if "embedding" not in name else 1.0)
    rng = np.random.default_rng(5)
    ids = rng.integers(0, cfg.vocab_size, size=(2, cfg.context_length + 1))
    x = torch.as_tensor(ids[:, :-1])
    y = torch.as_tensor(ids[:, 1:])
    model.train()
    loss, logits = model(x, y)
    loss.backward()
    out: dict[str, np.ndarray] = {
        "config": np.array([cfg.vocab_size, cfg.context_length, cfg.n_layer, cfg.n_embd]),
        "ids": ids,
        "loss": np.array(loss.item()),
        "logits": logits.detach().numpy(),
    }
    for name, p in model.named_parameters():
        out[f"param/{name}"] = p.detach().numpy()
        out[f"grad/{name}"] = p.grad.numpy()
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, loss {loss.item():.6f}")


if __name__ == "__main__":
    main()
