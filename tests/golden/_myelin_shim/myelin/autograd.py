"""Placeholders for myelin's fused LIF autograd functions (never called here)."""


def _unavailable(*_args, **_kwargs):
    raise RuntimeError("myelin LIF kernels are not available in this test shim")


triton_surrogate_lif_function = _unavailable
triton_surrogate_lif_recompute_function = _unavailable
