"""Test-only stand-in for the absent ``myelin`` dependency (git 68b8ebb).

It exists so that ``tests/golden/make_golden.py`` can import the reference's
``spikegpt.language`` in the build container and run its float64 WKV loop. None
of these names enter the WKV arithmetic: ``has_triton`` only gates dispatch
(reference ``src/spikegpt/wkv_triton.py:25,28``), and the LIF/surrogate names are
only touched by the spiking layers, which the golden script never runs.
"""
