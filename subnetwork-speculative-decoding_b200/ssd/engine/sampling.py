"""Sampling (temperature > 0) on the device: warped distributions, Gumbel
top-k drafting and multi-candidate speculative-sampling verification.

Placeholder until the sampling kernels land: every entry point raises, so
no sampling request silently falls back to a host implementation.
"""

from __future__ import annotations


def _unavailable(*_a, **_k):
    raise NotImplementedError("temperature > 0 needs the device sampling kernels, not built yet")


warp_probs_device = _unavailable
sampled_tree_build = _unavailable
sample_verify_device = _unavailable
sampled_autoregressive = _unavailable
sampled_speculative = _unavailable
