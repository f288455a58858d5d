# okc: problem=muse_prefill_layer
"""The Muse layer on prefill blocks (muse_prefill_layer/submission.py:84-218: the same weights,
inputs and outputs as muse_decode_layer, q_len 200-16384 tokens per request): `prepare(weights)`
and `kernel_fn(data, state)` of problems/muse_decode_layer.py, which take any q_len.  See that
module for the stages and for what a long block costs (projections in 256-row tcgen05 blocks,
experts in 2048-token passes, attention as one decode query row per token)."""

from __future__ import annotations

from okc_b200.problems.muse_decode_layer import kernel_fn, prepare  # noqa: F401

custom_kernel = kernel_fn
