"""Grouped expert operators for larger batches (mirror of ``exlr8/fast_prefill.py``).

Same signatures as the reference.  Rows are sorted by expert on the device
(the reference's ``_plan``/``_segment_table``, fast_prefill.py:19-46) and every
expert's tiles are decoded once per group of rows.  Matrix operands are
float16 hi/lo pieces with float32 accumulation, which is at least as exact as
the reference's ``half_dot`` experiment, so ``half_dot`` is accepted and has
no further effect.
"""

from __future__ import annotations

from .fast_decode import fast_expert_mlp
from .trellis import expert_linear, trellis_linear


def grouped_expert_linear(x, indices, packed, in_scale, out_scale, k, in_features, out_features, sharded_side=1, *,
                          half_dot=False):
    """Selected-expert linear over sorted rows (fast_prefill.py:151-165)."""
    return expert_linear(x, indices, packed, in_scale, out_scale, k, in_features, out_features, sharded_side)


def trellis_linear_prefill(x, packed, suh, svh, k, in_features, out_features, sharded_side=1):
    """One dense trellis matrix over many rows (fast_prefill.py:168-185)."""
    return trellis_linear(x, packed, suh, svh, k, in_features, out_features, sharded_side)


def grouped_expert_mlp(x, indices, packed, scales, k, hidden, intermediate, *, half_dot=False):
    """Gate/up/down with one expert sort (fast_prefill.py:188-211)."""
    return fast_expert_mlp(x, indices, packed, scales, k, hidden, intermediate)
