"""Grouped expert operators for larger batches (mirror of ``exlr8/fast_prefill.py``).

Same signatures as the reference.  Rows are sorted by expert on the device
(the reference's ``_plan``/``_segment_table``, fast_prefill.py:19-46, also
callable on its own as ``plan``) and every expert's tiles are decoded once
per group of rows.  Matrix operands are
float16 hi/lo pieces with float32 accumulation, which is at least as exact as
the reference's ``half_dot`` experiment, so ``half_dot`` is accepted and has
no further effect.
"""

from __future__ import annotations

import torch

from . import _lib
from .fast_decode import fast_expert_mlp
from .trellis import expert_linear, trellis_linear


def block_rows(rows, experts):
    """Rows per table block (fast_prefill.py:104-109 _block_rows): 8 for small
    segments (fewer discarded matrix rows), 32 otherwise."""
    return 8 if rows < experts * 8 else 32


def plan(indices, experts, block_rows=8):
    """``(sorted_ids, order, table, count)`` of fast_prefill.py:38-46 ``_plan``:
    the flattened slot ids sorted by expert (stable), their order, and the
    block table ``[3, blocks]`` (expert, first sorted row, length) of
    ``_segment_table`` (:19-35) with ``blocks = min(n, n // block_rows +
    experts)``; ``count`` (int32 tensor of one element) is the number of
    valid columns.  Computed on the GPU (the library's stable counting sort).
    Ids are returned as int32; ids >= ``experts`` sort after every valid id
    in slot order and get no table column."""
    device = _lib.require_cuda(indices)
    ids = indices.reshape(-1).to(torch.int32).contiguous()
    n = ids.numel()
    if not 1 <= experts <= 1024 or block_rows < 1:
        raise ValueError("plan takes 1..1024 experts and a positive block size")
    blocks = min(n, n // block_rows + experts)
    order = torch.empty(n, dtype=torch.int32, device=device)
    sorted_ids = torch.empty(n, dtype=torch.int32, device=device)
    table = torch.empty((3, max(blocks, 1)), dtype=torch.int32, device=device)
    count = torch.zeros(1, dtype=torch.int32, device=device)
    lib = _lib.lib()
    need = int(lib.exlr8_dispatch_plan_workspace(n, experts))
    workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
    _lib.check(lib.exlr8_dispatch_plan(ids.data_ptr(), n, experts, block_rows, order.data_ptr(),
                                       sorted_ids.data_ptr(), table.data_ptr(), table.shape[1], count.data_ptr(),
                                       workspace.data_ptr(), workspace.numel(), _lib.stream_handle(device)))
    return sorted_ids, order, table[:, :blocks], count


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
