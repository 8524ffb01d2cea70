"""The standalone dispatch plan (fast_prefill.py:19-46 ``_plan`` and
``_segment_table``) and combine (model.py:415-418) against NumPy.

The plan's expected values restate the reference in NumPy: a stable argsort
of the slot ids and, per expert in id order, ``ceil(count / block_rows)``
table columns (expert, first sorted row, length) -- the valid columns of
``_segment_table``'s vectorised formula.  Ids past the expert count sort
last in slot order and get no column (outside the reference's contract).
Bit-exact: integers.  The combine is bit-exact against the oracle's
restatement in every activation dtype.
"""

import numpy as np
import pytest

from helpers import host, torch_dtype
from oracle import trellis_oracle as ref

pytestmark = pytest.mark.gpu


def _expected_plan(ids, experts, block_rows):
    ids = np.asarray(ids, np.int64)
    key = np.where(ids < experts, ids, experts)
    order = np.argsort(key, kind="stable")
    valid = ids[ids < experts]
    counts = np.bincount(valid, minlength=experts)
    starts = np.cumsum(counts) - counts
    cols = []
    for e in range(experts):
        for j in range(-(-int(counts[e]) // block_rows)):
            cols.append((e, int(starts[e]) + j * block_rows, min(block_rows, int(counts[e]) - j * block_rows)))
    table = np.array(cols, np.int64).reshape(-1, 3).T
    return order, ids[order], table


def _check_plan(ids_np, experts, block_rows):
    import torch

    from mlxlr8_b200.fast_prefill import plan

    ids = torch.from_numpy(np.asarray(ids_np, np.int32)).cuda()
    sorted_ids, order, table, count = plan(ids, experts, block_rows)
    torch.cuda.synchronize()
    e_order, e_sorted, e_table = _expected_plan(ids_np, experts, block_rows)
    n = len(ids_np)
    assert table.shape[1] == min(n, n // block_rows + experts)
    np.testing.assert_array_equal(order.cpu().numpy(), e_order)
    np.testing.assert_array_equal(sorted_ids.cpu().numpy(), e_sorted)
    c = int(count.item())
    assert c == e_table.shape[1]
    np.testing.assert_array_equal(table.cpu().numpy()[:, :c], e_table)


@pytest.mark.parametrize("block_rows", [8, 32])
def test_plan_prefill_size(block_rows):
    """4096 tokens x 9 slots over 257 experts (the multi-CTA sort path)."""
    rng = np.random.default_rng(41)
    ids = np.concatenate([rng.integers(0, 256, (4096, 8)), np.full((4096, 1), 256)], axis=1).reshape(-1)
    _check_plan(ids, 257, block_rows)


@pytest.mark.parametrize("n", [0, 1, 9, 72, 4095])
def test_plan_decode_and_small_sizes(n):
    rng = np.random.default_rng(n)
    _check_plan(rng.integers(0, 257, n), 257, 8)


def test_plan_ragged_segments():
    """Empty experts, one expert with many rows, block boundaries at every
    remainder (fast_prefill tests' ragged segments, test_fast_prefill.py:60-78)."""
    ids = np.array([5] * 77 + [0] * 1 + [9] * 32 + [3] * 33 + [5] * 3 + [11] * 8 + [0] * 7, np.int64)
    np.random.default_rng(3).shuffle(ids)
    for block_rows in (8, 32):
        _check_plan(ids, 12, block_rows)


def test_plan_out_of_range_ids_sort_last():
    rng = np.random.default_rng(5)
    ids = rng.integers(0, 40, 5000)
    ids[rng.choice(5000, 37, replace=False)] = 40 + rng.integers(0, 1000, 37)
    _check_plan(ids, 40, 32)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_combine_matches_oracle(dtype):
    import torch

    from mlxlr8_b200.fast_router import combine

    rng = np.random.default_rng(17)
    tokens, h = 37, 6144
    td = torch_dtype(dtype)
    values = torch.from_numpy(rng.standard_normal((tokens, 9, h)).astype(np.float32)).cuda().to(td)
    scores = torch.from_numpy(rng.uniform(0.0, 1.0, (tokens, 8)).astype(np.float32)).cuda()
    residual = torch.from_numpy(rng.standard_normal((tokens, h)).astype(np.float32)).cuda().to(td)
    out = combine(values, scores, residual)
    torch.cuda.synchronize()
    expected = ref.combine(host(values), host(scores), host(residual), dtype)
    np.testing.assert_array_equal(host(out), expected)
