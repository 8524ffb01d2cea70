"""C-ABI library: loads on a CPU-only machine, exports every declared symbol,
and its host-side format checks raise the reference's errors."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from mlxlr8_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "exlr8_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(exlr8_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIBRARY))
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.EXPORTED)


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.exlr8_abi_version() == 1
    assert lib.exlr8_status_string(4).decode() == "packed byte count does not match the trellis dimensions"
    assert lib.exlr8_status_string(13).decode() == "Expert IDs must be in 0..256"


@pytest.mark.parametrize("args, message", [
    ((4, 4, 128, 128, 1), "byte count"),
    ((8192, 5, 128, 128, 1), "width must be 2, 3, or 4"),
    ((8192, 4, 100, 128, 1), "multiples of 128"),
    ((8192, 4, 128, 128, 3), "sharded_side"),
])
def test_format_errors_match_reference(args, message):
    from mlxlr8_b200.trellis import check_format

    nbytes, k, a, b, side = args
    with pytest.raises(ValueError, match=message):
        check_format(np_bytes(nbytes), k, a, b, side)


def np_bytes(n):
    import torch

    return torch.zeros(n, dtype=torch.uint8)


def test_format_counts_matrices():
    from mlxlr8_b200.trellis import check_format

    assert check_format(np_bytes(3 * 128 * 256 // 2), 4, 128, 256, 1) == 3
    assert check_format(np_bytes(2 * 128 * 256 * 3 // 8), 3, 256, 128, 2) == 2


def test_operators_fail_loudly_without_cuda(monkeypatch):
    import torch
    from mlxlr8_b200 import trellis

    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        trellis.mcg_codebook()


def _bad_struct(hidden=6144, intermediate=64, experts=257):
    """An expert struct whose dimensions no call accepts (intermediate 64)."""
    st = _lib.TrellisExperts()
    for i in range(3):
        st.packed[i] = 16
        st.packed_bytes[i] = experts * hidden * intermediate // 2
        st.in_scale[i] = 16
        st.out_scale[i] = 16
    st.scale_dtype = 1
    st.scale_experts = experts
    st.k = 4
    st.hidden = hidden
    st.intermediate = intermediate
    return st


@pytest.mark.parametrize("query, args", [
    ("exlr8_moe_layer_workspace", (1, 6144, 64, 257)),
    ("exlr8_moe_layer_workspace", (1, 100, 2048, 257)),
    ("exlr8_moe_layer_workspace", (-1, 6144, 2048, 257)),
    ("exlr8_expert_mlp_finish_workspace", (1, 6144, 0, 257)),
    ("exlr8_expert_mlp_workspace", (1, 9, 6144, 64, 257)),
    ("exlr8_expert_mlp_workspace", (1, 0, 6144, 2048, 257)),
    ("exlr8_expert_linear_workspace", (1, 9, 6144, 64, 257)),
    ("exlr8_shared_expert_workspace", (1, 6144, 64)),
    ("exlr8_joined_moe_layer_workspace", (1, 6144, 64, 257)),
    ("exlr8_dispatch_plan_workspace", (-1, 257)),
    ("exlr8_dispatch_plan_workspace", (36864, 0)),
    ("exlr8_dispatch_plan_workspace", (36864, 2048)),
])
def test_workspace_queries_reject_unusable_sizes(query, args):
    """Sizes no call accepts answer SIZE_MAX instead of dividing by a zero
    split count (the process used to die with SIGFPE)."""
    value = getattr(_lib.load(), query)(*args)
    assert value == ctypes.c_size_t(-1).value


def test_noalloc_rejects_a_bad_struct_before_sizing():
    """A malformed expert struct gets the same status as exlr8_moe_layer
    (trellis dimensions not multiples of 128), checked on the host before
    any size is derived from it, so no GPU is needed."""
    lib = _lib.load()
    st = _bad_struct()
    status = lib.exlr8_moe_layer_noalloc(16, 2, 16, 1, 16, 16, ctypes.byref(st), None, 16, None, None, None)
    assert status == 2
    assert lib.exlr8_status_string(status).decode() == "trellis dimensions must be positive multiples of 128"
    assert lib.exlr8_moe_layer_noalloc(16, 2, 16, 1, 16, 16, None, None, 16, None, None, None) == 11
    good = _bad_struct(hidden=256, intermediate=128)
    good.scale_experts = 3
    assert lib.exlr8_moe_layer_noalloc(16, 2, 16, 1, 16, 16, ctypes.byref(good), None, 16, None, None, None) == 5


def test_gemm_pair_switch_round_trips():
    """The SM-pair GEMM switch is host state: set, read back, restored."""
    lib = _lib.lib()
    previous = lib.exlr8_gemm_pair(0)
    try:
        assert previous == 1
        assert lib.exlr8_gemm_pair(-1) == 0
        assert lib.exlr8_gemm_pair(1) == 0
        assert lib.exlr8_gemm_pair(-1) == 1
    finally:
        lib.exlr8_gemm_pair(previous)


def test_dispatch_plan_and_combine_reject_bad_arguments_without_a_gpu():
    """Argument checks run before any device work: a table narrower than the
    reference's width, a block size of zero and an unknown dtype."""
    lib = _lib.lib()
    ws = lib.exlr8_dispatch_plan_workspace(100, 257)
    assert 0 < ws < ctypes.c_size_t(-1).value
    buf = ctypes.create_string_buffer(16)
    p = ctypes.addressof(buf)
    # width min(100, 100 // 8 + 257) = 100 columns; one fewer is refused
    narrow = lib.exlr8_dispatch_plan(p, 100, 257, 8, p, p, p, 99, p, p, ws, None)
    assert narrow != 0 and "argument" in lib.exlr8_status_string(narrow).decode().lower()
    assert lib.exlr8_dispatch_plan(p, 100, 257, 0, p, p, p, 100, p, p, ws, None) == narrow
    assert lib.exlr8_combine(p, p, p, 1, 128, 99, p, None) != 0


def test_host_buffer_entries_reject_bad_arguments_without_a_gpu():
    """exlr8_stage_in / exlr8_host_device_pointer check sizes, nulls and
    alignment before any CUDA call (codes EXLR8_ERR_ARG = 11, EXLR8_ERR_ALIGN
    = 9)."""
    lib = _lib.lib()
    out = ctypes.c_void_p(0)
    assert lib.exlr8_host_device_pointer(None, ctypes.byref(out)) == 11
    assert lib.exlr8_host_device_pointer(4096, None) == 11
    assert lib.exlr8_stage_in(4096, 8192, 12288, 16384, 0, None) == 0
    assert lib.exlr8_stage_in(4096, 8192, 12288, 16384, 24, None) == 11
    assert lib.exlr8_stage_in(4096, 8192, 12288, 16384, -16, None) == 11
    assert lib.exlr8_stage_in(None, 8192, 12288, 16384, 16, None) == 11
    assert lib.exlr8_stage_in(4096, 8192, 12288, 16392, 16, None) == 9
