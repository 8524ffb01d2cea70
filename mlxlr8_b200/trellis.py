"""Trellis codec and selected-expert operators (mirror of ``exlr8/trellis.py``).

Same function names, argument order and meaning as the reference module,
with torch CUDA tensors in place of MLX arrays.  ``packed`` buffers are the
EXLR8 "grouped128" bytes as stored in the checkpoint (uint8, contiguous);
side vectors are float16 or float32.  Every operator runs on the GPU through
``libexlr8_b200.so``; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def check_format(packed: torch.Tensor, k: int, in_features: int, out_features: int, sharded_side: int) -> int:
    """Number of matrices in ``packed`` (exlr8/trellis.py:53-64 ``_check_format``).

    Raises ``ValueError`` with the reference's messages.
    """
    count = ctypes.c_int64(0)
    _lib.check(_lib.lib().exlr8_check_format(_nbytes(packed), k, in_features, out_features, sharded_side,
                                             ctypes.byref(count)))
    return int(count.value)


def _words(packed: torch.Tensor) -> torch.Tensor:
    if packed.dtype != torch.uint8:
        packed = packed.view(torch.uint8) if packed.is_contiguous() else packed.contiguous().view(torch.uint8)
    return packed.contiguous()


def _ids(indices: torch.Tensor) -> torch.Tensor:
    if indices.dtype == torch.uint32:
        indices = indices.contiguous().view(torch.int32)
    elif indices.dtype != torch.int32:
        indices = indices.to(torch.int32)
    return indices.contiguous()


def _hadamard(x: torch.Tensor) -> torch.Tensor:
    """Normalised Hadamard transform of each 128-value block of the last axis
    (exlr8/trellis.py:134-137 ``_hadamard``), computed in float32 on the GPU."""
    device = _lib.require_cuda(x)
    features = x.shape[-1]
    if features % 128:
        raise ValueError("trellis dimensions must be positive multiples of 128")
    rows = x.numel() // features if features else 0
    src = x.to(torch.float32).contiguous()
    out = torch.empty_like(src)
    _lib.check(_lib.lib().exlr8_hadamard128(src.data_ptr(), rows, features, out.data_ptr(),
                                            _lib.stream_handle(device)))
    return out


def mcg_codebook(device=None, paired: bool = False) -> torch.Tensor:
    """All 65,536 codeword values as float16, evaluated by the CUDA decoder.

    Mirrors ``mcg_codebook`` (exlr8/trellis.py:43-50); ``paired`` selects the
    two-codeword vector path used inside the GEMV kernels.
    """
    device = torch.device(device) if device is not None else _lib.require_cuda()
    states = torch.arange(1 << 16, dtype=torch.int32, device=device)
    values = torch.empty(1 << 16, dtype=torch.float32, device=device)
    _lib.check(_lib.lib().exlr8_codebook(states.data_ptr(), values.data_ptr(), states.numel(), int(paired),
                                         _lib.stream_handle(device)))
    return values.to(torch.float16)


def decode_trellis(packed: torch.Tensor, k: int, in_features: int, out_features: int, sharded_side: int = 1,
                   matrix: int = 0) -> torch.Tensor:
    """Inner weights float32 [in, out] of matrix ``matrix`` (metal/decode.metal)."""
    device = _lib.require_cuda(packed)
    packed = _words(packed)
    inner = torch.empty(in_features, out_features, dtype=torch.float32, device=device)
    _lib.check(_lib.lib().exlr8_decode_trellis(packed.data_ptr(), _nbytes(packed), matrix, k, in_features,
                                               out_features, sharded_side, inner.data_ptr(),
                                               _lib.stream_handle(device)))
    return inner


def dequantize_trellis(packed, suh, svh, k, in_features, out_features, sharded_side=1) -> torch.Tensor:
    """Public dense matrix float32 [out, in] (exlr8/trellis.py:199-214)."""
    device = _lib.require_cuda(packed, suh, svh)
    packed = _words(packed)
    if check_format(packed, k, in_features, out_features, sharded_side) != 1:
        raise ValueError("dense dequantization requires one matrix")
    suh = suh.contiguous()
    svh = svh.to(suh.dtype).contiguous()
    weight = torch.empty(out_features, in_features, dtype=torch.float32, device=device)
    lib = _lib.lib()
    ws = _lib.workspace(lib.exlr8_dequantize_trellis_workspace(in_features, out_features), device)
    _lib.check(lib.exlr8_dequantize_trellis(packed.data_ptr(), _nbytes(packed), suh.data_ptr(), svh.data_ptr(),
                                            _lib.scale_code(suh), k, in_features, out_features, sharded_side,
                                            weight.data_ptr(), ws.data_ptr(), ws.numel(),
                                            _lib.stream_handle(device)))
    return weight


def expert_linear(x, indices, packed, in_scale, out_scale, k, in_features, out_features, sharded_side=1):
    """Apply selected experts; return ``[*indices.shape, out_features]``.

    Mirrors ``expert_linear`` (exlr8/trellis.py:172-196): ``x`` has one row
    per token (``x.shape[:-1] == indices.shape[:-1]``) or one row per expert
    slot (``x.shape[:-1] == indices.shape``); side vectors are
    ``[experts, in]`` and ``[experts, out]`` with signs included.  The output
    has the activation dtype.
    """
    device = _lib.require_cuda(x, indices, packed, in_scale, out_scale)
    packed = _words(packed)
    experts = check_format(packed, k, in_features, out_features, sharded_side)
    if x.shape[-1] != in_features:
        raise ValueError("activation width does not match in_features")
    if tuple(in_scale.shape) != (experts, in_features) or tuple(out_scale.shape) != (experts, out_features):
        raise ValueError("expert side vectors must contain full signed channel scales")
    if x.shape[:-1] == indices.shape:
        per_slot = 1
    elif x.shape[:-1] == indices.shape[:-1]:
        per_slot = 0
    else:
        raise ValueError("activation rows do not match the expert indices")
    ids = _ids(indices)
    slots = indices.shape[-1] if indices.dim() else 1
    tokens = ids.numel() // max(slots, 1)
    x = x.contiguous()
    in_scale = in_scale.contiguous()
    out_scale = out_scale.to(in_scale.dtype).contiguous()
    out = torch.empty(tuple(indices.shape) + (out_features,), dtype=x.dtype, device=device)
    lib = _lib.lib()
    ws = _lib.workspace(lib.exlr8_expert_linear_workspace(tokens, slots, in_features, out_features, experts), device)
    _lib.check(lib.exlr8_expert_linear(x.data_ptr(), _lib.act_code(x), per_slot, ids.data_ptr(), tokens, slots,
                                       packed.data_ptr(), _nbytes(packed), in_scale.data_ptr(), out_scale.data_ptr(),
                                       _lib.scale_code(in_scale), experts, k, in_features, out_features, sharded_side,
                                       out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle(device)))
    return out


def trellis_linear(x, packed, suh, svh, k, in_features, out_features, sharded_side=1):
    """Dense stored trellis matrix applied without decoded weights (trellis.py:157-169)."""
    packed = _words(packed)
    if check_format(packed, k, in_features, out_features, sharded_side) != 1:
        raise ValueError("dense trellis requires one matrix")
    if x.shape[-1] != in_features or suh.numel() != in_features or svh.numel() != out_features:
        raise ValueError("activation or side vector dimensions do not match")
    rows = x.numel() // in_features
    ids = torch.zeros(rows, 1, dtype=torch.int32, device=x.device)
    y = expert_linear(x.reshape(rows, in_features), ids, packed, suh.reshape(1, -1), svh.reshape(1, -1), k,
                      in_features, out_features, sharded_side)
    return y.reshape(tuple(x.shape[:-1]) + (out_features,))
