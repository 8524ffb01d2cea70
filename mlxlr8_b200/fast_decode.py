"""Selected-expert MLP for small batches (mirror of ``exlr8/fast_decode.py``).

``fast_expert_mlp`` / ``fast_expert_linear`` / ``compiled_expert_mlp_finish``
keep the reference's names and argument meaning.  The CUDA path decodes each
trellis tile once per expert and shares it across every row routed to that
expert, so ``reuse`` (the reference's 2-4 row tile sharing) is always on and
the flag is accepted for compatibility.  ``packed`` and ``scales`` are the
``ExpertLayer`` dictionaries: ``packed[p]`` uint8 bytes and
``scales[p] = (in_scale [E, in], out_scale [E, out])`` for p in gate/up/down.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .trellis import _ids, _nbytes, _words, check_format, expert_linear


def trellis_experts(packed, scales, k, hidden, intermediate):
    """Validate the expert dictionaries and build the C ``exlr8_trellis_experts``."""
    st = _lib.TrellisExperts()
    count = None
    dtype = scales["gate"][0].dtype
    keep = []
    for p, name in enumerate(("gate", "up", "down")):
        a, b, side = (intermediate, hidden, 2) if name == "down" else (hidden, intermediate, 1)
        buf = _words(packed[name])
        experts = check_format(buf, k, a, b, side)
        in_s, out_s = scales[name]
        if tuple(in_s.shape) != (experts, a) or tuple(out_s.shape) != (experts, b):
            raise ValueError("expert side vectors must contain full signed channel scales")
        if count is not None and experts != count:
            raise ValueError("packed byte count does not match the trellis dimensions")
        count = experts
        in_s = in_s.to(dtype).contiguous()
        out_s = out_s.to(dtype).contiguous()
        keep += [buf, in_s, out_s]
        st.packed[p] = buf.data_ptr()
        st.packed_bytes[p] = _nbytes(buf)
        st.in_scale[p] = in_s.data_ptr()
        st.out_scale[p] = out_s.data_ptr()
    st.scale_dtype = _lib.scale_code(scales["gate"][0])
    st.scale_experts = count
    st.k, st.hidden, st.intermediate = k, hidden, intermediate
    st._keep = keep  # keep the contiguous copies alive with the struct
    return st, count


def dense_expert(shared):
    """C ``exlr8_dense_expert`` for a (gate, up, down) bf16 triple, or None."""
    if shared is None:
        return None, []
    gate, up, down = (t.to(torch.bfloat16).contiguous() for t in shared)
    st = _lib.DenseExpert(gate.data_ptr(), up.data_ptr(), down.data_ptr())
    return st, [gate, up, down]


def fast_expert_linear(x, indices, packed, in_scale, out_scale, k, in_features, out_features, sharded_side=1):
    """Exact EXLR8 matrix applied to each selected expert row (fast_decode.py:153-165)."""
    return expert_linear(x, indices, packed, in_scale, out_scale, k, in_features, out_features, sharded_side)


def fast_expert_mlp(x, indices, packed, scales, k, hidden, intermediate, *, reuse=False, fp8=None,
                    expert_to_slot=None, workspace=None):
    """Gate/up, typed SwiGLU, down for every slot; ``[*indices.shape, hidden]``.

    Mirrors ``fast_expert_mlp`` (fast_decode.py:208-221).  ``fp8`` (cached
    gate/up/down E4M3 bytes in tile order, ``static_cache.StaticExpertCache``)
    and ``expert_to_slot`` (uint32 or int32 [experts], 0xFFFFFFFF = not cached)
    make the streaming decode read the cached experts' bytes instead of
    decoding their codes; the outputs are bit-equal either way, as the
    reference requires of the cache.  An optional uint8 ``workspace`` tensor is
    used instead of a fresh one when it is large enough (its dispatch header
    stays readable after the call).
    """
    if (fp8 is None) != (expert_to_slot is None):
        raise ValueError("fp8 bytes and expert_to_slot go together")
    if fp8 is not None and set(fp8) != {"gate", "up", "down"}:
        raise ValueError("fp8 must hold gate, up and down bytes")
    device = _lib.require_cuda(x, indices)
    if x.shape[-1] != hidden:
        raise ValueError("activation width does not match in_features")
    if x.shape[:-1] == indices.shape:
        per_slot = 1
    elif x.shape[:-1] == indices.shape[:-1]:
        per_slot = 0
    else:
        raise ValueError("activation rows do not match the expert indices")
    st, experts = trellis_experts(packed, scales, k, hidden, intermediate)
    ids = _ids(indices)
    slots = indices.shape[-1]
    tokens = ids.numel() // slots
    x = x.contiguous()
    out = torch.empty(tuple(indices.shape) + (hidden,), dtype=x.dtype, device=device)
    lib = _lib.lib()
    need = lib.exlr8_expert_mlp_workspace(tokens, slots, hidden, intermediate, experts)
    ws = workspace if workspace is not None and workspace.numel() >= need else _lib.workspace(need, device)
    if fp8 is None:
        _lib.check(lib.exlr8_expert_mlp(x.data_ptr(), _lib.act_code(x), per_slot, ids.data_ptr(), tokens, slots,
                                        st, out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle(device)))
        return out
    slot_map = _ids(expert_to_slot.reshape(-1))
    if slot_map.numel() != experts:
        raise ValueError("expert_to_slot needs one entry per expert")
    size = hidden * intermediate
    cache = _lib.StaticCache()
    counts = set()
    for i, p in enumerate(("gate", "up", "down")):
        b = fp8[p].reshape(-1)
        if b.dtype != torch.uint8 or b.device != device or b.numel() % size or not b.is_contiguous():
            raise ValueError("fp8 bytes must be contiguous uint8 with hidden * intermediate bytes per slot")
        counts.add(b.numel() // size)
        cache.fp8[i] = b.data_ptr()
    if len(counts) != 1:
        raise ValueError("fp8 gate, up and down must hold the same slots")
    cache.expert_to_slot = slot_map.data_ptr()
    cache.slots = counts.pop()
    _lib.check(lib.exlr8_expert_mlp_cached(x.data_ptr(), _lib.act_code(x), per_slot, ids.data_ptr(), tokens, slots,
                                           st, ctypes.byref(cache), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                           _lib.stream_handle(device)))
    return out


def expert_mlp_finish(x, indices, scores, residual, packed, scales, k, hidden, intermediate, shared=None):
    """Nine-slot MLP plus the routed/shared/residual sum (fast_decode.py:237-242)."""
    device = _lib.require_cuda(x, indices, scores, residual)
    rows = x.numel() // hidden
    st, experts = trellis_experts(packed, scales, k, hidden, intermediate)
    sh, keep = dense_expert(shared)
    ids = _ids(indices).reshape(rows, 9)
    sc = scores.to(torch.float32).contiguous().reshape(rows, 8)
    xr = x.contiguous().reshape(rows, hidden)
    res = residual.to(x.dtype).contiguous().reshape(rows, hidden)
    out = torch.empty_like(res)
    lib = _lib.lib()
    ws = _lib.workspace(lib.exlr8_expert_mlp_finish_workspace(rows, hidden, intermediate, experts), device)
    _lib.check(lib.exlr8_expert_mlp_finish(xr.data_ptr(), _lib.act_code(xr), ids.data_ptr(), sc.data_ptr(),
                                           res.data_ptr(), rows, st, sh, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                           _lib.stream_handle(device)))
    return out.reshape(residual.shape)


def compiled_expert_mlp_finish(expert):
    """Return ``apply(x, indices, scores, residual)`` (fast_decode.py:224-244).

    ``expert`` provides ``hidden``, ``intermediate``, ``packed``, ``scales`` and
    optionally ``k`` (default 4) and ``shared`` (a dense bf16 triple).  A
    joined MXFP4 expert (``expert.affine``) returns its own ``finish``.
    """
    affine = getattr(expert, "affine", None)
    if affine is not None:
        return affine.finish
    k = getattr(expert, "k", 4)
    shared = getattr(expert, "shared", None)

    def apply(x, indices, scores, residual):
        return expert_mlp_finish(x, indices, scores, residual, expert.packed, expert.scales, k, expert.hidden,
                                 expert.intermediate, shared)

    return apply
