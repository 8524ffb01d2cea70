"""A stack of MoE decoder blocks with the attention stubbed (exlr8 model.py:373-418).

Each block of the reference decoder layer is

    r, _ = self_attn(rms_norm(x, input_norm))       (stubbed: r = 0)
    h = x + r
    x = rms_norm(h, post_norm, eps)                  exlr8_residual_rms_norm
    return h + moe(x)                                the MoE layer, residual h

so with the attention stubbed the stack threads the hidden state through
``rms_norm`` and one MoE layer per block: ``MoELayer`` (one GPU, resident
trellis experts), ``JoinedMoELayer`` (MXFP4) or ``ExpertParallelMoE``
(experts sharded over the node's GPUs).  The reference model runs layers
3-77 this way (the first three are dense) plus the layer-78 block whose
experts are K3; any callable ``layer(x, residual) -> h + moe(x)`` fits.
"""

from __future__ import annotations

import torch

from . import _lib


def residual_rms_norm(x, weight, eps: float = 1e-5, residual=None, return_sum: bool = False):
    """``rms_norm(x + residual, weight, eps)`` in x's dtype
    (model.py:383-384; fast_norm.residual_rms_pair).  With ``return_sum`` the
    rounded sum ``h`` is returned as well."""
    device = _lib.require_cuda(x)
    hidden = x.shape[-1]
    if weight.shape != (hidden,):
        raise ValueError("norm weight must have one entry per hidden channel")
    x = x.contiguous()
    rows = x.numel() // hidden
    w = weight.to(x.dtype).contiguous()
    out = torch.empty_like(x)
    h = torch.empty_like(x) if return_sum else None
    res = residual.to(x.dtype).contiguous() if residual is not None else None
    _lib.check(_lib.lib().exlr8_residual_rms_norm(x.data_ptr(), res.data_ptr() if res is not None else None,
                                                  w.data_ptr(), _lib.act_code(x), rows, hidden, float(eps),
                                                  h.data_ptr() if h is not None else None, out.data_ptr(),
                                                  _lib.stream_handle(device)))
    return (h, out) if return_sum else out


class MoEStack:
    """Blocks of (post-attention norm weight [hidden], MoE layer) applied in
    order to the hidden state [tokens, hidden]."""

    def __init__(self, blocks, eps: float = 1e-5):
        self.blocks = [(w, layer) for w, layer in blocks]
        self.eps = eps

    def __len__(self):
        return len(self.blocks)

    def __call__(self, h, trace: bool = False):
        """The hidden state after every block; with ``trace`` also the list of
        (block input, normalised input, block output) per block."""
        steps = []
        for w, layer in self.blocks:
            xn = residual_rms_norm(h, w, self.eps)
            out = layer(xn, h)
            if trace:
                steps.append((h, xn, out))
            h = out
        return (h, steps) if trace else h
