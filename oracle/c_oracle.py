"""ctypes binding of the C oracle ``oracle/c/liboracle.so`` (TEST INFRASTRUCTURE ONLY).

Faster CPU checker and CPU baseline for the routed-MoE layer; pinned to the
NumPy oracle by ``tests/test_c_oracle.py``.  Build with ``make -C oracle/c``.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int64, c_uint16, c_uint32, c_void_p
from functools import lru_cache
from pathlib import Path

import numpy as np

from . import trellis_oracle as ref

LIBRARY = Path(__file__).resolve().parent / "c" / "liboracle.so"
DTYPE = {"float32": 0, "float16": 1, "bfloat16": 2}


@lru_cache(maxsize=1)
def lib():
    if not LIBRARY.exists():
        raise RuntimeError("C oracle not built: run `make -C oracle/c`")
    so = ctypes.CDLL(str(LIBRARY))
    so.oracle_expert_mlp_rows.restype = c_int
    so.oracle_expert_mlp_rows.argtypes = [c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p, POINTER(c_void_p),
                                          POINTER(c_void_p), c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]
    so.oracle_moe_layer.restype = c_int
    so.oracle_moe_layer.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    POINTER(c_void_p), POINTER(c_void_p), c_int, c_int, c_int, c_int, c_void_p,
                                    c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
    so.oracle_threads.restype = c_int
    return so


@lru_cache(maxsize=1)
def codebook_f32():
    return np.ascontiguousarray(ref.mcg_codebook().astype(np.float32))


def _p(a):
    return a.ctypes.data_as(c_void_p)


def _scale_arrays(scales):
    keep = []
    dtype = None
    ins, outs = [], []
    for p in ("gate", "up", "down"):
        a, b = scales[p]
        a = np.ascontiguousarray(a)
        b = np.ascontiguousarray(b)
        dtype = a.dtype
        keep += [a, b]
        ins.append(a.ctypes.data)
        outs.append(b.ctypes.data)
    code = 0 if dtype == np.float32 else 1
    return (c_void_p * 3)(*ins), (c_void_p * 3)(*outs), code, keep


def threads():
    return lib().oracle_threads()


def expert_mlp_rows(x, expert, packed, scales, k, hidden, intermediate, dtype="float32"):
    """Fused MLP of rows that all use `expert` (fast_decode.py:168-205 order)."""
    x = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, hidden))
    out = np.empty_like(x)
    ins, outs, code, keep = _scale_arrays(scales)
    words = [np.ascontiguousarray(packed[p]).view(np.uint32) for p in ("gate", "up", "down")]
    st = lib().oracle_expert_mlp_rows(_p(x), x.shape[0], int(expert), _p(words[0]), _p(words[1]), _p(words[2]), ins,
                                      outs, code, k, hidden, intermediate, DTYPE[dtype], _p(codebook_f32()), _p(out))
    if st:
        raise ValueError("C oracle rejected the arguments")
    return out


def moe_layer(x, residual, gate_weight, bias, packed, scales, k, hidden, intermediate, shared=None, dtype="bfloat16",
              logits=None):
    """Whole MoE layer (model.py:385-418); ``shared`` bf16 triple as uint16 bit arrays or None.
    ``logits`` [tokens][256] float32, if given, replaces the oracle's own gate product."""
    x = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, hidden))
    residual = np.ascontiguousarray(np.asarray(residual, np.float32).reshape(-1, hidden))
    tokens = x.shape[0]
    out = np.empty_like(x)
    ids = np.empty((tokens, 9), np.uint32)
    scores = np.empty((tokens, 8), np.float32)
    ins, outs, code, keep = _scale_arrays(scales)
    words = [np.ascontiguousarray(packed[p]).view(np.uint32) for p in ("gate", "up", "down")]
    wg = np.ascontiguousarray(gate_weight, np.float32)
    b = np.ascontiguousarray(bias, np.float32)
    sh = [None, None, None] if shared is None else [np.ascontiguousarray(s, np.uint16) for s in shared]
    lg = None if logits is None else np.ascontiguousarray(np.asarray(logits, np.float32).reshape(tokens, 256))
    st = lib().oracle_moe_layer(_p(x), _p(residual), tokens, _p(wg), _p(b), _p(words[0]), _p(words[1]), _p(words[2]),
                                ins, outs, code, k, hidden, intermediate,
                                None if sh[0] is None else _p(sh[0]), None if sh[1] is None else _p(sh[1]),
                                None if sh[2] is None else _p(sh[2]), DTYPE[dtype], _p(codebook_f32()), _p(out),
                                _p(ids), _p(scores), None if lg is None else _p(lg))
    if st:
        raise ValueError("C oracle rejected the arguments")
    return out, ids, scores
