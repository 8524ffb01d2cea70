"""NumPy restatement of the exlr8 routed-MoE arithmetic (TEST INFRASTRUCTURE ONLY).

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this
module; it is the checker, never the product.  Every function names the
reference line (package ``exlr8`` v0.1.21, paths relative to the reference
project root) whose arithmetic it restates.

Parity status: the codec functions (``round_e4m3``, ``mcg_codebook``,
``hadamard128``, ``decode_trellis``, ``dequantize``) are pinned bit-exact
against vectors produced by the reference's own NumPy functions
(``tests/golden/make_golden.py``).  The operator compositions (expert linear,
typed SwiGLU, router, combine, joined MXFP4) restate Metal/MLX code that cannot
run on this machine; they are pinned by the reference's own test formulas
(cited per function) and by the golden vectors computed with those formulas.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np

F32 = np.float32
DTYPES = ("float32", "float16", "bfloat16")


# ---------------------------------------------------------------------------
# Typed rounding helpers (emulate T(...) casts of the Metal kernels)
# ---------------------------------------------------------------------------

def round_bf16(values):
    """Round float32 values to bfloat16 (nearest, ties to even); return float32."""
    a = np.ascontiguousarray(np.asarray(values, dtype=F32))
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(F32)
    return np.where(np.isnan(a), a, out).astype(F32)


def round_f16(values):
    return np.asarray(values, dtype=F32).astype(np.float16).astype(F32)


def rounder(dtype):
    if dtype == "float32":
        return lambda v: np.asarray(v, dtype=F32)
    if dtype == "float16":
        return round_f16
    if dtype == "bfloat16":
        return round_bf16
    raise ValueError(f"unsupported dtype {dtype}")


def bf16_bits(values):
    """float32 values that are exact bfloat16 -> uint16 bit patterns."""
    return (np.asarray(round_bf16(values)).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits):
    return (np.asarray(bits, dtype=np.uint32) << 16).view(F32)


# ---------------------------------------------------------------------------
# Trellis codec: exlr8/trellis.py:22-109, metal/fast_decode_common.metal:4-38
# ---------------------------------------------------------------------------

def e4m3_levels():
    """The 127 non-negative finite E4M3 magnitudes, ascending (trellis.py:24-30)."""
    code = np.arange(127, dtype=np.int64)
    exponent, mantissa = code >> 3, code & 7
    subnormal = mantissa * 2.0 ** -9
    normal = (8 + mantissa) * np.exp2(exponent - 10.0)
    return np.where(exponent == 0, subnormal, normal).astype(F32)


def round_e4m3(values):
    """Nearest finite E4M3 value, ties to the even code, saturating at 448.

    Restates ``round_e4m3`` (trellis.py:22-40): the magnitude is clipped to 448,
    the two neighbouring levels are compared, and an exact tie picks the level
    whose code (index) is even.  The sign is copied back, so -0.0 stays -0.0.
    """
    values = np.asarray(values, dtype=F32)
    levels = e4m3_levels()
    mag = np.minimum(np.abs(values), F32(448.0))
    hi = np.clip(np.searchsorted(levels, mag), 0, 126)
    lo = np.maximum(hi - 1, 0)
    d_hi = levels[hi] - mag
    d_lo = mag - levels[lo]
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    return np.copysign(np.where(pick_hi, levels[hi], levels[lo]), values).astype(F32)


MCG_MULTIPLIER = 0xCBAC1FED
MCG_MASK = 0x8FFF8FFF
MCG_XOR = 0x3B603B60


@lru_cache(maxsize=1)
def mcg_codebook():
    """Value of every 16-bit trellis state as float16 (trellis.py:43-50).

    The state is multiplied by 0xCBAC1FED (mod 2^32), masked with 0x8FFF8FFF,
    xor-ed with 0x3B603B60; the two 16-bit halves are float16 numbers whose
    float16 sum, rounded to E4M3, is the weight value.
    """
    state = np.arange(1 << 16, dtype=np.uint64)
    word = ((state * MCG_MULTIPLIER) & 0xFFFFFFFF) & MCG_MASK ^ MCG_XOR
    word = word.astype(np.uint32)
    low = (word & 0xFFFF).astype(np.uint16).view(np.float16)
    high = (word >> 16).astype(np.uint16).view(np.float16)
    total = (low + high).astype(np.float16)  # one float16 rounding of the exact sum
    return round_e4m3(total.astype(F32)).astype(np.float16)


def hadamard128(x):
    """Normalised Sylvester transform in independent 128-channel blocks.

    Restates ``hadamard_reference`` (trellis.py:67-75): butterfly stages over
    index bits 1, 2, 4, ..., 64 in that order (a+b, a-b), then a multiply by
    float32(1/sqrt(128)).  The CUDA kernels use the same stage order, so the
    two agree bit for bit.
    """
    x = np.asarray(x, dtype=F32)
    y = x.reshape(-1, 128).copy()
    for bit in (1, 2, 4, 8, 16, 32, 64):
        v = y.reshape(-1, 128 // (2 * bit), 2, bit)
        a = v[:, :, 0, :].copy()
        b = v[:, :, 1, :].copy()
        v[:, :, 0, :] = a + b
        v[:, :, 1, :] = a - b
    return (y * F32(1.0 / math.sqrt(128.0))).reshape(x.shape)


def check_format(nbytes, k, in_features, out_features, sharded_side):
    """Validate a packed trellis buffer; return the matrix count (trellis.py:53-64)."""
    if k not in (2, 3, 4):
        raise ValueError("EXLR8 trellis width must be 2, 3, or 4")
    if in_features <= 0 or out_features <= 0 or in_features % 128 or out_features % 128:
        raise ValueError("trellis dimensions must be positive multiples of 128")
    if sharded_side not in (0, 1, 2):
        raise ValueError("sharded_side must be 0, 1, or 2")
    size = in_features * out_features * k // 8
    if nbytes == 0 or nbytes % size:
        raise ValueError("packed byte count does not match the trellis dimensions")
    return nbytes // size


def tile_index(expert, tk, tn, in_tiles, out_tiles, side):
    """Storage index of the 16x16 tile (tk, tn) of one expert.

    Side 1 (and 0) stores 128-column output blocks first, side 2 stores
    128-row input blocks first; inside a 128x128 block the input tile precedes
    the output tile (fast_decode_linear.metal:91-95, trellis.py:84-89).
    """
    e = np.asarray(expert, dtype=np.int64)
    tk = np.asarray(tk, dtype=np.int64)
    tn = np.asarray(tn, dtype=np.int64)
    if side == 2:
        return (((e * (in_tiles // 8) + tk // 8) * (out_tiles // 8) + tn // 8) * 8 + tk % 8) * 8 + tn % 8
    return ((e * (out_tiles // 8) + tn // 8) * in_tiles + tk) * 8 + tn % 8


@lru_cache(maxsize=3)
def codeword_geometry(k):
    """Per codeword i of a tile: (left word, right word, shift, row, col).

    Codeword i is the 16-bit window that ends at bit (i+1)*k + 256*k of the
    cyclic tile bitstream (trellis.py:91-96, decode.metal:19-23); its place in
    the 16x16 tile follows the tensor-core permutation (trellis.py:97-99).
    """
    i = np.arange(256, dtype=np.int64)
    words = 8 * k
    end = (i + 1) * k + 256 * k
    last = (end - 1) // 32
    left = (last - 1) % words
    right = last % words
    shift = (last + 1) * 32 - end
    lane, slot = i // 8, i % 8
    row = (lane % 4) * 2 + (slot & 1) + (slot & 2) * 4
    col = lane // 4 + (slot & 4) * 2
    return left, right, shift, row, col


def decode_codewords(words, k):
    """words [..., 8k] uint32 tiles -> codewords [..., 256] in trellis order."""
    left, right, shift, _, _ = codeword_geometry(k)
    w = np.asarray(words, dtype=np.uint64)
    merged = (w[..., left] << np.uint64(32)) | w[..., right]
    return ((merged >> shift.astype(np.uint64)) & np.uint64(0xFFFF)).astype(np.uint16)


def decode_trellis(packed, k, in_features, out_features, sharded_side=1, expert=0):
    """Decode one stored matrix to its inner weights [in, out] (float16 values).

    Restates ``decode_trellis_reference`` (trellis.py:78-102) for matrix
    ``expert`` of a packed buffer that may hold several matrices.
    """
    raw = np.ascontiguousarray(np.asarray(packed)).view(np.uint8).reshape(-1)
    check_format(raw.size, k, in_features, out_features, sharded_side)
    it, ot = in_features // 16, out_features // 16
    words = raw.view(np.uint32).reshape(-1, 8 * k)
    tk, tn = np.meshgrid(np.arange(it), np.arange(ot), indexing="ij")
    tiles = words[tile_index(expert, tk, tn, it, ot, sharded_side)]  # [it, ot, 8k]
    values = mcg_codebook()[decode_codewords(tiles, k)]  # [it, ot, 256]
    _, _, _, row, col = codeword_geometry(k)
    inner = np.empty((it, ot, 16, 16), dtype=np.float16)
    inner[:, :, row, col] = values
    return inner.transpose(0, 2, 1, 3).reshape(in_features, out_features)


def dequantize(packed, suh, svh, k, in_features, out_features, sharded_side=1, expert=0):
    """Public matrix [out, in] with both transforms and side scales (trellis.py:105-109)."""
    inner = decode_trellis(packed, k, in_features, out_features, sharded_side, expert).astype(F32)
    weight = hadamard128(hadamard128(inner).T)
    return weight * np.asarray(svh, F32)[:, None] * np.asarray(suh, F32)[None, :]


class DecodedCache:
    """Memo of decoded inner matrices keyed by (buffer id, expert)."""

    def __init__(self):
        self._store = {}

    def get(self, packed, k, a, b, side, expert):
        key = (id(packed), int(expert), k, a, b, side)
        if key not in self._store:
            self._store[key] = decode_trellis(packed, k, a, b, side, int(expert)).astype(F32)
        return self._store[key]


# ---------------------------------------------------------------------------
# Operators
# ---------------------------------------------------------------------------

def e4m3_code(values):
    """E4M3 byte of float16 values that are already E4M3 numbers
    (static_cache.py:11-22): sign in bit 7; a float16 exponent field of 9 or
    more is a normal E4M3 number (exponent field minus 8, top three fraction
    bits); fields 6..8 are the E4M3 subnormals m * 2^-9; zero keeps its sign."""
    bits = np.asarray(values, dtype=np.float16).view(np.uint16).astype(np.uint32)
    field = (bits >> 10) & 31
    fraction = bits & 1023
    code = (bits >> 8) & 0x80
    normal = field >= 9
    code = np.where(normal, code | ((field - 8) << 3) | (fraction >> 7), code)
    sub = (field >= 6) & (field < 9)
    shift = np.where(sub, 16 - field, 0)
    code = np.where(sub, code | ((1024 + fraction) >> shift), code)
    return code.astype(np.uint8)


def expand_static(packed, k, in_features, out_features, sharded_side=1):
    """Exact E4M3 bytes of every stored tile, in storage order
    (static_cache.py:29-42): tile t of the packed buffer becomes 256 bytes at
    256 * t, byte p holding the E4M3 code of the tile's codeword p (codeword
    8 * lane + j of the trellis order)."""
    raw = np.ascontiguousarray(np.asarray(packed)).view(np.uint8).reshape(-1)
    check_format(raw.size, k, in_features, out_features, sharded_side)
    words = raw.view(np.uint32).reshape(-1, 8 * k)
    return e4m3_code(mcg_codebook())[decode_codewords(words, k)].reshape(-1)


def slot_rows(x, indices, features):
    """Broadcast one row per token to one row per slot (trellis.py:185-190)."""
    x = np.asarray(x, dtype=F32)
    indices = np.asarray(indices)
    if x.shape[-1] != features:
        raise ValueError("activation width does not match in_features")
    if x.shape[:-1] == indices.shape:
        return x.reshape(-1, features)
    if x.shape[:-1] == indices.shape[:-1]:
        return np.broadcast_to(x[..., None, :], indices.shape + (features,)).reshape(-1, features)
    raise ValueError("activation rows do not match the expert indices")


def expert_linear(x, indices, packed, in_scale, out_scale, k, in_features, out_features,
                  sharded_side=1, dtype="float32", cache=None):
    """Selected-expert trellis linear: ``T(H(H(x*in_s[e]) @ W_e) * out_s[e])``.

    Restates ``expert_linear`` (trellis.py:172-196): the signed input scale and
    the input transform in float32, a float32 dot with the exact decoded
    weights, the output transform, the signed output scale, then one cast to
    the activation type.  Returns float32 values exactly representable in
    ``dtype``, shaped ``indices.shape + (out_features,)``.
    """
    indices = np.asarray(indices)
    raw = np.ascontiguousarray(np.asarray(packed)).view(np.uint8).reshape(-1)
    experts = check_format(raw.size, k, in_features, out_features, sharded_side)
    in_scale = np.asarray(in_scale, F32)
    out_scale = np.asarray(out_scale, F32)
    if in_scale.shape != (experts, in_features) or out_scale.shape != (experts, out_features):
        raise ValueError("expert side vectors must contain full signed channel scales")
    rows = slot_rows(x, indices, in_features)
    ids = indices.reshape(-1).astype(np.int64)
    xh = hadamard128(rows * in_scale[ids])
    cache = cache or DecodedCache()
    inner = np.empty((ids.size, out_features), dtype=F32)
    for e in np.unique(ids):
        sel = np.nonzero(ids == e)[0]
        inner[sel] = xh[sel] @ cache.get(raw, k, in_features, out_features, sharded_side, e)
    y = hadamard128(inner) * out_scale[ids]
    return rounder(dtype)(y).reshape(indices.shape + (out_features,))


def swiglu_typed(gate, up, dtype):
    """Typed SwiGLU ``T(T(g*sigmoid(g))*u)`` (fast_decode_common.metal:40-49).

    For a 16-bit T every operation of MLX's typed sigmoid rounds to T:
    ``tail = T(1/T(1+T(exp(|g|))))`` and ``sigmoid = g<0 ? tail : T(1-tail)``.
    """
    r = rounder(dtype)
    g = r(gate)
    u = r(up)
    with np.errstate(over="ignore"):
        e = r(np.exp(np.abs(g)).astype(F32))
    tail = r(F32(1.0) / r(F32(1.0) + e))
    sig = np.where(g < 0, tail, r(F32(1.0) - tail))
    return r(r(g * sig) * u)


def expert_mlp(x, indices, packed, scales, k, hidden, intermediate, dtype="float32", cache=None):
    """Gate/up linear, typed SwiGLU, down linear (experts.py:176-188)."""
    cache = cache or DecodedCache()
    gate = expert_linear(x, indices, packed["gate"], *scales["gate"], k, hidden, intermediate, 1, dtype, cache)
    up = expert_linear(x, indices, packed["up"], *scales["up"], k, hidden, intermediate, 1, dtype, cache)
    hidden_rows = swiglu_typed(gate, up, dtype)
    return expert_linear(hidden_rows, indices, packed["down"], *scales["down"], k, intermediate, hidden, 2,
                         dtype, cache)


def expert_mlp_fused(x, indices, packed, scales, k, hidden, intermediate, dtype="float32", cache=None):
    """Fused decode MLP order (fast_decode.py:168-205).

    Differs from :func:`expert_mlp` only in that gate/up stay float32 until the
    typed SwiGLU (fast_decode_gate_finish.metal:14-25) and the SwiGLU output is
    scaled and transformed in float32 before the down projection.
    """
    cache = cache or DecodedCache()
    indices = np.asarray(indices)
    ids = indices.reshape(-1).astype(np.int64)
    rows = slot_rows(x, indices, hidden)
    r = rounder(dtype)
    g_in, g_out = (np.asarray(s, F32) for s in scales["gate"])
    u_in, u_out = (np.asarray(s, F32) for s in scales["up"])
    d_in, d_out = (np.asarray(s, F32) for s in scales["down"])
    gate_raw = np.ascontiguousarray(np.asarray(packed["gate"])).view(np.uint8).reshape(-1)
    up_raw = np.ascontiguousarray(np.asarray(packed["up"])).view(np.uint8).reshape(-1)
    down_raw = np.ascontiguousarray(np.asarray(packed["down"])).view(np.uint8).reshape(-1)
    xg = hadamard128(rows * g_in[ids])
    xu = hadamard128(rows * u_in[ids])
    gi = np.empty((ids.size, intermediate), F32)
    ui = np.empty((ids.size, intermediate), F32)
    for e in np.unique(ids):
        sel = np.nonzero(ids == e)[0]
        gi[sel] = xg[sel] @ cache.get(gate_raw, k, hidden, intermediate, 1, e)
        ui[sel] = xu[sel] @ cache.get(up_raw, k, hidden, intermediate, 1, e)
    g = hadamard128(gi) * g_out[ids]
    u = hadamard128(ui) * u_out[ids]
    act = swiglu_typed(g, u, dtype) * d_in[ids]
    dx = hadamard128(act)
    di = np.empty((ids.size, hidden), F32)
    for e in np.unique(ids):
        sel = np.nonzero(ids == e)[0]
        di[sel] = dx[sel] @ cache.get(down_raw, k, intermediate, hidden, 2, e)
    out = r(hadamard128(di) * d_out[ids])
    return out.reshape(indices.shape + (hidden,))


def sigmoid_f32(v):
    """``1/(1+exp(|v|))`` with a sign select, in float32 (fast_router.metal:8-9)."""
    v = np.asarray(v, F32)
    with np.errstate(over="ignore"):
        y = (F32(1.0) / (F32(1.0) + np.exp(np.abs(v)))).astype(F32)
    return np.where(v < 0, y, F32(1.0) - y).astype(F32)


def route(logits, bias, top_k=8, scale=2.5, shared_id=256):
    """Fused router semantics (fast_router.metal:1-42).

    Select the top ``top_k`` of ``sigmoid(l) + bias`` (highest first, lowest
    expert id on a tie), weight each by its sigmoid, divide by
    ``1e-20 + sum`` accumulated in rank order, multiply by 2.5, and append the
    shared expert id.  Returns ids ``[..., top_k+1]`` uint32 and scores
    ``[..., top_k]`` float32.
    """
    logits = np.asarray(logits, F32)
    shape = logits.shape[:-1]
    n = logits.shape[-1]
    flat = logits.reshape(-1, n)
    original = sigmoid_f32(flat)
    choice = (original + np.asarray(bias, F32)[None, :]).astype(F32)
    rows = flat.shape[0]
    ids = np.empty((rows, top_k + 1), np.uint32)
    scores = np.empty((rows, top_k), F32)
    for r in range(rows):
        c = choice[r].copy()
        selected = []
        for rank in range(top_k):
            best = int(np.argmax(c))  # argmax returns the lowest index among equal maxima
            ids[r, rank] = best
            selected.append(original[r, best])
            c[best] = -np.inf
        total = F32(1e-20)
        for s in selected:
            total = F32(total + s)
        for rank, s in enumerate(selected):
            scores[r, rank] = F32(F32(s / total) * F32(scale))
        ids[r, top_k] = shared_id
    return ids.reshape(shape + (top_k + 1,)), scores.reshape(shape + (top_k,))


def route_experts(logits, bias, top_k=8, n_group=1, topk_group=1, norm_topk_prob=True, scale=2.5):
    """Reference router ``route_experts`` (model.py:111-132).

    Returns ids sorted ascending (``argpartition`` leaves the order
    unspecified) and the matching weights.
    """
    logits = np.asarray(logits, F32)
    scores = (F32(1.0) / (F32(1.0) + np.exp(-logits))).astype(F32)
    choice = scores + np.asarray(bias, F32)
    n = choice.shape[-1]
    if topk_group < n_group:
        grouped = choice.reshape(choice.shape[:-1] + (n_group, n // n_group))
        top2 = -np.sort(-grouped, axis=-1)[..., :2].sum(axis=-1)
        order = np.argsort(-top2, axis=-1, kind="stable")[..., :topk_group]
        keep = np.zeros(top2.shape, dtype=bool)
        np.put_along_axis(keep, order, True, axis=-1)
        choice = np.where(keep[..., None], grouped, -np.inf).reshape(choice.shape)
    ids = np.sort(np.argsort(-choice, axis=-1, kind="stable")[..., :top_k], axis=-1)
    weights = np.take_along_axis(scores, ids, axis=-1)
    if norm_topk_prob:
        weights = weights / (weights.sum(axis=-1, keepdims=True) + F32(1e-20))
    return ids.astype(np.uint32), (weights * F32(scale)).astype(F32)


def combine(values, scores, residual, dtype):
    """Routed weighted sum + shared + residual (fast_decode_finish_fused.metal:52-62).

    ``values`` [..., 9, h] typed expert outputs (slot 8 = shared), ``scores``
    [..., 8].  The float32 routed sum starts from slot 0 and adds slots 1..7
    in order (the MLX col_reduce order the fused kernel replicates); then
    ``T(routed)``, ``T(routed + shared)`` and ``T(residual + combined)``
    (model.py:415-418).
    """
    r = rounder(dtype)
    values = np.asarray(values, F32)
    scores = np.asarray(scores, F32)
    prod = values[..., :8, :] * scores[..., :, None]
    total = prod[..., 0, :] + F32(0.0)
    for s in range(1, 8):
        total = (prod[..., s, :] + F32(0.0)) + total
    routed = r(total)
    combined = r(routed + r(values[..., 8, :]))
    return r(np.asarray(residual, F32) + combined)


# ---------------------------------------------------------------------------
# bf16 shared expert (dense bf16 weights; the reference stores it as
# trellis slot 256, experts.py:116-124 -- both forms are supported)
# ---------------------------------------------------------------------------

def shared_bf16(x, w_gate, w_up, w_down, dtype="bfloat16"):
    """``T(T(swiglu(T(x@Wg^T), T(x@Wu^T))) @ Wd^T)`` with float32 accumulation."""
    r = rounder(dtype)
    x = np.asarray(x, F32)
    g = r(x @ np.asarray(w_gate, F32).T)
    u = r(x @ np.asarray(w_up, F32).T)
    h = swiglu_typed(g, u, dtype)
    return r(h @ np.asarray(w_down, F32).T)


# ---------------------------------------------------------------------------
# MXFP4 (joined_gather_order_common.metal:29-44, joined_gather_order.metal:19-20)
# ---------------------------------------------------------------------------

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=F32)


def e2m1_value(code):
    code = np.asarray(code, dtype=np.int64)
    mag = E2M1[code & 7]
    return np.where(code & 8, -mag, mag).astype(F32)


def e8m0_value(code):
    """``s == 0 ? 2^-127 : 2^(s-127)``, as float32."""
    code = np.asarray(code, dtype=np.int64)
    return np.where(code == 0, F32(2.0 ** -127), np.exp2(code - 127.0)).astype(F32)


def mxfp4_dequantize(weights, scales):
    """weights [E, n, k/8] uint32 (low nibble first), scales [E, n, k/32] uint8 -> [E, n, k]."""
    w = np.asarray(weights, dtype=np.uint32)
    nib = (w[..., None] >> (np.arange(8, dtype=np.uint32) * 4)) & 0xF
    values = e2m1_value(nib.reshape(w.shape[:-1] + (w.shape[-1] * 8,)))
    s = e8m0_value(np.asarray(scales))
    return (values * np.repeat(s, 32, axis=-1)).astype(F32)


def e8m0_encode(amax):
    """E8M0 code of blocks with largest magnitude ``amax`` under MLX 0.32.3
    ``quantize(mode="mxfp4")`` (fp_quantize: ``scale = amax / 6`` in float32,
    then the fp8_e8m0 conversion ``n = int(round(log2(scale)))`` clamped to
    [-127, 127], code n + 127).  log2 is the correctly rounded float32 value
    (through float64) and ``round`` is Metal's, half away from zero, so a
    scale whose float32 log2 is exactly n + 1/2 rounds away from zero.
    amax = 0 gives code 0; a non-finite amax gives 255."""
    amax = np.asarray(amax, F32)
    x = (amax / F32(6.0)).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        lf = np.log2(x.astype(np.float64)).astype(F32).astype(np.float64)
    n = np.where(lf >= 0, np.floor(lf + 0.5), np.ceil(lf - 0.5))
    n = np.nan_to_num(n, nan=0.0, posinf=127.0, neginf=-127.0)
    code = np.clip(n, -127, 127).astype(np.int64) + 127
    code = np.where(amax == 0, 0, code)
    code = np.where(np.isfinite(amax), code, 255)
    return code.astype(np.uint8)


def e2m1_encode(q):
    """E2M1 code of q (MLX fp4_e2m1 conversion): nearest of 0, .5, 1, 1.5, 2,
    3, 4, 6 with ties to the even code, saturating at 6; bit 3 = signbit(q);
    NaN -> 7."""
    q = np.asarray(q, F32)
    a = np.abs(q)
    m = ((a > 0.25).astype(np.uint32) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5) + (a >= 3.5) + (a > 5.0))
    code = np.where(np.signbit(q), np.uint32(8), np.uint32(0)) | m.astype(np.uint32)
    return np.where(np.isnan(q), np.uint32(7), code).astype(np.uint32)


def mxfp4_quantize(w):
    """MLX 0.32.3 ``quantize(w, mode="mxfp4")`` (group 32, bits 4) as used by
    joined_mxfp4.py:32 and dense_trellis.py:97-101: w [..., k] float32 ->
    (codes [..., k/8] uint32, eight E2M1 codes per word low nibble first;
    scales [..., k/32] uint8 E8M0).  Elements are coded from ``v / 2^e``
    with 2^e the decoded scale (2^-127 for code 0)."""
    w = np.asarray(w, F32)
    k = w.shape[-1]
    if k % 32:
        raise ValueError("mxfp4 quantisation needs a multiple of 32 values per row")
    g = w.reshape(w.shape[:-1] + (k // 32, 32))
    with np.errstate(invalid="ignore"):
        amax = np.max(np.abs(g), axis=-1)
    scales = e8m0_encode(amax)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        q = (g / e8m0_value(scales)[..., None]).astype(F32)
    nib = e2m1_encode(q).reshape(w.shape[:-1] + (k // 8, 8))
    codes = np.zeros(nib.shape[:-1], np.uint32)
    for j in range(8):
        codes |= nib[..., j] << np.uint32(4 * j)
    return codes, scales


def encode_joined(packed, scales, k, hidden, intermediate, experts=None):
    """``encode(expert)`` (joined_mxfp4.py:12-47): ``unit = sign(gate
    in-scale of matrix 0)``; every matrix of every projection decoded to inner
    [in, out] (decode.metal), gate/up rows times ``in_scale[e] * unit``
    (float32), quantised as ``inner.T`` with ``mxfp4_quantize``; gate and up
    joined along rows ([E, 2m, h/8], gate first).  ``experts`` restricts the
    matrices computed (the others stay zero); the fold product is formed in
    the scale dtype (fp16 * fp16 -> fp16 for fp16 scales) before the float32
    multiply, as the reference's MLX arrays do; returns (unit [h] float32,
    {"gate_up": (codes, scales), "down": (codes, scales)})."""
    h, m = hidden, intermediate
    count = np.asarray(packed["gate"]).size // (h * m * k // 8)
    keep = range(count) if experts is None else sorted(set(int(i) for i in experts))
    unit_typed = np.sign(np.asarray(scales["gate"][0])[0])  # in the scale dtype
    unit = unit_typed.astype(F32)
    out = {"gate_up": (np.zeros((count, 2 * m, h // 8), np.uint32), np.zeros((count, 2 * m, h // 32), np.uint8)),
           "down": (np.zeros((count, h, m // 8), np.uint32), np.zeros((count, h, m // 32), np.uint8))}
    for projection, offset in (("gate", 0), ("up", m), ("down", 0)):
        incoming, outgoing, side = (m, h, 2) if projection == "down" else (h, m, 1)
        target = out["down" if projection == "down" else "gate_up"]
        for e in keep:
            inner = decode_trellis(packed[projection], k, incoming, outgoing, side, e).astype(F32)
            if side == 1:
                # (scale * unit) in the scale dtype, then float32 (joined_mxfp4.py:22)
                fold = (np.asarray(scales[projection][0])[e] * unit_typed).astype(F32)
                inner = inner * fold[:, None]
            codes, sc = mxfp4_quantize(inner.T)
            target[0][e, offset:offset + outgoing] = codes
            target[1][e, offset:offset + outgoing] = sc
    return unit, out


def joined_slots(x, indices, unit, gate_up, down, scales, hidden, intermediate, dtype):
    """Joined MXFP4 slots (joined_mxfp4.py:90-134 + fast_decode_finish.metal).

    ``xh = H(x*unit)``; ``gu = xh @ Wgu[e]^T`` (gate rows first, up rows
    after, joined_mxfp4.py:41-45); typed SwiGLU of the transformed, scaled
    halves times the down input scale, transformed (joined_gate_finish.metal);
    down product; ``T(H(v)*out_down[e])``.
    ``gate_up``/``down`` are (weights, scales) MXFP4 pairs; ``scales`` maps
    "gate"/"up" to their out scales and "down" to (in, out).
    """
    indices = np.asarray(indices)
    ids = indices.reshape(-1).astype(np.int64)
    tokens = np.asarray(x, F32).reshape(-1, hidden)
    slots = indices.shape[-1]
    xh = hadamard128(tokens * np.asarray(unit, F32)[None, :])
    rows = xh[np.arange(ids.size) // slots]
    out = np.zeros((ids.size, hidden), F32)  # ids outside [0, experts) stay zero
    d_in, d_out = (np.asarray(s, F32) for s in scales["down"])
    g_out = np.asarray(scales["gate"], F32)
    u_out = np.asarray(scales["up"], F32)
    experts = np.asarray(gate_up[0]).shape[0]
    for e in np.unique(ids):
        if e < 0 or e >= experts:
            continue
        sel = np.nonzero(ids == e)[0]
        wgu = mxfp4_dequantize(gate_up[0][e:e + 1], gate_up[1][e:e + 1])[0]
        wd = mxfp4_dequantize(down[0][e:e + 1], down[1][e:e + 1])[0]
        gu = rows[sel] @ wgu.T
        g = hadamard128(gu[:, :intermediate]) * g_out[e]
        u = hadamard128(gu[:, intermediate:]) * u_out[e]
        act = hadamard128(swiglu_typed(g, u, dtype) * d_in[e])
        out[sel] = rounder(dtype)(hadamard128(act @ wd.T) * d_out[e])
    return out.reshape(indices.shape + (hidden,))


# ---------------------------------------------------------------------------
# Whole MoE layer (DecoderLayer MoE branch, model.py:385-418)
# ---------------------------------------------------------------------------

def router_logits(x, gate_weight):
    """``x.astype(f32) @ Wg^T`` (model.py:366-371, dense.py:158-159)."""
    return (np.asarray(x, F32) @ np.asarray(gate_weight, F32).T).astype(F32)


def moe_layer(x, residual, gate_weight, bias, packed, scales, k, hidden, intermediate,
              shared=None, dtype="bfloat16", logits=None, cache=None):
    """One routed-MoE layer: router, routed experts, shared expert, combine.

    ``shared`` is None when the shared expert is trellis slot 256 of
    ``packed``; otherwise a (w_gate, w_up, w_down) triple of bf16-valued
    float32 matrices in ``[out, in]`` layout.  Returns (out, ids, scores).
    """
    x = np.asarray(x, F32).reshape(-1, hidden)
    if logits is None:
        logits = router_logits(x, gate_weight)
    ids, scores = route(logits, bias)
    cache = cache or DecodedCache()
    if shared is None:
        values = expert_mlp_fused(x, ids, packed, scales, k, hidden, intermediate, dtype, cache)
    else:
        values = np.empty(ids.shape + (hidden,), F32)
        values[:, :8] = expert_mlp_fused(x, ids[:, :8], packed, scales, k, hidden, intermediate, dtype, cache)
        values[:, 8] = shared_bf16(x, *shared, dtype=dtype)
    out = combine(values, scores, residual, dtype)
    return out, ids, scores


def residual_rms_norm(x, weight, eps=1e-5, residual=None, dtype="bfloat16"):
    """Residual add + RMS norm in front of each MoE block (exlr8 model.py:373-384;
    the fused kernel of fast_norm.py:23-34 / metal/residual_rms.metal):
    h = T(x + residual); out = T(w * T(h * rsqrt(sum(h^2) / n + eps))), the sum
    of squares in float32.  Returns (h, out) as float32 arrays of T values."""
    rnd = rounder(dtype)
    h = np.asarray(x, np.float32)
    if residual is not None:
        h = rnd((h + np.asarray(residual, np.float32)).astype(np.float32))
    ss = np.sum(h * h, axis=-1, dtype=np.float32, keepdims=True)
    inv = (np.float32(1.0) / np.sqrt(ss / np.float32(h.shape[-1]) + np.float32(eps))).astype(np.float32)
    out = rnd((np.asarray(weight, np.float32) * rnd((h * inv).astype(np.float32))).astype(np.float32))
    return h, out
