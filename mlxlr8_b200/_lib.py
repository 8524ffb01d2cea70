"""ctypes binding of the C ABI in ``include/exlr8_b200.h``.

The CUDA library ``libexlr8_b200.so`` is built in-tree by
``python -m mlxlr8_b200.build``.  There is no CPU fallback: every operator
raises if the library is missing or no CUDA device is present.
"""

from __future__ import annotations

import ctypes
from ctypes import c_double, POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p
from functools import lru_cache
from pathlib import Path

import torch

LIBRARY = Path(__file__).resolve().with_name("libexlr8_b200.so")

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
SCALE_CODES = {torch.float32: 0, torch.float16: 1}

# Status codes whose reference behaviour is a ValueError.
VALUE_ERRORS = {1, 2, 3, 4, 5, 6, 7, 8, 13, 15}


class TrellisExperts(ctypes.Structure):
    _fields_ = [
        ("packed", c_void_p * 3),
        ("packed_bytes", c_int64 * 3),
        ("in_scale", c_void_p * 3),
        ("out_scale", c_void_p * 3),
        ("scale_dtype", c_int),
        ("scale_experts", c_int64),
        ("k", c_int),
        ("hidden", c_int),
        ("intermediate", c_int),
    ]


class StaticCache(ctypes.Structure):
    _fields_ = [("fp8", c_void_p * 3), ("expert_to_slot", c_void_p), ("slots", c_int64)]


class DenseExpert(ctypes.Structure):
    _fields_ = [("gate", c_void_p), ("up", c_void_p), ("down", c_void_p)]


class JoinedMXFP4Weights(ctypes.Structure):
    _fields_ = [
        ("gate_up", c_void_p),
        ("gate_up_scales", c_void_p),
        ("down", c_void_p),
        ("down_scales", c_void_p),
        ("unit", c_void_p),
        ("gate_out", c_void_p),
        ("up_out", c_void_p),
        ("down_in", c_void_p),
        ("down_out", c_void_p),
        ("scale_dtype", c_int),
        ("experts", c_int64),
        ("hidden", c_int),
        ("intermediate", c_int),
    ]


_SIGNATURES = {
    "exlr8_abi_version": (c_int, []),
    "exlr8_status_string": (c_char_p, [c_int]),
    "exlr8_last_cuda_error": (c_char_p, []),
    "exlr8_codebook": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "exlr8_check_format": (c_int, [c_int64, c_int, c_int, c_int, c_int, POINTER(c_int64)]),
    "exlr8_decode_trellis": (c_int, [c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "exlr8_expand_static_trellis": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "exlr8_dequantize_trellis_workspace": (c_size_t, [c_int, c_int]),
    "exlr8_dequantize_trellis": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                         c_void_p, c_void_p, c_size_t, c_void_p]),
    "exlr8_route": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "exlr8_dispatch_plan_workspace": (c_size_t, [c_int64, c_int]),
    "exlr8_dispatch_plan": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                                    c_void_p, c_size_t, c_void_p]),
    "exlr8_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "exlr8_router": (c_int, [c_void_p, c_int, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p]),
    "exlr8_expert_linear_workspace": (c_size_t, [c_int64, c_int, c_int, c_int, c_int64]),
    "exlr8_expert_linear": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p,
                                    c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                    c_size_t, c_void_p]),
    "exlr8_expert_mlp_workspace": (c_size_t, [c_int64, c_int, c_int, c_int, c_int64]),
    "exlr8_expert_mlp": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int64, c_int, POINTER(TrellisExperts),
                                 c_void_p, c_void_p, c_size_t, c_void_p]),
    "exlr8_expert_mlp_cached": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int64, c_int, POINTER(TrellisExperts),
                                        POINTER(StaticCache), c_void_p, c_void_p, c_size_t, c_void_p]),
    "exlr8_expert_mlp_finish_workspace": (c_size_t, [c_int64, c_int, c_int, c_int64]),
    "exlr8_expert_mlp_finish": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                        POINTER(TrellisExperts), POINTER(DenseExpert), c_void_p, c_void_p, c_size_t,
                                        c_void_p]),
    "exlr8_moe_layer_workspace": (c_size_t, [c_int64, c_int, c_int, c_int64]),
    "exlr8_moe_layer": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_void_p, c_void_p, POINTER(TrellisExperts),
                                POINTER(DenseExpert), c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "exlr8_host_device_pointer": (c_int, [c_void_p, POINTER(c_void_p)]),
    "exlr8_stage_in": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "exlr8_workspace_bad_ids": (c_int, [c_void_p, POINTER(c_int64), c_void_p]),
    "exlr8_profile_enable": (c_int, [c_int, c_int]),
    "exlr8_profile_read": (c_int, [c_int, POINTER(c_int64), POINTER(ctypes.c_double)]),
    "exlr8_moe_layer_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_void_p, c_void_p,
                                        POINTER(TrellisExperts), POINTER(DenseExpert), c_void_p, c_void_p, c_void_p,
                                        c_void_p]),
    "exlr8_codec_peak": (c_int, [c_int, POINTER(c_double), c_void_p, c_void_p]),
    "exlr8_gemm_pair": (c_int, [c_int]),
    "exlr8_tensor_peak": (c_int, [c_int, c_int, c_int, POINTER(c_double), c_void_p, c_void_p]),
    "exlr8_peer_write": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "exlr8_hadamard128": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "exlr8_mxfp4_quantize": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p]),
    "exlr8_mxfp4_encode_trellis": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int,
                                           c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "exlr8_mxfp4_prepared_scales_bytes": (c_size_t, [c_int64, c_int]),
    "exlr8_mxfp4_prepare_scales": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "exlr8_joined_workspace": (c_size_t, [c_int64, c_int, c_int, c_int, c_int64]),
    "exlr8_joined_slots": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int, POINTER(JoinedMXFP4Weights), c_void_p,
                                   c_void_p, c_size_t, c_void_p]),
    "exlr8_joined_finish": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                    POINTER(JoinedMXFP4Weights), c_void_p, c_void_p, c_size_t, c_void_p]),
    "exlr8_joined_moe_layer_workspace": (c_size_t, [c_int64, c_int, c_int, c_int64]),
    "exlr8_joined_moe_layer": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_void_p, c_void_p,
                                       POINTER(JoinedMXFP4Weights), c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                       c_void_p]),
    "exlr8_joined_status": (c_int, [c_void_p, c_int64, c_int, c_int64, c_void_p, c_void_p]),
    "exlr8_prefill_status": (c_int, [c_void_p, c_int64, c_int, c_int, c_int64, c_void_p, c_void_p]),
    "exlr8_ep_dispatch": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    "exlr8_ep_combine": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p,
                                 c_void_p]),
    "exlr8_residual_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int, c_float, c_void_p,
                                        c_void_p, c_void_p]),
    "exlr8_ep_peer_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "exlr8_ep_peer_offsets": (c_int, [c_int, c_int, c_int, c_int, POINTER(c_size_t), POINTER(c_size_t),
                                      POINTER(c_size_t)]),
    "exlr8_ep_peer_create": (c_int, [c_size_t, POINTER(c_void_p), c_void_p]),
    "exlr8_ep_peer_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "exlr8_ep_peer_close": (c_int, [c_void_p]),
    "exlr8_ep_peer_destroy": (c_int, [c_void_p]),
    "exlr8_ep_send": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_void_p]),
    "exlr8_ep_return": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                c_void_p]),
    "exlr8_expert_mlp_shared_workspace": (c_size_t, [c_int64, c_int, c_int, c_int64, c_int64]),
    "exlr8_expert_mlp_shared": (c_int, [c_void_p, c_int, c_void_p, c_int64, POINTER(TrellisExperts), c_void_p, c_int64,
                                        POINTER(DenseExpert), c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "exlr8_shared_expert_workspace": (c_size_t, [c_int64, c_int, c_int]),
    "exlr8_shared_expert": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, POINTER(DenseExpert), c_void_p, c_void_p,
                                    c_size_t, c_void_p]),
    "exlr8_router_logits_workspace": (c_size_t, [c_int64, c_int, c_int]),
    "exlr8_router_logits": (c_int, [c_void_p, c_int, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_size_t,
                                    c_void_p]),
}

EXPORTED = tuple(_SIGNATURES)


@lru_cache(maxsize=1)
def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library and declare every exported function."""
    target = Path(path) if path else LIBRARY
    if not target.exists():
        raise RuntimeError(f"{target.name} is not built: run `python -m mlxlr8_b200.build` "
                           "(the exlr8 B200 operators have no CPU fallback)")
    lib = ctypes.CDLL(str(target))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def lib() -> ctypes.CDLL:
    return load()


def check(status: int) -> None:
    if status == 0:
        return
    message = load().exlr8_status_string(status).decode()
    if status in VALUE_ERRORS:
        raise ValueError(message)
    detail = load().exlr8_last_cuda_error().decode()
    raise RuntimeError(f"{message} ({detail})" if detail else message)


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All operands must live on one CUDA device; there is no CPU path."""
    if not torch.cuda.is_available():
        raise RuntimeError("the exlr8 B200 operators need a CUDA device (no CPU fallback)")
    device = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError("exlr8 B200 operators take CUDA tensors")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("operands are on different devices")
    return device if device is not None else torch.device("cuda", torch.cuda.current_device())


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def host_device_pointer(t: torch.Tensor) -> int:
    """Device-accessible address of a page-locked host tensor's data, for a
    kernel that reads or writes it over PCIe (pageable memory is refused)."""
    ptr = c_void_p(0)
    check(load().exlr8_host_device_pointer(t.data_ptr(), ctypes.byref(ptr)))
    return int(ptr.value)


def act_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported activation dtype {t.dtype}") from None


def scale_code(t: torch.Tensor) -> int:
    try:
        return SCALE_CODES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported side-scale dtype {t.dtype}") from None


KERNEL_KINDS = ("router", "plan", "prep", "gate_up", "gate_finish", "down", "finish", "dense", "ep_send",
                "ep_return", "ep_combine", "norm")


def profile_enable(enable: bool, capacity: int = 65536) -> None:
    """Bracket every library launch on this thread with CUDA events."""
    check(load().exlr8_profile_enable(int(enable), capacity))


def profile_read() -> dict:
    """{kind: (launches, total_ms)} of the launches recorded since enabling."""
    out = {}
    for i, name in enumerate(KERNEL_KINDS):
        n = ctypes.c_int64(0)
        ms = ctypes.c_double(0.0)
        check(load().exlr8_profile_read(i, ctypes.byref(n), ctypes.byref(ms)))
        out[name] = (int(n.value), float(ms.value))
    return out


def prefill_status(workspace_tensor: torch.Tensor, tokens: int, slots: int, intermediate: int, experts: int):
    """[chunks, padded rows, gate/up units, down units, GEMM error] of the last
    trellis prefill call that used ``workspace_tensor``."""
    header = torch.zeros(8, dtype=torch.int32)
    check(load().exlr8_prefill_status(workspace_tensor.data_ptr(), tokens, slots, intermediate, experts,
                                      header.data_ptr(), stream_handle(workspace_tensor.device)))
    return header.tolist()[:5]


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
