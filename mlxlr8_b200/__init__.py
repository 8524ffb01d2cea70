"""exlr8 routed-MoE hot path for NVIDIA B200 (sm_100a).

Mirrors the expert-operator API of the reference package ``exlr8``
(GordoAR/MLXLR8): :mod:`.trellis`, :mod:`.fast_router`, :mod:`.fast_decode`,
:mod:`.fast_prefill`, :mod:`.experts`, plus :class:`.moe.MoELayer` for a whole
layer.  All compute runs in the in-tree CUDA library ``libexlr8_b200.so``
through the C ABI declared in ``include/exlr8_b200.h``.
"""

__version__ = "0.1.0"
