"""Generate the golden vectors in this directory from the reference's own code.

Run from the repository root on a machine that has the reference checkout:

    python tests/golden/make_golden.py /path/to/MLXLR8

It imports the reference's NumPy-only functions (``exlr8/trellis.py``:
``round_e4m3``, ``mcg_codebook``, ``hadamard_reference``,
``decode_trellis_reference``, ``dequantize_reference``) and the vendored
PonyExl3 CPU reference (``third_party/ponyexl3/ref/{trellis,perm,codebook}.py``)
by file path, and ``exlr8/static_cache.py`` (``expand_static_reference``,
``codebook_codes``) as a package module -- MLX is not needed for these -- and
evaluates them on seeded inputs.  Expected values for composite operators use the same formulas as the
reference's own tests (cited beside each case).  The output is
``tests/golden/golden.npz``; the tests never read the reference at run time.
"""

from __future__ import annotations

import importlib
import importlib.util
import sys
from pathlib import Path

import numpy as np


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def main(reference_root: str) -> None:
    root = Path(reference_root)
    trellis = _load(root / "exlr8" / "trellis.py", "ref_exlr8_trellis")
    pack = _load(root / "third_party/ponyexl3/ref/trellis.py", "ref_pony_trellis")
    perm = _load(root / "third_party/ponyexl3/ref/perm.py", "ref_pony_perm")
    out = {}

    # Full codebook (trellis.py:43-50; test_fast_decode.py:93-116, test_trellis.py:59-63).
    out["codebook_bits"] = trellis.mcg_codebook().view(np.uint16).copy()

    # E4M3 ties, saturation, signed zero and random values (test_trellis.py:48-57).
    codes = np.arange(127)
    e, f = codes >> 3, codes & 7
    levels = np.array([f_ * 2.0 ** -9 if e_ == 0 else (8 + f_) * 2.0 ** (e_ - 10)
                       for e_, f_ in zip(e, f)], np.float32)
    mid = (levels[:-1] + levels[1:]) / 2
    rng = np.random.default_rng(5)
    e4m3_in = np.concatenate([mid, -mid, np.array([500, -500, np.inf, -np.inf, 0.0, -0.0], np.float32),
                              rng.normal(0, 3, 4096).astype(np.float32),
                              rng.uniform(-0.02, 0.02, 1024).astype(np.float32)]).astype(np.float32)
    out["e4m3_in"] = e4m3_in
    out["e4m3_out"] = trellis.round_e4m3(e4m3_in).astype(np.float32)

    # Hadamard (trellis.py:67-75).
    h_in = rng.normal(size=(6, 384)).astype(np.float32)
    out["hadamard_in"] = h_in
    out["hadamard_out"] = trellis.hadamard_reference(h_in)

    # Bitstream, permutation and storage orders (test_trellis.py:32-45,65-70):
    # canonical tiles packed by PonyExl3, decoded by decode_trellis_reference.
    for k in (2, 3, 4):
        for side in (0, 1, 2):
            in_f, out_f = 128, 256
            r = np.random.default_rng(8)
            fresh = r.integers(0, 1 << k, (in_f // 16, out_f // 16, 256), dtype=np.uint16)
            canonical = pack.pack_trellis(fresh, k)
            if side == 2:
                stored = canonical.reshape(in_f // 128, 8, out_f // 128, 8, 16 * k).transpose(0, 2, 1, 3, 4)
            else:
                stored = canonical.reshape(in_f // 16, out_f // 128, 8, 16 * k).transpose(1, 0, 2, 3)
            packed = np.ascontiguousarray(stored).view(np.uint8).reshape(-1)
            inner = trellis.decode_trellis_reference(packed, k, in_f, out_f, side)
            codewords = pack.unpack_trellis(canonical, k)
            independent = trellis.mcg_codebook()[codewords][..., perm.tensor_core_perm_inverse()]
            independent = independent.reshape(in_f // 16, out_f // 16, 16, 16).transpose(0, 2, 1, 3)
            assert np.array_equal(inner.view(np.uint16), independent.reshape(in_f, out_f).view(np.uint16))
            out[f"decode_k{k}_s{side}_packed"] = packed
            out[f"decode_k{k}_s{side}_inner_bits"] = inner.view(np.uint16)

    # Direct K4 words (test_fast_decode.py:56-69).
    canonical = np.random.default_rng(235).integers(0, 65536, (16, 16, 64), dtype=np.uint16)
    out["k4_canonical"] = canonical
    out["k4_codewords"] = pack.unpack_trellis(canonical, 4)

    # Random packed bytes are valid bitstreams (test_fast_decode.py:119-129):
    # decode and dequantize several seeded matrices, sides 1 and 2, K 2..4.
    r = np.random.default_rng(181)
    for k in (2, 3, 4):
        for side in (1, 2):
            a, b = (128, 256) if side == 1 else (256, 128)
            packed = r.integers(0, 256, 2 * a * b * k // 8, dtype=np.uint8)
            suh = r.uniform(-0.3, 0.3, a).astype(np.float16)
            svh = r.uniform(-0.3, 0.3, b).astype(np.float16)
            second = packed[a * b * k // 8:]
            out[f"rand_k{k}_s{side}_packed"] = packed
            out[f"rand_k{k}_s{side}_inner1_bits"] = trellis.decode_trellis_reference(second, k, a, b, side).view(np.uint16)
            out[f"rand_k{k}_s{side}_suh"] = suh
            out[f"rand_k{k}_s{side}_svh"] = svh
            out[f"rand_k{k}_s{side}_dequant1"] = trellis.dequantize_reference(second, suh, svh, k, a, b, side).astype(np.float32)

    # Selected-expert linear (test_trellis.py:121-141 formula: dequantize_reference + einsum).
    r = np.random.default_rng(31)
    indices = np.array([[2, 0], [1, 2]], np.uint32)
    out["linear_ids"] = indices
    for side in (1, 2):
        weights = []
        for e_ in range(3):
            rr = np.random.default_rng(e_)
            weights.append(rr.integers(0, 256, 128 * 256 // 2, dtype=np.uint8))
        packed = np.concatenate(weights)
        suh = r.uniform(-0.3, 0.3, (3, 128)).astype(np.float16)
        svh = r.uniform(-0.3, 0.3, (3, 256)).astype(np.float16)
        matrices = np.stack([trellis.dequantize_reference(w, suh[e_], svh[e_], 4, 128, 256, side)
                             for e_, w in enumerate(weights)])
        out[f"linear_s{side}_packed"] = packed
        out[f"linear_s{side}_in_scale"] = suh
        out[f"linear_s{side}_out_scale"] = svh
        for per_slot in (0, 1):
            x = r.normal(size=(2, 2, 128) if per_slot else (2, 128)).astype(np.float32)
            rows = x if per_slot else np.broadcast_to(x[:, None, :], (2, 2, 128))
            out[f"linear_s{side}_p{per_slot}_x"] = x
            out[f"linear_s{side}_p{per_slot}_expected"] = np.einsum("bsi,bsoi->bso", rows, matrices[indices]).astype(np.float32)

    # Router (test_fast_router.py:13-46 independent NumPy expectation).
    for case in ("random", "bias", "ties", "saturated", "zero"):
        for rows in (1, 2, 3, 4):
            r = np.random.default_rng(28)
            host = r.normal(size=(1, rows, 256)).astype(np.float32)
            bias = r.normal(0, .2, 256).astype(np.float32)
            if case == "bias":
                bias[:8] = 4
            elif case == "ties":
                host[:] = .5
                bias[:] = 0
            elif case == "saturated":
                host *= 100
            elif case == "zero":
                host[:] = -1000
            with np.errstate(over="ignore"):
                small = 1 / (1 + np.exp(np.abs(host)))
            original = np.where(host < 0, small, 1 - small)
            expected = np.argsort(-(original + bias), axis=-1, kind="stable")[..., :8]
            weights = np.take_along_axis(original, expected, axis=-1)
            weights = weights / (weights.sum(axis=-1, keepdims=True) + 1e-20) * 2.5
            out[f"route_{case}_{rows}_logits"] = host
            out[f"route_{case}_{rows}_bias"] = bias
            out[f"route_{case}_{rows}_ids"] = expected.astype(np.uint32)
            out[f"route_{case}_{rows}_scores"] = weights.astype(np.float32)

    # Static hot-expert cache: exact E4M3 bytes in the stored tile order
    # (static_cache.py:11-45, expand_static_reference and codebook_codes; the
    # module needs the package for its relative import, and MLX only inside
    # functions not called here).
    sys.path.insert(0, str(root))
    static = importlib.import_module("exlr8.static_cache")
    out["static_codebook_codes"] = np.asarray(static.codebook_codes()).copy()
    r = np.random.default_rng(991)
    for k in (2, 3, 4):
        for side in (1, 2):
            a, b = (128, 256) if side == 1 else (256, 128)
            packed = r.integers(0, 256, 2 * a * b * k // 8, dtype=np.uint8)
            out[f"static_k{k}_s{side}_packed"] = packed
            out[f"static_k{k}_s{side}_bytes"] = np.asarray(static.expand_static_reference(packed, k, a, b, side))

    target = Path(__file__).with_name("golden.npz")
    np.savez_compressed(target, **out)
    print(f"wrote {target} ({target.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/MLXLR8")
    main(sys.argv[1])
