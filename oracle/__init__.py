"""CPU oracle for the routed-MoE hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in NumPy and plain C, the arithmetic of the reference
package ``exlr8`` (GordoAR/MLXLR8 v0.1.21) for its routed mixture-of-experts
path.  It exists to check the CUDA product and to time a CPU baseline.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline``
leg and its ``--impl reference`` arm) may import it.  The product package
``mlxlr8_b200`` never imports, links or executes anything under ``oracle/``.

Parity pinning: ``tests/golden/`` holds vectors produced by the reference's
own NumPy functions (``exlr8/trellis.py:22-109`` and the vendored PonyExl3
pack/unpack/permutation reference) by ``tests/golden/make_golden.py``; the
CPU test-suite checks this oracle against them.
"""
