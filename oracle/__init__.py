"""CPU oracle for the int4 decode/prefill hot path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only to check or time the reference algorithm. The product
package ``tritonforge_b200`` never imports it and has no CPU fallback.

Contents:

* :mod:`oracle.quant` -- numpy restatement of the reference's int4 group
  quantizer, packer, unpacker and dequantizer (``src/tritonforge/quant.py``),
  bit-exact, including IEEE fp32 division, round-half-even and the sign of
  zero that ``torch.clamp`` keeps.
* :mod:`oracle.ops` -- CPU restatements of the reference's PyTorch oracles
  (``src/tritonforge/reference.py``): int4 linear, residual + RMSNorm, plain
  RMSNorm and SwiGLU, with the same rounding points.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by running the reference's own ``quant.py`` and
``reference.py`` (``tests/golden/make_golden.py``).
"""

from . import ops, quant  # noqa: F401

__all__ = ["ops", "quant"]
