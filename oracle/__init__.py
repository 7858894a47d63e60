"""CPU oracle for the attention prologue -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package, and only as the checker or the timed CPU
baseline. The product (``flash_attn_prologue_b200``) never imports it.

* ``native``: the reference's ``native`` backend restated op for op on CPU
  tensors (flash_attn_prologue/functional.py:49-63 broadcasting, :89-94 math);
  its backward is autograd through the same ops, exactly as the reference's.
* ``fp64``: an independent float64 oracle in numpy -- vector-norm RMS and
  explicit 2x2 rotations as in the reference's tests/test_frontend_api.py:13-32,
  and a closed-form backward following the identities of the reference's
  backward kernel (flash_attn_prologue/fused_epilogue.py:1047-1126).

* ``inverse``: the reference's inverse (recompute-from-outputs) prologue
  (flash_attn_prologue/fused_epilogue.py:2560-2805): forward = ``native`` plus
  the per-row statistic r, backward restated op for op from the saved outputs.

* ``compare``: the output bar -- 1 ulp, or within the FP32 rounding band of
  the rotation's term magnitudes where its two products nearly cancel.

Pinning: tests/golden/ holds outputs and gradients produced by importing the
reference package itself (tests/golden/make_golden.py); tests/test_oracle_golden.py
checks both restatements against them.
"""
from .native import native_forward, native_forward_backward  # noqa: F401
from .fp64 import fp64_forward, fp64_backward  # noqa: F401
from .compare import check_outputs, term_magnitudes  # noqa: F401
from .inverse import inverse_backward, inverse_forward  # noqa: F401
