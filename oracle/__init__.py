"""CPU oracle for the HADS block-sparse attention path -- TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy, the algorithms of the reference project
(Hridambiswas/XSAKE) for the one hot path this repository accelerates:

* ``attention``  -- ``sparse_attention_reference`` and its autodiff backward
  (kernels/pallas/sparse_attention.py:45-91, :286-298);
* ``rowops``     -- ``jax.nn.softmax`` as called by ``fused_softmax`` and the
  LayerNorm formula of ``fused_layernorm`` (kernels/pallas/fused_softmax.py:26-36,87;
  kernels/pallas/fused_layernorm.py:26-51,116-119), with their backwards;
* ``hads``       -- entropy, the entropy->sparsity map and the seeded block-mask
  builder (kernels/hads/hads_pattern.py:36-223);
* ``inputs``     -- seeded synthetic inputs with the shapes and distributions of
  the benchmark configurations.

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``, and there only as
the expected results that GPU outputs are compared against, or as the timed CPU
baseline.  The product package ``xsake_b200``
never imports this package; its compute path is CUDA only.

Pinning: the reference's own tests hold no stored vectors.  The golden files
under ``tests/golden/`` were produced by executing the reference's own source
functions (read from the reference checkout) with a NumPy-backed stand-in for
``jax.numpy`` -- see ``tests/golden/make_golden.py``.  ``tests/test_oracle_golden.py``
checks every oracle function against those files.  Float results are therefore
pinned to the reference's code structure evaluated with NumPy arithmetic (JAX
itself is not installable here); block masks are pinned bit-exactly because the
reference builds them with NumPy alone.
"""

from . import attention, rowops, hads, inputs  # noqa: F401
