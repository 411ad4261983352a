"""CPU oracle for the KeSSie fog-attention hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, in numpy, the reference's
own PyTorch/HIP semantics for the path (fog weights, windowed fog attention,
RoPE remap, page evict / insert / gather and the page-table bookkeeping of
``KeSSiePagedKVCache``).  It is the checker for the CUDA library, never the
thing measured or shipped: only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / ``--impl reference`` legs may import it.  The
product path (``kessie_b200``) never imports it and fails loudly when the
CUDA library is missing.

Parity of this restatement is pinned by ``tests/golden/*.npz``, which were
produced by running the reference's own Python functions
(``kessie_hip_kernels.py``) on seeded inputs; see
``tests/golden/make_golden.py`` and ``tests/test_oracle_golden.py``.
"""

from .fog_oracle import *  # noqa: F401,F403
