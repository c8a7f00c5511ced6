"""CPU oracle of FastMD's per-step hot path -- TEST INFRASTRUCTURE ONLY.

Plain NumPy restatements of the reference algorithms (each function cites the
FastMD source file:line it restates). Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference legs may import this package, and
only as the checker or the timed CPU baseline: the product path
(``fastmd_b200``) never imports it and has no CPU fallback.

Pinning: the restatements are checked against golden vectors produced by the
reference's own code run in this container (``tests/golden/make_golden.py``:
the Triton gather-cat and CSR segment-sum kernels under TRITON_INTERPRET=1,
the torch backend of the Nose-Hoover chain, the dense FP64 neighbour search
of the reference's boundary tests). The MACE-architecture model has no
source in the reference (it lives in mace-torch 0.3.16, not vendored): its
oracle is a restatement of the published MACE equations and its parity is
"unpinned" (see oracle/mace.py).
"""
