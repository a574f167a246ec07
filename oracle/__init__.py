"""CPU oracle for the W4A8 MoE path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or as the timed CPU restatement of the reference.  The product
path (the package ``flagos-kernel-gen_b200``) never imports it.

Parity pinning: the grouped GEMM restatement is checked bit-for-bit against
golden vectors produced by running the reference's own PyTorch implementation
(docs/Task1.md:49-115), and the per-token quantiser against the reference's
own int8 quantiser (docs/Task3.md:58-67); see ``tests/golden/make_golden.py``.
The align, SiLU-mul requant and combine stages have no reference code; their
restatements here define the semantics ("parity unpinned by the reference").
"""
