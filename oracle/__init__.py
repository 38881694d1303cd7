"""CPU oracle for the fragment kernels — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline /
``--impl reference`` arm may import this package, and only as the checker or
the timed CPU reference — never as part of the product path.  The product
(``kernelproblems_b200``) never imports it and has no CPU fallback.

``oracle.fragments`` restates, with torch CPU ops, the torch reference graph
of every hot-path fragment of SherlockNoMad/KernelProblems (each function
cites the reference ``problem.py`` lines it follows), plus float64 versions of
the two column/segment reductions (dweight, embedding gradient) used for the
tighter fp32 checks.

Pinning: ``tests/golden/make_golden.py`` runs the reference ``Model`` modules
themselves on CPU on seeded inputs and records their outputs (sha256 of every
output plus sampled rows); ``tests/test_oracle_golden.py`` checks that these
restatements reproduce them bit for bit.  The neox rotate-half RoPE has no
reference implementation; it is tied to the reference's interleaved RoPE by
the pair-permutation identity in ``oracle.fragments.rope_neox_via_interleaved``.
"""
