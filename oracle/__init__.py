"""CPU oracle for the LITHE index-resident forward -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (integer / byte work) and plain torch CPU ops (the float
contractions, mirroring the reference's own torch code), the algorithm of the reference
implementation (JianJiang1995/LITHE) for the hot path:

  codebook_ref  -- Hadamard-9bit twin pools          (lithe/codebook.py)
  decode_ref    -- blocking, RVQ decode, 9-bit packing, packed layout
                   (lithe/quant.py, lithe/kernels/packed.py)
  sgmv_ref      -- per-sample routed LoRA delta       (lithe/serve.py,
                   lithe/kernels/shared.py reference)

It is pinned against fixtures generated from the reference itself
(tests/golden/make_golden.py, run where the reference is importable) and against the
known answers of the reference's own tests.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import it, and
only as the checker or the timed CPU baseline.  The product package (lithe_b200) never
imports it and has no CPU fallback.
"""
