"""CPU oracle for the GDN and NVFP4 hot path -- TEST INFRASTRUCTURE ONLY.

Everything under ``oracle/`` restates, on the CPU, the algorithms of the
reference RECANT package that the B200 kernels replace:

* ``oracle.gdn``    -- chunked Gated DeltaNet forward (recant/model/ops.py:21-54)
                      and its autograd backward, plus the varlen (cu_seqlens) and
                      GQA wrappers the B200 op adds;
* ``oracle.nvfp4``  -- randomized-Hadamard + NVFP4 quantizer, the 128x4 blocked
                      scale swizzle, dequantisation and the emulated GEMM
                      (recant/model/nvfp4.py:6-124), in numpy, bit-exact.
* ``oracle.segments`` -- the affine state folds (prefix / suffix / composition) of the
                      segmented and context-parallel op, as plain torch loops;
* ``oracle.inputs`` -- the seeded synthetic inputs of the benchmark configs.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
reference arms may import this package, and only as the checker or as the timed
CPU baseline.  The product package ``recant_b200`` never imports it: its ops run
only on the CUDA library and raise when the library is missing.

Pinning: ``tests/golden/make_golden.py`` runs the reference package itself on
seeded inputs and commits its outputs (hashes for the bit-exact quantizer,
fp32 arrays for GDN); ``tests/test_oracle_pins.py`` checks this oracle against
those fixtures.
"""
