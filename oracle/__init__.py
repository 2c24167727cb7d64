"""CPU oracle for the moe-stream expert-block hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped library imports this package:
only the tests under ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and there
only as the checker or as the timed CPU baseline.

It is a plain numpy restatement of the reference's algorithm:

* ``bf16``     -- round-to-nearest-even bfloat16 emulation on float32 arrays.
* ``quant``    -- MLX affine 4-bit quantisation (group 64, bf16 scales/biases,
                  eight nibbles per uint32, low nibble first) as used through
                  ``mx.quantize`` / ``mx.dequantize`` (test_kernel.py:57-60,
                  kernels.py:129-144).
* ``moe``      -- the two routers (engine_v3.py:467-483, engine_120b.py:65-75),
                  the gather_qmm expert block with MLX's bf16 rounding points
                  (engine_v3.py:588-600, engine_120b.py:130-145) and the fp32
                  dequantised reference of test_kernel.py:52-65.
* ``pool_sim`` -- ``ExpertPool``'s slot bookkeeping (engine_v3.py:303-464)
                  made deterministic: reads complete at the end of each
                  ``acquire``.
* ``torch_port`` -- the whole decode step (routers, speculation, pool
                  simulator with blob fills, expert math) vectorised in
                  float32 torch on the host: the timed CPU baseline.

Parity status. The slot-pool restatement is PINNED: it is checked against
fixtures produced by running the reference's own ``ExpertPool`` code
(``tests/golden/make_pool_golden.py``). The floating-point block (quantiser,
routers, expert math) is "parity unpinned": the reference computes it with
MLX 0.32 / mlx-lm 0.31, which are neither vendored nor installable here, so
the restatement is pinned only by the properties the reference's own tests
check (byte-exact pool contents, kernel error against the fp32 dequantised
reference no worse than 1.5x the bf16 MLX path's, routing invariants).
"""
