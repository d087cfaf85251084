"""CPU oracle for the tensor-parallel quantized decode path of shardcompute.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg (``cpu_baseline`` / ``--impl reference``) may use it, and only as
the checker or as the timed stand-in for the reference's CPU path.

What it restates (numpy, float64 unless a step is defined in fp16/fp32):

* ``mlx_affine``: the MLX group-wise affine quantization format the reference
  stores on disk (``mx.quantize`` / ``mx.dequantize`` /
  ``mx.quantized_matmul`` call sites in ``parallel/quantized_linear.py:168-176,
  206-214,435-443,472-480`` and ``parallel/embedding.py:338-349``).
* ``tp``: the reference's tensor-parallel layer math with the collectives
  simulated in-process, the way the reference's own tests do it
  (``tests/test_parallel_layers.py``, ``tests/test_integration.py``).
* ``sharder``: the shard layout written by ``model/sharder.py:100-255``.

Parity status
-------------
* TP split math, shard layout and collective semantics: pinned against the
  reference's own structural tests, restated in ``tests/test_oracle_pins.py``.
* Quantized arithmetic (pack order, dequant rounding, quantized_matmul):
  **parity unpinned**.  The arithmetic lives in the third-party MLX wheel
  (``requirements.txt:2``, ``mlx>=0.12.0``, unpinned, not vendored), MLX is not
  installed on either machine, and the reference ships no golden vectors for
  the quantized path.  The oracle follows MLX's published format:
  per group of ``g`` values along the last axis, ``w ~= s*q + b`` with
  ``q`` in ``[0, 2**bits - 1]``, packed little-endian inside each uint32
  (element j at bits ``[bits*j, bits*(j+1))``).
"""
