"""shardcompute_b200: the tensor-parallel quantized decode path of shardcompute on B200 (sm_100a).

The compute lives in ``libsc_b200.so`` (hand-written CUDA, C ABI in
``include/sc_b200.h``); this package is the host-side mirror of the
reference's ``parallel/`` / ``collectives/`` / ``model/`` interfaces.
"""

__version__ = "0.1.0"
