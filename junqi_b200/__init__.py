"""junqi_b200 -- B200-native batched JunQi environment.

The hot path (step, combat memory, beliefs, auto-reset, legal CSR / mask,
317-channel observation) runs in hand-written sm_100a kernels behind the C
ABI of ``libjq.so`` (``include/jq.h``).  ``junqi_b200.env.JunqiEnvB200`` is
the native Python API; ``junqi_b200.junqi_cuda`` mirrors the reference's
``junqi_cuda`` pybind module for drop-in use.
"""
__version__ = "0.1.0"
