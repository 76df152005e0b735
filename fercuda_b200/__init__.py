"""fercuda_b200: B200-native (sm_100a) drop-in for feRcuda's deterministic
tensor-op hot path. The product is the C ABI in fercuda_b200/lib
(libfercuda_capi.so, libptx_core.so, libptx_kernels.so); this package holds
the ctypes binding (capi), the seeded workload generators (synth) and the
multi-GPU transformer driver."""
from . import capi, synth  # noqa: F401

__all__ = ["capi", "synth"]
