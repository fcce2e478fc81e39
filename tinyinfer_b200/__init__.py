"""B200-native (sm_100a) MiniPrefix paged-KV Llama forward.

Layers:
  * device  -- ctypes binding of libmpb200.so (include/miniprefix_b200.h): CUDA
               kernels behind a thin C ABI.
  * host    -- ctypes binding of libmpb200_host.so (include/miniprefix_b200_host.h):
               the C++ page pool, prefix cache, KV manager, scheduler, engine and
               runner that drive the device layer.
  * synthetic -- seeded synthetic weights/tokens in the MPFX0001 orientation.
"""
__version__ = "0.1.0"
