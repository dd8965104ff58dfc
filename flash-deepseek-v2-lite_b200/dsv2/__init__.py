"""B200-native (sm_100a) decode kernels and runner for DeepSeek-V2-Lite.

Layers:
  dsv2._lib      ctypes binding of libdsv2.so (C ABI: include/dsv2.h)
  dsv2.ops       tensor-level wrappers (current torch stream, caller-owned outputs)
  dsv2.kernels   drop-in modules with the reference's names and signatures
                 (replacing heiheiha798/Flash-DeepSeeek-V2-Lite triton_kernels/*)
  dsv2.model     DeepSeek-V2-Lite shapes and load-time weight packing
  dsv2.engine    latent-cache decode engine with CUDA-graph replay (src/run.py runner)
  dsv2.run       command-line driver mirroring src/run.py
"""
from ._lib import LIB_PATH, Dsv2Error, load  # noqa: F401

__version__ = "1.0"
