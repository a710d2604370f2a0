"""chimera_b200 -- B200-native (sm_100a) implementation of the Chimera
multi-vector retrieval search path behind the reference's own interfaces.

* C ABI: include/chimera_b200.h, built into lib/libchimera_b200.so
* drop-in C++ API / CLI / pybind11 module: include/chimera/chimera_index.cuh,
  bin/gpu_build, bin/gpu_search, and the ``chimera`` extension module
* Python plumbing used by tests and the benchmark: :mod:`chimera_b200.capi`
"""
__version__ = "0.1.0"
