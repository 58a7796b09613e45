"""B200 (sm_100a) execution backend for mlir-cim22's software-simulated CIM path.

Submodules:
  abi      ctypes mirror of include/cim22_cuda.h data structures
  native   binding of libcim22_cuda.so (transaction runner, session, dispatch)
  cim_ops  CIM layers and Host glue over CUDA tensors
"""

__all__ = ["abi", "native", "cim_ops"]
