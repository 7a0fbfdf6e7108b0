"""B200-native (sm_100a) decode-step hot path of the ios_kernels LLM runtime.

Modules:
  _lib    ctypes binding of libb200dec.so (C ABI in include/b200dec.h)
  ops     torch-facing wrappers of every entry point (GEMV family, attention, small ops)
  tp      tensor-parallel sharding of a Llama-style decoder's weights
  engine  DecodeEngine: weights, paged KV pools and the decode-step handle for one rank
  build   nvcc build of the library (in-tree)
"""

__all__ = ["_lib", "ops", "tp", "engine", "build"]
