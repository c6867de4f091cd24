"""distrain_b200: a Blackwell-native asynchronous distributed trainer (Distrain protocol).

Subpackages:
  models    flat-parameter transformer engine (sm_100a kernels) + fp32 oracle
  ops       ctypes bindings of the sm_100a kernel library
  parallel  delta compression, coordinator merge, in-box transport, node runtime, tensor parallel
  utils     checkpoint/delta codecs, data loaders, storage, metrics
"""
__version__ = "0.1.0"
