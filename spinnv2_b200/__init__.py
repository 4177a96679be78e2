"""SPINNV2 B200: a CUDA (sm_100a) execution target for SPINNV2's SPK runtime.

  spinnv2_b200.compiler  SIR graphs, passes, cuda_b200 kernel specs, memory
                         plan, SPK writer, INT8 quantisation, config builders
  spinnv2_b200.runtime   ctypes driver of libspkv2_runtime.so (the C-ABI
                         CUDA runtime built from spinnv2_b200/csrc)
  spinnv2_b200.spk       SPK reader
  spinnv2_b200.shard     batch-sharded multi-GPU inference
"""

__version__ = "0.1.0"
