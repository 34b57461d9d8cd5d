"""LatticeQuant KV-cache compression on NVIDIA B200 (sm_100a).

E8 lattice quantisation -> parity-aware symbols -> bit-level rANS lanes ->
dequantisation / fused decode attention, as hand-written CUDA behind a C ABI
(include/latticequant_b200.h), with the reference's Python API on top:

  latticequant_b200.core.*                  e8_quantizer, entropy_coder, gpu_ans,
                                            compact_storage, triton_dequant, pipeline
  latticequant_b200.llm.compressed_kv_cache CompressedKVCache
  latticequant_b200.allocation.eval_alloc   VariableRateKVCache

There is no CPU fallback: every compute call runs the CUDA library.
"""
__version__ = "0.1.0"
