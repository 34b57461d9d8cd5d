"""Reference-compatible core modules (e8_quantizer, entropy_coder, gpu_ans,
compact_storage, triton_dequant) backed by the B200 CUDA library."""
