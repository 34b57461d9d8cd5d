"""Mixed-rate KV cache (allocation/eval_alloc.py: VariableRateKVCache)."""
