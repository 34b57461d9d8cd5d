"""Reference-compatible KV-cache integration (llm/compressed_kv_cache.py)."""
