"""VariableRateKVCache -- per-layer, per-K/V bit rates (allocation/eval_alloc.py:56-145).

Like the reference it sets ``self.bits`` before each ``_compress_tensor`` call
and skips CompressedKVCache's (3, 4, 5) assertion by initialising the
DynamicCache base directly.  The rest of the reference module (PPL drivers,
water-filling allocation) is research tooling and out of scope.
"""
from __future__ import annotations

from typing import Dict, List, Optional

from transformers.cache_utils import DynamicCache

from .. import codec
from ..llm.compressed_kv_cache import CompressedKVCache


class VariableRateKVCache(CompressedKVCache):
    """bits_schedule: [{'K': 3, 'V': 5}, {'K': 4, 'V': 4}, ...], one dict per layer."""

    def __init__(self, bits_schedule: List[Dict[str, int]], eval_only_no_entropy: bool = True,
                 tile_blocks: Optional[int] = codec.DEFAULT_TILE_BLOCKS, table_mode: str = "device"):
        DynamicCache.__init__(self)
        self.bits = 4  # overridden per _compress_tensor call
        self.eval_only_no_entropy = eval_only_no_entropy
        self.bits_schedule = bits_schedule
        self.tile_blocks = tile_blocks
        self.table_mode = table_mode
        if not hasattr(self, 'key_cache'):
            self.key_cache = []
        if not hasattr(self, 'value_cache'):
            self.value_cache = []
        self._comp_keys = []
        self._comp_values = []
        self.total_vectors = 0
        self._model_dtype = None

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """Compress K and V at this layer's scheduled rates (allocation/eval_alloc.py:87-145)."""
        schedule = self.bits_schedule[layer_idx] if layer_idx < len(self.bits_schedule) else {'K': 4, 'V': 4}
        device = key_states.device
        if self._model_dtype is None:
            self._model_dtype = key_states.dtype
        self.bits = schedule['K']
        comp_k, k_dec_new = self._compress_tensor(key_states)
        self.bits = schedule['V']
        comp_v, v_dec_new = self._compress_tensor(value_states)
        return self._store(layer_idx, device, key_states, value_states, comp_k, k_dec_new, comp_v, v_dec_new)
