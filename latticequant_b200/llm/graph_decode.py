"""Decode steps of a transformers causal LM over a CompressedAttentionKVCache,
captured once in a CUDA graph and replayed.

Eager decoding pays the Python and launch cost of every layer's projections,
cache update and attention each step (about a millisecond per layer for an
8B-shaped model), which caps tokens/s once the fused attention is fast.  The
step here is recorded with torch.cuda.graph and replayed: the token ids, the
position ids and the cache's tail slot are static device tensors the captured
step advances itself, and the cache's host bookkeeping runs after each replay
(CompressedAttentionKVCache.enter_graph / graph_advance).  When the tails are
full (every `tail_tokens` tokens) they are encoded eagerly, as an eager
update() would; the captured step is replayed on (its tail slot back at 0)
when the flush left every buffer it reads in place (the compact layout's
dequantised tails go to a buffer whose length the attention reads on the
device), and captured again when it did not (a new or recoded part, a buffer
that had to grow).  The reference decodes eagerly (llm/e2e_eval.py:212); the
tokens are the same greedy tokens.
"""
from __future__ import annotations

import time
from typing import Optional

import torch

from .compressed_attention import CompressedAttentionKVCache


class GraphedDecodeStep:
    """Greedy decode steps of `model` (bound to `cache`) from a CUDA graph.

    step(ids) takes the (B, 1) ids of the current tokens on the device and
    returns the (B, 1) ids of the next ones (a static tensor, overwritten by
    the next step); `logits` holds the step's last-position logits."""

    def __init__(self, model, cache: CompressedAttentionKVCache, keep_logits: bool = False):
        self.model, self.cache, self.keep_logits = model, cache, keep_logits
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.captures = 0
        self.capture_s = 0.0  # host wall time spent in captures (warm-up run included)

    def _body(self):
        out = self.model(self.s_ids, past_key_values=self.cache, position_ids=self.s_pos,
                         cache_position=self.s_cpos, use_cache=True, logits_to_keep=1)
        lg = out.logits[:, -1]
        if self.keep_logits:
            self.logits.copy_(lg)
        self.s_out.copy_(lg.argmax(-1, keepdim=True))
        self.s_pos.add_(1)
        self.s_cpos.add_(1)
        self.s_idx.add_(1)

    def _capture(self, ids: torch.Tensor):
        t0 = time.perf_counter()
        c, dev = self.cache, ids.device
        B = ids.shape[0]
        pos = c.get_seq_length(0)
        n_tail = c._state[0].n_tail
        self.s_ids = ids.clone()
        self.s_pos = torch.full((B, 1), pos, dtype=torch.long, device=dev)
        self.s_cpos = torch.tensor([pos], dtype=torch.long, device=dev)
        self.s_idx = torch.tensor([n_tail], dtype=torch.long, device=dev)
        self.s_out = torch.empty(B, 1, dtype=torch.long, device=dev)
        self.sig = c.graph_signature()
        if self.keep_logits:
            self.logits = torch.empty(B, self.model.config.vocab_size, dtype=torch.float32, device=dev)
        c.enter_graph(self.s_idx)
        # one eager run of the step on a side stream (kernels, workspaces and
        # prepared attention ops come into being), then the counters back
        saved = (self.s_pos.clone(), self.s_cpos.clone(), self.s_idx.clone())
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.s_pos.copy_(saved[0])
        self.s_cpos.copy_(saved[1])
        self.s_idx.copy_(saved[2])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self._body()
        self.captures += 1
        self.capture_s += time.perf_counter() - t0

    def release(self):
        """Drop the captured graph (before destroy_process_group when the step
        holds collectives)."""
        self.graph = None
        self.cache.exit_graph()

    @torch.no_grad()
    def step(self, ids: torch.Tensor) -> torch.Tensor:
        c = self.cache
        if self.graph is not None and c.tail_full():
            c.flush_tails()
            if c.graph_signature() == self.sig:
                self.s_idx.zero_()  # the same buffers: replay on from tail slot 0
            else:
                self.release()
        if self.graph is None:
            c.flush_tails()
            if any(st.tail_raw_k is None for st in c._state):  # the first decode step runs eagerly
                out = self.model(ids, past_key_values=c, use_cache=True, logits_to_keep=1)
                lg = out.logits[:, -1]
                if self.keep_logits:
                    self.logits = lg.float()
                return lg.argmax(-1, keepdim=True)
            self._capture(ids)
        self.s_ids.copy_(ids)
        self.graph.replay()
        c.graph_advance(1)
        return self.s_out
