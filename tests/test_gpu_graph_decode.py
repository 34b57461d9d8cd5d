"""CUDA-graph decode steps (llm.graph_decode.GraphedDecodeStep) against eager
decoding through the same CompressedAttentionKVCache: a tiny Llama, teacher-
forced on the eager run's greedy tokens for 150 steps (two tail flushes), for
both cache layouts.  Flushed tails are attended from a dequantised buffer
whose length the attention reads on the device, so the captured step stays
valid across a flush while the buffer has room; at this 128-token context it
is reserved for one tail, so the first flush keeps the capture and the
second (the buffer doubles) takes a new one: two captures in all.  The graphed step attends over the
whole tail with a mask where the eager one takes its filled slots, so fp32
sums round differently and the bf16 model turns that into ulp-level changes:
logits within 2e-2 of the eager step's (relative to the step's largest
logit, the bar of the eager hook test) and the same greedy token in at least
95% of the rows.  A wrong position or cache slot is far outside that."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout", ["rans", "compact"])
def test_graphed_steps_match_eager(layout):
    from transformers import LlamaConfig, LlamaForCausalLM

    from latticequant_b200.llm.compressed_attention import CompressedAttentionKVCache
    from latticequant_b200.llm.graph_decode import GraphedDecodeStep

    torch.manual_seed(2)
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=1024)
    model = LlamaForCausalLM(cfg).to("cuda", torch.bfloat16).eval()
    ids = torch.randint(0, 512, (2, 128), device="cuda")
    steps = 150
    with torch.no_grad():
        eager = CompressedAttentionKVCache(4, tail_tokens=64, layout=layout).bind(model)
        out = model(ids, past_key_values=eager, use_cache=True)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        toks, ref = [], []
        for _ in range(steps):
            toks.append(nxt)
            lg = model(nxt, past_key_values=eager, use_cache=True).logits[:, -1].float()
            ref.append(lg)
            nxt = lg.argmax(-1, keepdim=True)
        cache = CompressedAttentionKVCache(4, tail_tokens=64, layout=layout).bind(model)
        model(ids, past_key_values=cache, use_cache=True)
        g = GraphedDecodeStep(model, cache, keep_logits=True)
        worst, same = 0.0, 0
        for t in range(steps):
            g.step(toks[t])
            worst = max(worst, ((g.logits - ref[t]).abs().amax() / ref[t].abs().amax()).item())
            same += int((g.logits.argmax(-1) == ref[t].argmax(-1)).sum())
        g.release()
    assert g.captures == 2
    assert cache.get_seq_length(0) == 128 + steps == eager.get_seq_length(0)
    assert cache.flags() == 0
    assert worst < 2e-2, worst
    assert same >= 0.95 * steps * 2, same
