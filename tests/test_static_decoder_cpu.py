"""The host logic of bench.py's CUDA-graph generation mode, run eagerly on
the CPU: greedy decoding with a static KV cache whose step keeps the
position, the causal mask and the cache slot on the device (so that one
captured step can be replayed per token) gives Transformers' own greedy
tokens, also after a warm-up and a rewind (what the capture does before
the timed replays)."""

import pytest
import torch
from transformers import AutoModelForCausalLM, LlamaConfig, Qwen2Config

import bench


def _model(kind):
    common = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                  intermediate_size=128, vocab_size=97)
    config = LlamaConfig(**common) if kind == "llama" else Qwen2Config(**common, tie_word_embeddings=True)
    config._attn_implementation = "eager"
    torch.manual_seed(0)
    return AutoModelForCausalLM.from_config(config, dtype=torch.bfloat16).eval()


@pytest.mark.parametrize("kind", ["llama", "qwen2"])
@pytest.mark.parametrize("batch", [1, 3])
def test_static_steps_match_generate(kind, batch):
    model = _model(kind)
    prompt = torch.randint(97, (batch, 9), generator=torch.Generator().manual_seed(batch))
    new = 7
    with torch.no_grad():
        want = model.generate(prompt, max_new_tokens=new, min_new_tokens=new, do_sample=False, use_cache=True,
                              pad_token_id=0)[:, prompt.shape[1]:]
        first, step, rewind = bench.static_decoder(model, prompt, new, torch.device("cpu"))
        for _ in range(3):  # the warm-up before a capture writes positions the replays rewrite
            step()
        rewind()
        got = torch.cat([first[:, None]] + [step()[:, None] for _ in range(new - 1)], 1)
    assert torch.equal(got, want)
