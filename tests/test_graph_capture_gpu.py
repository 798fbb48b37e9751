"""A compressed model's one-token step captured in a CUDA graph.

The runtime's forward pre-hooks enqueue the decode launches (and the
side-stream prefetches of the overlapped schedule) on the capturing stream,
so the graph holds them. Replayed token after token, the compressed model
must generate exactly the uncompressed model's greedy tokens, and the
workspaces must be rewritten by each replay (they are filled with 0xA5
before the replays)."""

import copy

import pytest
import torch
from transformers import AutoModelForCausalLM, LlamaConfig

import bench
from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_model_for_gpu
from neuralzip_b200.setup import NeuralZipSetup

pytestmark = pytest.mark.gpu


def _replayed_tokens(model, prompt, new_tokens, fill=None):
    device = prompt.device
    stream = torch.cuda.current_stream(device)
    with torch.no_grad():
        first, step, rewind = bench.static_decoder(model, prompt, new_tokens, device)
        side = torch.cuda.Stream(device=device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step()
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            nxt = step()
        rewind()
        if fill is not None:
            fill()
        steps = []
        for _ in range(new_tokens - 1):
            graph.replay()
            steps.append(nxt.clone())
        torch.cuda.synchronize(device)
        del graph
    return torch.cat([first[:, None], torch.stack(steps, 1)], 1)


@pytest.mark.parametrize("blocks_per_launch", [1, "auto"])
def test_captured_step_matches_uncompressed(blocks_per_launch):
    config = LlamaConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                         intermediate_size=512, vocab_size=512)
    config._attn_implementation = "eager"
    torch.manual_seed(0)
    with torch.device("cuda:0"):
        model = AutoModelForCausalLM.from_config(config, dtype=torch.bfloat16).eval()
    uncompressed = copy.deepcopy(model)
    runtime = NeuralZipRuntime.attach(model, export_model_for_gpu(model, NeuralZipSetup().build(model)),
                                      device="cuda:0", blocks_per_launch=blocks_per_launch)
    assert runtime.overlap == (blocks_per_launch == 1)
    prompt = torch.randint(512, (2, 12), generator=torch.Generator().manual_seed(1)).to("cuda:0")

    def fill():
        for workspace in runtime.workspaces.values():
            workspace.view(torch.uint8).fill_(0xA5)

    want = _replayed_tokens(uncompressed, prompt, 10)
    got = _replayed_tokens(model, prompt, 10, fill)
    assert torch.equal(got, want)
    runtime.check_status()
