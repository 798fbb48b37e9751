"""The drop-in Python API: neuralzip(), the HF wrapper (format v3), stats and
the runtime on real modules. GPU tests restate the reference's end-to-end
kernel checks (scripts/_experiment_kernel_checks.py:124-198, :260-318)."""

import copy
import json
import tempfile
from pathlib import Path

import pytest
import torch
from torch import nn

import helpers as H
from neuralzip_b200 import neuralzip
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu import pretrained
from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_model_for_gpu
from neuralzip_b200.setup import NeuralZipSetup


def exact(a, b):
    return torch.equal(a.cpu().contiguous().view(torch.uint8), b.cpu().contiguous().view(torch.uint8))


def tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    config = LlamaConfig(vocab_size=32, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                         num_attention_heads=8, num_key_value_heads=2)
    config._attn_implementation = "eager"
    model = LlamaForCausalLM(config).bfloat16().eval()
    with torch.no_grad():
        for module in model.modules():
            if isinstance(module, nn.Linear):
                pattern = torch.tensor([0.25, 0.25, 0.5, 0.5], dtype=torch.bfloat16)
                module.weight.copy_(pattern.repeat(module.weight.numel() // 4).view_as(module.weight))
    return model


def test_v3_checkpoint_save_and_manual_decode_cpu():
    """save_pretrained writes storage v2 inside safetensors plus
    config.neuralzip (v3); decoding it restores every tensor bit for bit."""
    model = tiny_llama()
    expected = {name: tensor.clone() for name, tensor in model.state_dict().items()}
    setup = neuralzip.setup(model, chunk_size=8192)
    neuralzip(setup)
    with tempfile.TemporaryDirectory() as folder:
        model.save_pretrained(folder)
        config = json.loads((Path(folder) / "config.json").read_text())
        meta = config["neuralzip"]
        assert meta["format"] == "neuralzip" and meta["version"] == 3 and meta["encoding"] == "storage"
        assert model.neuralzip_stats.representation == "storage"
        assert model.neuralzip_stats.compressed_bytes < model.neuralzip_stats.raw_bytes
        blob, storage, resident = pretrained._Checkpoint.read(Path(folder))
        assert storage["version"] == 2 and not any(n.startswith(pretrained.PREFIX) for n in resident)
        state = pretrained._decoded_state(blob, storage, resident, meta.get("aliases", {}))
    assert set(state) >= set(expected)
    assert all(exact(state[name], tensor) for name, tensor in expected.items())


def test_export_stats_cpu():
    model = tiny_llama()
    setup = neuralzip.setup(model, chunk_size=8192)
    exported = export_model_for_gpu(model, setup)
    stats = pretrained._export_stats(model, exported, setup, 0.0)
    assert stats.representation == "gpu"
    unique = {pretrained._storage_key(t): t for t in model.state_dict().values()}
    assert stats.raw_bytes == sum(t.numel() * t.element_size() for t in unique.values())
    assert stats.compressed_bytes < stats.raw_bytes
    assert 0 < stats.stream_ratio < 1 and 0 < stats.exponent_ratio < 1


class PatternModel(nn.Module):
    def __init__(self, dtype):
        super().__init__()
        self.layers = nn.ModuleList([nn.Linear(257, 513, bias=False, dtype=dtype),
                                     nn.Linear(513, 17, bias=False, dtype=dtype)])

    def forward(self, inputs):
        for layer in self.layers:
            inputs = layer(inputs)
        return inputs


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_pattern_model_runtime(dtype):
    model = PatternModel(dtype).eval()
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(H.pattern_weights(p.numel(), dtype).view_as(p))
    named = dict(model.named_parameters())
    expected = {name: tensor.detach().clone() for name, tensor in named.items()}
    setup = NeuralZipSetup(chunk_size=8192).build(named)
    baseline = copy.deepcopy(model).cuda()
    inputs = torch.ones(1, 257, dtype=dtype, device="cuda")
    with torch.no_grad():
        output = baseline(inputs).cpu()
    del baseline
    key = next(iter(setup.chunk_codebooks))
    ids = list(setup.chunk_codebooks[key])
    ids[len(ids) // 2] = None  # a raw fragment between compressed chunks
    setup.chunk_codebooks[key] = tuple(ids)
    exported = export_model_for_gpu(model, setup)
    assert any(g.codebook_id == -1 for g in exported.groups)
    if DTYPES[dtype].exponent_stream is not None:
        assert any(g.codebook.vocab for g in exported.groups)
    stats = pretrained._export_stats(model, exported, setup, 0.0)
    assert stats.raw_bytes == sum(p.numel() * p.element_size() for p in expected.values())
    runtime = NeuralZipRuntime.attach(model, exported, device="cuda:0")
    assert all("weight" not in model.get_submodule(b.module_name)._parameters for b in exported.bindings)
    for workspace in runtime.workspaces.values():
        workspace.view(torch.uint8).fill_(0xA5)
    restored = dict(runtime.materialized_weights())
    assert all(exact(restored[name], tensor) for name, tensor in expected.items())
    for workspace in runtime.workspaces.values():
        workspace.view(torch.uint8).fill_(0xA5)
    with torch.no_grad():
        assert exact(model(inputs), output), "forward did not reconstruct exact weights"
    runtime.check_status()


@pytest.mark.gpu
def test_hf_wrapper_ordinary_load_and_compressed_reload():
    from transformers import LlamaForCausalLM

    reference = tiny_llama()
    expected_state = {name: tensor.clone() for name, tensor in reference.state_dict().items()}
    setup = neuralzip.setup(reference, chunk_size=8192)
    tokens = torch.arange(16, device="cuda").reshape(1, -1)
    with torch.no_grad():
        expected_logits = reference.cuda()(tokens, use_cache=False).logits.cpu()
    with tempfile.TemporaryDirectory(prefix="nzb200-hf-") as folder:
        original_path, compressed_path = Path(folder) / "original", Path(folder) / "compressed"
        reference.cpu().save_pretrained(original_path)
        neuralzip(setup, device="cuda:0")
        for source in (original_path, compressed_path):
            restored = LlamaForCausalLM.from_pretrained(source, dtype=torch.bfloat16, attn_implementation="eager")
            runtime = restored.neuralzip_runtime
            assert any(group.codebook.vocab for group in runtime.export.groups)
            assert restored.neuralzip_stats.representation in ("gpu", "storage")
            actual = dict(restored.state_dict())
            actual.update(runtime.materialized_weights())
            assert set(actual) == set(expected_state)
            assert all(exact(actual[name], tensor) for name, tensor in expected_state.items())
            for workspace in runtime.workspaces.values():
                workspace.view(torch.uint8).fill_(0xA5)
            with torch.no_grad():
                assert exact(restored(tokens, use_cache=False).logits.cpu(), expected_logits)
            if source == original_path:
                restored.save_pretrained(compressed_path)
                assert restored.neuralzip_stats.representation == "storage"


@pytest.mark.gpu
def test_tied_embedding_qwen2_logits_bitwise():
    """Config 3's architecture family (Qwen2, tied embeddings): the tied
    lm_head/embedding stays resident, every other linear weight is decoded
    per block, and logits equal the uncompressed model's bit for bit."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    config = Qwen2Config(vocab_size=128, hidden_size=128, intermediate_size=352, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=True)
    config._attn_implementation = "eager"
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(config).bfloat16().eval().cuda()
    tokens = torch.arange(24, device="cuda").reshape(1, -1)
    with torch.no_grad():
        expected = model(tokens, use_cache=False).logits.clone()
    setup = neuralzip.setup(model, chunk_size=8192)
    exported = export_model_for_gpu(model, setup)
    names = {b.tensor_name for b in exported.bindings}
    assert "lm_head.weight" not in names and "model.embed_tokens.weight" not in names
    runtime = NeuralZipRuntime.attach(model, exported, device="cuda:0")
    for workspace in runtime.workspaces.values():
        workspace.view(torch.uint8).fill_(0xA5)
    with torch.no_grad():
        assert exact(model(tokens, use_cache=False).logits, expected)
    runtime.check_status()
