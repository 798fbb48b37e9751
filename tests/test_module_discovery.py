"""Which weights become compressed, and where their decode hooks go.

The reference's module checks (scripts/_experiment_module_checks.py:185-224,
fixtures :27-60) run candidate discovery (neuralzip/gpu/inference.py:232-285)
over torchvision CNNs, a dilated/grouped/reflect-padded Conv2d, a
Sequential, a nested ModuleList model, a MultiheadAttention whose out_proj
the parent reads functionally, and GPT-2 (transformers Conv1D); with CUDA,
each model is compressed, its workspaces are filled with 0xA5, and weights
and outputs must equal the uncompressed model's bit for bit. The same cases
run here: discovery on the CPU, the compressed forward on the GPU.
"""

import copy
from collections import Counter

import pytest
import torch
from torch import nn
from transformers import GPT2Config, GPT2LMHeadModel
from transformers.pytorch_utils import Conv1D

from neuralzip_b200.gpu.inference import (
    NeuralZipRuntime,
    _binding_module,
    _gpu_candidates,
    _unique_candidates,
    export_model_for_gpu,
)
from neuralzip_b200.setup import NeuralZipSetup

torchvision = pytest.importorskip("torchvision")


class DepthwiseBlock(nn.Module):
    """A depthwise 3x3 convolution followed by a pointwise Linear."""

    def __init__(self, width=32):
        super().__init__()
        self.conv = nn.Conv2d(width, width, 3, padding=1, groups=width)
        self.linear = nn.Linear(width, width)

    def forward(self, x):
        return self.linear(self.conv(x).permute(0, 2, 3, 1)).permute(0, 3, 1, 2)


class NestedStages(nn.Module):
    """stages[0] holds a downsampling conv and a ModuleList of blocks: the
    blocks, not the stage, are the decode blocks."""

    def __init__(self, width=32):
        super().__init__()
        stage = nn.Module()
        stage.downsample = nn.Conv2d(width, width, 1)
        stage.blocks = nn.ModuleList([DepthwiseBlock(width), DepthwiseBlock(width)])
        self.stages = nn.ModuleList([stage])

    def forward(self, x):
        for stage in self.stages:
            x = stage.downsample(x)
            for block in stage.blocks:
                x = block(x)
        return x


class SelfAttention(nn.Module):
    """MultiheadAttention reads out_proj.weight itself (functional call),
    never calling the out_proj Linear."""

    def __init__(self, width=256, heads=4):
        super().__init__()
        self.before = nn.Linear(width, width)
        self.attention = nn.MultiheadAttention(width, heads, batch_first=True)

    def forward(self, x):
        x = self.before(x)
        return self.attention(x, x, x, need_weights=False)[0]


def _cases():
    models = torchvision.models
    return {
        "resnet18": (lambda: models.resnet18(weights=None), {"x": (1, 3, 224, 224)}),
        "convnext_tiny": (lambda: models.convnext_tiny(weights=None), {"x": (1, 3, 224, 224)}),
        "efficientnet_b0": (lambda: models.efficientnet_b0(weights=None), {"x": (1, 3, 224, 224)}),
        "conv2d": (lambda: nn.Conv2d(32, 32, 3, padding=2, dilation=2, groups=4, padding_mode="reflect"),
                   {"input": (1, 32, 16, 16)}),
        "sequential": (lambda: nn.Sequential(nn.Conv2d(3, 32, 3, padding=1), nn.ReLU(),
                                             nn.Conv2d(32, 32, 3, padding=1, groups=32)),
                       {"input": (1, 3, 16, 16)}),
        "nested": (NestedStages, {"x": (1, 32, 16, 16)}),
        "multihead_attention": (SelfAttention, {"x": (1, 17, 256)}),
        "gpt2": (lambda: GPT2LMHeadModel(GPT2Config(vocab_size=64, n_positions=32, n_embd=32, n_layer=2, n_head=4)),
                 {"input_ids": None}),
    }


CASES = _cases()
# Small models whose random init would leave few distinct exponents get a
# repeating pattern instead (as the reference checks do); for the attention
# model each weight module gets its own scale, so that blocks sharing the
# workspace must overwrite each other's bytes.
PATTERNED = ("conv2d", "sequential", "nested", "multihead_attention")


def _build(name):
    torch.manual_seed(7)
    factory, _ = CASES[name]
    model = factory().eval().to(torch.bfloat16)
    if name in PATTERNED:
        with torch.no_grad():
            for index, module in enumerate(model.modules(), 1):
                if isinstance(module, (nn.Linear, nn.Conv2d)):
                    base = torch.tensor([0.03125, 0.03125, -0.0625, -0.0625], dtype=torch.bfloat16)
                    if name == "multihead_attention":
                        base = base * index
                    reps = (module.weight.numel() + 3) // 4
                    module.weight.copy_(base.repeat(reps)[:module.weight.numel()].reshape(module.weight.shape))
    return model


def _inputs(name, device):
    _, shapes = CASES[name]
    g = torch.Generator().manual_seed(11)
    out = {}
    for key, shape in shapes.items():
        if key == "input_ids":
            out[key] = torch.arange(16).reshape(1, -1).to(device)
        else:
            out[key] = torch.randn(shape, generator=g).to(device=device, dtype=torch.bfloat16)
    return out


def _expected_weights(model):
    """Weights discovery must pick: every Linear/Conv2d/Conv1D weight that
    no other module shares."""
    uses = Counter(id(p) for _, p in model.named_parameters(remove_duplicate=False))
    return {
        (f"{n}.weight" if n else "weight"): m.weight.detach().clone()
        for n, m in model.named_modules(remove_duplicate=False)
        if isinstance(m, (nn.Linear, nn.Conv2d, Conv1D)) and uses[id(m.weight)] == 1
    }


def _bits(t):
    return t.detach().cpu().contiguous().reshape(-1).view(torch.uint8)


@pytest.mark.parametrize("name", sorted(CASES))
def test_discovery(name):
    model = _build(name)
    blocks, candidates = _gpu_candidates(model)
    candidates = _unique_candidates(model, candidates)
    expected = _expected_weights(model)
    assert expected
    assert sorted(c.tensor_name for c in candidates) == sorted(expected)
    # No block is nested inside another block.
    assert not any(a != b and b.startswith(a + ".") for a in blocks for b in blocks)
    if name == "nested":
        assert blocks == ("stages.0.downsample", "stages.0.blocks.0", "stages.0.blocks.1")
    if name == "gpt2":  # tied lm_head / wte is shared, so not a candidate
        assert "lm_head.weight" not in expected and any(n.endswith("c_attn.weight") for n in expected)
    if name == "multihead_attention":
        assert "attention.out_proj.weight" in expected


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_compressed_forward_is_bitwise(name):
    torch.backends.cudnn.benchmark = False
    torch.backends.cudnn.deterministic = True
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    model = _build(name)
    expected = _expected_weights(model)
    inputs = _inputs(name, "cuda:0")
    with torch.inference_mode():
        reference = copy.deepcopy(model).to("cuda:0")
        out = reference(**inputs)
        want = (out if isinstance(out, torch.Tensor) else out.logits).cpu()
        del reference
    uses = []
    if name == "multihead_attention":
        def parent_reads_projection(module, _args):
            assert torch.equal(_bits(module.out_proj.weight), _bits(expected["attention.out_proj.weight"]))
            uses.append(True)

        def projection_never_called(_module, _args):
            raise AssertionError("out_proj must be read by its parent, not called")

        model.attention.register_forward_pre_hook(parent_reads_projection)
        model.attention.out_proj.register_forward_pre_hook(projection_never_called)
    setup = NeuralZipSetup().build(model)
    exported = export_model_for_gpu(model, setup)
    assert exported.groups
    if name == "multihead_attention":  # the functional projection stays compressed
        assert any(g.block_name == "attention.out_proj" and g.codebook.vocab for g in exported.groups)
    for binding in exported.bindings:
        assert _binding_module(model, binding).weight.shape == binding.shape
    runtime = NeuralZipRuntime.attach(model, exported, device="cuda:0")
    for workspace in runtime.workspaces.values():
        workspace.view(torch.uint8).fill_(0xA5)
    restored = dict(runtime.materialized_weights())
    assert set(restored) == {b.tensor_name for b in exported.bindings}
    for key, tensor in restored.items():
        assert torch.equal(_bits(tensor), _bits(expected[key])), key
    with torch.inference_mode():
        for _ in range(2):
            for workspace in runtime.workspaces.values():
                workspace.view(torch.uint8).fill_(0xA5)
            out = model(**inputs)
            got = out if isinstance(out, torch.Tensor) else out.logits
            assert got.shape == want.shape and torch.equal(_bits(got), _bits(want)), name
    runtime.check_status()
    if name == "multihead_attention":
        assert len(uses) == 2
