"""The overlapped decode schedule (side stream, 2..4 rotating workspaces).

Every case compares against the uncompressed model bit for bit and against
the sequential schedule (the reference's: decode on the compute stream
right before each block)."""

import copy

import pytest
import torch
from torch import nn

from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_model_for_gpu
from neuralzip_b200.setup import NeuralZipSetup

pytestmark = pytest.mark.gpu


class Stack(nn.Module):
    def __init__(self, widths, dtype):
        super().__init__()
        self.layers = nn.ModuleList(
            nn.Sequential(nn.Linear(a, b, bias=False, dtype=dtype), nn.SiLU()) for a, b in zip(widths, widths[1:]))

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return x


def build(n_layers, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    widths = [512 + 64 * (i % 3) for i in range(n_layers + 1)]
    model = Stack(widths, dtype).eval()
    with torch.no_grad():
        for p in model.parameters():
            p.copy_((torch.randn(p.shape, generator=g) * 0.05).to(dtype))
    setup = NeuralZipSetup(chunk_size=64 << 10).build(dict(model.named_parameters()))
    return model, setup


def exact(a, b):
    return torch.equal(a.cpu().view(torch.uint8), b.cpu().view(torch.uint8))


@pytest.mark.parametrize("n_layers,depth,per_launch", [
    (2, 2, 1), (5, 2, 1), (6, 2, 1), (2, 3, 1), (5, 3, 1), (7, 4, 1), (3, 4, 1),
    (5, 2, 2), (6, 2, 3), (7, 3, 2), (4, 2, 4), (9, 2, 4)])
def test_overlap_matches_uncompressed_and_sequential(n_layers, depth, per_launch):
    model, setup = build(n_layers)
    x = torch.randn(4, model.layers[0][0].in_features, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    with torch.no_grad():
        expected = copy.deepcopy(model).cuda()(x.cuda()).cpu()
    sequential = copy.deepcopy(model)
    overlapped = copy.deepcopy(model)
    rt_seq = NeuralZipRuntime.attach(sequential, export_model_for_gpu(sequential, setup), device="cuda:0", overlap=False,
                                     blocks_per_launch=per_launch)
    rt_ovl = NeuralZipRuntime.attach(overlapped, export_model_for_gpu(overlapped, setup), device="cuda:0",
                                     prefetch_depth=depth, blocks_per_launch=per_launch)
    assert not rt_seq.overlap and rt_ovl.prefetch_depth == (depth if rt_ovl.overlap else 1)
    assert rt_ovl.overlap == (n_layers > per_launch)
    for ws in list(rt_ovl.workspaces.values()) + list(rt_seq.workspaces.values()):
        ws.view(torch.uint8).fill_(0xA5)
    with torch.no_grad():
        for _ in range(3):  # repeated forwards exercise the wrap-around prefetch
            assert exact(overlapped(x.cuda()), expected)
            assert exact(sequential(x.cuda()), expected)
    rt_ovl.check_status()


@pytest.mark.parametrize("depth,per_launch", [(2, 1), (3, 1), (2, 2), (2, 3)])
def test_out_of_order_blocks_and_materialize(depth, per_launch):
    model, setup = build(4)
    reference = copy.deepcopy(model).cuda()
    runtime = NeuralZipRuntime.attach(model, export_model_for_gpu(model, setup), device="cuda:0", prefetch_depth=depth,
                                      blocks_per_launch=per_launch)
    x = torch.randn(2, model.layers[0][0].in_features).to(torch.bfloat16).cuda()
    with torch.no_grad():
        model(x)  # leaves a prefetch of block 0 pending for the next forward
        for i in (2, 0, 3, 1, 1, 3, 2):
            layer_in = torch.randn(2, model.layers[i][0].in_features).to(torch.bfloat16).cuda()
            assert exact(model.layers[i](layer_in), reference.layers[i](layer_in))
    weights = dict(runtime.materialized_weights())
    for name, tensor in reference.named_parameters():
        assert exact(weights[name], tensor)
    with torch.no_grad():  # single-block decodes leave no unit marked whole
        assert exact(model(x), reference(x))
