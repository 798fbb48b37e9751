"""Host-to-host bulk decode (neuralzip_b200.gpu.bulk.HostDecoder): pieces
pipelined over three streams must leave every tensor bit-exact in pinned
host memory, for any piece count and across repeated calls."""

import pytest
import torch

from neuralzip_b200.gpu.bulk import HostDecoder
from neuralzip_b200.gpu.inference import export_tensors_for_gpu
from neuralzip_b200.setup import NeuralZipSetup

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("pieces", [1, 3, 16])
def test_host_decoder_round_trip(pieces):
    g = torch.Generator().manual_seed(7)
    named = {
        "w0": (torch.randn(512, 2048, generator=g) * 0.02).to(torch.bfloat16),
        "w1": (torch.randn(257, 999, generator=g) * 1.0).to(torch.bfloat16),
        "w2": (torch.randn(129, 513, generator=g) * 0.1).to(torch.float32),
        "w3": (torch.randn(256, 1024, generator=g) * 0.02).to(torch.float16),
    }
    setup = NeuralZipSetup(chunk_size=64 << 10).build(named)
    host = HostDecoder(export_tensors_for_gpu(named, setup), "cuda:0", pieces=pieces)
    assert 1 <= len(host.pieces) <= pieces
    for _ in range(2):
        for out in host.host_outputs.values():
            out.view(torch.uint8).fill_(0xA5)
        host.decode()
        host.synchronize()
        decoded = host.tensors()
        for name, tensor in named.items():
            assert torch.equal(decoded[name].view(torch.uint8), tensor.view(torch.uint8)), name
    host.check_status()
