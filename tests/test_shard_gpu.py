"""Sharded bulk decode on the GPU: each rank's shard (contiguous,
byte-balanced groups rebased into its own workspace) decodes through the
runtime to exactly its pieces of the original tensors. All ranks are run
one after another on cuda:0; there is no exchange between them."""

import pytest
import torch

from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_tensors_for_gpu
from neuralzip_b200.gpu.shard import shard_export
from neuralzip_b200.setup import NeuralZipSetup

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3, 8])
def test_each_shard_decodes_its_pieces(world):
    g = torch.Generator().manual_seed(5)
    named = {
        "w0": (torch.randn(512, 2048, generator=g) * 0.02).to(torch.bfloat16),
        "w1": (torch.randn(300, 1000, generator=g) * 1.0).to(torch.bfloat16),
        "w2": (torch.randn(129, 513, generator=g) * 0.1).to(torch.float32),
        "w3": (torch.randn(256, 1024, generator=g) * 0.02).to(torch.float16),
    }
    setup = NeuralZipSetup(chunk_size=64 << 10).build(named)
    export = export_tensors_for_gpu(named, setup)
    covered = {name: torch.zeros(t.numel(), dtype=torch.int32) for name, t in named.items()}
    for rank in range(world):
        shard = shard_export(export, rank, world)
        if not shard.export.groups:
            continue
        runtime = NeuralZipRuntime(None, shard.export, "cuda:0")
        for block in shard.export.block_order:
            runtime._decode_block(block)
        torch.cuda.synchronize()
        runtime.check_status()
        for piece in shard.pieces:
            t = named[piece.tensor_name]
            ws = runtime.workspaces[t.dtype]
            got = ws[piece.workspace_offset:piece.workspace_offset + piece.numel].cpu()
            want = t.reshape(-1)[piece.tensor_offset:piece.tensor_offset + piece.numel]
            assert torch.equal(got.view(torch.uint8), want.view(torch.uint8)), (rank, piece)
            covered[piece.tensor_name][piece.tensor_offset:piece.tensor_offset + piece.numel] += 1
    assert all(bool((c == 1).all()) for c in covered.values())
