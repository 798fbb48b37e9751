"""Host logic of the multi-GPU bulk decode, run as two gloo ranks on CPU.

Each rank builds the same export, takes its shard (contiguous, byte-balanced
groups, no exchange), and checks on the CPU (oracle tile reader) that its
pieces decode to its part of the original tensors. The ranks then gather
what they own: every element of every tensor must belong to exactly one
rank. bench.py's max-over-ranks timing reduction runs on the same group."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tensors():
    g = torch.Generator().manual_seed(3)
    return {
        "a": (torch.randn(64, 2048, generator=g) * 0.02).to(torch.bfloat16),
        "b": (torch.randn(40, 1000, generator=g) * 1.0).to(torch.bfloat16),
        "c": (torch.randn(33, 517, generator=g) * 0.1).to(torch.float32),
        "d": (torch.randn(96, 1024, generator=g) * 0.02).to(torch.float16),
    }


def _worker(rank, world, port, failures):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        import bench
        import helpers as H
        from neuralzip_b200.gpu.inference import export_tensors_for_gpu
        from neuralzip_b200.gpu.shard import shard_export
        from neuralzip_b200.setup import NeuralZipSetup
        from oracle import oracle as O

        dist.init_process_group("gloo", rank=rank, world_size=world)
        named = _tensors()
        setup = NeuralZipSetup(chunk_size=8192).build(named)
        export = export_tensors_for_gpu(named, setup)
        shard = shard_export(export, rank, world)
        # Decode this rank's groups on the CPU into its own workspace.
        workspaces = {}
        for group in shard.export.groups:
            spec = group.encoded.dtype
            ws = workspaces.setdefault(spec.torch_dtype, {})
            sym = group.encoded.symbols
            if group.codebook.max_bits:
                sel = O.tile_decode(np.frombuffer(sym.bitstream, dtype=np.uint32),
                                    np.frombuffer(sym.lane_bits, np.uint16), np.asarray(sym.tile_offsets),
                                    group.encoded.numel, group.codebook.code_lengths, group.codebook.code_values,
                                    group.codebook.vocab)
            else:
                sel = np.frombuffer(sym.bitstream, dtype=np.uint8)
            lanes = [np.frombuffer(s, np.uint8) if i != spec.gpu_stream else sel
                     for i, s in enumerate(group.encoded.streams)]
            raw = O.restore(lanes, spec)
            ws[group.workspace_offset] = raw
        owned = []
        for piece in shard.pieces:
            t = named[piece.tensor_name]
            es = t.element_size()
            expected = t.reshape(-1)[piece.tensor_offset:piece.tensor_offset + piece.numel].view(torch.uint8)
            ws = workspaces[t.dtype]
            got = b"".join(bytes(ws[off]) for off in sorted(ws)
                           if piece.workspace_offset <= off < piece.workspace_offset + piece.numel)
            assert got == expected.numpy().tobytes(), piece
            assert piece.workspace_offset * es % 128 == 0
            owned.append((piece.tensor_name, piece.tensor_offset, piece.numel))
        everything = [None] * world
        dist.all_gather_object(everything, (owned, shard.decoded_bytes))
        cover = {name: np.zeros(t.numel(), dtype=np.int32) for name, t in named.items()}
        for ranges, _ in everything:
            for name, start, n in ranges:
                cover[name][start:start + n] += 1
        assert all((c == 1).all() for c in cover.values()), "each element on exactly one rank"
        sizes = [b for _, b in everything]
        biggest = max(g.encoded.numel * g.encoded.dtype.element_size for g in export.groups)
        assert max(sizes) - min(sizes) <= 2 * biggest, sizes
        assert bench.max_over_ranks(float(rank + 1), world) == float(world)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # reported to the parent process
        failures.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.timeout(600)
def test_two_rank_shards_cover_everything_once():
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(540)
    for p in procs:
        if p.is_alive():
            p.kill()
    messages = []
    while not failures.empty():
        messages.append(failures.get())
    assert not messages, messages
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_partition_is_balanced_and_contiguous():
    from neuralzip_b200.gpu.shard import partition

    class G:
        def __init__(self, n):
            self.encoded = type("E", (), {"numel": n, "dtype": type("D", (), {"element_size": 2})})

    groups = [G(n) for n in [131072] * 37 + [5000, 131072, 77]]
    for world in (1, 2, 3, 4, 8):
        ranges = partition(groups, world)
        assert ranges[0][0] == 0 and ranges[-1][1] == len(groups)
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        loads = [sum(g.encoded.numel for g in groups[s:e]) for s, e in ranges]
        assert max(loads) - min(loads) <= 2 * 131072
    assert partition(groups[:3], 8)[-1][1] == 3
