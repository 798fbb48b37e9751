"""Bulk decode split across GPUs of one node, one process per GPU.

Every group (one source chunk) decodes on its own: it needs only its
bitstream, sub-stream lengths, tile offsets, raw lanes and decode table
(neuralzip/gpu/cuda/decode.cu:335-359 reads the same per-group inputs). So a
checkpoint is split into contiguous ranges of groups, one per rank, balanced
by decoded bytes; each rank uploads and decodes only its range, from and
into its own HBM, and no data crosses between ranks.

A rank's groups are rebased into a workspace of their own: each tensor the
range touches becomes one piece (a contiguous run of its elements), and the
pieces of a block lie side by side, 128-byte aligned.
"""

from __future__ import annotations

import bisect
from collections import defaultdict
from dataclasses import dataclass, replace

from neuralzip_b200.gpu.inference import LinearWeightBinding, NeuralZipModelExport, _aligned


@dataclass(frozen=True)
class ShardPiece:
    """The part of one tensor that a rank decodes."""

    block_name: str
    tensor_name: str
    tensor_offset: int      # first element of the piece within the tensor
    numel: int
    workspace_offset: int   # where the piece starts in the rank's block workspace


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    export: NeuralZipModelExport
    pieces: tuple[ShardPiece, ...]
    decoded_bytes: int


def group_bytes(group):
    return group.encoded.numel * group.encoded.dtype.element_size


def partition(groups, world):
    """[start, end) group ranges for `world` ranks: contiguous in export
    order, each boundary at the group edge nearest to an equal split of the
    decoded bytes."""
    if world < 1:
        raise ValueError("world must be at least 1.")
    prefix = [0]
    for group in groups:
        prefix.append(prefix[-1] + group_bytes(group))
    total = prefix[-1]
    bounds = [0]
    for k in range(1, world):
        target = total * k / world
        j = bisect.bisect_left(prefix, target)
        if j > 0 and (j == len(prefix) or target - prefix[j - 1] <= prefix[j] - target):
            j -= 1
        bounds.append(max(bounds[-1], min(j, len(groups))))
    bounds.append(len(groups))
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def shard_export(export, rank, world):
    """The groups of `rank` out of `world`, rebased into the rank's own
    workspace (see the module docstring)."""
    if not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world).")
    start, end = partition(export.groups, world)[rank]
    mine = export.groups[start:end]
    # Pieces: a contiguous run of each tensor's groups.
    runs = {}
    for group in mine:
        full = group.bindings[0]
        offset = group.workspace_offset - full.workspace_offset
        key = (group.block_name, full.tensor_name)
        first, count = runs.get(key, (offset, 0))
        runs[key] = (first, count + group.encoded.numel)
    cursor = defaultdict(int)
    pieces, bindings = {}, {}
    for group in mine:
        full = group.bindings[0]
        key = (group.block_name, full.tensor_name)
        if key in pieces:
            continue
        spec = group.encoded.dtype
        ws_key = (group.block_name, spec.torch_dtype)
        base = _aligned(cursor[ws_key], spec.element_size)
        first, count = runs[key]
        pieces[key] = ShardPiece(group.block_name, full.tensor_name, first, count, base)
        bindings[key] = LinearWeightBinding(full.module_name, full.tensor_name, (count,), count, base)
        cursor[ws_key] = base + count
    rebased = []
    for group in mine:
        full = group.bindings[0]
        key = (group.block_name, full.tensor_name)
        piece = pieces[key]
        offset = group.workspace_offset - full.workspace_offset
        rebased.append(replace(group, bindings=(bindings[key],),
                               workspace_offset=piece.workspace_offset + offset - piece.tensor_offset))
    return Shard(rank, world, NeuralZipModelExport(tuple(rebased)), tuple(pieces.values()),
                 sum(group_bytes(g) for g in mine))
