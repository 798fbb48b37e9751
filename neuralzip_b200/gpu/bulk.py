"""Host-to-host bulk decode: compressed arrays in pinned host memory in,
decoded weights in pinned host memory out.

This is the path behind ``materialized_weights``-style uses, where the
reference decodes on the CPU (neuralzip/native/decode_queue.h:1-113, one
chunk per worker). Here the export is cut into pieces of consecutive groups,
balanced by decoded bytes, and three CUDA streams pipeline them: piece i+1 is
copied host->device while piece i decodes and piece i-1 is copied
device->host, so the two copy directions and the decode overlap. Each
piece's groups are contiguous both in the compressed arena and, per dtype,
in the output workspace, so every copy is one cudaMemcpyAsync.
"""

from __future__ import annotations

from collections import defaultdict

import torch

from neuralzip_b200.gpu.inference import NeuralZipRuntime
from neuralzip_b200.gpu.shard import partition


class HostDecoder:
    """Pipelined decode of one export from and to pinned host memory.

    ``host_arena`` holds the compressed arrays (filled from the export; a
    caller may refill it, e.g. from storage, before each ``decode``) and
    ``host_outputs[dtype]`` receives the decoded element words at the same
    offsets as the runtime's workspace. ``decode`` only enqueues work;
    ``synchronize`` waits for it."""

    def __init__(self, export, device, *, pieces=8):
        if len(export.block_order) != 1:
            raise ValueError("HostDecoder takes a single-block export (export_tensors_for_gpu).")
        self.device = torch.device(device)
        self.runtime = NeuralZipRuntime(None, export, self.device, overlap=False)
        rt = self.runtime
        block = export.block_order[0]
        items = rt._groups_by_block[block]
        self.host_arena = torch.empty(rt.arena.numel(), dtype=torch.uint8, pin_memory=True)
        self.host_arena.copy_(torch.from_numpy(rt.arena_host))
        self.host_outputs = {dtype: torch.empty(ws.numel(), dtype=dtype, pin_memory=True)
                             for dtype, ws in rt.workspaces.items()}
        self.pieces = []
        for start, end in partition([item.group for item in items], max(1, int(pieces))):
            if start == end:
                continue
            chunk = items[start:end]
            # A single block's items are the export's groups in order.
            lo, hi = rt.arena_ranges[start][0], rt.arena_ranges[end - 1][1]
            outputs = defaultdict(lambda: [None, 0])
            for item in chunk:
                dtype = item.group.encoded.dtype.torch_dtype
                begin = item.group.workspace_offset
                span = outputs[dtype]
                span[0] = begin if span[0] is None else min(span[0], begin)
                span[1] = max(span[1], begin + item.group.encoded.numel)
            self.pieces.append((lo, hi, dict(outputs), rt._prepare(chunk)))
        self.h2d = torch.cuda.Stream(device=self.device)
        self.compute = torch.cuda.Stream(device=self.device)
        self.d2h = torch.cuda.Stream(device=self.device)
        n = len(self.pieces)
        self._loaded = [torch.cuda.Event() for _ in range(n)]
        self._decoded = [torch.cuda.Event() for _ in range(n)]
        self._done = torch.cuda.Event()
        self.h2d_bytes = int(self.host_arena.numel())
        self.d2h_bytes = int(sum(t.numel() * t.element_size() for t in self.host_outputs.values()))

    def decode(self, stream=None):
        """Enqueues H2D, decode and D2H of every piece; the work starts after
        what is already on `stream` (default: the current stream) and `stream`
        waits for its end."""
        rt = self.runtime
        after = stream or torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(after)
        for s in (self.h2d, self.compute, self.d2h):
            s.wait_event(start)
        for i, (lo, hi, outputs, batches) in enumerate(self.pieces):
            with torch.cuda.stream(self.h2d):
                rt.arena[lo:hi].copy_(self.host_arena[lo:hi], non_blocking=True)
                self._loaded[i].record(self.h2d)
            self.compute.wait_event(self._loaded[i])
            rt._decoder.decode_batches(batches, self.compute)
            self._decoded[i].record(self.compute)
            self.d2h.wait_event(self._decoded[i])
            with torch.cuda.stream(self.d2h):
                for dtype, (begin, end) in outputs.items():
                    self.host_outputs[dtype][begin:end].copy_(rt.workspaces[dtype][begin:end], non_blocking=True)
        self._done.record(self.d2h)
        after.wait_event(self._done)

    def synchronize(self):
        self._done.synchronize()

    def check_status(self):
        for _, _, _, batches in self.pieces:
            for prepared in batches:
                self.runtime._decoder.check_status(prepared)

    def tensors(self):
        """Decoded tensors as views of the pinned host outputs, by name."""
        out = {}
        for item in self.runtime._groups_by_block[self.runtime.export.block_order[0]]:
            for binding in item.group.bindings:
                if binding.tensor_name not in out:
                    dtype = item.group.encoded.dtype.torch_dtype
                    flat = self.host_outputs[dtype][binding.workspace_offset:binding.workspace_offset + binding.numel]
                    out[binding.tensor_name] = flat.view(binding.shape)
        return out
