"""Compressed GPU representation and the per-block runtime.

Mirrors the public surface of neuralzip/gpu/inference.py: ``GPUCodebook``,
``GPUEncodedSymbols``, ``GPUEncoded``, ``encode_gpu_native``,
``LinearWeightBinding``, ``GPUWeightGroup``, ``NeuralZipModelExport``,
``export_model_for_gpu`` and ``NeuralZipRuntime`` (attach, workspaces,
``_decode_block``, ``materialized_weights``), with the same semantics for
candidate discovery (inference.py:219-285), chunk grouping (one group per
source chunk, raw fragments included, a tensor skipped when its fragments are
not smaller than raw, inference.py:288-336) and weight binding.

The encoded form is the tile layout of include/nz_b200.h rather than the
reference's segment/gap layout (the GPU layout is an in-memory format that
is never persisted). The runtime uploads every group into one device arena
with a single host-to-device copy instead of one small tensor per array per
group (inference.py:393-432), and decodes a block with one launch per dtype
instead of one per (layout, staging) pair.
"""

from __future__ import annotations

import functools
from collections import defaultdict
from dataclasses import dataclass, field
import weakref

import numpy as np
import torch
from torch import nn

from neuralzip_b200 import _native
from neuralzip_b200.dtypes import DTYPES, DTypeSpec
from neuralzip_b200.gpu import decoder as gpu_decoder
from neuralzip_b200.utils import _stream_chunk_size

try:  # transformers is optional for the core path
    from transformers.pytorch_utils import Conv1D
except Exception:  # pragma: no cover - exercised only without transformers
    class Conv1D(nn.Module):  # type: ignore[no-redef]
        pass

RUNTIME_ATTRIBUTE = "neuralzip_runtime"
_GPU_WEIGHT_TYPES = (nn.Linear, nn.Conv2d, Conv1D)
ARENA_ALIGN = 128
WORKSPACE_ALIGN_BYTES = 128


@dataclass(frozen=True)
class GPUCodebook:
    """Code lengths/values of one codebook and its tile decode table.

    Validation mirrors neuralzip/gpu/inference.py:28-75: singleton codes are
    at most 12 bits, pair (mixed) codes at most 56, the alphabet must match
    the pair vocabulary, and every 12-bit prefix must decode."""

    code_lengths: tuple[int, ...]
    code_values: tuple[int, ...]
    vocab: bytes = b""
    max_bits: int = field(init=False)
    decode_lut: object = field(init=False, repr=False, compare=False)
    native: object = field(init=False, repr=False, compare=False)

    def __post_init__(self):
        longest = max(self.code_lengths, default=0)
        if longest > (56 if self.vocab else 12):
            raise ValueError("The GPU codebook exceeds its decoder's code-length limit.")
        object.__setattr__(self, "max_bits", min(12, longest))
        if not longest:
            object.__setattr__(self, "decode_lut", ())
            object.__setattr__(self, "native", None)
            return
        if len(self.code_lengths) != 256 + len(self.vocab) // 2:
            raise ValueError("The GPU alphabet does not match its pair vocabulary.")
        if len(self.code_values) != len(self.code_lengths):
            raise ValueError("Code values must match code lengths.")
        try:
            book = _native.NativeCodebook(bytes(self.code_lengths), self.code_values, bytes(self.vocab))
        except ValueError as error:
            if "prefix" in str(error) or "cover" in str(error):
                raise ValueError("The Huffman codebook does not cover every prefix.") from error
            raise
        object.__setattr__(self, "native", book)
        object.__setattr__(self, "decode_lut", book.lut())

    @property
    def table_words(self):
        """Words of the decode table the kernel stages (entries, plus the
        long-code tables when a code is longer than 12 bits)."""
        if self.native is None:
            return 0
        return (self.native.table_words + 3) // 4 * 4


@dataclass(frozen=True)
class GPUEncodedSymbols:
    """Huffman-coded selected lane of one group in the tile layout.

    ``bitstream``: little-endian 32-bit words, bit 31 earliest, zero padded;
    ``lane_bits``: uint16 bit length per 256-element sub-stream;
    ``tile_offsets``: bit offset of each 8192-element tile. A raw fragment
    keeps its bytes in ``bitstream`` with empty sync metadata
    (neuralzip/gpu/inference.py:319-324)."""

    bitstream: bytes
    bit_length: int
    symbol_count: int
    lane_bits: bytes
    tile_offsets: tuple[int, ...]

    @property
    def compressed_bytes(self):
        return len(self.bitstream) + len(self.lane_bits) + 4 * len(self.tile_offsets)

    # Names of the reference layout's sync metadata.
    @property
    def packed_gaps(self):
        return self.lane_bits

    @property
    def output_positions(self):
        return self.tile_offsets


@dataclass(frozen=True)
class GPUEncoded:
    dtype: DTypeSpec
    numel: int
    streams: tuple  # Indexed by byte-lane ID: raw lane bytes (bytes-like) or GPUEncodedSymbols.

    @property
    def raw_bytes(self):
        return self.numel * self.dtype.element_size

    @property
    def compressed_bytes(self):
        return sum(s.compressed_bytes if isinstance(s, GPUEncodedSymbols) else len(s) for s in self.streams)

    @property
    def symbols(self):
        (symbols,) = (s for s in self.streams if isinstance(s, GPUEncodedSymbols))
        return symbols


@functools.lru_cache(maxsize=4096)
def codebook_from_header(header, vocab=b""):
    """GPUCodebook of a serialized table (Huff0 header or "NZM1" mixed
    header), via export_code_table semantics (binding_helpers.h:103-123)."""
    lengths, values, _longest = _native.export_code_table(header, max_bits=56, vocab=vocab)
    return GPUCodebook(tuple(lengths), values, bytes(vocab))


def _dtype_struct(spec, stream_id):
    if stream_id != spec.gpu_stream:
        raise ValueError("GPU stream_id does not match the dtype's coded lane.")
    return _native.dtype_struct(spec.element_size, spec.bit_reorder, spec.mantissa_bits,
                                spec.exponent_bits, stream_id)


def encode_with_codebook(raw, book, *, dtype, stream_id):
    """Packs raw element bytes with a GPUCodebook into a GPUEncoded."""
    dt = _dtype_struct(dtype, stream_id)
    bits, lens, tile_off, lanes, bit_length = _native.pack_chunk(book.native, raw, dt)
    numel = len(raw) // dtype.element_size
    streams = [lane.tobytes() if lane is not None else None for lane in lanes]
    streams[stream_id] = GPUEncodedSymbols(bits.tobytes(), int(bit_length), numel, lens.tobytes(),
                                           tuple(int(x) for x in tile_off))
    return GPUEncoded(dtype, numel, tuple(streams))


def encode_gpu_native(raw, codebook_header, *, dtype, stream_id, vocab=b"", codebook_handle=None):
    """Encodes one chunk's selected lane with a serialized codebook
    (neuralzip/gpu/inference.py:111-131). ``codebook_handle`` may be a
    GPUCodebook to skip re-reading the header."""
    raw = bytes(raw)
    book = codebook_handle if isinstance(codebook_handle, GPUCodebook) else codebook_from_header(
        bytes(codebook_header), bytes(vocab))
    return encode_with_codebook(raw, book, dtype=dtype, stream_id=stream_id)


def encode_raw_fragment(raw, *, dtype, stream_id):
    """Raw fragment: every lane stored as bytes, the selected one wrapped."""
    raw = _as_bytes_array(raw)
    lanes = _native.split_lanes(raw, _dtype_struct(dtype, stream_id))
    numel = len(raw) // dtype.element_size
    streams = [_view(lane) for lane in lanes]
    streams[stream_id] = GPUEncodedSymbols(streams[stream_id], 8 * numel, numel, b"", ())
    return GPUEncoded(dtype, numel, tuple(streams))


@dataclass(frozen=True)
class LinearWeightBinding:
    module_name: str
    tensor_name: str
    shape: tuple[int, ...]
    numel: int
    workspace_offset: int


@dataclass(frozen=True)
class GPUWeightGroup:
    block_name: str
    codebook_id: int
    codebook: GPUCodebook
    encoded: GPUEncoded
    bindings: tuple[LinearWeightBinding, ...]
    workspace_offset: int

    @property
    def layout(self):
        dtype = self.encoded.dtype
        return (
            dtype.element_size, bool(dtype.bit_reorder), dtype.mantissa_bits, dtype.exponent_bits,
            dtype.gpu_stream, bool(self.codebook.vocab), max(self.codebook.code_lengths, default=0) > 32,
        )


@dataclass(frozen=True)
class NeuralZipModelExport:
    groups: tuple[GPUWeightGroup, ...]

    @property
    def block_order(self):
        return tuple(dict.fromkeys(group.block_name for group in self.groups))

    @property
    def bindings(self):
        return tuple(dict.fromkeys(binding for group in self.groups for binding in group.bindings))

    @property
    def workspace_sizes(self):
        sizes = {}
        for group in self.groups:
            dtype = group.encoded.dtype.torch_dtype
            sizes[dtype] = max(sizes.get(dtype, 0), group.workspace_offset + group.encoded.numel)
        return sizes


@dataclass(frozen=True)
class _Candidate:
    block_name: str
    module_name: str
    tensor_name: str
    parameter: nn.Parameter = field(repr=False, compare=False)


def _join(parent, child):
    return f"{parent}.{child}" if parent and child else parent or child


def _decode_hook_module(model, block_name):
    """The module whose forward pre-hook decodes `block_name`. A
    MultiheadAttention reads out_proj.weight itself without calling the
    Linear, so that block's hook goes on the attention module."""
    parent_name, _, child_name = block_name.rpartition(".")
    if child_name == "out_proj" and isinstance(model.get_submodule(parent_name), nn.MultiheadAttention):
        return model.get_submodule(parent_name)
    return model.get_submodule(block_name)


def _linears_only_in_nested_lists(element, path):
    """True when `element` (an item of a ModuleList) holds ModuleLists of
    its own and every Linear inside it sits inside an item of one of them:
    then the element is only a container and its inner items are the
    blocks."""
    inner = tuple(
        _join(_join(path, name), item) + "."
        for name, module in element.named_modules(remove_duplicate=False)
        if isinstance(module, nn.ModuleList) and module is not element
        for item, child in module._modules.items() if child is not None
    )
    if not inner:
        return False
    return all((_join(path, name) + ".").startswith(inner)
               for name, module in element.named_modules(remove_duplicate=False) if isinstance(module, nn.Linear))


def _list_blocks(module, path=""):
    """Decode blocks under `module`, in module order: each item of a
    ModuleList met on the way down is a block, unless it is only a
    container of further ModuleLists (then the search continues inside
    it); nothing inside a block is searched."""
    blocks = []
    for name, child in module._modules.items():
        if child is None:
            continue
        child_path = _join(path, name)
        if isinstance(child, nn.ModuleList):
            for item, element in child._modules.items():
                if element is None:
                    continue
                item_path = _join(child_path, item)
                if _linears_only_in_nested_lists(element, item_path):
                    blocks.extend(_list_blocks(element, item_path))
                else:
                    blocks.append(item_path)
        else:
            blocks.extend(_list_blocks(child, child_path))
    return blocks


def _gpu_candidates(model):
    """(decode block names, candidates): every Linear, Conv2d and Conv1D
    weight (a Parameter), assigned to the list block that contains it, or
    hooked on its own module when no block does (discovery semantics of
    neuralzip/gpu/inference.py:232-274)."""
    blocks = _list_blocks(model)
    candidates = []
    for module_name, module in model.named_modules(remove_duplicate=False):
        weight = module._parameters.get("weight") if isinstance(module, _GPU_WEIGHT_TYPES) else None
        if not isinstance(weight, nn.Parameter):
            continue
        owner = next((b for b in blocks if module_name == b or module_name.startswith(b + ".")), module_name)
        candidates.append(_Candidate(owner, module_name, _join(module_name, "weight"), weight))
    return tuple(dict.fromkeys(c.block_name for c in candidates)), tuple(candidates)


def _unique_candidates(model, candidates):
    """Candidates whose weight is non-empty and owned by no other module
    (tied or shared parameters stay resident)."""
    owners = defaultdict(int)
    for _name, parameter in model.named_parameters(remove_duplicate=False):
        owners[id(parameter)] += 1
    return tuple(c for c in candidates if c.parameter.numel() and owners[id(c.parameter)] == 1)


def _aligned(offset, element_size):
    step = max(1, WORKSPACE_ALIGN_BYTES // element_size)
    return (offset + step - 1) // step * step


def _view(array):
    """Read-only byte view of a numpy array (no copy)."""
    return memoryview(np.ascontiguousarray(array).view(np.uint8)).toreadonly()


def _as_bytes_array(data):
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data).reshape(-1).view(np.uint8)
    return np.frombuffer(data, dtype=np.uint8)


def _pack_parallel(items, threads=0):
    """Packs (raw bytes, GPUCodebook, spec) items on the native thread pool
    (nz_pack_many) and returns one GPUEncoded per item."""
    results = [None] * len(items)
    by_spec = defaultdict(list)
    for index, (raw, book, spec) in enumerate(items):
        by_spec[spec].append(index)
    for spec, indices in by_spec.items():
        dt = _dtype_struct(spec, spec.gpu_stream)
        jobs, keep = [], []
        for index in indices:
            raw, book, _ = items[index]
            raw_array = _as_bytes_array(raw)
            numel = len(raw_array) // spec.element_size
            words, n_lens, n_tiles = _native.pack_bound(numel, book.native.longest)
            bits = np.empty(words, dtype=np.uint32)
            lens = np.empty(n_lens, dtype=np.uint16)
            tile_off = np.empty(n_tiles, dtype=np.uint32)
            lanes = [None if lane == spec.gpu_stream else np.empty(numel, dtype=np.uint8)
                     for lane in range(spec.element_size)]
            job = _native.PackJob()
            job.codebook = book.native.handle.value
            job.raw = raw_array.ctypes.data if numel else None
            job.numel = numel
            job.bits, job.bits_cap_words = bits.ctypes.data, words
            job.lens, job.lens_cap = lens.ctypes.data, n_lens
            job.tile_off, job.tiles_cap = tile_off.ctypes.data, n_tiles
            for lane in range(4):
                job.lanes[lane] = lanes[lane].ctypes.data if lane < len(lanes) and lanes[lane] is not None else None
            jobs.append(job)
            keep.append((index, raw_array, bits, lens, tile_off, lanes, numel, book))
        done = _native.pack_many(jobs, dt, threads)
        for job, (index, _raw, bits, lens, tile_off, lanes, numel, book) in zip(done, keep):
            streams = [_view(lane) if lane is not None else None for lane in lanes]
            streams[spec.gpu_stream] = GPUEncodedSymbols(
                _view(bits[:job.words_used].copy()), int(job.bit_length), numel, _view(lens),
                tuple(tile_off.tolist()))
            results[index] = GPUEncoded(spec, numel, tuple(streams))
    return results


def _assemble(entries, compressor, threads=0):
    """One GPU group per source chunk (neuralzip/gpu/inference.py:288-336).
    entries: (block_name, module_name, tensor_name, tensor) in export order.
    Tensor offsets inside a block workspace are rounded up to 128 bytes so
    every group's output is 16-byte aligned for the vector stores."""
    payloads = {int(p.codebook_id): p for p in compressor.export_codebooks()}
    codebooks = {-1: GPUCodebook((), ())}
    workspace_offsets = defaultdict(int)
    planned = []
    for block_name, module_name, tensor_name, tensor in entries:
        spec = DTYPES[tensor.dtype]
        stream_id = spec.gpu_stream
        modes = compressor.chunk_modes(tensor_name, tensor, stream_id)
        step = _stream_chunk_size(compressor.chunk_size, spec.element_size)
        raw = tensor.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy()
        chunks = []
        for chunk, mode in enumerate(modes):
            start = chunk * step
            part = raw[start * spec.element_size:(start + step) * spec.element_size]
            codebook_id = mode.codebook_id if mode.kind != "raw" else -1
            if codebook_id not in codebooks:
                payload = payloads[codebook_id]
                codebooks[codebook_id] = codebook_from_header(bytes(payload.codebook), bytes(payload.vocab))
            chunks.append((start, part, codebook_id))
        planned.append((block_name, module_name, tensor_name, tensor, spec, raw, chunks))
    coded = [(part, codebooks[cid], spec) for *_, spec, _raw, chunks in planned for _s, part, cid in chunks if cid != -1]
    packed = iter(_pack_parallel(coded, threads))
    groups = []
    for block_name, module_name, tensor_name, tensor, spec, raw, chunks in planned:
        ws_key = (block_name, tensor.dtype)
        workspace_offset = _aligned(workspace_offsets[ws_key], spec.element_size)
        binding = LinearWeightBinding(module_name, tensor_name, tuple(tensor.shape), tensor.numel(), workspace_offset)
        fragments = []
        for start, part, cid in chunks:
            encoded = next(packed) if cid != -1 else encode_raw_fragment(part, dtype=spec, stream_id=spec.gpu_stream)
            fragments.append(GPUWeightGroup(block_name, cid, codebooks[cid], encoded, (binding,),
                                            workspace_offset + start))
        if sum(group.encoded.compressed_bytes for group in fragments) >= len(raw):
            continue
        groups.extend(fragments)
        workspace_offsets[ws_key] = workspace_offset + tensor.numel()
    return NeuralZipModelExport(tuple(groups))


def _assemble_export(block_order, candidates, compressor, threads=0):
    block_index = {name: index for index, name in enumerate(block_order)}
    ordered = sorted(candidates, key=lambda c: (block_index[c.block_name], c.module_name))
    return _assemble([(c.block_name, c.module_name, c.tensor_name, c.parameter) for c in ordered], compressor,
                     threads)


def export_tensors_for_gpu(named_tensors, setup, *, block_name="tensors", threads=0):
    """Exports a mapping of floating tensors as one block (bulk decode, no
    model): every tensor is bound under its own name."""
    from neuralzip_b200.compressor import NeuralZipCompressor

    items = [(str(name), tensor) for name, tensor in dict(named_tensors).items()
             if torch.is_tensor(tensor) and tensor.dtype in DTYPES and tensor.numel()]
    compressor = NeuralZipCompressor(setup, gpu=True)
    compressor.prepare_gpu_transfer_target(items)
    return _assemble([(block_name, name, name, tensor) for name, tensor in items], compressor, threads)


def export_model_for_gpu(model, setup, *, allowed_dtypes=DTYPES, threads=0):
    """Exports the frozen chunk tables, including adaptive singleton/pair
    codes (neuralzip/gpu/inference.py:339-358)."""
    from neuralzip_b200.compressor import NeuralZipCompressor

    blocks, candidates = _gpu_candidates(model)
    candidates = _unique_candidates(model, candidates)
    candidates = tuple(
        c for c in candidates
        if c.parameter.dtype in DTYPES and c.parameter.dtype in allowed_dtypes and c.parameter.is_contiguous()
    )
    if not candidates:
        return NeuralZipModelExport(())
    compressor = NeuralZipCompressor(setup, gpu=True)
    compressor.prepare_gpu_transfer_target(tuple((c.tensor_name, c.parameter) for c in candidates))
    return _assemble_export(blocks, candidates, compressor, threads)


def _binding_module(model, binding):
    module = model.get_submodule(binding.module_name)
    if not isinstance(module, _GPU_WEIGHT_TYPES):
        raise TypeError(f"{binding.module_name!r} is not a supported weight module.")
    return module


def _group_arrays(group):
    """Host arrays of one group in upload order: name -> uint8 view."""
    encoded = group.encoded
    symbols = encoded.symbols
    stream = encoded.dtype.gpu_stream
    arrays = {}
    if group.codebook.max_bits:
        arrays["bits"] = symbols.bitstream
        arrays["lens"] = symbols.lane_bits
        arrays["tile_off"] = np.asarray(symbols.tile_offsets, dtype=np.uint32).tobytes()
    for lane, data in enumerate(encoded.streams):
        if lane == stream:
            if not group.codebook.max_bits:
                arrays[f"lane{lane}"] = symbols.bitstream
        else:
            arrays[f"lane{lane}"] = data
    return arrays


@dataclass(frozen=True)
class _UploadedGroup:
    group: GPUWeightGroup
    device: object  # decoder.DeviceGroup

    @property
    def layout(self):
        return self.group.layout


def _current_stream_handle(index):
    """Raw cudaStream_t of torch's current stream on device `index`."""
    return torch.cuda.current_stream(index).cuda_stream


if hasattr(torch._C, "_cuda_getCurrentRawStream"):
    _current_stream_handle = torch._C._cuda_getCurrentRawStream  # noqa: F811  (same value, no Stream object)


# "auto" launch units decode at least this many bytes where blocks are
# smaller: a launch of one small layer (tens of MB) is a single wave of tiles
# whose time is the tiles' serial decode latency, while a few such layers in
# one launch keep every warp busy with several tiles.
AUTO_UNIT_BYTES = 256 << 20


def _plan_units(exported, blocks_per_launch):
    """Consecutive blocks decoded by one launch: fixed-size runs, or with
    "auto" greedy runs whose decoded bytes stay within the largest block's
    or AUTO_UNIT_BYTES, whichever is larger."""
    blocks = exported.block_order
    if blocks_per_launch != "auto":
        per_unit = max(1, int(blocks_per_launch))
        return [tuple(blocks[i:i + per_unit]) for i in range(0, len(blocks), per_unit)]
    size = defaultdict(int)
    for group in exported.groups:
        size[group.block_name] += group.encoded.numel * group.encoded.dtype.element_size
    limit = max(max(size.values(), default=0), AUTO_UNIT_BYTES)
    units, current, total = [], [], 0
    for name in blocks:
        if current and total + size[name] > limit:
            units.append(tuple(current))
            current, total = [], 0
        current.append(name)
        total += size[name]
    if current:
        units.append(tuple(current))
    return units


class NeuralZipRuntime:
    """Runtime attached to one model on one CUDA device.

    Blocks are decoded in units of consecutive blocks: ``blocks_per_launch``
    blocks (1 decodes block by block as the reference does), or with "auto"
    (the default) as many as fit in the size of the largest block or in
    AUTO_UNIT_BYTES (256 MiB) if that is larger, so the workspace is no
    larger than with single blocks or than 256 MiB a slot. One launch per dtype
    covers a unit, and the blocks of a unit lie side by side in one
    workspace slot. Fewer, larger launches cost less host time per token and
    lose less to the start and end of each launch.

    With ``overlap`` (the default when there are two or more units) every
    dtype gets ``prefetch_depth`` slots (2 = ping-pong): unit k decodes into
    slot k % depth, and while unit k runs, units k + 1 .. k + depth - 1 of
    the same forward are already being decoded on a side stream (the first
    unit of a forward is decoded by its own hook, so no forward depends on
    workspace contents left by the previous one). The two streams are ordered with
    CUDA events only: the compute stream waits for "unit k decoded" before
    unit k runs, and the side stream waits for "everything before unit k
    enqueued" before it reuses a slot, which covers the slot's previous
    reader (a prefetch whose slot is still used by the current or a later
    unit is skipped and done when that unit is reached).

    The first block of a unit decodes it (or waits for its prefetch); the
    other blocks only check that their unit is the one in the slot. A block
    reached out of order decodes its unit first; the direct
    ``_decode_block`` / ``materialized_weights`` calls drain pending side
    decodes and decode one block on the current stream, as the reference
    does (neuralzip/gpu/inference.py:476-509). ``workspaces[dtype]`` covers
    all slots."""

    def __init__(self, model, exported, device, *, overlap=True, prefetch_depth=2, blocks_per_launch="auto"):
        self.model = model
        self.export = exported
        self.device = torch.device(device)
        self._decoder = gpu_decoder.default_decoder()
        self._hook_handles = []
        self._units = _plan_units(exported, blocks_per_launch)
        self.blocks_per_launch = blocks_per_launch
        n = len(self._units)
        self.overlap = bool(overlap) and n > 1
        depth = max(2, int(prefetch_depth)) if self.overlap else 1
        self.prefetch_depth = depth
        self._unit_of = {name: k for k, unit in enumerate(self._units) for name in unit}
        self._slot = [k % depth for k in range(n)]
        # Workspace: each block's extent per dtype, blocks of a unit side by side.
        extent = defaultdict(int)
        for group in exported.groups:
            key = (group.block_name, group.encoded.dtype.torch_dtype)
            extent[key] = max(extent[key], group.workspace_offset + group.encoded.numel)
        dtypes = tuple(dict.fromkeys(group.encoded.dtype.torch_dtype for group in exported.groups))
        self._block_base = {}
        slot_elems = defaultdict(int)
        for unit in self._units:
            for dtype in dtypes:
                size = DTYPES[dtype].element_size
                cursor = 0
                for name in unit:
                    self._block_base[(name, dtype)] = cursor
                    cursor = _aligned(cursor + extent.get((name, dtype), 0), size)
                slot_elems[dtype] = max(slot_elems[dtype], cursor)
        self._slot_elems = dict(slot_elems)
        self.workspaces = {
            dtype: torch.empty(size * depth, dtype=dtype, device=self.device)
            for dtype, size in self._slot_elems.items()
        }
        self._side = torch.cuda.Stream(device=self.device) if self.overlap else None
        # Decode tables: one row of LUT_WORDS words per codebook id.
        book_ids = sorted({g.codebook_id for g in exported.groups if g.codebook.max_bits})
        self._lut_rows = {cid: row for row, cid in enumerate(book_ids)}
        books = {g.codebook_id: g.codebook for g in exported.groups}
        if book_ids:
            table = np.stack([np.asarray(books[cid].decode_lut, dtype=np.uint32) for cid in book_ids])
            self.decode_tables = torch.from_numpy(table).to(self.device)
        else:
            self.decode_tables = torch.zeros((1, _native.LUT_WORDS), dtype=torch.int32, device=self.device)
        # One arena for every group's arrays.
        offsets = []
        cursor = 0
        for group in exported.groups:
            placed = {}
            for name, data in _group_arrays(group).items():
                cursor = (cursor + ARENA_ALIGN - 1) // ARENA_ALIGN * ARENA_ALIGN
                placed[name] = (cursor, data)
                cursor += len(data)
            offsets.append(placed)
        host = np.zeros(max(cursor, 1), dtype=np.uint8)
        for placed in offsets:
            for start, data in placed.values():
                host[start:start + len(data)] = np.frombuffer(data, dtype=np.uint8)
        # Byte range of each group's arrays in the arena (groups are placed in order).
        self.arena_ranges = tuple(
            (min(start for start, _ in placed.values()), max(start + len(data) for start, data in placed.values()))
            for placed in offsets)
        self.arena_host = host
        self.arena = torch.from_numpy(host).to(self.device)
        base = self.arena.data_ptr()
        lut_base = self.decode_tables.data_ptr()
        row_bytes = _native.LUT_WORDS * 4
        uploaded = []
        for group, placed in zip(exported.groups, offsets):
            spec = group.encoded.dtype

            def addr(name, placed=placed):
                return base + placed[name][0] if name in placed else 0

            start = group.workspace_offset + self._buffer_offset(group.block_name, spec.torch_dtype)
            output = self.workspaces[spec.torch_dtype][start:start + group.encoded.numel]
            coded = bool(group.codebook.max_bits)
            row = self._lut_rows.get(group.codebook_id) if coded else None
            device_group = gpu_decoder.DeviceGroup(
                spec=spec, numel=group.encoded.numel,
                lut_index=row if coded else _native.RAW_LUT,
                lut_ptr=lut_base + row * row_bytes if coded else 0,
                lut_words=group.codebook.table_words,
                bits=addr("bits"), lens=addr("lens"), tile_off=addr("tile_off"),
                lanes=tuple(addr(f"lane{lane}") for lane in range(4)),
                out=output.data_ptr(), output=output,
                tile_words=gpu_decoder.tile_copy_words(group.encoded.symbols.tile_offsets,
                                                       group.encoded.symbols.bit_length) if coded else 0,
            )
            uploaded.append(_UploadedGroup(group, device_group))
        by_block = defaultdict(list)
        for item in uploaded:
            by_block[item.group.block_name].append(item)
        self._groups_by_block = {name: tuple(by_block[name]) for name in exported.block_order}
        self._prepared_batches = {name: self._prepare(items) for name, items in self._groups_by_block.items()}
        self._unit_batches = [
            self._prepared_batches[unit[0]] if len(unit) == 1
            else self._prepare([item for name in unit for item in self._groups_by_block[name]])
            for unit in self._units
        ]
        # The schedule (native): slot residency, pending side decodes, events.
        with torch.cuda.device(self.device):
            self._schedule = _native.Schedule([[p.launch for p in batches] for batches in self._unit_batches],
                                              depth, self._side.cuda_stream if self._side is not None else 0)
        weakref.finalize(self, self._schedule.close)
        torch.cuda.synchronize(self.device)

    def _prepare(self, items):
        """Prepared launches over `items` (uploaded groups of any dtypes):
        one for the dtype with the most elements and, if there are others,
        one more launch that mixes all of them. The big launch runs alone
        and fills every SM; small dtypes are latency-bound and decode faster
        in a launch of their own geometry than as extra CTAs of the big one
        (the reference keeps one launch per layout)."""
        by_dtype = defaultdict(list)
        for item in items:
            by_dtype[item.group.encoded.dtype.torch_dtype].append(item.device)
        main = max(by_dtype, key=lambda dtype: sum(d.numel for d in by_dtype[dtype]))
        rest = [d for dtype, devices in by_dtype.items() if dtype != main for d in devices]
        batches = [self._decoder.prepare_batch(by_dtype[main])]
        if rest:
            batches.append(self._decoder.prepare_batch(rest))
        return tuple(batches)

    @classmethod
    def attach(cls, model, exported, *, device=None, overlap=True, prefetch_depth=2, blocks_per_launch="auto"):
        if hasattr(model, RUNTIME_ATTRIBUTE):
            raise RuntimeError("This model already has a NeuralZip runtime.")
        if not exported.groups:
            raise ValueError("The setup produced no GPU-compressible weights.")
        if device is None:
            current = next(model.parameters()).device
            device = current if current.type == "cuda" else "cuda"
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("NeuralZip GPU inference requires a CUDA device.")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        decoder = gpu_decoder.default_decoder()
        for group in exported.groups:
            decoder.prepare_group(device.index, group)
        for binding in exported.bindings:
            module = _binding_module(model, binding)
            module._parameters.pop("weight", None)
            module.__dict__.pop("weight", None)
        model.to(device).eval()
        runtime = cls(model, exported, device, overlap=overlap, prefetch_depth=prefetch_depth,
                      blocks_per_launch=blocks_per_launch)
        runtime._install()
        return runtime

    def _buffer_offset(self, block_name, dtype):
        slot = self._slot[self._unit_of[block_name]]
        return slot * self._slot_elems[dtype] + self._block_base[(block_name, dtype)]

    def _binding_view(self, block_name, dtype, binding):
        offset = binding.workspace_offset + self._buffer_offset(block_name, dtype)
        return self.workspaces[dtype][offset:offset + binding.numel].view(binding.shape)

    def _install(self):
        for name, items in self._groups_by_block.items():
            for item in items:
                for binding in item.group.bindings:
                    _binding_module(self.model, binding).__dict__["weight"] = self._binding_view(
                        name, item.group.encoded.dtype.torch_dtype, binding)
        heads = {unit[0] for unit in self._units}
        for block_name in self.export.block_order:
            hook = self._make_hook(self._unit_of[block_name], int(block_name in heads))
            handle = _decode_hook_module(self.model, block_name).register_forward_pre_hook(hook, prepend=True)
            self._hook_handles.append(handle)
        setattr(self.model, RUNTIME_ATTRIBUTE, self)

    def _make_hook(self, unit, head):
        """Forward pre-hook of one block: one native call
        (nz_schedule_enter) on the current stream."""
        enter, handle, index = self._schedule.enter_fn, self._schedule.handle, self.device.index

        def hook(_module, _args):
            status = enter(handle, unit, head, _current_stream_handle(index))
            if status:
                _native.check(status)

        return hook

    def _pre_hook(self, block_name, _module=None, _args=None):
        """Runs the forward pre-hook of `block_name` by hand."""
        unit = self._unit_of[block_name]
        self._make_hook(unit, int(self._units[unit][0] == block_name))(_module, _args)

    def _drain(self, stream):
        """Makes `stream` wait for every pending side-stream decode."""
        self._schedule.drain(stream.cuda_stream)

    def _decode_unit(self, unit, stream):
        """Decodes a whole unit on `stream` (after pending side decodes)."""
        self._schedule.decode_unit(unit, stream.cuda_stream)

    def _decode_block(self, block_name, _module=None, _args=None):
        """Decodes one block on the current stream (reference semantics)."""
        stream = torch.cuda.current_stream(self.device)
        self._drain(stream)
        self._decoder.decode_batches(self._prepared_batches[block_name], stream)
        unit = self._unit_of[block_name]
        self._schedule.mark(unit, len(self._units[unit]) == 1)

    def check_status(self):
        """Raises if any decode launch reported a corrupt table."""
        for batches in list(self._prepared_batches.values()) + list(self._unit_batches):
            for prepared in batches:
                self._decoder.check_status(prepared)

    @torch.no_grad()
    def materialized_weights(self):
        """Yield compressed weights as bit-exact CPU tensors, one block at a
        time (neuralzip/gpu/inference.py:495-509). While a block's weights
        are copied to the host, the next block is already decoding on a side
        stream when it decodes into another workspace slot, so the decode
        hides behind the copies."""
        stream = torch.cuda.current_stream(self.device)
        self._drain(stream)
        order = self.export.block_order
        side = torch.cuda.Stream(device=self.device)

        def start(name):
            # On the side stream, after everything enqueued on `stream` so far
            # (which covers the previous reader of the block's slot).
            after = torch.cuda.Event()
            after.record(stream)
            side.wait_event(after)
            self._decoder.decode_batches(self._prepared_batches[name], side)
            done = torch.cuda.Event()
            done.record(side)
            return done

        def slot(name):
            return self._slot[self._unit_of[name]]

        # The slots are overwritten block by block: the next forward must
        # decode every unit again, even if this generator is left early.
        for unit in range(len(self._units)):
            self._schedule.mark(unit, 0)
        yielded = set()
        try:
            pending = start(order[0]) if order else None
            for index, block_name in enumerate(order):
                stream.wait_event(pending)
                following = order[index + 1] if index + 1 < len(order) else None
                ahead = following is not None and slot(following) != slot(block_name)
                pending = start(following) if ahead else None
                for item in self._groups_by_block[block_name]:
                    for binding in item.group.bindings:
                        if binding.tensor_name in yielded:
                            continue
                        yielded.add(binding.tensor_name)
                        weight = self._binding_view(block_name, item.group.encoded.dtype.torch_dtype, binding)
                        yield binding.tensor_name, weight.detach().to("cpu", copy=True)
                if following is not None and not ahead:
                    pending = start(following)
        finally:
            stream.wait_stream(side)
