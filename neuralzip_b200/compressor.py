"""Storage-format compressor: encodes named tensors into storage v2 and back.

Public surface of neuralzip/compressor.py:16-187: ``NeuralZipCompressor``
(setup, threads, direct_batch_bytes, gpu) with ``encode`` ->
(blob, metadata, storage statistics, seconds), ``decode`` -> {name: tensor},
``export_codebooks``, ``load_codebooks``, ``prepare_storage_transfer_target``
and ``prepare_gpu_transfer_target``.

How a tensor's chunks are coded is a transfer plan: for every (tensor name,
dtype, byte lane) the setup's codebook ids are resolved once into
``ChunkMode`` records, taking the first of

1. the chunk-level assignment of a tensor of that name (or its fallback
   name: lm_head reuses tied embeddings) and the same element count;
2. that tensor's pooled singleton table, for every chunk;
3. a per-dtype global table (files in ``codebooks/``), for every chunk;
4. raw.

Encoding runs the native packer (``huff0.compress_direct_storage``) over the
plan and ``StorageWriter`` writes the metadata; decoding is one native pass
over the checkpoint's chunk table (``StorageReader.decode``), the decode
tables built once per codebook and kept while the codebook is unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from pathlib import Path

import torch

from neuralzip_b200 import huff0
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.payloads import CodebookPayload
from neuralzip_b200.setup import NeuralZipSetup
from neuralzip_b200.storage import StorageReader, StorageWriter
from neuralzip_b200.utils import _stream_chunk_size, time_call

# A tensor without a plan of its own borrows the plan of these names (tied
# output embeddings, as the reference's transfer fallback does).
_NAME_FALLBACKS = {"lm_head.weight": ("model.embed_tokens.weight",)}
_MISSING = object()


@dataclass(frozen=True)
class ChunkMode:
    """How one source chunk of one byte lane is stored."""

    kind: str = "raw"          # "raw", "shared_huff0" or "mixed_huffman"
    codebook_id: int = -1
    codebook: object = None    # huff0.Huff0Codebook (host tables) when coded


RAW = ChunkMode()


class NeuralZipCompressor:
    def __init__(self, setup=None, *, threads=0, direct_batch_bytes=128 << 20, gpu=False):
        setup = NeuralZipSetup() if setup is None else NeuralZipSetup.load(setup)
        self.min_saving_bytes = setup.min_saving_bytes
        self.chunk_size = setup.chunk_size
        self.compression_threshold = setup.compression_threshold
        self.threads = int(threads)
        # Decode writes every chunk straight into its tensor, so the whole
        # checkpoint is one native pass; the budget is kept for callers.
        self.direct_batch_bytes = int(direct_batch_bytes)
        self._books = list(setup.codebooks)
        self._coded = {book.codebook_id: ChunkMode(book.mode, book.codebook_id,
                                                   huff0.build_codebook_from_header(book.codebook, vocab=book.vocab))
                       for book in setup.codebooks}
        self._chunk_ids = dict(setup.chunk_codebooks)     # (name, dtype, lane, numel) -> ids per chunk
        self._pooled_ids = dict(setup.tensor_codebooks)   # (name, dtype, lane) -> id or None
        self._global = {key: self._mode(cid) for key, cid in setup.global_codebooks.items()}
        self._plan = {}                                   # (name, dtype, lane) -> tuple[ChunkMode]
        self._tables = {}                                 # codebook id -> host decode table
        self._payload_by_id = {}
        if gpu:
            self._add_global_codebooks()
        self.load_codebooks(self._books)

    # ---- plan -------------------------------------------------------------

    def _mode(self, codebook_id):
        return RAW if codebook_id is None else self._coded[codebook_id]

    def _resolve(self, name, dtype_name, lane, numel, count):
        for candidate in (name, *_NAME_FALLBACKS.get(name, ())):
            pooled = self._pooled_ids.get((candidate, dtype_name, lane), _MISSING)
            if pooled is _MISSING:
                continue
            ids = self._chunk_ids.get((candidate, dtype_name, lane, numel))
            if ids is not None:
                return tuple(self._mode(cid) for cid in ids)
            return (self._mode(pooled),) * count
        return (self._global.get((dtype_name, lane), RAW),) * count

    def prepare_storage_transfer_target(self, named_tensors):
        """Resolves the per-chunk modes of every byte lane of these tensors."""
        plan = {}
        for name, tensor in named_tensors:
            spec = DTYPES[tensor.dtype]
            step = _stream_chunk_size(self.chunk_size, spec.element_size)
            count = -(-tensor.numel() // step)
            for lane in spec.stream_ids:
                plan[(str(name), spec.name, int(lane))] = self._resolve(str(name), spec.name, int(lane),
                                                                        tensor.numel(), count)
        self._plan = plan

    def prepare_gpu_transfer_target(self, named_tensors):
        self.prepare_storage_transfer_target(named_tensors)

    def chunk_modes(self, name, tensor, lane=None):
        """The planned ChunkMode of every source chunk of `tensor`'s byte
        lane `lane` (default: its coded lane)."""
        spec = DTYPES[tensor.dtype]
        return self._plan[(str(name), spec.name, int(spec.gpu_stream if lane is None else lane))]

    # ---- codebooks ----------------------------------------------------------

    def _add_global_codebooks(self):
        """Optional per-dtype tables shipped as files (DTypeSpec.global_codebooks)."""
        next_id = max((book.codebook_id for book in self._books), default=-1) + 1
        for spec in DTYPES.values():
            for lane, filename in spec.global_codebooks:
                key = (spec.name, lane)
                path = Path(__file__).with_name("codebooks") / filename
                if key in self._global or not path.is_file():
                    continue
                header = path.read_bytes()
                self._books.append(CodebookPayload(next_id, lane, spec.name, codebook=header))
                self._global[key] = ChunkMode("shared_huff0", next_id, huff0.build_codebook_from_header(header))
                next_id += 1

    def export_codebooks(self):
        return tuple(self._books)

    def load_codebooks(self, codebooks):
        """Makes `codebooks` the ones decode reads; host decode tables are
        kept for ids whose table and vocabulary did not change. Only the
        small tables are copied, never views into a checkpoint."""
        payloads = {book.codebook_id: replace(book, codebook=bytes(book.codebook), vocab=bytes(book.vocab))
                    for book in codebooks}
        self._tables = {cid: table for cid, table in self._tables.items()
                        if self._payload_by_id.get(cid) == payloads.get(cid)}
        self._payload_by_id = payloads

    def _decode_table(self, codebook_id, dtype_name, lane, mode):
        book = self._payload_by_id.get(codebook_id)
        if book is None or (book.dtype, book.stream_id, book.mode) != (dtype_name, lane, mode):
            raise ValueError("Chunk codebook does not match its tensor stream.")
        if codebook_id not in self._tables:
            self._tables[codebook_id] = huff0.build_decodebook(book.codebook, vocab=book.vocab)
        return self._tables[codebook_id]

    # ---- encode / decode --------------------------------------------------------

    def encode(self, named_tensors):
        named_tensors = tuple(named_tensors)
        self._add_global_codebooks()
        self.prepare_storage_transfer_target(named_tensors)
        result, seconds = time_call(self._encode, named_tensors)
        return *result, seconds

    def _encode(self, named_tensors):
        specs, used = [], set()
        for name, tensor in named_tensors:
            spec = DTYPES[tensor.dtype]
            modes = self.chunk_modes(name, tensor)
            used.update(mode.codebook_id for mode in modes if mode.kind != "raw")
            raw = tensor.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy()
            specs.append((raw, spec, spec.gpu_stream, _stream_chunk_size(self.chunk_size, spec.element_size), modes))
        writer = StorageWriter(book for book in self._books if book.codebook_id in used)
        packed, chunk_lists = huff0.compress_direct_storage(
            specs, writer.prefix, min_saving_bytes=self.min_saving_bytes, threads=self.threads,
            compression_threshold=self.compression_threshold)
        return writer.finish(named_tensors, specs, packed, chunk_lists)

    def decode(self, blob, metadata):
        reader = StorageReader(blob, metadata)
        self.load_codebooks(reader.codebooks())
        return reader.decode(self._decode_table, threads=self.threads)
