"""Storage format v2: one byte blob plus JSON metadata.

The format is the reference's (neuralzip/storage.py:21-39 and :105-164 name
the keys; neuralzip/native/direct_storage.h:137-191 lays out the blob), so a
checkpoint written by either implementation loads in the other:

* metadata ``{version: 2, codebooks: [{id, stream, dtype, mode,
  codebook: [offset, len], vocab: [offset, len]}], tensors: [{name, shape,
  dtype, element_size, numel, bit_reorder, groups}]}`` where ``groups`` has
  one list per byte lane of ``{mode, symbols, codebook, payload: [offset,
  len]}`` per source chunk;
* the blob holds the codebook prefix (each header, then its vocabulary),
  then the raw lanes, then the compacted selected-lane payloads.

Here a ``StorageWriter`` lays out the prefix and turns the packer's chunk
lists (``huff0.compress_direct_storage``) into metadata, and a
``StorageReader`` checks every span once and then either exposes payload
records (``unpack_storage``) or builds the chunk table that one native call
(``nz_storage_decode``) decodes, merges and restores on the host cores.
"""

from __future__ import annotations

import numpy as np
import torch

from neuralzip_b200 import _native
from neuralzip_b200.payloads import ByteGroupPayload, CodebookPayload, StreamChunk, TensorPayload, storage_bytes

FORMAT_VERSION = 2


def _codebook_layout(codebooks):
    """(prefix bytes, codebook metadata entries) for `codebooks` in order."""
    prefix = bytearray()
    entries = []
    for book in codebooks:
        header_at = len(prefix)
        prefix += book.codebook
        vocab_at = len(prefix)
        prefix += book.vocab
        entries.append({"id": int(book.codebook_id), "stream": int(book.stream_id), "dtype": str(book.dtype),
                        "mode": str(book.mode), "codebook": [header_at, vocab_at - header_at],
                        "vocab": [vocab_at, len(prefix) - vocab_at]})
    return prefix, entries


class StorageWriter:
    """Blob prefix and metadata of one checkpoint. ``prefix`` goes first in
    the packer's output buffer; ``finish`` writes the metadata for what the
    packer produced."""

    def __init__(self, codebooks):
        self.codebooks = tuple(codebooks)
        self.prefix, self._entries = _codebook_layout(self.codebooks)

    def finish(self, named_tensors, specs, packed, chunk_lists):
        """(blob tensor, metadata, storage statistics). ``chunk_lists[t][lane]``
        holds (mode, symbols, codebook id or -1, offset, size) per chunk.
        Codebooks that no chunk ended up using (every chunk of theirs fell
        back to raw) are dropped, and offsets past the prefix move down by
        the bytes removed."""
        used = {cid for lanes in chunk_lists for lane in lanes for (_m, _s, cid, _o, _n) in lane}
        kept = tuple(book for book in self.codebooks if book.codebook_id in used)
        entries, shift, old_end = self._entries, 0, len(self.prefix)
        if len(kept) != len(self.codebooks):
            prefix, entries = _codebook_layout(kept)
            shift = old_end - len(prefix)
            packed[:old_end] = prefix
        tensors = []
        for (name, tensor), spec, lanes in zip(named_tensors, specs, chunk_lists, strict=True):
            dtype = spec[1]
            tensors.append({
                "name": str(name), "shape": [int(d) for d in tensor.shape], "dtype": dtype.name,
                "element_size": dtype.element_size, "numel": int(tensor.numel()),
                "bit_reorder": int(dtype.bit_reorder),
                "groups": [[{"mode": str(mode), "symbols": int(symbols), "codebook": int(cid) if cid >= 0 else None,
                             "payload": [int(offset) - (shift if offset >= old_end else 0), int(size)]}
                            for mode, symbols, cid, offset, size in lane] for lane in lanes],
            })
        blob = torch.frombuffer(packed, dtype=torch.uint8) if packed else torch.empty(0, dtype=torch.uint8)
        metadata = {"version": FORMAT_VERSION, "codebooks": entries, "tensors": tensors}
        return blob, metadata, storage_bytes(kept, tensors, blob.numel())


class StorageReader:
    """A checkpoint's blob and metadata, every span checked against the blob."""

    def __init__(self, blob, metadata):
        if int(metadata["version"]) != FORMAT_VERSION:
            raise ValueError("Unsupported NeuralZip storage checkpoint.")
        if torch.is_tensor(blob):
            blob = blob.detach().cpu().contiguous().reshape(-1).numpy()
        array = np.frombuffer(memoryview(blob).cast("B"), dtype=np.uint8) if not isinstance(blob, np.ndarray) \
            else np.ascontiguousarray(blob.reshape(-1).view(np.uint8))
        self.blob = array
        self.metadata = metadata

    def span(self, span):
        offset, size = (int(v) for v in span)
        if offset < 0 or size < 0 or offset + size > len(self.blob):
            raise ValueError("A NeuralZip storage span is outside its data tensor.")
        return offset, size

    def view(self, span):
        offset, size = self.span(span)
        return memoryview(self.blob[offset:offset + size]).toreadonly()

    def codebooks(self):
        return tuple(CodebookPayload(codebook_id=e["id"], stream_id=e["stream"], dtype=e["dtype"], mode=e["mode"],
                                     codebook=self.view(e["codebook"]), vocab=self.view(e["vocab"]))
                     for e in self.metadata["codebooks"])

    def tensors(self):
        return tuple(
            TensorPayload(name=t["name"], shape=tuple(t["shape"]), dtype=t["dtype"], element_size=t["element_size"],
                          numel=t["numel"], bit_reorder=t["bit_reorder"],
                          groups=tuple(ByteGroupPayload(chunks=tuple(
                              StreamChunk(mode=c["mode"], symbol_count=c["symbols"], codebook_id=c["codebook"],
                                          payload=self.view(c["payload"])) for c in lane)) for lane in t["groups"]))
            for t in self.metadata["tensors"])

    def decode(self, decode_table, threads=0):
        """{name: tensor} decoded on the host cores in one native call.
        ``decode_table(codebook_id, tensor_dtype, lane, mode)`` returns the
        host table (a NativeCodebook) of a compressed chunk's codebook."""
        from neuralzip_b200.dtypes import DTYPES

        specs = {spec.name: spec for spec in DTYPES.values()}
        entries = self.metadata["tensors"]
        n_pieces = sum(len(t["groups"][0]) if t["groups"] else 0 for t in entries)
        n_lanes = sum(len(t["groups"][0]) * len(t["groups"]) if t["groups"] else 0 for t in entries)
        pieces = np.zeros(n_pieces, dtype=_native.STORAGE_PIECE_DTYPE)
        lanes = np.zeros(max(n_lanes, 1), dtype=_native.STORAGE_LANE_DTYPE)
        blob_at = self.blob.ctypes.data
        lanes_at = lanes.ctypes.data
        tables, outputs = [], []
        p = k = 0
        for t in entries:
            es, numel, groups = int(t["element_size"]), int(t["numel"]), t["groups"]
            if es not in (2, 4) or numel < 0:
                raise ValueError("Invalid decoded width or element count.")
            if len(groups) != es:
                raise ValueError("Decode needs one group per byte stream.")
            if any(len(lane) != len(groups[0]) for lane in groups):
                raise ValueError("Unaligned chunk groups.")
            spec = specs[t["dtype"]]
            out = np.empty(numel * es, dtype=np.uint8)
            outputs.append((t, out))
            first = 0
            for c in range(len(groups[0])):
                count = int(groups[0][c]["symbols"])
                if count < 0 or count > numel - first:
                    raise ValueError("Chunk exceeds its tensor element count.")
                if any(int(lane[c]["symbols"]) != count for lane in groups):
                    raise ValueError("Unaligned chunk boundaries.")
                piece = pieces[p]
                piece["lanes"], piece["out"], piece["count"] = lanes_at + k * lanes.itemsize, \
                    out.ctypes.data + first * es, count
                piece["elem_size"], piece["reorder"] = es, int(t["bit_reorder"])
                piece["mant_bits"], piece["exp_bits"] = spec.mantissa_bits, spec.exponent_bits
                for lane_index, lane in enumerate(groups):
                    chunk = lane[c]
                    mode = _native.CHUNK_MODES.get(chunk["mode"])
                    if mode is None:
                        raise ValueError("Unsupported decoded chunk mode.")
                    offset, size = self.span(chunk["payload"])
                    record = lanes[k]
                    record["payload"], record["payload_size"], record["mode"] = blob_at + offset, size, mode
                    if mode != _native.CHUNK_RAW:
                        if chunk["codebook"] is None:
                            raise ValueError("Compressed chunk needs a decode table.")
                        table = decode_table(int(chunk["codebook"]), t["dtype"], lane_index, chunk["mode"])
                        tables.append(table)
                        record["codebook"] = table.handle.value
                    k += 1
                first += count
                p += 1
            if first != numel:
                raise ValueError("Byte stream does not reconstruct exactly numel values.")
        _native.storage_decode(pieces, threads)
        del tables
        result = {}
        for t, out in outputs:
            dtype = getattr(torch, t["dtype"])
            shape = tuple(int(d) for d in t["shape"])
            result[t["name"]] = torch.from_numpy(out).view(dtype).reshape(shape) if out.size else \
                torch.empty(shape, dtype=dtype)
        return result


def unpack_storage(blob, metadata):
    """(codebook payloads, tensor payloads) of a checkpoint, as read-only
    views into its blob (the caller keeps the blob alive and unchanged)."""
    reader = StorageReader(blob, metadata)
    return reader.codebooks(), reader.tensors()
