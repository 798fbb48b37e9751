"""Payload records, statistics and canonical byte accounting.

The records are the reference's public data types, with their names and
fields (neuralzip/payloads.py:14-95): NeuralZipStats (model.neuralzip_stats),
CodebookPayload, StreamChunk, ByteGroupPayload and TensorPayload, so pickles
and attribute access carry over. storage_bytes() applies the same byte
accounting, so the statistics of a checkpoint agree between the two
implementations.
"""

from dataclasses import dataclass

from neuralzip_b200.dtypes import DTYPES

RAW_CHUNK_METADATA_BYTES = 17
SHARED_CHUNK_METADATA_BYTES = 25
CHUNK_METADATA_BYTES = {
    "raw": RAW_CHUNK_METADATA_BYTES,
    "shared_huff0": SHARED_CHUNK_METADATA_BYTES,
    "mixed_huffman": SHARED_CHUNK_METADATA_BYTES,
}


@dataclass(frozen=True)
class NeuralZipStats:
    setup_seconds: float
    encoding_seconds: float
    raw_bytes: int
    compressed_bytes: int
    exponent_raw_bytes: int | None
    exponent_compressed_bytes: int | None
    representation: str = "storage"
    decoding_seconds: float = 0.0
    runtime_encoding_seconds: float = 0.0
    stream_raw_bytes: int | None = None
    stream_compressed_bytes: int | None = None

    @property
    def compression_ratio(self):
        return self.compressed_bytes / self.raw_bytes if self.raw_bytes else 1.0

    @property
    def exponent_ratio(self):
        if self.exponent_raw_bytes is None or self.exponent_compressed_bytes is None:
            return None
        return self.exponent_compressed_bytes / self.exponent_raw_bytes if self.exponent_raw_bytes else 1.0

    @property
    def stream_ratio(self):
        """Selected GPU lanes plus their codebooks; excludes resident lanes."""
        if not self.stream_raw_bytes or self.stream_compressed_bytes is None:
            return None
        return self.stream_compressed_bytes / self.stream_raw_bytes

    @property
    def total_seconds(self):
        return self.setup_seconds + self.encoding_seconds


@dataclass(frozen=True)
class CodebookPayload:
    codebook_id: int
    stream_id: int
    dtype: str
    mode: str = "shared_huff0"
    codebook: bytes | memoryview = b""
    vocab: bytes | memoryview = b""

    @property
    def metadata_bytes(self):
        return _codebook_size(self)


@dataclass(frozen=True)
class StreamChunk:
    mode: str
    symbol_count: int
    payload: bytes | memoryview = b""
    codebook_id: int | None = None

    @property
    def payload_bytes(self):
        return len(self.payload)

    @property
    def metadata_bytes(self):
        return CHUNK_METADATA_BYTES[self.mode]

    @property
    def compressed_bytes(self):
        return self.metadata_bytes + self.payload_bytes


@dataclass(frozen=True)
class ByteGroupPayload:
    chunks: tuple


@dataclass(frozen=True)
class TensorPayload:
    name: str
    shape: tuple
    dtype: str
    element_size: int
    numel: int
    groups: tuple
    bit_reorder: int = 0

    @property
    def raw_bytes(self):
        return self.numel * self.element_size


# ---- canonical size of the stored metadata -------------------------------------
#
# compressed_bytes counts the blob plus the size the metadata would take in a
# canonical binary serialization, not the JSON actually written (the
# accounting of neuralzip/payloads.py:97-174): length-prefixed strings (4-byte
# length) and byte strings (8-byte length), 8-byte integers, 4-byte stream
# ids; per chunk 17 bytes raw or 25 bytes coded.


def _text(value):
    return 4 + len(str(value).encode("utf-8"))


def _blob(value):
    return 8 + len(value)


# File header: magic (4), version (2), format name, codebook and tensor counts (8 each).
_HEADER_BYTES = 4 + 2 + _text("neuralzip") + 8 + 8


def _codebook_size(codebook):
    """id (8), stream (4), dtype, mode, and the header and vocabulary."""
    return 8 + 4 + _text(codebook.dtype) + _text(codebook.mode) + _blob(codebook.codebook) + _blob(codebook.vocab)


def _tensor_fields(entry):
    """name, dtype, element size + numel + reorder flag (24), the shape
    (8 per dimension) and the lane count (8)."""
    return _text(entry["name"]) + _text(entry["dtype"]) + 24 + 8 * len(entry["shape"]) + 8


def _lane_fields(lane):
    """chunk count (8) and each chunk's record."""
    return 8 + sum(CHUNK_METADATA_BYTES[chunk["mode"]] for chunk in lane)


def storage_bytes(codebooks, tensors, blob_bytes):
    """{raw_bytes, compressed_bytes, exponent_raw_bytes,
    exponent_compressed_bytes} of a checkpoint from its codebooks, tensor
    metadata entries and blob size. The exponent figures cover the lanes
    that are a pure exponent (and the codebooks of those lanes); they are
    None when a non-empty tensor has no such lane."""
    specs = {spec.name: spec for spec in DTYPES.values()}
    structure = _HEADER_BYTES + sum(_codebook_size(b) - len(b.codebook) - len(b.vocab) for b in codebooks)
    raw = exponent_raw = exponent_stored = 0
    exponent_lanes = set()
    exponent_defined = True
    for entry in tensors:
        spec = specs[entry["dtype"]]
        lane_of_exponent = spec.exponent_stream
        raw += entry["numel"] * entry["element_size"]
        structure += _tensor_fields(entry)
        if lane_of_exponent is None:
            exponent_defined = exponent_defined and not entry["numel"]
        else:
            exponent_raw += entry["numel"]
            exponent_lanes.add((spec.name, lane_of_exponent))
        for lane_index, lane in enumerate(entry["groups"]):
            fields = _lane_fields(lane)
            structure += fields
            if lane_index == lane_of_exponent:
                exponent_stored += fields - 8 + sum(chunk["payload"][1] for chunk in lane)
    exponent_stored += sum(_codebook_size(b) for b in codebooks if (b.dtype, b.stream_id) in exponent_lanes)
    return {
        "raw_bytes": int(raw),
        "compressed_bytes": int(blob_bytes + structure),
        "exponent_raw_bytes": int(exponent_raw) if exponent_defined else None,
        "exponent_compressed_bytes": int(exponent_stored) if exponent_defined else None,
    }
