"""Codebook builders and the CPU codec entry points.

Same functions as neuralzip/huff0.py:1-74 (count_mixed_tokens,
build_mixed_codebook, build_codebook_from_counts, build_codebook_from_header,
build_decodebook, export_code_table, compress_direct_storage,
decompress_mixed_streams_many), implemented over libnzb200's host codec
instead of the nanobind/zstd extension. A codebook handle is a host table
object (NativeCodebook) rather than a PyCapsule.
"""

from __future__ import annotations

import heapq
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

from neuralzip_b200 import _native

MAX_BLOCK_SIZE = 128 * 1024  # Huff0 block limit (HUF_BLOCKSIZE_MAX)
MAX_HISTOGRAM_TOTAL = (1 << 30) - 1
MAX_WORKERS = 16  # neuralzip/native/common.h:146


@dataclass(frozen=True)
class Huff0Codebook:
    handle: object
    codebook: bytes


def _workers(threads, jobs, total_bytes):
    """Worker count of the reference's pool (common.h:134-150)."""
    import os

    count = threads if threads > 0 else (os.cpu_count() or 1)
    count = max(1, min(count, MAX_WORKERS, jobs))
    return 1 if total_bytes < (512 << 10) else count


def count_mixed_tokens(chunks, vocab):
    """Greedy pair/singleton token counts that do not cross chunk
    boundaries (mixed_huffman.h:96-115)."""
    vocab = bytes(vocab)
    if len(vocab) % 2 or len(vocab) > 508:
        raise RuntimeError("Invalid mixed pair vocabulary.")
    counts = np.zeros(256 + len(vocab) // 2, dtype=np.uint64)
    for chunk in chunks:
        _native.count_tokens(chunk, vocab, counts)
    return tuple(int(c) for c in counts)


def build_mixed_codebook(counts, vocab, *, prior_count=1):
    """Huffman lengths over singleton + pair tokens with heapq tie-breaking
    by insertion serial (neuralzip/huff0.py:19-36), as an "NZM1" header."""
    heap = [(int(count) + prior_count, i, i) for i, count in enumerate(counts)]
    heapq.heapify(heap)
    serial = len(heap)
    while len(heap) > 1:
        left, _, a = heapq.heappop(heap)
        right, _, b = heapq.heappop(heap)
        heapq.heappush(heap, (left + right, serial, (a, b)))
        serial += 1
    lengths = bytearray(len(counts))
    stack = [(heap[0][2], 0)]
    while stack:
        node, depth = stack.pop()
        if isinstance(node, int):
            lengths[node] = max(1, depth)
        else:
            stack.extend((child, depth + 1) for child in node)
    return build_codebook_from_header(b"NZM1" + bytes(lengths), vocab=vocab)


def _scaled_counts(symbol_counts, prior_count):
    """Histogram scaling of parse_symbol_counts (binding_helpers.h:9-66):
    shift counts down until their total plus priors stays below 2^30."""
    counts = [int(c) for c in symbol_counts]
    if len(counts) != 256:
        raise ValueError("symbol_counts must contain exactly 256 entries.")
    if any(c < 0 for c in counts):
        raise OverflowError("Huff0 symbol counts must be non-negative.")
    prior_total = prior_count * 256
    if prior_total >= MAX_HISTOGRAM_TOTAL:
        raise ValueError("prior_count is too large for a 256-symbol Huff0 table.")
    available = MAX_HISTOGRAM_TOTAL - prior_total
    shift = 0
    if sum(counts) > available:
        for shift in range(1, 64):
            if sum(max(1, c >> shift) for c in counts if c) <= available:
                break
        else:
            raise OverflowError("Huff0 symbol count overflow.")
    return np.array([(max(1, c >> shift) if c else 0) + prior_count for c in counts], dtype=np.uint64)


def build_codebook_from_counts(symbol_counts, *, prior_count=0, max_bits=11):
    """Singleton table from a 256-bin histogram, serialized as a Huff0
    header (build_codebook_from_counts, binding_helpers.h:68-90). Raises
    RuntimeError when the alphabet cannot be serialized."""
    if not (1 <= int(max_bits) <= 12):
        raise ValueError("max_bits must be in [1, 12].")
    if prior_count < 0:
        raise ValueError("prior_count must fit in unsigned.")
    counts = _scaled_counts(symbol_counts, int(prior_count))
    header, _lengths = _native.huff0_build(counts, int(max_bits))
    return build_codebook_from_header(header)


def build_codebook_from_header(codebook, *, vocab=b""):
    """Host encode/decode tables of a serialized table (Huff0 or "NZM1")."""
    codebook = bytes(codebook)
    vocab = bytes(vocab)
    if not codebook:
        raise RuntimeError("Huff0 codebook header is empty.")
    lengths, values, _longest = _native.export_code_table(codebook, max_bits=56, vocab=vocab)
    return Huff0Codebook(_native.NativeCodebook(lengths, values, vocab), codebook)


def build_decodebook(codebook, *, vocab=b""):
    return build_codebook_from_header(codebook, vocab=vocab).handle


def export_code_table(codebook, *, max_bits=12, vocab=b""):
    return _native.export_code_table(bytes(codebook), max_bits=int(max_bits), vocab=bytes(vocab))


# ---- storage container (neuralzip/native/direct_storage.h, decode_queue.h) ----

SHARED_CHUNK_METADATA_BYTES = 25


def _selected_and_raw_lanes(data, element_size, bit_reorder, mantissa_bits, exponent_bits, stream_id):
    raw = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
    dt = _native.dtype_struct(element_size, bit_reorder, mantissa_bits, exponent_bits, stream_id)
    return _native.split_lanes(raw, dt)


def compress_direct_storage(tensor_specs, prefix, *, min_saving_bytes=0, threads=0, compression_threshold=0.95):
    """Encodes one selected lane per tensor into one buffer laid out as
    prefix | raw lanes | compacted selected-lane payloads and returns
    (bytearray, groups) where groups[t][lane] lists (mode, symbols,
    codebook_id, offset, size) per chunk (direct_storage.h:72-214).

    tensor_specs: (data, dtype spec, stream_id, chunk_size, modes), modes
    holding one compressor.ChunkMode per source chunk (the reference's
    Python wrapper takes the same tuple, neuralzip/huff0.py:40-53)."""
    if min_saving_bytes < 0 or threads < 0:
        raise ValueError("min_saving_bytes and threads must be non-negative.")
    if not (0 < compression_threshold <= 1):
        raise ValueError("compression_threshold must be in (0, 1].")
    prefix = bytes(prefix)
    requests = []
    total_symbols = total_bytes = 0
    jobs = []
    for index, (data, spec, stream_id, chunk_size, modes) in enumerate(tensor_specs):
        data = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
        es = spec.element_size
        if len(data) % es:
            raise ValueError("Direct storage input must contain complete elements.")
        symbols = len(data) // es
        starts = list(range(0, symbols, int(chunk_size)))
        if len(modes) != len(starts):
            raise ValueError("Each source chunk needs exactly one frozen mode.")
        requests.append(dict(data=data, spec=spec, stream=int(stream_id), symbols=symbols,
                             symbol_offset=total_symbols, raw_offset=total_bytes - total_symbols, modes=modes,
                             first_job=len(jobs)))
        for j, start in enumerate(starts):
            jobs.append((index, start, min(int(chunk_size), symbols - start), j))
        total_symbols += symbols
        total_bytes += len(data)
    output = bytearray(len(prefix) + total_bytes)
    output[:len(prefix)] = prefix
    view = np.frombuffer(output, dtype=np.uint8)
    raw_base = len(prefix)
    selected_base = len(prefix) + total_bytes - total_symbols
    results = [None] * len(jobs)
    lanes_cache = {}

    def lanes_of(index):
        if index not in lanes_cache:
            r = requests[index]
            spec = r["spec"]
            lanes_cache[index] = _selected_and_raw_lanes(r["data"], spec.element_size, spec.bit_reorder,
                                                         spec.mantissa_bits, spec.exponent_bits, r["stream"])
        return lanes_cache[index]

    for index in range(len(requests)):  # lane split once per tensor
        lanes = lanes_of(index)
        r = requests[index]
        for lane in range(r["spec"].element_size):
            if lane == r["stream"]:
                continue
            slot = lane - (lane > r["stream"])
            base = raw_base + r["raw_offset"] + slot * r["symbols"]
            view[base:base + r["symbols"]] = lanes[lane]

    def run(j):
        index, start, length, local = jobs[j]
        r = requests[index]
        mode = r["modes"][local]
        symbols = lanes_of(index)[r["stream"]][start:start + length]
        budget = int(length * compression_threshold) - SHARED_CHUNK_METADATA_BYTES
        kind, book = mode.kind, mode.codebook
        payload = b""
        if budget > 0 and kind == "shared_huff0":
            payload = _native.huff0_encode(book.handle, symbols, length) if length <= MAX_BLOCK_SIZE else b""
            if len(payload) > budget:
                payload = b""
        elif budget > 0 and kind == "mixed_huffman":
            payload = _native.mixed_encode(book.handle, symbols, budget)
        if payload and len(payload) + min_saving_bytes < length and \
                len(payload) + SHARED_CHUNK_METADATA_BYTES < length * compression_threshold:
            results[j] = (kind, payload)
        else:
            results[j] = ("raw", symbols.tobytes())

    workers = _workers(threads, len(jobs), total_bytes)
    if workers > 1:
        with ThreadPoolExecutor(workers) as pool:
            list(pool.map(run, range(len(jobs))))
    else:
        for j in range(len(jobs)):
            run(j)
    cursor = selected_base
    offsets = []
    for kind, payload in results:
        offsets.append(cursor)
        view[cursor:cursor + len(payload)] = np.frombuffer(payload, dtype=np.uint8)
        cursor += len(payload)
    del view
    output[cursor:] = b""
    groups = []
    for index, r in enumerate(requests):
        tensor_groups = []
        for lane in range(r["spec"].element_size):
            chunks = []
            for j in range(r["first_job"], r["first_job"] + len(r["modes"])):
                _, start, length, local = jobs[j]
                if lane == r["stream"]:
                    kind, payload = results[j]
                    mode = r["modes"][local]
                    cid = -1 if kind == "raw" else mode.codebook_id
                    chunks.append((kind, length, cid, offsets[j], len(payload)))
                else:
                    slot = lane - (lane > r["stream"])
                    chunks.append(("raw", length, -1, raw_base + r["raw_offset"] + start + slot * r["symbols"],
                                   length))
            tensor_groups.append(tuple(chunks))
        groups.append(tuple(tensor_groups))
    return output, tuple(groups)


# (mantissa, exponent) bits of the element layouts storage holds, by
# (element size, reorder): bf16, fp32 and fp16 (neuralzip/dtypes.py:53-83).
_WIDTH_FIELDS = {(2, 1): (7, 8), (4, 1): (23, 8), (2, 0): (10, 5), (4, 0): (23, 8)}


def decompress_mixed_streams_many(tensor_specs, *, threads=0):
    """Decodes tensors from per-lane chunk lists (decode_queue.h:1-113):
    spec = (element_size, bit_reorder, numel, groups) where groups[lane] is a
    sequence of (mode, payload, symbol_count, decodebook). Returns one
    bytearray of element bytes per tensor. One native call
    (nz_storage_decode) decodes, merges and restores every chunk."""
    if threads < 0:
        raise ValueError("threads must be non-negative.")
    pieces, lane_records, keep, outputs = [], [], [], []
    for element_size, bit_reorder, numel, groups in tensor_specs:
        if element_size not in (2, 4) or numel < 0:
            raise ValueError("Invalid decoded width or element count.")
        if len(groups) != element_size:
            raise ValueError("Decode needs one group per byte stream.")
        if any(len(lane) != len(groups[0]) for lane in groups):
            raise ValueError("Unaligned chunk groups.")
        mant_bits, exp_bits = _WIDTH_FIELDS[(element_size, int(bool(bit_reorder)))]
        out = bytearray(numel * element_size)
        outputs.append(out)
        out_at = np.frombuffer(out, dtype=np.uint8).ctypes.data if numel else 0
        first = 0
        for c in range(len(groups[0])):
            count = int(groups[0][c][2])
            if count < 0 or count > numel - first:
                raise ValueError("Chunk exceeds its tensor element count.")
            if any(int(lane[c][2]) != count for lane in groups):
                raise ValueError("Unaligned chunk boundaries.")
            records = []
            for mode, payload, symbols, book in (lane[c] for lane in groups):
                code = _native.CHUNK_MODES.get(mode)
                if code is None:
                    raise ValueError("Unsupported decoded chunk mode.")
                if code != _native.CHUNK_RAW and book is None:
                    raise ValueError("Compressed chunk needs a decode table.")
                data = np.frombuffer(memoryview(payload).cast("B"), dtype=np.uint8)
                keep.append(data)
                records.append((data.ctypes.data if len(data) else 0, len(data),
                                book.handle.value if book is not None else 0, code, 0))
            lane_records.append(np.array(records, dtype=_native.STORAGE_LANE_DTYPE))
            pieces.append((lane_records[-1].ctypes.data, out_at + first * element_size, count, element_size,
                           int(bool(bit_reorder)), mant_bits, exp_bits, 0, 0))
            first += count
        if first != numel:
            raise ValueError("Byte stream does not reconstruct exactly numel values.")
    _native.storage_decode(np.array(pieces, dtype=_native.STORAGE_PIECE_DTYPE), threads)
    return outputs
