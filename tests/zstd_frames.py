"""Zstandard frames around Huff0 literal blocks (RFC 8878), for pinning the
product's Huff0 code against the zstd library installed on this image.

The reference's singleton (shared_huff0) tables and payloads come from zstd's
Huff0 (neuralzip/native/codebooks.h:20-39, 60-68, 131-141, 156-206), which
is not in the reference tree. The system libzstd (1.5.5 here) writes the
same two structures inside every frame whose literals it Huffman-codes: a
Huffman tree description (RFC 8878 section 4.2.1) and 4-stream Huffman data
(section 4.2.2, "Huffman-coded Streams"). This module

* asks zstd for frames that carry only literals (ZSTD_compressSequences with
  no sequences, so the regenerated literals are exactly the input),
* parses a frame down to its literals section (sections 3.1.1, 3.1.1.2 and
  3.1.1.3.1), and
* assembles a frame from a tree description and 4 streams written by the
  product, for zstd's own decoder to check.
"""

from __future__ import annotations

import ctypes
import ctypes.util

ZSTD_MAGIC = b"\x28\xb5\x2f\xfd"


class _Sequence(ctypes.Structure):
    _fields_ = [("offset", ctypes.c_uint), ("litLength", ctypes.c_uint), ("matchLength", ctypes.c_uint),
                ("rep", ctypes.c_uint)]


def library():
    """The system libzstd through ctypes, or None when it is absent."""
    path = ctypes.util.find_library("zstd")
    if not path:
        return None
    lib = ctypes.CDLL(path)
    lib.ZSTD_versionString.restype = ctypes.c_char_p
    lib.ZSTD_compressBound.restype = ctypes.c_size_t
    lib.ZSTD_compressBound.argtypes = [ctypes.c_size_t]
    lib.ZSTD_createCCtx.restype = ctypes.c_void_p
    lib.ZSTD_freeCCtx.argtypes = [ctypes.c_void_p]
    lib.ZSTD_isError.argtypes = [ctypes.c_size_t]
    lib.ZSTD_isError.restype = ctypes.c_uint
    lib.ZSTD_getErrorName.argtypes = [ctypes.c_size_t]
    lib.ZSTD_getErrorName.restype = ctypes.c_char_p
    lib.ZSTD_compressSequences.restype = ctypes.c_size_t
    lib.ZSTD_compressSequences.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.POINTER(_Sequence), ctypes.c_size_t, ctypes.c_void_p,
                                           ctypes.c_size_t]
    lib.ZSTD_decompress.restype = ctypes.c_size_t
    lib.ZSTD_decompress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
    return lib


def _check(lib, n):
    if lib.ZSTD_isError(n):
        raise RuntimeError(lib.ZSTD_getErrorName(n).decode())
    return n


def literals_frame(lib, data):
    """A zstd frame of `data` with no matches: every block is literals only."""
    data = bytes(data)
    cap = lib.ZSTD_compressBound(len(data))
    out = ctypes.create_string_buffer(cap)
    src = ctypes.create_string_buffer(data, len(data))
    cctx = lib.ZSTD_createCCtx()
    try:
        n = _check(lib, lib.ZSTD_compressSequences(cctx, out, cap, None, 0, src, len(data)))
    finally:
        lib.ZSTD_freeCCtx(cctx)
    return out.raw[:n]


def decompress(lib, frame, size):
    out = ctypes.create_string_buffer(max(size, 1))
    src = ctypes.create_string_buffer(bytes(frame), len(frame))
    n = _check(lib, lib.ZSTD_decompress(out, size, src, len(frame)))
    return out.raw[:n]


def frame_blocks(frame):
    """[(block type, block content)] of a frame (RFC 8878 section 3.1.1)."""
    frame = bytes(frame)
    if frame[:4] != ZSTD_MAGIC:
        raise ValueError("not a zstd frame")
    descriptor = frame[4]
    pos = 5
    fcs_flag, single_segment, dict_flag = descriptor >> 6, (descriptor >> 5) & 1, descriptor & 3
    if not single_segment:
        pos += 1  # window descriptor
    pos += (0, 1, 2, 4)[dict_flag]
    pos += (1 if single_segment else 0, 2, 4, 8)[fcs_flag]
    blocks = []
    while True:
        header = int.from_bytes(frame[pos:pos + 3], "little")
        pos += 3
        last, kind, size = header & 1, (header >> 1) & 3, header >> 3
        content = frame[pos:pos + (1 if kind == 1 else size)]
        pos += len(content)
        blocks.append((kind, content))
        if last:
            return blocks


def tree_description_size(data):
    """Bytes of the Huffman tree description at the start of `data`
    (section 4.2.1: a header byte < 128 is followed by that many bytes of
    FSE-coded weights; one >= 128 by (byte - 127) 4-bit weights)."""
    head = data[0]
    return 1 + head if head < 128 else 1 + (head - 127 + 1) // 2


def literals_section(block):
    """(regenerated size, stream count, tree description, stream data, rest)
    of a compressed block's Huffman-coded literals section (3.1.1.3.1)."""
    block = bytes(block)
    kind, size_format = block[0] & 3, (block[0] >> 2) & 3
    if kind != 2:
        raise ValueError(f"literals section type {kind} is not Huffman-coded with a tree")
    header_size, bits = {0: (3, 10), 1: (3, 10), 2: (4, 14), 3: (5, 18)}[size_format]
    value = int.from_bytes(block[:header_size], "little")
    regenerated = (value >> 4) & ((1 << bits) - 1)
    compressed = (value >> (4 + bits)) & ((1 << bits) - 1)
    body = block[header_size:header_size + compressed]
    tree = tree_description_size(body)
    return regenerated, 1 if size_format == 0 else 4, body[:tree], body[tree:], block[header_size + compressed:]


def literals_only_frame(tree, streams, regenerated):
    """One frame holding one compressed block: a Huffman-coded literals
    section (`tree` + 4 `streams`, the jump table included) and an empty
    sequences section. Single segment, content size given, no checksum."""
    compressed = len(tree) + len(streams)
    if regenerated >= 1 << 18 or compressed >= 1 << 18:
        raise ValueError("literals too large for one section")
    size_format, header_size, bits = (1, 3, 10) if max(regenerated, compressed) < 1 << 10 else \
        (2, 4, 14) if max(regenerated, compressed) < 1 << 14 else (3, 5, 18)
    value = 2 | (size_format << 2) | (regenerated << 4) | (compressed << (4 + bits))
    block = value.to_bytes(header_size, "little") + bytes(tree) + bytes(streams) + b"\x00"
    if len(block) >= 1 << 17:
        raise ValueError("block too large")
    block_header = (1 | (2 << 1) | (len(block) << 3)).to_bytes(3, "little")
    # Frame header: single segment, 4-byte content size (flag 2), no dictionary, no checksum.
    descriptor = (2 << 6) | (1 << 5)
    return ZSTD_MAGIC + bytes([descriptor]) + regenerated.to_bytes(4, "little") + block_header + block
