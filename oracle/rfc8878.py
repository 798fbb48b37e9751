"""Huff0 (RFC 8878) decoding restated in Python: TEST INFRASTRUCTURE ONLY.

The reference's singleton tables and shared_huff0 payloads are zstd Huff0
structures (neuralzip/native/codebooks.h:60-68 reads a table with
HUF_readCTable, :156-206 decodes a 4-stream block with
HUF_decompress4X_usingDTable). zstd itself is not in the reference tree, so
this module restates the published format, independently of the product's
C++ (neuralzip_b200/csrc/nz_huff0.cpp, nz_storage.cpp):

* section 4.1.1, FSE table description (accuracy log, normalized counts,
  "less than 1" probabilities, repeat flags) and the FSE decoding table
  (symbol spread with step (size >> 1) + (size >> 3) + 3);
* section 4.2.1, Huffman tree description: FSE-compressed weights (two
  interleaved states over a backward bitstream) or 4-bit direct weights, the
  implied last weight, code length = max_bits + 1 - weight, and prefix codes
  handed out from the lowest weight (longest code) up, in symbol order;
* section 4.2.2, Huffman-coded streams: 4 streams behind a 6-byte jump
  table, each read backward from its end marker, the first three
  regenerating (size + 3) / 4 bytes.

It is pinned against frames written by the system libzstd
(tests/golden/make_huff0_golden.py, tests/test_huff0_zstd_pin.py). Only
tests import it; the product never does.
"""

from __future__ import annotations

import numpy as np


def _highbit(v):
    return int(v).bit_length() - 1


def read_fse_table_description(data):
    """(accuracy log, normalized counts, bytes used) of an FSE table
    description (section 4.1.1.1); counts of -1 mean "less than 1"."""
    bits = int.from_bytes(bytes(data), "little")
    pos = 0

    def take(n):
        nonlocal pos
        value = (bits >> pos) & ((1 << n) - 1)
        pos += n
        return value

    log = take(4) + 5
    remaining = (1 << log) + 1
    threshold = 1 << log
    width = log + 1
    counts = []
    while remaining > 1:
        largest = 2 * threshold - 1 - remaining
        low = (bits >> pos) & (threshold - 1)
        if low < largest:
            value = low
            pos += width - 1
        else:
            value = (bits >> pos) & (2 * threshold - 1)
            pos += width
            if value >= threshold:
                value -= largest
        count = value - 1
        remaining -= abs(count)
        counts.append(count)
        if count == 0:
            while True:
                repeat = take(2)
                counts.extend([0] * repeat)
                if repeat != 3:
                    break
        while remaining < threshold:
            width -= 1
            threshold >>= 1
    if remaining != 1:
        raise ValueError("FSE counts do not sum to the table size")
    return log, counts, (pos + 7) // 8


def fse_decoding_table(counts, log):
    """[(symbol, bits to read, baseline)] per state (section 4.1.1.2)."""
    size = 1 << log
    symbol = [0] * size
    high = size - 1
    for s, c in enumerate(counts):
        if c == -1:
            symbol[high] = s
            high -= 1
    step, mask, position = (size >> 1) + (size >> 3) + 3, size - 1, 0
    for s, c in enumerate(counts):
        for _ in range(max(c, 0)):
            symbol[position] = s
            position = (position + step) & mask
            while position > high:
                position = (position + step) & mask
    following = [1 if c == -1 else max(c, 0) for c in counts]
    table = []
    for state in range(size):
        s = symbol[state]
        nxt = following[s]
        following[s] += 1
        n = log - _highbit(nxt)
        table.append((s, n, (nxt << n) - size))
    return table


class BackwardBits:
    """Bits of a backward bitstream (read from just below the end marker of
    the last byte towards bit 0 of the first); reads past the start yield
    zeros and set `overflow`."""

    def __init__(self, data):
        data = bytes(data)
        if not data or data[-1] == 0:
            raise ValueError("backward bitstream without an end marker")
        self.value = int.from_bytes(data, "little")
        self.left = 8 * (len(data) - 1) + _highbit(data[-1])
        self.overflow = False

    def read(self, n):
        if n == 0:
            return 0
        if n > self.left:
            value = (self.value & ((1 << self.left) - 1)) << (n - self.left) if self.left > 0 else 0
            self.left -= n
            self.overflow = True
            return value
        self.left -= n
        return (self.value >> self.left) & ((1 << n) - 1)


def decode_fse_weights(data):
    """Weights of an FSE-compressed weight block (section 4.2.1.2)."""
    log, counts, used = read_fse_table_description(data)
    table = fse_decoding_table(counts, log)
    bits = BackwardBits(data[used:])
    states = [bits.read(log), bits.read(log)]
    weights = []
    k = 0
    while True:
        s, n, base = table[states[k]]
        weights.append(s)
        states[k] = base + bits.read(n)
        if bits.left < 0:
            weights.append(table[states[1 - k]][0])
            return weights
        k = 1 - k


def tree_description(data):
    """(256 code lengths, bytes used) of a Huffman tree description
    (section 4.2.1)."""
    head = data[0]
    if head < 128:
        weights = decode_fse_weights(bytes(data[1:1 + head]))
        used = 1 + head
    else:
        n = head - 127
        packed = data[1:1 + (n + 1) // 2]
        weights = [(packed[i // 2] >> (0 if i % 2 else 4)) & 15 for i in range(n)]
        used = 1 + (n + 1) // 2
    total = sum(1 << (w - 1) for w in weights if w)
    max_bits = _highbit(total) + 1
    rest = (1 << max_bits) - total
    if rest & (rest - 1):
        raise ValueError("the implied last weight is not a power of two")
    weights.append(_highbit(rest) + 1)
    lengths = [0] * 256
    for s, w in enumerate(weights):
        if w:
            lengths[s] = max_bits + 1 - w
    return lengths, used


def canonical_codes(lengths):
    """Code value per symbol: from the longest length to the shortest, in
    symbol order within a length, counting up from zero."""
    codes = [0] * len(lengths)
    value, current = 0, max(lengths)
    for length in range(current, 0, -1):
        value >>= current - length
        current = length
        for s, l in enumerate(lengths):
            if l == length:
                codes[s] = value
                value += 1
    return codes


def _stream(lengths, codes, data, count, max_bits):
    table = [None] * (1 << max_bits)
    for s, (l, c) in enumerate(zip(lengths, codes)):
        if l:
            for w in range(c << (max_bits - l), (c + 1) << (max_bits - l)):
                table[w] = (s, l)
    data = bytes(data)
    total = 8 * (len(data) - 1) + _highbit(data[-1])
    bits = np.unpackbits(np.frombuffer(data, dtype=np.uint8), bitorder="little")[:total][::-1]
    bits = np.concatenate([bits, np.zeros(max_bits, dtype=np.uint8)]).astype(np.int64)
    windows = np.zeros(total + 1, dtype=np.int64)
    for j in range(max_bits):
        windows = (windows << 1) | bits[j:j + total + 1]
    windows = windows.tolist()
    out = bytearray()
    pos = 0
    for _ in range(count):
        entry = table[windows[pos]] if pos <= total else None
        if entry is None:
            raise ValueError("invalid Huffman code")
        out.append(entry[0])
        pos += entry[1]
    if pos != total:
        raise ValueError("stream not fully consumed")
    return bytes(out)


def decode_4streams(lengths, data, count):
    """Bytes of a 4-stream Huffman block (jump table + streams)."""
    codes = canonical_codes(lengths)
    max_bits = max(lengths)
    sizes = [int.from_bytes(data[2 * i:2 * i + 2], "little") for i in range(3)]
    sizes.append(len(data) - 6 - sum(sizes))
    segment = (count + 3) // 4
    out, pos = bytearray(), 6
    for i, size in enumerate(sizes):
        n = segment if i < 3 else count - 3 * segment
        out += _stream(lengths, codes, data[pos:pos + size], n, max_bits)
        pos += size
    return bytes(out)
