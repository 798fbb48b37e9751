"""Fixture builders shared by the CPU and GPU tests.

The cases restate the reference's own kernel checks
(scripts/_experiment_kernel_checks.py in the reference project):
  * ``segment_book(max_bits)``: the complete canonical tree with 258 leaves
    whose deepest codes have `max_bits` bits, one common pair token of
    length 1 (:59-73);
  * ``segment_symbols()``: 70,000 copies of the common pair's byte, every
    byte three times and an odd tail (:74-76);
  * ``lanes_with(symbols, spec)``: arbitrary non-selected lane bytes,
    non-finite patterns included (:79-84);
  * ``long_code_book()``: the histogram whose pair count is 2^52, forcing
    codes longer than 12 bits (:214-222);
  * ``pattern_weights``: the repeating [0.25 x4, 0.5 x2, 1 x2] pattern (:134-145).
"""

import heapq

import numpy as np
import torch

from neuralzip_b200.dtypes import DTYPES

VOCAB = bytes((127, 127, 125, 126))


def segment_lengths(max_bits):
    chain = max_bits - 8
    remaining = 258 - chain
    lengths = list(range(2, chain + 1))
    lengths += [max_bits - 1] * (256 - remaining) + [max_bits] * (2 * remaining - 256)
    lengths.insert(256, 1)
    return bytes(lengths)


def segment_symbols():
    return np.array([127] * 70000 + list(range(256)) * 3 + [125, 126, 126], dtype=np.uint8)


def huffman_lengths_heap(counts, prior_count=1):
    """Huffman lengths with heapq tie-breaking by serial (the reference's
    build_mixed_codebook, neuralzip/huff0.py:19-36)."""
    heap = [(int(c) + prior_count, i, i) for i, c in enumerate(counts)]
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
    return bytes(lengths)


def long_code_lengths():
    counts = [1 << (i // 8) for i in range(258)]
    counts[256] = 1 << 52
    return huffman_lengths_heap(counts)


def lanes_with(symbols, spec):
    """Raw element bytes whose selected lane is `symbols` and whose other
    lanes are arbitrary (0..255 repeating), non-finite patterns included."""
    stream_id = spec.gpu_stream
    reordered = np.arange(len(symbols) * spec.element_size, dtype=np.uint32).astype(np.uint8)
    reordered[stream_id::spec.element_size] = symbols
    return spec.reorder_bytes(reordered.tobytes(), restore=True)


def gaussian_raw(numel, sigma, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    t = (torch.randn(numel, generator=g) * sigma).to(dtype)
    return t.view(torch.uint8).numpy().tobytes()


def pattern_weights(numel, dtype, pattern=(0.25, 0.25, 0.25, 0.25, 0.5, 0.5, 1, 1)):
    p = torch.tensor(pattern, dtype=dtype)
    return p.repeat((numel + len(pattern) - 1) // len(pattern))[:numel]


def selected_lane(raw, spec):
    return np.frombuffer(spec.reorder_bytes(raw), dtype=np.uint8)[spec.gpu_stream::spec.element_size]


def greedy_token_counts(symbols, vocab):
    """Greedy pair parse counts (neuralzip/native/mixed_huffman.h:85-115)."""
    lookup = np.zeros(65536, dtype=np.int32)
    for i in range(0, len(vocab), 2):
        lookup[vocab[i] | (vocab[i + 1] << 8)] = 256 + i // 2
    counts = np.zeros(256 + len(vocab) // 2, dtype=np.int64)
    s = symbols.tolist()
    n = len(s)
    i = 0
    while i < n:
        t = lookup[s[i] | (s[i + 1] << 8)] if i + 1 < n else 0
        if t:
            counts[t] += 1
            i += 2
        else:
            counts[s[i]] += 1
            i += 1
    return counts


def top_pairs(symbols, k=254):
    sym = symbols.astype(np.uint32)
    pairs = np.bincount(sym[:-1] | (sym[1:] << 8), minlength=65536)
    observed = np.flatnonzero(pairs)
    order = np.argsort(-pairs[observed], kind="stable")
    return np.sort(observed[order[:k]]).astype("<u2").tobytes()


def mixed_book_for(symbols, k=64):
    """(lengths, vocab) of a mixed table fitted to `symbols`."""
    vocab = top_pairs(symbols, k)
    return huffman_lengths_heap(greedy_token_counts(symbols, vocab)), vocab


SPECS = list(DTYPES.values())
