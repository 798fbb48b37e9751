"""CPU checks of the product packer and decode tables (no GPU needed).

The packer's tile layout is read back by the oracle's independent
bit-by-bit reader (oz_tile_decode) and by a step-for-step model of the
kernel's lane loop over the product's decode table (tests/kernel_model.py);
both must return the selected lane exactly.
"""

import numpy as np
import pytest
import torch

import helpers as H
import kernel_model as KM
from neuralzip_b200 import _native
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu.inference import GPUCodebook, encode_raw_fragment, encode_with_codebook
from oracle import oracle as O


def _roundtrip(raw, spec, book, model=True):
    enc = encode_with_codebook(raw, book, dtype=spec, stream_id=spec.gpu_stream)
    sym = enc.symbols
    bits = np.frombuffer(sym.bitstream, dtype=np.uint32)
    lens = np.frombuffer(sym.lane_bits, dtype=np.uint16)
    tile_off = np.asarray(sym.tile_offsets, dtype=np.uint32)
    expected = H.selected_lane(raw, spec)
    got = O.tile_decode(bits, lens, tile_off, enc.numel, book.code_lengths, book.code_values, book.vocab)
    assert np.array_equal(got, expected)
    if model:
        modeled = KM.decode_group(np.asarray(book.decode_lut), bits, lens, tile_off, enc.numel,
                                  lut_words=book.table_words)
        assert np.array_equal(modeled, expected)
    lanes = O.split(raw, spec)
    for lane, data in enumerate(enc.streams):
        if lane != spec.gpu_stream:
            assert data == lanes[lane].tobytes()
    assert sum(int(x) for x in lens) == sym.bit_length
    return enc


@pytest.mark.parametrize("max_bits", [12, 13, 20, 31, 32, 33, 56])
def test_segment_books_roundtrip(max_bits):
    lengths = H.segment_lengths(max_bits)
    values = O.mixed_codes(lengths)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in values), H.VOCAB)
    # Codes of 13..31 bits decode through the canonical tables (the entries
    # and those tables are staged); longer ones walk the suffix tree too.
    if max_bits == 12:
        assert book.table_words == _native.LUT_CANON
    elif max_bits <= 31:
        assert book.table_words == _native.LUT_TREE
    else:
        assert book.table_words > _native.LUT_TREE
    for spec in DTYPES.values():
        raw = H.lanes_with(H.segment_symbols(), spec)
        _roundtrip(raw, spec, book, model=spec.name == "bfloat16")


def test_long_code_book_roundtrip():
    lengths = H.long_code_lengths()
    values = O.mixed_codes(lengths)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in values), H.VOCAB)
    assert book.native.tree_nodes > 0
    symbols = np.array([127] * 70000 + list(range(256)) * 3 + [126], dtype=np.uint8)
    _roundtrip(H.lanes_with(symbols, DTYPES[torch.bfloat16]), DTYPES[torch.bfloat16], book)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_gaussian_singleton_and_mixed(dtype):
    spec = DTYPES[dtype]
    raw = H.gaussian_raw(70001, 0.02, dtype, 1)
    sel = H.selected_lane(raw, spec)
    header, _ = _native.huff0_build(np.bincount(sel, minlength=256) + 1, 12)
    lengths, values, _, _ = _native.huff0_read(header)
    _roundtrip(raw, spec, GPUCodebook(tuple(lengths), values))
    if spec.exponent_stream is not None:
        lengths, vocab = H.mixed_book_for(sel)
        _roundtrip(raw, spec, GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab))


def test_pairs_never_straddle_substreams():
    # The pair (7, 7) everywhere: elements 255 and 256 of a group must not
    # form a pair, since they belong to different sub-streams.
    counts = [1] * 256 + [10_000]
    counts[7] = 1000
    lengths = H.huffman_lengths_heap(counts)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), bytes((7, 7)))
    symbols = np.full(257 * 3, 7, dtype=np.uint8)
    spec = DTYPES[torch.bfloat16]
    _roundtrip(H.lanes_with(symbols, spec), spec, book)


def test_raw_fragment_lanes():
    spec = DTYPES[torch.float32]
    raw = H.gaussian_raw(1001, 0.5, torch.float32, 2)
    enc = encode_raw_fragment(raw, dtype=spec, stream_id=3)
    lanes = O.split(raw, spec)
    assert enc.symbols.bitstream == lanes[3].tobytes()
    assert all(enc.streams[i] == lanes[i].tobytes() for i in range(3))


def test_empty_and_tiny_groups():
    lengths = H.segment_lengths(12)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), H.VOCAB)
    spec = DTYPES[torch.bfloat16]
    for n in (1, 2, 255, 256, 257, 8191, 8192, 8193):
        _roundtrip(H.lanes_with(np.full(n, 127, dtype=np.uint8), spec), spec, book)
    enc = encode_with_codebook(b"", book, dtype=spec, stream_id=1)
    assert enc.numel == 0 and enc.symbols.bit_length == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_merge_arithmetic_model_restores_elements(dtype):
    """The kernel's byte-wise undo of the sign/exponent reorder (four
    elements per step: bit selects, shifts and byte permutes) rebuilds the
    original elements from the oracle's lane split."""
    spec = DTYPES[dtype]
    es = spec.element_size
    rng = np.random.default_rng(7)
    raw = rng.integers(0, 256, size=4 * es * 256, dtype=np.uint8)
    raw[:4 * es * 4] = 0xFF  # all-ones and all-zero words
    raw[4 * es * 4:4 * es * 8] = 0
    lanes = O.split(raw, spec)

    def word(lane, i):
        return int.from_bytes(lanes[lane][4 * i:4 * i + 4].tobytes(), "little")

    for i in range(256):
        if es == 2:
            words = KM.merge_bf16_words(word(0, i), word(1, i))
        else:
            words = KM.merge_fp32_words(word(0, i), word(1, i), word(2, i), word(3, i))
        got = b"".join(w.to_bytes(4, "little") for w in words)
        assert got == raw[4 * es * i:4 * es * (i + 1)].tobytes(), i


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_random_long_code_books_decode_through_canonical_tables(seed):
    """Random skewed histograms over 256 bytes and 254 pairs give codes of
    up to 31 bits; they decode through the canonical limit/offset/leaf
    tables (no suffix tree staged), identically in the kernel model and the
    oracle's bit-by-bit reader."""
    rng = np.random.default_rng(100 + seed)
    counts = (rng.pareto(0.6 + 0.1 * seed, size=510) * 10).astype(np.int64) + 1
    counts[rng.integers(0, 510, size=8)] = 1 << 24  # a few dominant tokens push the rest long
    lengths = H.huffman_lengths_heap(counts)
    longest = max(lengths)
    if not 13 <= longest <= 31:
        pytest.skip(f"longest code {longest} is outside the canonical range")
    vocab = rng.choice(65536, size=254, replace=False).astype("<u2").tobytes()
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
    assert book.table_words == _native.LUT_TREE
    spec = DTYPES[torch.bfloat16]
    symbols = rng.integers(0, 256, size=3 * 8192 + 77, dtype=np.uint8)
    _roundtrip(H.lanes_with(symbols, spec), spec, book)


def test_long_codes_in_any_order_within_a_length_use_the_limit_tables():
    """The limit tables need only that each length's codes are consecutive
    values and that longer codes have larger left-justified values: the
    symbols of one length may take them in any order."""
    lengths = H.segment_lengths(20)
    canonical = [int(v) for v in O.mixed_codes(lengths)]
    values = list(canonical)
    for length in set(lengths):
        idx = [i for i, n in enumerate(lengths) if n == length]
        for i, j in zip(idx, reversed(idx)):
            values[i] = canonical[j]
    book = GPUCodebook(tuple(lengths), tuple(values), H.VOCAB)
    assert book.table_words == _native.LUT_TREE
    spec = DTYPES[torch.bfloat16]
    _roundtrip(H.lanes_with(H.segment_symbols(), spec), spec, book)


def test_non_canonical_long_codes_use_the_suffix_tree():
    """Codes with every bit flipped (still a complete prefix code, but the
    longest codes now have the smallest values) cannot use the limit
    tables: the kernel walks the suffix tree instead, with the same
    result."""
    lengths = H.segment_lengths(20)
    values = [(1 << n) - 1 - int(v) for n, v in zip(lengths, O.mixed_codes(lengths))]
    book = GPUCodebook(tuple(lengths), tuple(values), H.VOCAB)
    assert book.table_words > _native.LUT_TREE
    spec = DTYPES[torch.bfloat16]
    _roundtrip(H.lanes_with(H.segment_symbols(), spec), spec, book)
