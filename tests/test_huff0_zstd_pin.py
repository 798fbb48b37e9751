"""The singleton (Huff0) path pinned against zstd's own output and decoder.

The reference codes singleton chunks with zstd's Huff0 (table headers from
HUF_writeCTable_wksp, neuralzip/native/codebooks.h:20-39, read back with
HUF_readCTable, :60-68; payloads from HUF_compress4X_usingCTable, :131-141,
decoded by HUF_decompress4X_usingDTable, :156-206). zstd is not in the
reference tree; tests/golden/zstd_huff0_vectors.npz holds literals-only
frames that the system zstd library (1.5.5) wrote for seeded byte lanes
(tests/golden/make_huff0_golden.py). Pinned here:

* decode direction: the Huffman tree descriptions and 4-stream blocks zstd
  wrote decode to the input bytes through the RFC 8878 restatement in
  oracle/rfc8878.py and through the product's reader and decoder, and the
  two agree on every code length and code;
* stream bytes: for zstd's code lengths, the product's 4-stream encoder
  writes zstd's stream bytes exactly;
* encode direction (needs libzstd at test time): headers and blocks the
  product writes, for its own tables and for zstd's lengths, wrapped in a
  zstd frame, decode in zstd's decoder to the input.

Not pinned, and checked as a bound instead: the product's length-limited
Huffman lengths equal zstd's on some histograms and differ by a few symbols
on others (zstd's length-limiting heuristic is not published outside its
source); and its FSE-coded weight headers pick a different accuracy log
from zstd's, so header bytes differ while describing the same lengths.
"""

from pathlib import Path

import numpy as np
import pytest

import zstd_frames as Z
from neuralzip_b200 import _native
from oracle import rfc8878 as R

GOLDEN = np.load(Path(__file__).with_name("golden") / "zstd_huff0_vectors.npz")
CASES = sorted(k[:-len("_frame")] for k in GOLDEN.files if k.endswith("_frame"))
ZSTD = Z.library()
needs_zstd = pytest.mark.skipif(ZSTD is None, reason="libzstd not found")


def _case(name):
    frame = GOLDEN[f"{name}_frame"].tobytes()
    (_kind, block), = Z.frame_blocks(frame)
    regenerated, _streams, tree, streams, _rest = Z.literals_section(block)
    data = GOLDEN[f"{name}_data"].tobytes()
    assert regenerated == len(data)
    return tree, streams, data


def _cost(lengths, data):
    counts = np.bincount(np.frombuffer(data, dtype=np.uint8), minlength=256)
    return int((counts * np.frombuffer(bytes(lengths), dtype=np.uint8).astype(np.int64)).sum())


def test_fixture_is_from_zstd():
    assert bytes(GOLDEN["zstd_version"]).startswith(b"1.")
    assert len(CASES) >= 7


@pytest.mark.parametrize("name", CASES)
def test_oracle_decodes_zstd_blocks(name):
    tree, streams, data = _case(name)
    lengths, used = R.tree_description(tree)
    assert used == len(tree)
    assert R.decode_4streams(lengths, streams, len(data)) == data


@pytest.mark.parametrize("name", CASES)
def test_product_reads_zstd_tables_and_decodes_zstd_blocks(name):
    tree, streams, data = _case(name)
    lengths, values, table_log, used = _native.huff0_read(tree)
    oracle_lengths, _ = R.tree_description(tree)
    oracle_codes = R.canonical_codes(oracle_lengths)
    assert used == len(tree) and table_log == max(oracle_lengths)
    assert lengths == bytes(oracle_lengths)
    assert [v for v, l in zip(values, lengths) if l] == [c for c, l in zip(oracle_codes, oracle_lengths) if l]
    book = _native.NativeCodebook(lengths, np.asarray(values, dtype=np.uint64))
    assert _native.huff0_decode(book, streams, len(data)).tobytes() == data
    # The same table through the export path the GPU codebooks use.
    export_lengths, export_values, longest = _native.export_code_table(tree, 12)
    assert export_lengths == lengths and longest == table_log


@pytest.mark.parametrize("name", CASES)
def test_product_streams_are_zstd_bytes(name):
    tree, streams, data = _case(name)
    lengths, values, _, _ = _native.huff0_read(tree)
    book = _native.NativeCodebook(lengths, np.asarray(values, dtype=np.uint64))
    assert _native.huff0_encode(book, np.frombuffer(data, dtype=np.uint8), len(streams) + 64) == streams


@pytest.mark.parametrize("name", CASES)
def test_product_length_builder_against_zstd(name):
    """For zstd's table log, the product's length-limited Huffman code is a
    complete prefix code whose cost on the data is within 0.1% of zstd's."""
    tree, _streams, data = _case(name)
    zstd_lengths, _ = R.tree_description(tree)
    counts = np.bincount(np.frombuffer(data, dtype=np.uint8), minlength=256).astype(np.uint64)
    _header, lengths = _native.huff0_build(counts, max(zstd_lengths))
    assert max(lengths) <= max(zstd_lengths)
    assert sum(2.0 ** -l for l in lengths if l) == 1.0
    assert all((l > 0) == (c > 0) for l, c in zip(lengths, counts))
    assert _cost(lengths, data) <= _cost(zstd_lengths, data) * 1.001


@needs_zstd
@pytest.mark.parametrize("name", CASES)
def test_zstd_decodes_product_tables_and_blocks(name):
    """The setup's singleton tables (histogram + prior 1, at most 12 bits,
    neuralzip/setup.py:170-176) and the storage payloads the product writes
    for them decode in zstd's own decoder."""
    _tree, _streams, data = _case(name)
    counts = np.bincount(np.frombuffer(data, dtype=np.uint8), minlength=256).astype(np.uint64)
    for prior in (0, 1):
        header, lengths = _native.huff0_build(counts + prior, 12)
        _, values, _, used = _native.huff0_read(header)
        assert used == len(header)
        assert R.tree_description(header)[0] == list(lengths)  # the oracle reads it alike
        book = _native.NativeCodebook(lengths, np.asarray(values, dtype=np.uint64))
        block = _native.huff0_encode(book, np.frombuffer(data, dtype=np.uint8), 2 * len(data) + 64)
        assert block
        assert Z.decompress(ZSTD, Z.literals_only_frame(header, block, len(data)), len(data)) == data


@needs_zstd
@pytest.mark.parametrize("name", CASES)
def test_zstd_decodes_product_header_for_zstd_lengths(name):
    """A header the product writes for zstd's own lengths describes zstd's
    table: zstd decodes zstd's streams under it."""
    tree, streams, data = _case(name)
    zstd_lengths = np.frombuffer(bytes(R.tree_description(tree)[0]), dtype=np.uint8).astype(np.int64)
    longest = int(zstd_lengths.max())
    dyadic = np.where(zstd_lengths > 0, 1 << (longest - zstd_lengths), 0).astype(np.uint64)
    header, lengths = _native.huff0_build(dyadic, longest)
    assert lengths == bytes(zstd_lengths.astype(np.uint8))
    assert Z.decompress(ZSTD, Z.literals_only_frame(header, streams, len(data)), len(data)) == data
    if tree[0] >= 128:  # 4-bit direct weights: one encoding, so the same bytes
        assert header == tree


@needs_zstd
def test_one_bit_code_beside_twelve_bit_codes_stays_readable_by_zstd():
    """A byte value with probability near one half next to rare values
    (e.g. exact zeros of a pruned tensor) would give a 1-bit code beside
    12-bit codes, i.e. weight 12, which zstd rejects in FSE-coded weights;
    the product builds that table with 11 bits, and zstd decodes it."""
    rng = np.random.default_rng(5)
    counts = np.zeros(256)
    counts[:64] = np.maximum(1, np.round(1e6 * 0.3 ** np.arange(64)))
    data = rng.choice(256, size=4096, p=counts / counts.sum()).astype(np.uint8)
    header, lengths = _native.huff0_build(counts.astype(np.uint64), 12)
    assert header[0] < 128 and max(lengths) == 11 and min(l for l in lengths if l) == 1
    _, values, _, _ = _native.huff0_read(header)
    book = _native.NativeCodebook(lengths, np.asarray(values, dtype=np.uint64))
    block = _native.huff0_encode(book, data, 4 * len(data) + 64)
    assert Z.decompress(ZSTD, Z.literals_only_frame(header, block, len(data)), len(data)) == data.tobytes()
