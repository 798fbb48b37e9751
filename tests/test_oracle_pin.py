"""The oracle and the product pinned to the reference's own outputs.

tests/golden/reference_vectors.npz was produced by the reference's native
code compiled unchanged from its sources (tests/golden/make_golden.py over
oracle/_ref): canonical mixed codes (make_mixed_table), reference GPU
layouts (encode_gpu_layout) and mixed CPU frames (encode_mixed_block_into).
These tests run without the reference tree. Where oracle/_ref is present
(a checkout that can build it), random cases are compared with it too.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import helpers as H
from neuralzip_b200 import _native
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu.inference import GPUCodebook
from oracle import oracle as O

GOLDEN = np.load(Path(__file__).with_name("golden") / "reference_vectors.npz")
BOOKS = ("seg12", "seg32", "seg33", "seg56", "long", "gauss")
LAYOUTS = {"seg33_bf16": ("seg33", torch.bfloat16), "seg12_fp32": ("seg12", torch.float32),
           "gauss_bf16": ("gauss", torch.bfloat16), "single_bf16": ("single", torch.bfloat16)}


def _book(name):
    lengths = GOLDEN[f"{name}_lengths"].tobytes()
    vocab = GOLDEN[f"{name}_vocab"].tobytes() if f"{name}_vocab" in GOLDEN else b""
    return lengths, vocab, GOLDEN[f"{name}_codes"]


@pytest.mark.parametrize("name", BOOKS)
def test_canonical_codes_match_reference(name):
    lengths, vocab, codes = _book(name)
    assert np.array_equal(O.mixed_codes(lengths), codes)  # oracle restatement
    got_lengths, got_values, longest = _native.export_code_table(b"NZM1" + lengths, 56, vocab)  # product
    assert got_lengths == lengths and np.array_equal(np.array(got_values, dtype=np.uint64), codes)
    assert longest == max(lengths)


@pytest.mark.parametrize("case", sorted(LAYOUTS))
def test_reference_gpu_layout_restatement(case):
    book, dtype = LAYOUTS[case]
    lengths, vocab, codes = _book(book)
    spec = DTYPES[dtype]
    raw = GOLDEN[f"{case}_raw"].tobytes()
    sel = O.split(raw, spec)[spec.gpu_stream]
    layout = O.ref_encode(sel, lengths, codes, vocab)
    assert np.array_equal(layout["bitstream"], GOLDEN[f"{case}_bitstream"])
    assert np.array_equal(layout["packed_gaps"], GOLDEN[f"{case}_packed_gaps"])
    assert np.array_equal(layout["positions"], GOLDEN[f"{case}_positions"])
    assert [layout["bit_length"], layout["max_bits"]] == [int(x) for x in GOLDEN[f"{case}_meta"]]
    # The reference kernel semantics restated by the oracle reproduce the lane.
    lut, max_bits = O.ref_lut(lengths, codes, vocab)
    assert np.array_equal(O.ref_decode(layout, lut, max_bits, bool(vocab), len(sel)), sel)


@pytest.mark.parametrize("book", ("seg12", "seg56", "gauss"))
def test_mixed_frames_match_reference(book):
    lengths, vocab, codes = _book(book)
    data = GOLDEN[f"frame_{book}_data"]
    frame = GOLDEN[f"frame_{book}"].tobytes()
    assert O.mixed_frame_encode(data, lengths, codes, vocab) == frame  # oracle
    native = _native.NativeCodebook(lengths, None, vocab)
    assert _native.mixed_encode(native, data, len(data) + 64) == frame  # product encoder
    assert np.array_equal(O.mixed_frame_decode(frame, lengths, codes, vocab, len(data)), data)
    assert np.array_equal(_native.mixed_decode(native, frame, len(data)), data)  # product decoder


def test_singleton_header_reads_back():
    header = GOLDEN["single_header"].tobytes()
    lengths, values, table_log, used = _native.huff0_read(header)
    assert used == len(header)
    assert lengths == GOLDEN["single_lengths"].tobytes()
    assert np.array_equal(np.array(values, dtype=np.uint64), GOLDEN["single_codes"])
    assert table_log == max(lengths)


@pytest.mark.parametrize("seed", range(3))
def test_oracle_lut_matches_product_decode(seed):
    """The oracle's reference-layout decode and the product's tile decode
    (CPU kernel model) agree on random gaussian chunks."""
    import kernel_model as KM
    from neuralzip_b200.gpu.inference import encode_with_codebook

    spec = DTYPES[torch.bfloat16]
    raw = H.gaussian_raw(20000 + seed, [0.02, 0.2, 1.0][seed], torch.bfloat16, 100 + seed)
    sel = H.selected_lane(raw, spec)
    lengths, vocab = H.mixed_book_for(sel, 60)
    codes = O.mixed_codes(lengths)
    layout = O.ref_encode(sel, lengths, codes, vocab)
    lut, max_bits = O.ref_lut(lengths, codes, vocab)
    ref = O.ref_decode(layout, lut, max_bits, True, len(sel))
    book = GPUCodebook(tuple(lengths), tuple(int(c) for c in codes), vocab)
    enc = encode_with_codebook(raw, book, dtype=spec, stream_id=1)
    sym = enc.symbols
    got = KM.decode_group(np.asarray(book.decode_lut), np.frombuffer(sym.bitstream, dtype=np.uint32),
                          np.frombuffer(sym.lane_bits, dtype=np.uint16), np.asarray(sym.tile_offsets), enc.numel,
                          lut_words=book.table_words)
    assert np.array_equal(ref, sel) and np.array_equal(got, ref)


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref needs the reference sources")
@pytest.mark.parametrize("seed", range(4))
def test_oracle_against_reference_native_random(seed):
    rng = np.random.default_rng(seed)
    spec = [DTYPES[torch.bfloat16], DTYPES[torch.float32]][seed % 2]
    raw = H.gaussian_raw(int(rng.integers(1, 40000)), float(rng.choice([0.002, 0.02, 1.0])), spec.torch_dtype, seed)
    sel = H.selected_lane(raw, spec)
    lengths, vocab = H.mixed_book_for(sel, int(rng.integers(1, 254)))
    codes = O.mixed_codes(lengths)
    assert np.array_equal(codes, O.ref_mixed_codes_native(lengths, vocab))
    mine = O.ref_encode(sel, lengths, codes, vocab)
    theirs = O.ref_gpu_layout_native(raw, spec, spec.gpu_stream, lengths, codes, vocab)
    for key in ("bitstream", "packed_gaps", "positions"):
        assert np.array_equal(mine[key], theirs[key])
    assert O.mixed_frame_encode(sel, lengths, codes, vocab) == O.ref_mixed_encode_native(sel, lengths, vocab)
