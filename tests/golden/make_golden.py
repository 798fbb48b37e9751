"""Generates tests/golden/reference_vectors.npz from the reference's own code.

Run in a checkout where the reference sources exist (oracle/Makefile builds
oracle/_ref/libnzref.so from them): ``python tests/golden/make_golden.py``.
Every array comes from the reference's native functions compiled unchanged
(make_mixed_table, encode_gpu_layout, encode_mixed_block_into), except the
singleton table, whose header the system zstd library writes (zstd's Huff0
is the reference's singleton codec and is not in its tree); the inputs are
seeded and restated here. The fixtures let the CPU tests pin the oracle
and the product without the reference tree.
"""

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT), str(ROOT / "tests")]

import helpers as H  # noqa: E402
from neuralzip_b200.dtypes import DTYPES  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).with_name("reference_vectors.npz")


def main():
    O.build()
    if not O.ref_available():
        raise SystemExit("oracle/_ref is not built: the reference sources are needed.")
    arrays = {}
    # 1. Canonical codes of the reference kernel checks' segment books and
    #    the long-code book (make_mixed_table, mixed_huffman.h:5-57).
    books = {f"seg{b}": (H.segment_lengths(b), H.VOCAB) for b in (12, 32, 33, 56)}
    books["long"] = (H.long_code_lengths(), H.VOCAB)
    for name, (lengths, vocab) in books.items():
        arrays[f"{name}_lengths"] = np.frombuffer(lengths, dtype=np.uint8)
        arrays[f"{name}_vocab"] = np.frombuffer(vocab, dtype=np.uint8)
        arrays[f"{name}_codes"] = O.ref_mixed_codes_native(lengths, vocab)
    # 2. Reference GPU layouts (encode_gpu_layout, gpu_layout.h:185-241).
    cases = {
        "seg33_bf16": ("seg33", torch.bfloat16, H.lanes_with(H.segment_symbols()[:20000], DTYPES[torch.bfloat16])),
        "seg12_fp32": ("seg12", torch.float32, H.lanes_with(H.segment_symbols()[60000:], DTYPES[torch.float32])),
    }
    raw = H.gaussian_raw(9001, 0.02, torch.bfloat16, 11)
    sel = H.selected_lane(raw, DTYPES[torch.bfloat16])
    lengths, vocab = H.mixed_book_for(sel, 40)
    arrays["gauss_lengths"] = np.frombuffer(lengths, dtype=np.uint8)
    arrays["gauss_vocab"] = np.frombuffer(vocab, dtype=np.uint8)
    arrays["gauss_codes"] = O.ref_mixed_codes_native(lengths, vocab)
    cases["gauss_bf16"] = ("gauss", torch.bfloat16, raw)
    # A singleton table exercises the 4-bit gap path. Its header is the
    # Huffman tree description the system zstd library writes for these
    # bytes (a literals-only frame); the lengths and codes are read from it
    # by the RFC 8878 restatement in oracle/rfc8878.py, not by the product.
    import zstd_frames as Z
    from oracle import rfc8878 as R

    zstd = Z.library()
    if zstd is None:
        raise SystemExit("libzstd is needed for the singleton table.")
    (_kind, block), = Z.frame_blocks(Z.literals_frame(zstd, bytes(sel)))
    header = Z.literals_section(block)[2]
    s_lengths, _used = R.tree_description(header)
    arrays["single_lengths"] = np.asarray(s_lengths, dtype=np.uint8)
    arrays["single_codes"] = np.asarray(R.canonical_codes(s_lengths), dtype=np.uint64)
    arrays["single_header"] = np.frombuffer(header, dtype=np.uint8)
    cases["single_bf16"] = ("single", torch.bfloat16, raw)
    for case, (book, dtype, data) in cases.items():
        spec = DTYPES[dtype]
        lengths = arrays[f"{book}_lengths"].tobytes()
        vocab = arrays.get(f"{book}_vocab", np.zeros(0, np.uint8)).tobytes()
        codes = arrays[f"{book}_codes"]
        layout = O.ref_gpu_layout_native(data, spec, spec.gpu_stream, lengths, codes, vocab)
        arrays[f"{case}_raw"] = np.frombuffer(data, dtype=np.uint8)
        for key in ("bitstream", "packed_gaps", "positions"):
            arrays[f"{case}_{key}"] = layout[key]
        arrays[f"{case}_meta"] = np.array([layout["bit_length"], layout["max_bits"]], dtype=np.uint64)
    # 3. Mixed CPU frames (encode_mixed_block_into, mixed_huffman.h:127-178).
    for book in ("seg12", "seg56", "gauss"):
        lengths = arrays[f"{book}_lengths"].tobytes()
        vocab = arrays[f"{book}_vocab"].tobytes()
        data = sel if book == "gauss" else H.segment_symbols()[:30001]
        arrays[f"frame_{book}_data"] = np.asarray(data, dtype=np.uint8)
        arrays[f"frame_{book}"] = np.frombuffer(O.ref_mixed_encode_native(data, lengths, vocab), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(arrays)} arrays)")


if __name__ == "__main__":
    main()
