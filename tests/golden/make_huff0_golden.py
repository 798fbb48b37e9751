"""Generates tests/golden/zstd_huff0_vectors.npz: Huff0 structures written by
the system zstd library, for pinning the singleton (shared_huff0) path.

The reference's singleton tables and payloads are zstd Huff0 (table header:
HUF_writeCTable_wksp, neuralzip/native/codebooks.h:20-39; payload:
HUF_compress4X_usingCTable, :131-141); zstd at the reference's pinned
revision is not in its tree and cannot be fetched. The zstd library on this
image (libzstd 1.5.5) writes the same two structures in every frame whose
literals it Huffman-codes: a Huffman tree description (RFC 8878 4.2.1) and a
4-stream block (4.2.2). For each seeded case below, zstd compresses the bytes
as a literals-only frame (ZSTD_compressSequences with no sequences, so the
literals are exactly the input); the fixture keeps that frame and the input.

Run ``python tests/golden/make_huff0_golden.py`` where libzstd is present.
The cases are byte lanes the Huffman stage codes: bf16 exponent bytes of
N(0, sigma) for sigma in config 2's set (config 1's sigma 0.02 at the full
128 KiB chunk size), fp16's byte 1 (sign, exponent, 2 mantissa bits), fp32's
exponent byte, an odd-sized chunk, and a 13-symbol alphabet that zstd
describes with 4-bit direct weights.
"""

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT), str(ROOT / "tests")]

import helpers as H  # noqa: E402
import zstd_frames as Z  # noqa: E402
from neuralzip_b200.dtypes import DTYPES  # noqa: E402

OUT = Path(__file__).with_name("zstd_huff0_vectors.npz")


def cases():
    lanes = {}
    for name, dtype, sigma, n, seed in (
        ("bf16_s0.02_128k", torch.bfloat16, 0.02, 131072, 1),
        ("bf16_s0.002", torch.bfloat16, 0.002, 32768, 2),
        ("bf16_s1.0", torch.bfloat16, 1.0, 32768, 3),
        ("fp16_s0.02", torch.float16, 0.02, 32768, 4),
        ("fp32_s0.02", torch.float32, 0.02, 32768, 5),
        ("bf16_s0.2_odd", torch.bfloat16, 0.2, 5001, 6),
    ):
        spec = DTYPES[dtype]
        lanes[name] = bytes(H.selected_lane(H.gaussian_raw(n, sigma, dtype, seed), spec))
    rng = np.random.default_rng(7)
    p = 0.5 ** np.arange(1, 14)
    lanes["alphabet13"] = rng.choice(13, size=4096, p=p / p.sum()).astype(np.uint8).tobytes()
    return lanes


def main():
    lib = Z.library()
    if lib is None:
        raise SystemExit("libzstd was not found.")
    arrays = {"zstd_version": np.frombuffer(lib.ZSTD_versionString(), dtype=np.uint8)}
    for name, data in cases().items():
        frame = Z.literals_frame(lib, data)
        if Z.decompress(lib, frame, len(data)) != data:
            raise SystemExit(f"{name}: zstd does not round-trip")
        (kind, block), = Z.frame_blocks(frame)
        regenerated, streams, _tree, _data, rest = Z.literals_section(block)
        if (kind, regenerated, streams, rest) != (2, len(data), 4, b"\x00"):
            raise SystemExit(f"{name}: not a single literals-only block with 4 streams")
        arrays[f"{name}_frame"] = np.frombuffer(frame, dtype=np.uint8)
        arrays[f"{name}_data"] = np.frombuffer(data, dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(arrays)} arrays)")


if __name__ == "__main__":
    main()
