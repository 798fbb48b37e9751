"""ctypes wrappers over the CPU oracle (liboracle.so) and the reference shim
(_ref/libnzref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker; the product (neuralzip_b200/)
never imports it. See nz_oracle.c for the reference file:line each function
restates.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libnzref.so"

_oracle = None
_ref = None


def build():
    """Runs oracle/Makefile (the reference part only where its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True, capture_output=True)


def _vp(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None and len(a) else None


def lib():
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists() or ORACLE_LIB.stat().st_mtime < (HERE / "nz_oracle.c").stat().st_mtime:
            build()
        _oracle = ctypes.CDLL(str(ORACLE_LIB))
    return _oracle


def ref_available():
    return REF_LIB.exists()


def ref():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise FileNotFoundError("oracle/_ref/libnzref.so is not built (reference sources absent).")
        _ref = ctypes.CDLL(str(REF_LIB))
        _ref.ref_mixed_decodebook.restype = ctypes.c_void_p
        _ref.ref_mixed_decodebook_free.argtypes = [ctypes.c_void_p]
    return _ref


def _check(status, which="oracle"):
    if status != 0:
        if which == "ref":
            buf = ctypes.create_string_buffer(512)
            ref().ref_last_error(buf, 512)
            raise RuntimeError(buf.value.decode())
        raise RuntimeError(f"oracle check failed at nz_oracle.c:{lib().oz_error_line()}")


def u8(data):
    return np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8))


# ---- restatement -------------------------------------------------------------

def mixed_codes(lengths):
    lengths = u8(lengths)
    codes = np.zeros(len(lengths), dtype=np.uint64)
    _check(lib().oz_mixed_codes(_vp(lengths), ctypes.c_uint32(len(lengths)), _vp(codes)))
    return codes


def ref_lut(lengths, values, vocab=b""):
    """(lut uint32 array, max_bits) with GPUCodebook.decode_lut semantics."""
    lengths = u8(lengths)
    values = np.ascontiguousarray(np.asarray(values, dtype=np.uint64))
    vocab = u8(vocab)
    cap = 4096 + 2 * 64 * 512 + 16
    out = np.zeros(cap, dtype=np.uint32)
    n, mb = ctypes.c_uint32(), ctypes.c_uint32()
    _check(lib().oz_ref_lut(_vp(lengths), _vp(values), ctypes.c_uint32(len(lengths)), _vp(vocab),
                            ctypes.c_uint32(len(vocab)), _vp(out), ctypes.c_uint32(cap),
                            ctypes.byref(n), ctypes.byref(mb)))
    return out[:n.value].copy(), mb.value


def split(raw, spec):
    """All byte lanes (reordered) of raw element bytes."""
    raw = u8(raw)
    es = spec.element_size
    numel = len(raw) // es
    lanes = [np.zeros(numel, dtype=np.uint8) for _ in range(es)]
    ptrs = (ctypes.c_void_p * es)(*[lane.ctypes.data for lane in lanes])
    _check(lib().oz_split(_vp(raw), ctypes.c_uint64(numel), es, int(spec.bit_reorder), spec.mantissa_bits,
                          spec.exponent_mask.bit_length(), ptrs))
    return lanes


def restore(lanes, spec):
    es = spec.element_size
    numel = len(lanes[0])
    lanes = [np.ascontiguousarray(lane, dtype=np.uint8) for lane in lanes]
    out = np.zeros(numel * es, dtype=np.uint8)
    ptrs = (ctypes.c_void_p * es)(*[lane.ctypes.data for lane in lanes])
    _check(lib().oz_restore(ptrs, ctypes.c_uint64(numel), es, int(spec.bit_reorder), spec.mantissa_bits,
                            spec.exponent_mask.bit_length(), _vp(out)))
    return out


def ref_encode(symbols, lengths, codes, vocab=b""):
    """Reference GPU layout of one selected lane: dict with bitstream, gaps
    (one byte per segment), packed_gaps, positions, bit_length, max_bits."""
    symbols = u8(symbols)
    lengths = u8(lengths)
    codes = np.ascontiguousarray(np.asarray(codes, dtype=np.uint64))
    vocab = u8(vocab)
    numel = len(symbols)
    bit_cap = numel * 7 + 16
    bitstream = np.zeros(bit_cap, dtype=np.uint8)
    gap_cap = (bit_cap // 4096 + 2) * 512
    gaps = np.zeros(gap_cap, dtype=np.uint8)
    positions = np.zeros(bit_cap // 4096 + 4, dtype=np.uint32)
    nb, ng, npos, bl, mb = (ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64(),
                            ctypes.c_uint32())
    _check(lib().oz_ref_encode(_vp(symbols), ctypes.c_uint64(numel), _vp(lengths), _vp(codes),
                               ctypes.c_uint32(len(lengths)), _vp(vocab), ctypes.c_uint32(len(vocab)),
                               _vp(bitstream), ctypes.c_uint64(bit_cap), ctypes.byref(nb), _vp(gaps),
                               ctypes.c_uint64(gap_cap), ctypes.byref(ng), _vp(positions),
                               ctypes.c_uint64(len(positions)), ctypes.byref(npos), ctypes.byref(bl),
                               ctypes.byref(mb)))
    g = gaps[:ng.value].copy()
    packed = g.copy()
    if not len(vocab):
        packed = np.zeros(len(g) // 2 + len(g) % 2, dtype=np.uint8)
        lib().oz_pack_gaps(_vp(g), ctypes.c_uint64(len(g)), _vp(packed))
    return {"bitstream": bitstream[:nb.value].copy(), "gaps": g, "packed_gaps": packed,
            "positions": positions[:npos.value].copy(), "bit_length": bl.value, "max_bits": mb.value}


def ref_decode(layout, lut, max_bits, mixed, numel):
    """Decodes a reference-layout group (kernel semantics) to exponent bytes."""
    out = np.zeros(numel, dtype=np.uint8)
    bitstream = layout["bitstream"]
    lut = np.ascontiguousarray(lut, dtype=np.uint32)
    _check(lib().oz_ref_decode(_vp(lut), int(bool(mixed)), ctypes.c_uint32(max_bits), _vp(bitstream),
                               ctypes.c_uint64(len(bitstream)), _vp(layout["gaps"]), _vp(layout["positions"]),
                               ctypes.c_uint64(numel), _vp(out)))
    return out


def mixed_frame_encode(data, lengths, codes, vocab, cap=None):
    data = u8(data)
    lengths = u8(lengths)
    codes = np.ascontiguousarray(np.asarray(codes, dtype=np.uint64))
    vocab = u8(vocab)
    cap = len(data) + 64 if cap is None else cap
    out = np.zeros(cap, dtype=np.uint8)
    size = ctypes.c_uint64()
    _check(lib().oz_mixed_frame_encode(_vp(data), ctypes.c_uint64(len(data)), _vp(lengths), _vp(codes),
                                       _vp(vocab), ctypes.c_uint32(len(vocab)), _vp(out), ctypes.c_uint64(cap),
                                       ctypes.byref(size)))
    return out[:size.value].tobytes()


def mixed_frame_decode(frame, lengths, codes, vocab, expected):
    frame = u8(frame)
    lengths = u8(lengths)
    codes = np.ascontiguousarray(np.asarray(codes, dtype=np.uint64))
    vocab = u8(vocab)
    out = np.zeros(expected, dtype=np.uint8)
    _check(lib().oz_mixed_frame_decode(_vp(frame), ctypes.c_uint64(len(frame)), _vp(lengths), _vp(codes),
                                       ctypes.c_uint32(len(lengths)), _vp(vocab), _vp(out),
                                       ctypes.c_uint64(expected)))
    return out


def tile_decode(bits, lens, tile_off, numel, lengths, codes, vocab=b""):
    """Independent reader of the B200 tile layout (selected lane bytes)."""
    bits = np.ascontiguousarray(bits, dtype=np.uint32)
    lens = np.ascontiguousarray(lens, dtype=np.uint16)
    tile_off = np.ascontiguousarray(tile_off, dtype=np.uint32)
    lengths = u8(lengths)
    codes = np.ascontiguousarray(np.asarray(codes, dtype=np.uint64))
    vocab = u8(vocab)
    out = np.zeros(numel, dtype=np.uint8)
    _check(lib().oz_tile_decode(_vp(bits), ctypes.c_uint64(len(bits)), _vp(lens), _vp(tile_off),
                                ctypes.c_uint64(numel), _vp(lengths), _vp(codes), ctypes.c_uint32(len(lengths)),
                                _vp(vocab), _vp(out)))
    return out


# ---- the reference's own code (oracle/_ref) ------------------------------------

def ref_mixed_codes_native(lengths, vocab):
    header = u8(b"NZM1" + bytes(lengths))
    vocab = u8(vocab)
    codes = np.zeros(len(header) - 4, dtype=np.uint64)
    _check(ref().ref_mixed_codes(_vp(header), ctypes.c_size_t(len(header)), _vp(vocab),
                                 ctypes.c_size_t(len(vocab)), _vp(codes)), "ref")
    return codes


def ref_gpu_layout_native(raw, spec, stream_id, lengths, codes, vocab=b""):
    raw = u8(raw)
    es = spec.element_size
    numel = len(raw) // es
    lengths = u8(lengths)
    codes = np.ascontiguousarray(np.asarray(codes, dtype=np.uint64))
    vocab = u8(vocab)
    cap = numel * 7 + 16
    bitstream = np.zeros(cap, dtype=np.uint8)
    gaps = np.zeros((cap // 4096 + 2) * 512, dtype=np.uint8)
    positions = np.zeros(cap // 4096 + 4, dtype=np.uint32)
    lanes = [None if lane == stream_id else np.zeros(numel, dtype=np.uint8) for lane in range(es)]
    ptrs = (ctypes.c_void_p * es)(*[(lane.ctypes.data if lane is not None else None) for lane in lanes])
    nb, ng, npos = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    bl, mb = ctypes.c_uint64(), ctypes.c_uint32()
    _check(ref().ref_gpu_layout(_vp(raw), ctypes.c_size_t(numel), es, int(spec.bit_reorder), spec.mantissa_bits,
                                spec.exponent_mask.bit_length(), stream_id, _vp(lengths), _vp(codes),
                                ctypes.c_uint32(len(lengths)), _vp(vocab), ctypes.c_size_t(len(vocab)),
                                _vp(bitstream), ctypes.byref(nb), _vp(gaps), ctypes.byref(ng), _vp(positions),
                                ctypes.byref(npos), ctypes.byref(bl), ctypes.byref(mb), ptrs), "ref")
    return {"bitstream": bitstream[:nb.value].copy(), "packed_gaps": gaps[:ng.value].copy(),
            "positions": positions[:npos.value].copy(), "bit_length": bl.value, "max_bits": mb.value,
            "lanes": lanes}


def ref_mixed_encode_native(data, lengths, vocab, cap=None):
    data = u8(data)
    header = u8(b"NZM1" + bytes(lengths))
    vocab = u8(vocab)
    cap = len(data) + 64 if cap is None else cap
    out = np.zeros(max(cap, 1), dtype=np.uint8)
    size = ctypes.c_size_t()
    _check(ref().ref_mixed_encode(_vp(data), ctypes.c_size_t(len(data)), _vp(header), ctypes.c_size_t(len(header)),
                                  _vp(vocab), ctypes.c_size_t(len(vocab)), _vp(out), ctypes.c_size_t(cap),
                                  ctypes.byref(size)), "ref")
    return out[:size.value].tobytes()


def ref_mixed_decode_native(frame, lengths, vocab, expected):
    frame = u8(frame)
    header = u8(b"NZM1" + bytes(lengths))
    vocab = u8(vocab)
    out = np.zeros(expected, dtype=np.uint8)
    _check(ref().ref_mixed_decode(_vp(frame), ctypes.c_size_t(len(frame)), _vp(header), ctypes.c_size_t(len(header)),
                                  _vp(vocab), ctypes.c_size_t(len(vocab)), _vp(out), ctypes.c_size_t(expected)),
           "ref")
    return out


class RefChunk(ctypes.Structure):
    _fields_ = [("payload", ctypes.c_void_p), ("payload_size", ctypes.c_uint64), ("book", ctypes.c_void_p),
                ("lanes", ctypes.c_void_p * 4), ("out", ctypes.c_void_p), ("numel", ctypes.c_uint64),
                ("elem_size", ctypes.c_uint32), ("reorder", ctypes.c_uint32), ("stream_id", ctypes.c_uint32),
                ("pad", ctypes.c_uint32)]


class RefDecodebook:
    def __init__(self, lengths, vocab):
        header = u8(b"NZM1" + bytes(lengths))
        vocab_a = u8(vocab)
        self._keep = (header, vocab_a)
        self.handle = ref().ref_mixed_decodebook(_vp(header), ctypes.c_size_t(len(header)), _vp(vocab_a),
                                                 ctypes.c_size_t(len(vocab_a)))
        if not self.handle:
            _check(1, "ref")

    def __del__(self):
        if getattr(self, "handle", None):
            ref().ref_mixed_decodebook_free(self.handle)
            self.handle = None


def ref_decode_chunks(chunks, threads=0):
    array = (RefChunk * len(chunks))(*chunks)
    _check(ref().ref_decode_chunks(array, ctypes.c_size_t(len(chunks)), int(threads)), "ref")
