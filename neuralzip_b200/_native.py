"""ctypes binding of libnzb200.so (the C ABI in include/nz_b200.h).

Everything that crosses this boundary is a plain pointer, size or struct.
Status codes become the exceptions the reference raises for the same
conditions (neuralzip/native/common.h:59-63 and nanobind's translation):
ValueError, TypeError, OverflowError and RuntimeError.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

import os

# NZB200_LIBRARY may point at another build of the same ABI (e.g. a debug build).
LIBRARY = Path(os.environ.get("NZB200_LIBRARY") or Path(__file__).resolve().parent / "_lib" / "libnzb200.so")

LANE_ELEMS = 256
TILE_LANES = 32
TILE_ELEMS = LANE_ELEMS * TILE_LANES
LUT_BITS = 12
LUT_ENTRIES = 1 << LUT_BITS
TREE_MAX_NODES = 512
LUT_CANON = 2 * LUT_ENTRIES
CANON_WORDS = 64 + 512
LUT_TREE = LUT_CANON + CANON_WORDS
LUT_WORDS = LUT_TREE + 2 * TREE_MAX_NODES
MAX_CODE_BITS = 56
BITS_PAD_WORDS = 16
RAW_LUT = 0xFFFFFFFF
ABI_VERSION = 4
LAYOUT_BF16, LAYOUT_FP16, LAYOUT_FP32 = 0, 1, 2

OK, EVALUE, ETYPE, EOVERFLOW, ERUNTIME, ECUDA = range(6)
_ERRORS = {EVALUE: ValueError, ETYPE: TypeError, EOVERFLOW: OverflowError, ERUNTIME: RuntimeError,
           ECUDA: RuntimeError}

u8p = ctypes.POINTER(ctypes.c_uint8)
u16p = ctypes.POINTER(ctypes.c_uint16)
u32p = ctypes.POINTER(ctypes.c_uint32)
u64p = ctypes.POINTER(ctypes.c_uint64)
sizep = ctypes.POINTER(ctypes.c_size_t)


class Dtype(ctypes.Structure):
    _fields_ = [("elem_size", ctypes.c_uint32), ("reorder", ctypes.c_uint32),
                ("mant_bits", ctypes.c_uint32), ("exp_bits", ctypes.c_uint32),
                ("stream_id", ctypes.c_uint32)]


class PackJob(ctypes.Structure):
    _fields_ = [("codebook", ctypes.c_void_p), ("raw", ctypes.c_void_p), ("numel", ctypes.c_uint64),
                ("bits", ctypes.c_void_p), ("bits_cap_words", ctypes.c_uint64),
                ("lens", ctypes.c_void_p), ("lens_cap", ctypes.c_uint64),
                ("tile_off", ctypes.c_void_p), ("tiles_cap", ctypes.c_uint64),
                ("lanes", ctypes.c_void_p * 4), ("bit_length", ctypes.c_uint64),
                ("words_used", ctypes.c_uint64), ("status", ctypes.c_int32), ("pad", ctypes.c_int32)]


class Launch(ctypes.Structure):
    _fields_ = [("warps_per_cta", ctypes.c_uint32), ("n_ctas", ctypes.c_uint32), ("groups", ctypes.c_uint64),
                ("works", ctypes.c_uint64), ("ctas", ctypes.c_uint64), ("luts", ctypes.c_uint64),
                ("status", ctypes.c_uint64), ("scratch", ctypes.c_uint64), ("queues", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32)]


# Device descriptor records (numpy views of the C structs).
GROUP_DTYPE = np.dtype([("bits", "<u8"), ("lens", "<u8"), ("tile_off", "<u8"), ("lanes", "<u8", (4,)),
                        ("out", "<u8"), ("numel", "<u4"), ("lut", "<u4")])
WORK_DTYPE = np.dtype([("group", "<u4"), ("tile", "<u4")])
CTA_DTYPE = np.dtype([("lut", "<u4"), ("begin", "<u4"), ("end", "<u4"), ("lut_words", "<u2"), ("layout", "<u2"),
                      ("queue", "<u4"), ("reserved", "<u4")])
assert GROUP_DTYPE.itemsize == 72 and WORK_DTYPE.itemsize == 8 and CTA_DTYPE.itemsize == 24
# Host storage-decode records (nz_storage_lane, nz_storage_piece).
CHUNK_RAW, CHUNK_HUFF0, CHUNK_MIXED = 0, 1, 2
CHUNK_MODES = {"raw": CHUNK_RAW, "shared_huff0": CHUNK_HUFF0, "mixed_huffman": CHUNK_MIXED}
STORAGE_LANE_DTYPE = np.dtype([("payload", "<u8"), ("payload_size", "<u8"), ("codebook", "<u8"), ("mode", "<u4"),
                               ("reserved", "<u4")])
STORAGE_PIECE_DTYPE = np.dtype([("lanes", "<u8"), ("out", "<u8"), ("count", "<u8"), ("elem_size", "<u4"),
                                ("reorder", "<u4"), ("mant_bits", "<u4"), ("exp_bits", "<u4"),
                                ("stream_id", "<u4"), ("reserved", "<u4")])
assert STORAGE_LANE_DTYPE.itemsize == 32 and STORAGE_PIECE_DTYPE.itemsize == 48

EXPORTS = (
    "nz_export_code_table", "nz_codebook_create", "nz_codebook_destroy", "nz_codebook_info",
    "nz_codebook_lut", "nz_codebook_table_words", "nz_huff0_build", "nz_huff0_read", "nz_pack_bound", "nz_pack_chunk",
    "nz_pack_many", "nz_split_lanes", "nz_exponent_histograms", "nz_count_tokens", "nz_mixed_encode", "nz_mixed_decode",
    "nz_huff0_encode", "nz_huff0_decode", "nz_storage_decode", "nz_cluster_chunks", "nz_decode_launch", "nz_decode_launch_noalloc", "nz_decode_launch_many", "nz_decode_occupancy", "nz_decode_smem_bytes",
    "nz_decode_tile_words",
    "nz_schedule_create", "nz_schedule_destroy", "nz_schedule_enter", "nz_schedule_decode_unit",
    "nz_schedule_drain", "nz_schedule_mark", "nz_last_error",
    "nz_abi_version",
)

_lock = threading.Lock()
_lib = None


def library_path():
    return LIBRARY


def load():
    """Loads the library, building it first when it is absent and nvcc exists."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIBRARY.exists():
            from neuralzip_b200 import build as _build

            _build.build()
        lib = ctypes.CDLL(str(LIBRARY))
        _declare(lib)
        if lib.nz_abi_version() != ABI_VERSION:
            raise RuntimeError("libnzb200.so ABI version mismatch.")
        _lib = lib
        return lib


def _declare(lib):
    c = ctypes
    sig = {
        "nz_export_code_table": [c.c_void_p, c.c_size_t, c.c_void_p, c.c_size_t, c.c_uint32, c.c_void_p,
                                 c.c_void_p, c.c_uint32, u32p, u32p],
        "nz_codebook_create": [c.c_void_p, c.c_void_p, c.c_uint32, c.c_void_p, c.c_uint32,
                               c.POINTER(c.c_void_p)],
        "nz_codebook_destroy": [c.c_void_p],
        "nz_codebook_info": [c.c_void_p, u32p, u32p],
        "nz_codebook_lut": [c.c_void_p, c.c_void_p, c.c_uint32],
        "nz_codebook_table_words": [c.c_void_p, u32p],
        "nz_huff0_build": [c.c_void_p, c.c_uint32, c.c_void_p, c.c_size_t, sizep, c.c_void_p],
        "nz_huff0_read": [c.c_void_p, c.c_size_t, c.c_void_p, c.c_void_p, u32p, sizep],
        "nz_pack_bound": [c.c_uint64, c.c_uint32, u64p, u64p, u64p],
        "nz_pack_chunk": [c.c_void_p, c.c_void_p, c.c_uint64, c.POINTER(Dtype), c.c_void_p, c.c_uint64,
                          c.c_void_p, c.c_uint64, c.c_void_p, c.c_uint64, c.c_void_p, u64p, u64p],
        "nz_pack_many": [c.POINTER(PackJob), c.c_uint64, c.POINTER(Dtype), c.c_int32],
        "nz_split_lanes": [c.c_void_p, c.c_uint64, c.POINTER(Dtype), c.c_void_p],
        "nz_count_tokens": [c.c_void_p, c.c_uint64, c.c_void_p, c.c_uint32, c.c_void_p],
        "nz_exponent_histograms": [c.c_void_p, c.c_uint64, c.POINTER(Dtype), c.c_uint64, c.c_void_p],
        "nz_mixed_encode": [c.c_void_p, c.c_void_p, c.c_uint64, c.c_void_p, c.c_uint64, u64p],
        "nz_mixed_decode": [c.c_void_p, c.c_void_p, c.c_uint64, c.c_void_p, c.c_uint64],
        "nz_huff0_encode": [c.c_void_p, c.c_void_p, c.c_uint64, c.c_void_p, c.c_uint64, u64p],
        "nz_huff0_decode": [c.c_void_p, c.c_void_p, c.c_uint64, c.c_void_p, c.c_uint64],
        "nz_storage_decode": [c.c_void_p, c.c_uint64, c.c_int32],
        "nz_cluster_chunks": [c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p, c.c_uint64, c.c_uint32, c.c_double,
                              c.c_int32, c.c_void_p, c.c_void_p, c.c_uint64, u64p],
        "nz_decode_launch": [c.POINTER(Launch), c.c_void_p],
        "nz_decode_launch_noalloc": [c.POINTER(Launch), c.c_void_p],
        "nz_decode_occupancy": [c.c_uint32, u32p],
        "nz_decode_launch_many": [c.POINTER(Launch), c.c_uint32, c.c_void_p],
        "nz_schedule_create": [c.POINTER(Launch), u32p, c.c_uint32, c.c_uint32, c.c_void_p, c.POINTER(c.c_void_p)],
        "nz_schedule_destroy": [c.c_void_p],
        "nz_schedule_enter": [c.c_void_p, c.c_uint32, c.c_uint32, c.c_void_p],
        "nz_schedule_decode_unit": [c.c_void_p, c.c_uint32, c.c_void_p],
        "nz_schedule_drain": [c.c_void_p, c.c_void_p],
        "nz_schedule_mark": [c.c_void_p, c.c_uint32, c.c_uint32],
        "nz_decode_smem_bytes": [c.c_uint32, u32p],
        "nz_decode_tile_words": [c.c_uint32, u32p],
        "nz_last_error": [c.c_char_p, c.c_size_t],
        "nz_abi_version": [],
    }
    for name, argtypes in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = c.c_int


def check(status):
    if status == OK:
        return
    buf = ctypes.create_string_buffer(1024)
    _lib.nz_last_error(buf, len(buf))
    raise _ERRORS.get(status, RuntimeError)(buf.value.decode("utf-8", "replace"))


def _ptr(array):
    return ctypes.c_void_p(array.ctypes.data) if array is not None else None


def dtype_struct(element_size, reorder, mantissa_bits, exponent_bits, stream_id):
    return Dtype(int(element_size), int(bool(reorder)), int(mantissa_bits), int(exponent_bits),
                 int(stream_id))


# ---- codebooks --------------------------------------------------------------

def export_code_table(header, max_bits=12, vocab=b""):
    """(lengths bytes, values tuple, longest) like _huff0_cpp.export_code_table."""
    lib = load()
    header = np.frombuffer(bytes(header), dtype=np.uint8)
    vocab = np.frombuffer(bytes(vocab), dtype=np.uint8)
    cap = 256 + len(vocab) // 2
    lengths = np.zeros(max(cap, 256), dtype=np.uint8)
    values = np.zeros(max(cap, 256), dtype=np.uint64)
    nsym, longest = ctypes.c_uint32(), ctypes.c_uint32()
    check(lib.nz_export_code_table(_ptr(header), len(header), _ptr(vocab) if len(vocab) else None,
                                   len(vocab), int(max_bits), _ptr(lengths), _ptr(values),
                                   len(lengths), ctypes.byref(nsym), ctypes.byref(longest)))
    n = nsym.value
    return bytes(lengths[:n]), tuple(int(v) for v in values[:n]), longest.value


class NativeCodebook:
    """Owns an nz_codebook handle built from lengths (and optional values)."""

    def __init__(self, lengths, values=None, vocab=b""):
        lib = load()
        self._lib = lib
        self.lengths = np.ascontiguousarray(np.frombuffer(bytes(lengths), dtype=np.uint8))
        vocab = bytes(vocab)
        self.vocab = vocab
        vocab_array = np.frombuffer(vocab, dtype=np.uint8) if vocab else None
        values_array = None
        if values is not None:
            values_array = np.ascontiguousarray(np.asarray(values, dtype=np.uint64))
        handle = ctypes.c_void_p()
        check(lib.nz_codebook_create(_ptr(self.lengths), _ptr(values_array), len(self.lengths),
                                     _ptr(vocab_array), len(vocab), ctypes.byref(handle)))
        self.handle = handle
        longest, nodes = ctypes.c_uint32(), ctypes.c_uint32()
        check(lib.nz_codebook_info(handle, ctypes.byref(longest), ctypes.byref(nodes)))
        self.longest = longest.value
        self.tree_nodes = nodes.value
        words = ctypes.c_uint32()
        check(lib.nz_codebook_table_words(handle, ctypes.byref(words)))
        self.table_words = words.value

    def lut(self):
        out = np.zeros(LUT_WORDS, dtype=np.uint32)
        check(self._lib.nz_codebook_lut(self.handle, _ptr(out), LUT_WORDS))
        return out

    def __del__(self):
        handle = getattr(self, "handle", None)
        if handle is not None and handle.value:
            self._lib.nz_codebook_destroy(handle)
            self.handle = None


def huff0_build(counts, max_bits=12):
    """(Huff0 header bytes, lengths) for a 256-bin histogram (priors included)."""
    lib = load()
    counts = np.ascontiguousarray(np.asarray(counts, dtype=np.uint64))
    if counts.shape != (256,):
        raise ValueError("symbol_counts must contain exactly 256 entries.")
    out = np.zeros(512, dtype=np.uint8)
    lengths = np.zeros(256, dtype=np.uint8)
    size = ctypes.c_size_t()
    check(lib.nz_huff0_build(_ptr(counts), int(max_bits), _ptr(out), len(out), ctypes.byref(size),
                             _ptr(lengths)))
    return bytes(out[:size.value]), bytes(lengths)


def huff0_read(header):
    """(lengths bytes, values tuple, table_log, consumed) of a Huff0 header."""
    lib = load()
    header = np.frombuffer(bytes(header), dtype=np.uint8)
    lengths = np.zeros(256, dtype=np.uint8)
    values = np.zeros(256, dtype=np.uint16)
    log, used = ctypes.c_uint32(), ctypes.c_size_t()
    check(lib.nz_huff0_read(_ptr(header), len(header), _ptr(lengths), _ptr(values), ctypes.byref(log),
                            ctypes.byref(used)))
    return bytes(lengths), tuple(int(v) for v in values), log.value, used.value


# ---- packer -------------------------------------------------------------------

def pack_bound(numel, longest):
    lib = load()
    words, lens, tiles = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
    check(lib.nz_pack_bound(int(numel), int(longest), ctypes.byref(words), ctypes.byref(lens),
                            ctypes.byref(tiles)))
    return words.value, lens.value, tiles.value


def pack_chunk(codebook, raw, dt):
    """Packs one group. Returns (bits u32, lens u16, tile_off u32, lanes list, bit_length)."""
    lib = load()
    raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray, memoryview))
                               else raw.reshape(-1).view(np.uint8))
    numel = len(raw) // dt.elem_size
    if len(raw) % dt.elem_size:
        raise RuntimeError("Input must contain complete elements.")
    cap_words, n_lens, n_tiles = pack_bound(numel, codebook.longest)
    bits = np.empty(cap_words, dtype=np.uint32)
    lens = np.empty(n_lens, dtype=np.uint16)
    tile_off = np.empty(n_tiles, dtype=np.uint32)
    lanes = [None if lane == dt.stream_id else np.empty(numel, dtype=np.uint8)
             for lane in range(dt.elem_size)]
    lane_ptrs = (ctypes.c_void_p * 4)(*[(lane.ctypes.data if lane is not None else None)
                                         for lane in lanes + [None] * (4 - len(lanes))])
    bit_length, used = ctypes.c_uint64(), ctypes.c_uint64()
    check(lib.nz_pack_chunk(codebook.handle, _ptr(raw), numel, ctypes.byref(dt), _ptr(bits), cap_words,
                            _ptr(lens), n_lens, _ptr(tile_off), n_tiles, lane_ptrs,
                            ctypes.byref(bit_length), ctypes.byref(used)))
    return bits[:used.value].copy(), lens, tile_off, lanes, bit_length.value


def split_lanes(raw, dt, selected_only=False):
    """Reorders and splits every byte lane (raw fragments); with
    `selected_only`, only the selected lane is written (the others are
    None)."""
    lib = load()
    raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray, memoryview))
                               else raw.reshape(-1).view(np.uint8))
    numel = len(raw) // dt.elem_size
    lanes = [np.empty(numel, dtype=np.uint8) if not selected_only or lane == dt.stream_id else None
             for lane in range(dt.elem_size)]
    lane_ptrs = (ctypes.c_void_p * 4)(*[None if lane is None else lane.ctypes.data for lane in lanes]
                                      + [None] * (4 - len(lanes)))
    check(lib.nz_split_lanes(_ptr(raw), numel, ctypes.byref(dt), lane_ptrs))
    return lanes


def pack_many(jobs, dt, threads=0):
    lib = load()
    array = (PackJob * len(jobs))(*jobs)
    check(lib.nz_pack_many(array, len(jobs), ctypes.byref(dt), int(threads)))
    return array


# ---- CPU storage codec ------------------------------------------------------------

def _bytes_array(data):
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data.reshape(-1).view(np.uint8))
    return np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)


def count_tokens(data, vocab=b"", counts=None):
    """Adds greedy pair-parse token counts of `data` into `counts`."""
    lib = load()
    data = _bytes_array(data)
    vocab = bytes(vocab)
    if counts is None:
        counts = np.zeros(256 + len(vocab) // 2, dtype=np.uint64)
    vocab_array = np.frombuffer(vocab, dtype=np.uint8) if vocab else None
    check(lib.nz_count_tokens(_ptr(data) if len(data) else None, len(data), _ptr(vocab_array), len(vocab),
                              _ptr(counts)))
    return counts


def exponent_histograms(raw, dt, step):
    """(chunks, 256) exponent histograms of consecutive `step`-element chunks."""
    lib = load()
    raw = _bytes_array(raw)
    numel = len(raw) // dt.elem_size
    chunks = (numel + step - 1) // step
    out = np.zeros((chunks, 256), dtype=np.uint64)
    check(lib.nz_exponent_histograms(_ptr(raw) if numel else None, numel, ctypes.byref(dt), int(step), _ptr(out)))
    return out


def _encode(fn, codebook, data, cap, measure):
    lib = load()
    data = _bytes_array(data)
    written = ctypes.c_uint64()
    out = None if measure else np.empty(max(int(cap), 1), dtype=np.uint8)
    check(getattr(lib, fn)(codebook.handle, _ptr(data) if len(data) else None, len(data), _ptr(out), int(cap),
                           ctypes.byref(written)))
    return written.value if measure else out[:written.value].tobytes()


def mixed_encode(codebook, data, cap, measure=False):
    """Mixed frame bytes (b"" when it does not fit cap), or its size when measuring."""
    return _encode("nz_mixed_encode", codebook, data, cap, measure)


def huff0_encode(codebook, data, cap, measure=False):
    """Huff0 4-stream block bytes (b"" when it does not fit cap), or its size."""
    return _encode("nz_huff0_encode", codebook, data, cap, measure)


def mixed_decode(codebook, frame, expected, out=None):
    lib = load()
    frame = _bytes_array(frame)
    out = np.empty(expected, dtype=np.uint8) if out is None else out
    check(lib.nz_mixed_decode(codebook.handle, _ptr(frame), len(frame), _ptr(out), int(expected)))
    return out


def huff0_decode(codebook, block, count, out=None):
    lib = load()
    block = _bytes_array(block)
    out = np.empty(count, dtype=np.uint8) if out is None else out
    check(lib.nz_huff0_decode(codebook.handle, _ptr(block), len(block), _ptr(out), int(count)))
    return out


def cluster_chunks(distributions, weights, classes, forced, threshold, share=True):
    """(assignment per chunk, centroids) of nz_cluster_chunks."""
    lib = load()
    distributions = np.ascontiguousarray(distributions, dtype=np.float64)
    count, bins = distributions.shape
    weights = np.ascontiguousarray(weights, dtype=np.float64)
    classes = np.ascontiguousarray(classes, dtype=np.int32)
    forced = np.ascontiguousarray(forced, dtype=np.uint8)
    assign = np.zeros(count, dtype=np.uint32)
    centroids = np.zeros((max(count, 1), bins), dtype=np.float64)
    n = ctypes.c_uint64()
    check(lib.nz_cluster_chunks(_ptr(distributions), _ptr(weights), _ptr(classes), _ptr(forced), count, bins,
                                float(threshold), int(bool(share)), _ptr(assign), _ptr(centroids), len(centroids),
                                ctypes.byref(n)))
    return assign, centroids[:n.value]


def storage_decode(pieces, threads=0):
    """Decodes storage pieces (a STORAGE_PIECE_DTYPE array whose `lanes`
    point at STORAGE_LANE_DTYPE records) on the host cores; the caller keeps
    every buffer the records point at alive during the call."""
    lib = load()
    pieces = np.ascontiguousarray(pieces, dtype=STORAGE_PIECE_DTYPE)
    check(lib.nz_storage_decode(_ptr(pieces) if len(pieces) else None, len(pieces), int(threads)))


# ---- decode -----------------------------------------------------------------------

def decode_smem_bytes(warps_per_cta=8):
    lib = load()
    out = ctypes.c_uint32()
    check(lib.nz_decode_smem_bytes(int(warps_per_cta), ctypes.byref(out)))
    return out.value


def decode_tile_words(warps_per_cta):
    """Bitstream words of one tile a warp stages in shared memory."""
    lib = load()
    out = ctypes.c_uint32()
    check(lib.nz_decode_tile_words(int(warps_per_cta), ctypes.byref(out)))
    return out.value


def decode_occupancy(warps_per_cta):
    """Resident decode CTAs per SM on the current CUDA device."""
    lib = load()
    out = ctypes.c_uint32()
    check(lib.nz_decode_occupancy(int(warps_per_cta), ctypes.byref(out)))
    return out.value


def layout_code(element_size, bit_reorder, mantissa_bits, exponent_bits, stream_id):
    """NZ_LAYOUT_* of a DTypeSpec's GPU layout, or None if the kernel has none."""
    return {(2, True, 7, 8, 1): LAYOUT_BF16, (2, False, 10, 5, 1): LAYOUT_FP16,
            (4, True, 23, 8, 3): LAYOUT_FP32}.get(
        (int(element_size), bool(bit_reorder), int(mantissa_bits), int(exponent_bits), int(stream_id)))


class Schedule:
    """Owns an nz_schedule (the native per-block decode schedule)."""

    def __init__(self, unit_launches, depth, side_stream_handle):
        lib = load()
        launches = [launch for unit in unit_launches for launch in unit]
        first = [0]
        for unit in unit_launches:
            first.append(first[-1] + len(unit))
        array = (Launch * max(1, len(launches)))(*launches)
        first_array = (ctypes.c_uint32 * len(first))(*first)
        handle = ctypes.c_void_p()
        check(lib.nz_schedule_create(array, first_array, len(unit_launches), int(depth),
                                     ctypes.c_void_p(int(side_stream_handle) or None), ctypes.byref(handle)))
        self.handle = handle
        self._lib = lib
        self.enter_fn = lib.nz_schedule_enter  # bound once: the hook's only call

    def enter(self, unit, head, stream_handle):
        status = self.enter_fn(self.handle, unit, head, stream_handle)
        if status:
            check(status)

    def decode_unit(self, unit, stream_handle):
        check(self._lib.nz_schedule_decode_unit(self.handle, int(unit), ctypes.c_void_p(int(stream_handle) or None)))

    def drain(self, stream_handle):
        check(self._lib.nz_schedule_drain(self.handle, ctypes.c_void_p(int(stream_handle) or None)))

    def mark(self, unit, whole):
        check(self._lib.nz_schedule_mark(self.handle, int(unit), int(bool(whole))))

    def close(self):
        if self.handle:
            self._lib.nz_schedule_destroy(self.handle)
            self.handle = ctypes.c_void_p()


def decode_launch_many(launches, stream_handle):
    """Enqueues several launches as one step on a CUDA stream handle: the
    largest on the stream, the others on the library's side streams."""
    lib = load()
    array = (Launch * len(launches))(*launches)
    check(lib.nz_decode_launch_many(array, len(launches), ctypes.c_void_p(int(stream_handle) or None)))


def decode_launch(launch, stream_handle):
    """Enqueues the tile decode on a CUDA stream handle (an int)."""
    lib = load()
    check(lib.nz_decode_launch(ctypes.byref(launch), ctypes.c_void_p(int(stream_handle) or None)))


def decode_launch_noalloc(launch, stream_handle):
    """nz_decode_launch_noalloc: the same decode, its work-queue counters in
    the library's own device memory (for callers that cannot allocate);
    launch.scratch is ignored."""
    lib = load()
    check(lib.nz_decode_launch_noalloc(ctypes.byref(launch), ctypes.c_void_p(int(stream_handle) or None)))
