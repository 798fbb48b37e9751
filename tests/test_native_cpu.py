"""C ABI, host codec and setup checks that need no GPU."""

import ctypes
import pickle
import re
from pathlib import Path

import numpy as np
import pytest
import torch
from torch import nn

import helpers as H
from neuralzip_b200 import _native, huff0
from neuralzip_b200.compressor import NeuralZipCompressor
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu.inference import GPUCodebook, export_model_for_gpu
from neuralzip_b200.setup import NeuralZipSetup, _dtype_struct
from oracle import oracle as O

HEADER = Path(__file__).resolve().parents[1] / "include" / "nz_b200.h"


def test_library_exports_every_declared_symbol():
    declared = set(re.findall(r"^int (nz_\w+)\(", HEADER.read_text(), flags=re.M))
    assert declared == set(_native.EXPORTS)
    lib = ctypes.CDLL(str(_native.library_path()))
    for name in declared:
        assert hasattr(lib, name), name
    assert _native.load().nz_abi_version() == _native.ABI_VERSION == 4


def test_struct_layouts_match_header(tmp_path):
    """sizeof/offsetof of the C structs (compiled from the header) equal the
    Python mirrors used to build device descriptors."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    probe = tmp_path / "probe.c"
    probe.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "nz_b200.h"\n'
        'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(nz_group), sizeof(nz_work),'
        ' sizeof(nz_cta), sizeof(nz_launch), sizeof(nz_pack_job), sizeof(nz_dtype),'
        ' offsetof(nz_launch, n_ctas), offsetof(nz_group, numel)); return 0;}\n')
    subprocess.run([cc, f"-I{HEADER.parent}", str(probe), "-o", str(tmp_path / "probe")], check=True)
    sizes = [int(x) for x in subprocess.run([str(tmp_path / "probe")], capture_output=True, text=True,
                                            check=True).stdout.split()]
    assert sizes == [_native.GROUP_DTYPE.itemsize, _native.WORK_DTYPE.itemsize, _native.CTA_DTYPE.itemsize,
                     ctypes.sizeof(_native.Launch), ctypes.sizeof(_native.PackJob), ctypes.sizeof(_native.Dtype),
                     _native.Launch.n_ctas.offset, _native.GROUP_DTYPE.fields["numel"][1]]


def test_error_mapping():
    with pytest.raises(RuntimeError, match="Duplicate mixed pair"):
        _native.export_code_table(b"NZM1" + bytes([9] * 258), 56, bytes((1, 2, 1, 2)))
    with pytest.raises(RuntimeError, match="256 singletons"):
        _native.export_code_table(b"NZM1" + bytes([8] * 100), 56)
    with pytest.raises(ValueError, match="max_bits"):
        _native.export_code_table(b"NZM1" + bytes([8] * 256), 0)
    with pytest.raises(RuntimeError, match="Incomplete"):
        _native.export_code_table(b"NZM1" + bytes([9] * 256), 56)
    with pytest.raises(ValueError, match="code-length limit"):
        GPUCodebook(tuple([13] + [8] * 255), tuple(range(256)))
    with pytest.raises(ValueError, match="alphabet"):
        GPUCodebook(tuple([8] * 257), tuple(range(257)))
    with pytest.raises(ValueError):
        _native.dtype_struct(3, 0, 7, 8, 1) and _native.split_lanes(b"\0" * 6, _native.dtype_struct(3, 0, 7, 8, 1))
    with pytest.raises(RuntimeError, match="at least two"):
        huff0.build_codebook_from_counts([5] + [0] * 255, prior_count=0, max_bits=12)
    with pytest.raises(ValueError, match="256 entries"):
        huff0.build_codebook_from_counts([1] * 10)


@pytest.mark.parametrize("seed", range(8))
def test_huff0_headers_round_trip(seed):
    rng = np.random.default_rng(seed)
    counts = np.zeros(256, dtype=np.uint64)
    present = rng.choice(256, size=int(rng.integers(2, 257)), replace=False)
    counts[present] = rng.geometric(0.02 if seed % 2 else 0.3, size=len(present))
    book = huff0.build_codebook_from_counts(counts, prior_count=seed % 2, max_bits=12)
    lengths, values, table_log, used = _native.huff0_read(book.codebook)
    assert used == len(book.codebook) and table_log <= 12
    lengths = np.frombuffer(lengths, dtype=np.uint8)
    present_mask = (counts + (seed % 2)) > 0
    assert np.array_equal(lengths > 0, present_mask)
    kraft = sum(2.0 ** -int(length) for length in lengths if length)
    assert kraft == 1.0
    # Canonical values: longest codes first, symbol order within a length.
    order = sorted((-int(length), s) for s, length in enumerate(lengths) if length)
    codes = [(int(lengths[s]), values[s]) for _, s in order]
    assert len(set(codes)) == len(codes)
    # Huff0 4-stream blocks round trip through the product codec.
    weights = (counts + (seed % 2)).astype(np.float64)
    data = rng.choice(256, size=20000, p=weights / weights.sum()).astype(np.uint8)
    block = _native.huff0_encode(book.handle, data, 2 * len(data))
    assert block and np.array_equal(_native.huff0_decode(book.handle, block, len(data)), data)


def test_empty_batch_and_zero_cta_launch():
    """An empty batch is refused on the host; a launch with no CTAs is a
    no-op that touches no device state (so it runs without a GPU)."""
    from neuralzip_b200.gpu import decoder as gpu_decoder

    with pytest.raises(ValueError, match="at least one group"):
        gpu_decoder.default_decoder().prepare_batch([])
    launch = _native.Launch()
    launch.n_ctas = 0
    _native.decode_launch(launch, 0)
    launch.n_ctas = 1
    with pytest.raises(ValueError, match="Null device"):
        _native.decode_launch(launch, 0)


def test_uniform_alphabet_is_left_raw():
    setup = NeuralZipSetup()
    assert setup._singleton(np.full(256, 100, dtype=np.uint64)) is None


class Model(nn.Module):
    def __init__(self, dtype):
        super().__init__()
        self.layers = nn.ModuleList([nn.Linear(257, 513, bias=False, dtype=dtype),
                                     nn.Linear(513, 17, bias=False, dtype=dtype)])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_storage_round_trip_and_export(dtype):
    """The reference's CPU kernel check (_experiment_kernel_checks.py:134-174):
    pattern weights, chunk_size 8192, bitwise storage round trip, packed
    codebooks where the dtype has a pure exponent lane, and a raw fragment
    between compressed chunks in the GPU export."""
    model = Model(dtype)
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(H.pattern_weights(p.numel(), dtype).view_as(p))
    named = dict(model.named_parameters())
    setup = NeuralZipSetup(chunk_size=8192).build(named)
    blob, metadata, sizes, seconds = NeuralZipCompressor(setup, threads=1).encode(named.items())
    assert metadata["version"] == 2 and sizes["compressed_bytes"] < sizes["raw_bytes"]
    decoded = NeuralZipCompressor().decode(blob, metadata)
    assert all(torch.equal(decoded[n].view(torch.uint8), t.detach().view(torch.uint8)) for n, t in named.items())
    key = next(iter(setup.chunk_codebooks))
    ids = list(setup.chunk_codebooks[key])
    ids[len(ids) // 2] = None
    setup.chunk_codebooks[key] = tuple(ids)
    exported = export_model_for_gpu(model, setup)
    assert {b.tensor_name for b in exported.bindings} == set(named)
    assert any(g.codebook_id == -1 for g in exported.groups)
    if DTYPES[dtype].exponent_stream is not None:
        assert any(g.codebook.vocab for g in exported.groups), "packed route not exercised"
    # Every group decodes (CPU reader) to its slice of the original.
    for g in exported.groups:
        spec = g.encoded.dtype
        sym = g.encoded.symbols
        binding = g.bindings[0]
        start = g.workspace_offset - binding.workspace_offset
        raw = named[binding.tensor_name].detach().reshape(-1)[start:start + g.encoded.numel]
        expected = H.selected_lane(raw.view(torch.uint8).numpy().tobytes(), spec)
        if g.codebook.max_bits:
            got = O.tile_decode(np.frombuffer(sym.bitstream, dtype=np.uint32), np.frombuffer(sym.lane_bits, np.uint16),
                                np.asarray(sym.tile_offsets), g.encoded.numel, g.codebook.code_lengths,
                                g.codebook.code_values, g.codebook.vocab)
        else:
            got = np.frombuffer(sym.bitstream, dtype=np.uint8)
        assert np.array_equal(got, expected)


def test_setup_pickle_and_options():
    named = {"a.weight": (torch.randn(64, 4096) * 0.02).to(torch.bfloat16),
             "b.weight": (torch.randn(64, 4096) * 1.0).to(torch.bfloat16)}
    setup = NeuralZipSetup(chunk_size=64 << 10).build(named)
    again = pickle.loads(pickle.dumps(setup))
    assert again.chunk_codebooks == setup.chunk_codebooks and len(again.codebooks) == len(setup.codebooks)
    assert NeuralZipSetup.load(again) is again
    forced = NeuralZipSetup(chunk_size=64 << 10, cluster_map={"a.weight": 7, "b.weight": 7}).build(named)
    ids = {i for v in forced.chunk_codebooks.values() for i in v}
    assert len(ids) == 1  # one forced cluster for both tensors
    off = NeuralZipSetup(enable_shared_codebooks=False, enable_packed_codebooks=False).build(named)
    assert off.codebooks == () and all(i is None for v in off.chunk_codebooks.values() for i in v)
    singleton_only = NeuralZipSetup(chunk_size=64 << 10, enable_packed_codebooks=False).build(named)
    assert all(b.mode == "shared_huff0" for b in singleton_only.codebooks)
    with pytest.raises(ValueError):
        NeuralZipSetup(chunk_size=2)


def test_multithreaded_pack_matches_single_chunk():
    spec = DTYPES[torch.bfloat16]
    raw = H.gaussian_raw(3 * 131072 + 5, 0.02, torch.bfloat16, 9)
    sel = H.selected_lane(raw, spec)
    lengths, vocab = H.mixed_book_for(sel)
    book = GPUCodebook(tuple(lengths), tuple(int(c) for c in O.mixed_codes(lengths)), vocab)
    from neuralzip_b200.gpu.inference import _pack_parallel, encode_with_codebook

    parts = [raw[i:i + 2 * 131072] for i in range(0, len(raw), 2 * 131072)]
    many = _pack_parallel([(np.frombuffer(p, dtype=np.uint8), book, spec) for p in parts], threads=4)
    for part, enc in zip(parts, many):
        one = encode_with_codebook(part, book, dtype=spec, stream_id=1)
        assert bytes(enc.symbols.bitstream) == bytes(one.symbols.bitstream)
        assert bytes(enc.symbols.lane_bits) == bytes(one.symbols.lane_bits)
        assert enc.symbols.tile_offsets == one.symbols.tile_offsets


def test_config1_storage_round_trip():
    """BASELINE config 1 on the CPU path: a 4096x4096 bf16 N(0, 0.02) tensor
    (seed 0), 256 KiB chunks, JS threshold 0.05, singleton (Huff0) codes
    only; storage v2 encode and decode are bit-exact and the export packs
    every chunk with a singleton table."""
    g = torch.Generator().manual_seed(0)
    named = {"w": (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.bfloat16)}
    setup = NeuralZipSetup(chunk_size=256 << 10, cluster_js_threshold=0.05,
                           enable_packed_codebooks=False).build(named)
    assert setup.codebooks and all(b.mode == "shared_huff0" for b in setup.codebooks)
    blob, metadata, sizes, _ = NeuralZipCompressor(setup, threads=4).encode(named.items())
    assert sizes["compressed_bytes"] < sizes["raw_bytes"]
    decoded = NeuralZipCompressor().decode(blob, metadata)
    assert torch.equal(decoded["w"].view(torch.uint8), named["w"].view(torch.uint8))
    from neuralzip_b200.gpu.inference import export_tensors_for_gpu

    export = export_tensors_for_gpu(named, setup)
    assert len(export.groups) == 128 and all(not g.codebook.vocab and g.codebook.max_bits for g in export.groups)


def test_decode_geometry_fits_shared_memory():
    """Each CTA width's shared memory (table + per-warp staging rows and
    tile-bitstream copy) keeps its resident CTAs within an SM's 228 KB."""
    resident = {24: 1, 16: 1, 8: 2, 4: 3}
    copy_words = {24: 956, 16: 1960, 8: 1332, 4: 1292}
    for nw, ctas in resident.items():
        smem = _native.decode_smem_bytes(nw)
        assert smem <= 232448 and ctas * (smem + 1024) <= 233472
        assert _native.decode_tile_words(nw) == copy_words[nw]
    with pytest.raises(ValueError):
        _native.decode_tile_words(12)


def test_tile_copy_words_matches_kernel_bounds():
    from neuralzip_b200.gpu.decoder import tile_copy_words

    # Tiles at bits [0, 100), [100, 5000), [5000, 5001): the copy runs from
    # the 16-byte boundary at or below the first bit to 12..15 words past
    # the word of the last one.
    assert tile_copy_words([0, 100, 5000], 5001) == max(((100 >> 5) + 16) & ~3,
                                                         (((5000 >> 5) + 16) & ~3) - ((100 >> 5) & ~3),
                                                         (((5001 >> 5) + 16) & ~3) - ((5000 >> 5) & ~3))
    assert tile_copy_words([], 0) == 0


def _js(a, b):
    m = 0.5 * (a + b)
    left = np.sum(a[a > 0] * np.log2(a[a > 0] / m[a > 0]))
    right = np.sum(b[b > 0] * np.log2(b[b > 0] / m[b > 0]))
    return float(np.sqrt(max(0.5 * left + 0.5 * right, 0.0)))


@pytest.mark.parametrize("share", [True, False])
def test_native_clustering_matches_sequential_rule(share):
    """nz_cluster_chunks against the clustering rule of
    neuralzip/setup.py:91-141 restated step by step in numpy: nearest
    centroid of the same class (earliest on ties), joined within the
    threshold or when forced, centroids weight-averaged after each chunk."""
    rng = np.random.default_rng(4)
    protos = rng.dirichlet(np.full(256, 0.05), size=5)
    n = 300
    dists = np.stack([rng.dirichlet(protos[rng.integers(5)] * 400 + 1e-3) for _ in range(n)])
    weights = rng.integers(1000, 5000, size=n).astype(np.float64)
    classes = rng.integers(0, 3, size=n).astype(np.int32)
    forced = (rng.random(n) < 0.1).astype(np.uint8)
    threshold = 0.3
    assign, centroids = _native.cluster_chunks(dists, weights, classes, forced, threshold, share=share)
    cls, cent, wts, expect = [], [], [], []
    for i in range(n):
        best, best_d = None, None
        for c in range(len(cls)) if share else ():
            if cls[c] != classes[i]:
                continue
            d = _js(dists[i], cent[c])
            if best is None or d < best_d:
                best, best_d = c, d
        if best is None or (not forced[i] and best_d > threshold):
            best = len(cls)
            cls.append(classes[i]); cent.append(dists[i].copy()); wts.append(0.0)
        total = wts[best] + weights[i]
        cent[best] = (cent[best] * wts[best] + dists[i] * weights[i]) / total
        wts[best] = total
        expect.append(best)
    assert assign.tolist() == expect
    assert len(centroids) == len(cls) and np.allclose(centroids, np.stack(cent), rtol=0, atol=1e-12)
    if not share:
        assert len(cls) == n


def _gaussian_checkpoint():
    g = torch.Generator().manual_seed(9)
    named = {"a": (torch.randn(64, 4096, generator=g) * 0.02).to(torch.bfloat16),
             "b": (torch.randn(40, 1000, generator=g) * 0.5).to(torch.float16),
             "c": torch.randn(33, 517, generator=g) * 0.1}
    setup = NeuralZipSetup(chunk_size=8192).build(named)
    blob, metadata, _sizes, _seconds = NeuralZipCompressor(setup, threads=2).encode(named.items())
    return named, setup, blob, metadata


def test_native_storage_decode_matches_the_per_chunk_wrapper():
    """The one-call storage decode (nz_storage_decode) and the per-lane
    chunk-list wrapper (huff0.decompress_mixed_streams_many, the reference's
    decode-queue signature) give the original bytes for singleton, mixed and
    raw chunks of bf16, fp16 and fp32 tensors."""
    from neuralzip_b200 import huff0
    from neuralzip_b200.storage import StorageReader

    named, setup, blob, metadata = _gaussian_checkpoint()
    modes = {c["mode"] for t in metadata["tensors"] for lane in t["groups"] for c in lane}
    assert {"raw", "shared_huff0", "mixed_huffman"} <= modes
    for threads in (1, 3):
        decoded = NeuralZipCompressor(setup, threads=threads).decode(blob, metadata)
        assert all(torch.equal(decoded[n].view(torch.uint8), t.view(torch.uint8)) for n, t in named.items())
    reader = StorageReader(blob, metadata)
    books = {b.codebook_id: huff0.build_decodebook(b.codebook, vocab=b.vocab) for b in reader.codebooks()}
    specs = [(t.element_size, t.bit_reorder, t.numel,
              [[(c.mode, c.payload, c.symbol_count, books.get(c.codebook_id)) for c in lane.chunks]
               for lane in t.groups]) for t in reader.tensors()]
    for out, t in zip(huff0.decompress_mixed_streams_many(specs, threads=2), reader.tensors()):
        assert bytes(out) == named[t.name].reshape(-1).view(torch.uint8).numpy().tobytes()


def test_native_storage_decode_reports_corrupt_chunks():
    """A corrupted coded payload fails the whole call with the decoder's
    message; inconsistent metadata is rejected before any decoding."""
    import copy

    named, setup, blob, metadata = _gaussian_checkpoint()
    coded = next(c for t in metadata["tensors"] for lane in t["groups"] for c in lane if c["mode"] == "shared_huff0")
    bad = blob.clone()
    offset, size = coded["payload"]
    bad[offset + 6:offset + size] = 0xFF  # streams of garbage behind an intact jump table
    with pytest.raises(ValueError):
        NeuralZipCompressor(setup).decode(bad, metadata)
    broken = copy.deepcopy(metadata)
    raw = next(c for t in broken["tensors"] for lane in t["groups"] for c in lane if c["mode"] == "raw")
    raw["payload"][1] -= 1
    with pytest.raises(ValueError, match="Raw payload size mismatch"):
        NeuralZipCompressor(setup).decode(blob, broken)
    broken = copy.deepcopy(metadata)
    broken["tensors"][0]["groups"][0][0]["symbols"] += 1
    with pytest.raises(ValueError, match="Unaligned chunk boundaries|exceeds"):
        NeuralZipCompressor(setup).decode(blob, broken)


def _reordered_words(raw, spec):
    """numpy restatement of DTypeSpec.reorder_bytes on whole words."""
    w = raw.view(np.uint16 if spec.element_size == 2 else np.uint32).astype(np.uint64)
    if spec.bit_reorder:
        mant = (1 << spec.mantissa_bits) - 1
        sign = 1 << spec.mantissa_bits
        expm = ((1 << spec.exponent_bits) - 1) << (spec.mantissa_bits + 1)
        w = (w & mant) | ((w >> spec.exponent_bits) & sign) | ((w << 1) & expm)
    return w


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("numel", [0, 1, 7, (1 << 20) + 5, 3 << 20])
def test_split_lanes_threaded_and_selected_only(dtype, numel):
    """nz_split_lanes splits large inputs in 1 Mi-element blocks on the
    host's threads and skips lanes whose buffer is NULL; every lane equals
    the reorder restated in numpy."""
    spec = DTYPES[dtype]
    raw = (torch.randn(numel, generator=torch.Generator().manual_seed(numel)) * 0.02).to(dtype)
    raw = raw.view(torch.uint8).numpy()
    dt = _dtype_struct(spec)
    words = _reordered_words(raw, spec)
    lanes = _native.split_lanes(raw, dt)
    for lane in range(spec.element_size):
        assert np.array_equal(lanes[lane], ((words >> (8 * lane)) & 0xFF).astype(np.uint8))
    only = _native.split_lanes(raw, dt, selected_only=True)
    assert [lane is None for lane in only] == [k != spec.gpu_stream for k in range(spec.element_size)]
    assert np.array_equal(only[spec.gpu_stream], lanes[spec.gpu_stream])


def test_split_lanes_requires_the_selected_lane():
    spec = DTYPES[torch.bfloat16]
    raw = np.zeros(16, dtype=np.uint8)
    lib = _native.load()
    keep = np.empty(8, dtype=np.uint8)
    lanes = (ctypes.c_void_p * 4)(keep.ctypes.data, None, None, None)  # lane 1 is bf16's selected lane
    assert lib.nz_split_lanes(raw.ctypes.data, 8, ctypes.byref(_dtype_struct(spec)), lanes) != 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_exponent_histograms_match_numpy(dtype):
    """Per-chunk exponent-field histograms, counted on the host's threads,
    with a ragged last chunk."""
    spec = DTYPES[dtype]
    numel = 5 * 131072 + 999
    raw = (torch.randn(numel, generator=torch.Generator().manual_seed(3)) * 0.3).to(dtype).view(torch.uint8).numpy()
    step = 131072
    hist = np.asarray(_native.exponent_histograms(raw, _dtype_struct(spec), step)).reshape(-1, 256)
    w = raw.view(np.uint16 if spec.element_size == 2 else np.uint32).astype(np.int64)
    e = (w >> spec.mantissa_bits) & ((1 << spec.exponent_bits) - 1)
    want = np.stack([np.bincount(e[s:s + step], minlength=256) for s in range(0, numel, step)])
    assert np.array_equal(hist.astype(np.int64), want)


@pytest.mark.parametrize("size", [0, 3, (1 << 22) - 1, (1 << 22) + 1, 3 * (1 << 22) + 17])
def test_byte_counts_across_blocks(size):
    """count_tokens without a pair vocabulary (4 Mi-byte blocks on the
    host's threads) equals a plain byte count."""
    data = np.random.default_rng(size).integers(0, 256, size, dtype=np.uint8)
    counts = np.asarray(_native.count_tokens(data, b""))
    assert np.array_equal(counts[:256].astype(np.int64), np.bincount(data, minlength=256))


@pytest.mark.parametrize("size", [1, 2, 3, 5, 4096 + 3, 131072])
def test_mixed_decode_lockstep_round_trips(size):
    """The host mixed decoder runs a frame's four lanes in lockstep; frames
    of every size (including lanes with unequal token counts) decode back
    to their bytes."""
    raw = H.gaussian_raw(max(size, 64), 0.02, torch.bfloat16, size)
    sel = H.selected_lane(raw, DTYPES[torch.bfloat16])[:size]
    lengths, vocab = H.mixed_book_for(sel)
    book = _native.NativeCodebook(lengths, None, vocab)
    frame = _native.mixed_encode(book, sel, 4 * size + 64)
    assert np.array_equal(_native.mixed_decode(book, frame, size), sel)


def test_mixed_decode_rejects_corrupt_frames():
    raw = H.gaussian_raw(20000, 0.02, torch.bfloat16, 9)
    sel = H.selected_lane(raw, DTYPES[torch.bfloat16])
    lengths, vocab = H.mixed_book_for(sel)
    book = _native.NativeCodebook(lengths, None, vocab)
    frame = bytearray(_native.mixed_encode(book, sel, 4 * len(sel) + 64))
    n = len(sel)
    cases = {
        "truncated": bytes(frame[:-1]),
        "trailing byte": bytes(frame) + b"\0",
        "token count + 1": (int.from_bytes(frame[:4], "little") + 1).to_bytes(4, "little") + bytes(frame[4:]),
        "bit count - 1": bytes(frame[:4]) + (int.from_bytes(frame[4:8], "little") - 1).to_bytes(4, "little") + bytes(frame[8:]),
        "short header": bytes(frame[:31]),
    }
    for what, bad in cases.items():
        with pytest.raises(ValueError):
            _native.mixed_decode(book, bad, n)
            pytest.fail(what)
    with pytest.raises(ValueError):  # one byte more expected than the frame holds
        _native.mixed_decode(book, bytes(frame), n + 1)
