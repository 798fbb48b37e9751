"""GPU parity of the tile decode kernel against the oracle (bit-exact).

Every expected tensor is computed on the CPU by the oracle: the reference
GPU layout is encoded and decoded with the reference's kernel semantics
(oracle/nz_oracle.c: oz_ref_encode / oz_ref_decode) and the lanes merged
(oz_restore). The oracle output is also checked against the original bits,
which is the reference's own criterion for every decode.
"""

import numpy as np
import pytest
import torch
from torch import nn

import helpers as H
from neuralzip_b200 import _native
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu import decoder as gpu_decoder
from neuralzip_b200.gpu.inference import (
    GPUCodebook,
    GPUWeightGroup,
    LinearWeightBinding,
    NeuralZipModelExport,
    NeuralZipRuntime,
    encode_raw_fragment,
    encode_with_codebook,
)
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def exact(a, b):
    return torch.equal(a.cpu().contiguous().view(torch.uint8), b.cpu().contiguous().view(torch.uint8))


def oracle_expected(raw, spec, lengths, values, vocab):
    """Oracle decode of the reference GPU layout, merged with the raw lanes."""
    lanes = O.split(raw, spec)
    sel = lanes[spec.gpu_stream]
    layout = O.ref_encode(sel, lengths, values, vocab)
    lut, max_bits = O.ref_lut(lengths, values, vocab)
    decoded = O.ref_decode(layout, lut, max_bits, bool(vocab), len(sel))
    lanes[spec.gpu_stream] = decoded
    out = O.restore(lanes, spec)
    assert out.tobytes() == bytes(raw), "oracle does not reproduce the original bits"
    return out


def single_group_model(raw, spec, book):
    original = torch.frombuffer(bytearray(raw), dtype=spec.torch_dtype).reshape(1, -1)
    model = nn.Module()
    model.layers = nn.ModuleList([nn.Linear(original.numel(), 1, bias=False, dtype=spec.torch_dtype)])
    with torch.no_grad():
        model.layers[0].weight.copy_(original)
    encoded = encode_with_codebook(raw, book, dtype=spec, stream_id=spec.gpu_stream)
    binding = LinearWeightBinding("layers.0", "layers.0.weight", tuple(original.shape), original.numel(), 0)
    export = NeuralZipModelExport((GPUWeightGroup("layers.0", 0, book, encoded, (binding,), 0),))
    return model, export, original


@pytest.mark.parametrize("max_bits", [12, 13, 20, 31, 32, 33, 56])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_segment_boundaries(max_bits, dtype):
    spec = DTYPES[dtype]
    lengths = H.segment_lengths(max_bits)
    values = O.mixed_codes(lengths)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in values), H.VOCAB)
    raw = H.lanes_with(H.segment_symbols(), spec)
    expected = oracle_expected(raw, spec, lengths, values, H.VOCAB)
    model, export, original = single_group_model(raw, spec, book)
    runtime = NeuralZipRuntime.attach(model, export, device="cuda:0")
    for _ in range(2):
        for workspace in runtime.workspaces.values():
            workspace.view(torch.uint8).fill_(0xA5)
        got = dict(runtime.materialized_weights())["layers.0.weight"]
        assert exact(got, original)
        assert got.view(torch.uint8).numpy().tobytes() == expected.tobytes()
    runtime.check_status()


def test_long_codes_bf16():
    spec = DTYPES[torch.bfloat16]
    lengths = H.long_code_lengths()
    assert max(lengths) > 12
    values = O.mixed_codes(lengths)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in values), H.VOCAB)
    assert book.native.tree_nodes > 0
    symbols = np.array([127] * 70000 + list(range(256)) * 3 + [126], dtype=np.uint8)
    raw = H.lanes_with(symbols, spec)
    expected = oracle_expected(raw, spec, lengths, values, H.VOCAB)
    model, export, original = single_group_model(raw, spec, book)
    runtime = NeuralZipRuntime.attach(model, export, device="cuda:0")
    got = dict(runtime.materialized_weights())["layers.0.weight"]
    assert exact(got, original)
    assert got.view(torch.uint8).numpy().tobytes() == expected.tobytes()


def _gaussian_export(spec, numel, sigmas, chunk, seed=0, raw_chunk=None, mixed=True):
    """One tensor cut into `chunk`-element groups with per-chunk sigma;
    singleton and mixed codebooks alternate, one chunk may stay raw."""
    pieces = [H.gaussian_raw(min(chunk, numel - s), sigmas[i % len(sigmas)], spec.torch_dtype, seed + i)
              for i, s in enumerate(range(0, numel, chunk))]
    raw = b"".join(pieces)
    original = torch.frombuffer(bytearray(raw), dtype=spec.torch_dtype).reshape(1, -1)
    binding = LinearWeightBinding("layers.0", "layers.0.weight", tuple(original.shape), numel, 0)
    groups, books = [], {}
    for i, piece in enumerate(pieces):
        sel = H.selected_lane(piece, spec)
        start = i * chunk
        if raw_chunk is not None and i == raw_chunk:
            enc = encode_raw_fragment(piece, dtype=spec, stream_id=spec.gpu_stream)
            groups.append(GPUWeightGroup("layers.0", -1, GPUCodebook((), ()), enc, (binding,), start))
            continue
        if mixed and spec.exponent_stream is not None and i % 2 == 1:
            lengths, vocab = H.mixed_book_for(sel)
            book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
        else:
            header, _ = _native.huff0_build(np.bincount(sel, minlength=256) + 1, 12)
            lengths, values, _, _ = _native.huff0_read(header)
            book = GPUCodebook(tuple(lengths), values)
        books[i] = book
        enc = encode_with_codebook(piece, book, dtype=spec, stream_id=spec.gpu_stream)
        groups.append(GPUWeightGroup("layers.0", i, book, enc, (binding,), start))
    return raw, original, NeuralZipModelExport(tuple(groups))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_multi_codebook_batch_with_raw_fragment(dtype):
    spec = DTYPES[dtype]
    numel = 5 * 131072 + 4099  # odd tail chunk
    raw, original, export = _gaussian_export(spec, numel, [0.02, 0.002, 0.2, 1.0], 131072, raw_chunk=2)
    model = nn.Module()
    model.layers = nn.ModuleList([nn.Linear(numel, 1, bias=False, dtype=dtype)])
    runtime = NeuralZipRuntime.attach(model, export, device="cuda:0")
    for workspace in runtime.workspaces.values():
        workspace.view(torch.uint8).fill_(0xA5)
    got = dict(runtime.materialized_weights())["layers.0.weight"]
    assert exact(got, original)
    runtime.check_status()


def _device_group(raw, spec, book, out_tensor, arena, lut_index=0):
    """Uploads one group by hand; returns its DeviceGroup. Groups of one
    batch that use different tables need different `lut_index` values."""
    enc = encode_with_codebook(raw, book, dtype=spec, stream_id=spec.gpu_stream)
    sym = enc.symbols
    pieces = {"bits": sym.bitstream, "lens": sym.lane_bits,
              "tile_off": np.asarray(sym.tile_offsets, dtype=np.uint32).tobytes()}
    for lane, data in enumerate(enc.streams):
        if lane != spec.gpu_stream:
            pieces[f"lane{lane}"] = data
    addr = {}
    for name, data in pieces.items():
        t = torch.frombuffer(bytearray(data), dtype=torch.uint8).to("cuda")
        arena.append(t)
        addr[name] = t.data_ptr()
    lut = torch.from_numpy(np.asarray(book.decode_lut, dtype=np.uint32).view(np.int32)).to("cuda")
    arena.append(lut)
    return gpu_decoder.DeviceGroup(
        spec=spec, numel=enc.numel, lut_index=lut_index, lut_ptr=lut.data_ptr(),
        lut_words=book.table_words, bits=addr["bits"], lens=addr["lens"], tile_off=addr["tile_off"],
        lanes=tuple(addr.get(f"lane{lane}", 0) for lane in range(4)), out=out_tensor.data_ptr(),
        output=out_tensor)


@pytest.mark.parametrize("offset_elems", [0, 1, 3])
def test_guard_bytes_and_unaligned_outputs(offset_elems):
    """Writes stay inside [out, out + numel); unaligned outputs take the
    scalar path and still match."""
    spec = DTYPES[torch.bfloat16]
    numel = 3 * 8192 + 777
    raw = H.gaussian_raw(numel, 0.02, torch.bfloat16, 7)
    sel = H.selected_lane(raw, spec)
    lengths, vocab = H.mixed_book_for(sel)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
    guard = 4096
    buffer = torch.full((numel + 2 * guard,), -1, dtype=torch.int16, device="cuda")
    out = buffer[guard + offset_elems:guard + offset_elems + numel].view(torch.bfloat16)
    arena = []
    dg = _device_group(raw, spec, book, out, arena)
    decoder = gpu_decoder.default_decoder()
    prepared = decoder.prepare_batch([dg])
    decoder.decode_batch(prepared)
    torch.cuda.synchronize()
    host = buffer.cpu()
    assert bytes(out.cpu().view(torch.uint8).numpy()) == raw
    assert (host[:guard + offset_elems] == -1).all()
    assert (host[guard + offset_elems + numel:] == -1).all()
    decoder.check_status(prepared)


def test_c_abi_launch_by_hand():
    """Builds nz_group / nz_work / nz_cta records directly and calls
    nz_decode_launch, without the Python decoder."""
    spec = DTYPES[torch.float32]
    numel = 2 * 8192 + 5
    raw = H.gaussian_raw(numel, 0.02, torch.float32, 3)
    sel = H.selected_lane(raw, spec)
    lengths, vocab = H.mixed_book_for(sel)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
    out = torch.empty(numel, dtype=torch.float32, device="cuda")
    arena = []
    dg = _device_group(raw, spec, book, out, arena)
    groups = np.zeros(1, dtype=_native.GROUP_DTYPE)
    groups[0] = (dg.bits, dg.lens, dg.tile_off, dg.lanes, dg.out, numel, 0)
    works = np.array([(0, t) for t in range(dg.tiles)], dtype=_native.WORK_DTYPE)
    ctas = np.array([(0, 0, dg.tiles, dg.lut_words, _native.LAYOUT_FP32, 0, 0)], dtype=_native.CTA_DTYPE)
    luts = np.array([dg.lut_ptr], dtype=np.uint64)
    dev = [torch.from_numpy(a.view(np.uint8).copy()).cuda() for a in (groups, works, ctas, luts)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    launch = _native.Launch()
    launch.warps_per_cta = 4
    launch.groups, launch.works, launch.ctas, launch.luts = (t.data_ptr() for t in dev)
    launch.status = status.data_ptr()
    launch.n_ctas = 1
    _native.decode_launch(launch, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert bytes(out.cpu().view(torch.uint8).numpy()) == raw
    assert int(status.item()) == 0
    # A CTA that names no known layout writes nothing and reports status 3.
    out.view(torch.int32).fill_(-1)
    ctas["layout"] = 7
    dev[2].copy_(torch.from_numpy(ctas.view(np.uint8).copy()))
    _native.decode_launch(launch, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 3
    assert bool((out.view(torch.int32) == -1).all())


def test_c_abi_work_queues_by_hand():
    """CTAs that name one queue share their range through the launch
    scratch: every tile is decoded once, and the last CTA sets the counters
    back to zero, so the next launch on the same scratch works too."""
    spec = DTYPES[torch.bfloat16]
    numel = 9 * 8192 + 77
    raw = H.gaussian_raw(numel, 0.02, torch.bfloat16, 5)
    sel = H.selected_lane(raw, spec)
    lengths, vocab = H.mixed_book_for(sel)
    book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
    out = torch.empty(numel, dtype=torch.bfloat16, device="cuda")
    arena = []
    dg = _device_group(raw, spec, book, out, arena)
    groups = np.zeros(1, dtype=_native.GROUP_DTYPE)
    groups[0] = (dg.bits, dg.lens, dg.tile_off, dg.lanes, dg.out, numel, 0)
    works = np.array([(0, t) for t in range(dg.tiles)], dtype=_native.WORK_DTYPE)
    ctas = np.array([(0, 0, dg.tiles, dg.lut_words, _native.LAYOUT_BF16, 0, 0)] * 3, dtype=_native.CTA_DTYPE)
    luts = np.array([dg.lut_ptr], dtype=np.uint64)
    dev = [torch.from_numpy(a.view(np.uint8).copy()).cuda() for a in (groups, works, ctas, luts)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(2, dtype=torch.int32, device="cuda")
    launch = _native.Launch()
    launch.warps_per_cta = 4
    launch.groups, launch.works, launch.ctas, launch.luts = (t.data_ptr() for t in dev)
    launch.status = status.data_ptr()
    launch.n_ctas = 3
    launch.scratch, launch.queues = scratch.data_ptr(), 1
    for _ in range(3):
        out.view(torch.int16).fill_(-1)
        _native.decode_launch(launch, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert bytes(out.cpu().view(torch.uint8).numpy()) == raw
        assert int(status.item()) == 0
        assert scratch.tolist() == [0, 0]
    # A CTA naming a queue the launch does not have writes nothing and
    # reports status 4; the counters still end at zero.
    out.view(torch.int16).fill_(-1)
    ctas["queue"] = 7
    dev[2].copy_(torch.from_numpy(ctas.view(np.uint8).copy()))
    _native.decode_launch(launch, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 4
    assert bool((out.view(torch.int16) == -1).all())
    assert scratch.tolist() == [0, 0]


@pytest.mark.parametrize("work_queues", [False, True])
def test_fixed_ranges_and_work_queues_decode_alike(work_queues):
    """The launch plan with per-CTA ranges and with shared queues gives the
    same bits over a batch of several codebooks, twice in a row."""
    spec = DTYPES[torch.bfloat16]
    decoder = gpu_decoder.TileDecoder()
    decoder.work_queues = work_queues
    outs, devs, raws, arena = [], [], [], []
    for seed, sigma in enumerate((0.02, 0.5, 0.002)):
        numel = (5 + seed) * 8192 + 31 * seed
        raw = H.gaussian_raw(numel, sigma, torch.bfloat16, 10 + seed)
        sel = H.selected_lane(raw, spec)
        lengths, vocab = H.mixed_book_for(sel)
        book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
        out = torch.empty(numel, dtype=torch.bfloat16, device="cuda")
        devs.append(_device_group(raw, spec, book, out, arena, lut_index=seed))
        outs.append(out)
        raws.append(raw)
    batch = decoder.prepare_batch(devs)
    for _ in range(2):
        for out in outs:
            out.view(torch.int16).fill_(-1)
        decoder.decode_batch(batch)
        torch.cuda.synchronize()
        decoder.check_status(batch)
        for out, raw in zip(outs, raws):
            assert bytes(out.cpu().view(torch.uint8).numpy()) == raw


def test_launch_rejects_bad_geometry():
    launch = _native.Launch()
    launch.warps_per_cta = 5
    launch.n_ctas = 1
    launch.groups = launch.works = launch.ctas = launch.luts = 1
    with pytest.raises(ValueError):
        _native.decode_launch(launch, 0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_tiny_and_ragged_groups(dtype):
    """Groups of 1, 7, 9, 255, 257 and 8193 elements in one launch (partial
    sub-streams, partial tiles, scalar tails), singleton and mixed books."""
    spec = DTYPES[dtype]
    decoder = gpu_decoder.default_decoder()
    arena, groups, expected = [], [], []
    for i, numel in enumerate((1, 7, 9, 255, 257, 8193)):
        raw = H.gaussian_raw(numel, [0.02, 1.0][i % 2], dtype, 40 + i)
        sel = H.selected_lane(raw, spec)
        if spec.exponent_stream is not None and i % 2:
            lengths, vocab = H.mixed_book_for(sel)
            book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
        else:
            header, _ = _native.huff0_build(np.bincount(sel, minlength=256) * 64 + 1, 12)
            lengths, values, _, _ = _native.huff0_read(header)
            book = GPUCodebook(tuple(lengths), values)
        out = torch.full((numel,), -1, dtype=torch.int16 if spec.element_size == 2 else torch.int32,
                         device="cuda").view(dtype)
        groups.append(_device_group(raw, spec, book, out, arena, lut_index=i))
        expected.append(raw)
    prepared = decoder.prepare_batch(groups)
    decoder.decode_batch(prepared)
    torch.cuda.synchronize()
    for g, raw in zip(groups, expected):
        assert bytes(g.output.cpu().view(torch.uint8).numpy()) == raw
    decoder.check_status(prepared)


def test_one_launch_mixes_layouts():
    """bf16, fp16 and fp32 groups (singleton, mixed and raw) in one batch:
    one launch, each CTA runs its own layout."""
    decoder = gpu_decoder.default_decoder()
    arena, groups, expected = [], [], []
    index = 0
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        spec = DTYPES[dtype]
        for numel, sigma in ((3 * 8192 + 11, 0.02), (131072, 1.0)):
            raw = H.gaussian_raw(numel, sigma, dtype, 60 + index)
            sel = H.selected_lane(raw, spec)
            if spec.exponent_stream is not None and sigma > 0.5:
                lengths, vocab = H.mixed_book_for(sel)
                book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
            else:
                header, _ = _native.huff0_build(np.bincount(sel, minlength=256) + 1, 12)
                lengths, values, _, _ = _native.huff0_read(header)
                book = GPUCodebook(tuple(lengths), values)
            out = torch.full((numel,), -1, dtype=torch.int16 if spec.element_size == 2 else torch.int32,
                             device="cuda").view(dtype)
            groups.append(_device_group(raw, spec, book, out, arena, lut_index=index))
            expected.append(raw)
            index += 1
    prepared = decoder.prepare_batch(groups)
    assert prepared.layout == (_native.LAYOUT_BF16, _native.LAYOUT_FP16, _native.LAYOUT_FP32)
    decoder.decode_batch(prepared)
    torch.cuda.synchronize()
    for g, raw in zip(groups, expected):
        assert bytes(g.output.cpu().view(torch.uint8).numpy()) == raw
    decoder.check_status(prepared)


def test_config1_single_tensor_singleton():
    """BASELINE config 1 on the GPU: 128 singleton-coded chunks of one
    4096x4096 bf16 tensor decode bit-exactly through the runtime."""
    from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_tensors_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    g = torch.Generator().manual_seed(0)
    named = {"w": (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.bfloat16)}
    setup = NeuralZipSetup(chunk_size=256 << 10, cluster_js_threshold=0.05, enable_packed_codebooks=False).build(named)
    export = export_tensors_for_gpu(named, setup)
    runtime = NeuralZipRuntime(None, export, "cuda:0")
    runtime.workspaces[torch.bfloat16].view(torch.uint8).fill_(0xA5)
    got = dict(runtime.materialized_weights())["w"]
    assert torch.equal(got.reshape(-1).view(torch.uint8), named["w"].reshape(-1).view(torch.uint8))
    runtime.check_status()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_same_process_decodes_on_two_devices():
    """The kernel's shared-memory opt-in belongs to each device's context:
    one process decodes the same tensors on cuda:0 and on cuda:1, with the
    24-warp (232 KB) CTAs on both."""
    from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_tensors_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    g = torch.Generator().manual_seed(3)
    named = {f"w{i}": (torch.randn(1024, 8192, generator=g) * 0.02).to(torch.bfloat16) for i in range(20)}
    export = export_tensors_for_gpu(named, NeuralZipSetup().build(named))
    for device in ("cuda:0", "cuda:1"):
        runtime = NeuralZipRuntime(None, export, device)
        batch = runtime._prepared_batches[export.block_order[0]][0]
        assert batch.warps_per_cta == 24
        runtime.workspaces[torch.bfloat16].view(torch.uint8).fill_(0xA5)
        got = dict(runtime.materialized_weights())
        for name, tensor in named.items():
            assert torch.equal(got[name].reshape(-1).view(torch.uint8), tensor.reshape(-1).view(torch.uint8))
        runtime.check_status()
