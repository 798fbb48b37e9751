"""The allocation-free decode launch, nz_decode_launch_noalloc (B200).

Some callers cannot allocate device memory: a plugin running inside a
serving process whose memory pool has already reserved all of HBM, or a host
path that must not call cudaMalloc because cudaMalloc may synchronize the
device. For them the library keeps the decode's work-queue counters in its
own device memory, and this entry point uses those instead of a scratch
buffer from the caller. These tests drive it through the C ABI, several
times in a row on a stream of the caller's, with batches of one and of three
work queues, and compare its output with the regular launch's, bit for bit (integer
work: the tolerance is zero, as in every other decode test).

The file is named to be collected last, so that a run stopping at the
first failure has run every other test before it.
"""

import numpy as np
import pytest
import torch

import helpers as H
from neuralzip_b200 import _native
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu import decoder as gpu_decoder
from neuralzip_b200.gpu.inference import GPUCodebook, encode_with_codebook
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _upload(raw, spec, book, out, keep, lut_index):
    """One group in device memory (bitstream, lengths, tile offsets, raw
    lanes, decode table) as a DeviceGroup."""
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
        keep.append(t)
        addr[name] = t.data_ptr()
    lut = torch.from_numpy(np.asarray(book.decode_lut, dtype=np.uint32).view(np.int32)).to("cuda")
    keep.append(lut)
    return gpu_decoder.DeviceGroup(
        spec=spec, numel=enc.numel, lut_index=lut_index, lut_ptr=lut.data_ptr(), lut_words=book.table_words,
        bits=addr["bits"], lens=addr["lens"], tile_off=addr["tile_off"],
        lanes=tuple(addr.get(f"lane{lane}", 0) for lane in range(4)), out=out.data_ptr(), output=out,
        tile_words=gpu_decoder.tile_copy_words(sym.tile_offsets, sym.bit_length))


def test_noalloc_launch_matches_regular_launch():
    spec = DTYPES[torch.bfloat16]
    decoder = gpu_decoder.TileDecoder()
    decoder.work_queues = True  # the CTAs of each table share one work queue
    keep, outs, raws, groups = [], [], [], []
    for seed, sigma in enumerate((0.02, 0.3, 0.004)):
        numel = (6 + seed) * 8192 + 123 * seed
        raw = H.gaussian_raw(numel, sigma, torch.bfloat16, 40 + seed)
        lengths, vocab = H.mixed_book_for(H.selected_lane(raw, spec))
        book = GPUCodebook(tuple(lengths), tuple(int(v) for v in O.mixed_codes(lengths)), vocab)
        out = torch.empty(numel, dtype=torch.bfloat16, device="cuda")
        groups.append(_upload(raw, spec, book, out, keep, seed))
        outs.append(out)
        raws.append(raw)
    batch = decoder.prepare_batch(groups)
    assert batch.launch.queues == 3
    stream = torch.cuda.current_stream()

    # The regular launch, with the batch's own scratch buffer.
    decoder.decode_batch(batch, stream)
    torch.cuda.synchronize()
    decoder.check_status(batch)
    expected = [out.clone() for out in outs]
    for out, raw in zip(expected, raws):
        assert bytes(out.cpu().view(torch.uint8).numpy()) == raw

    # Allocation-free launches on a stream of the caller's own (the first
    # one in the process also sets up the library's counters), alternating
    # between a one-queue batch and the three-queue batch: each launch finds
    # every counter it uses, including the finished-CTA count at index
    # `queues`, set back to zero by the launch before it.
    single = decoder.prepare_batch(groups[:1])
    assert single.launch.queues == 1
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for current in (single, batch, single, batch):
            for out in outs:
                out.view(torch.int16).fill_(-1)
            _native.decode_launch_noalloc(current.launch, side.cuda_stream)
            side.synchronize()
            decoder.check_status(current)
            decoded = outs[:1] if current is single else outs
            for out, ref in zip(decoded, expected):
                assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
            for out in outs[len(decoded):]:
                assert bool((out.view(torch.int16) == -1).all())


def test_noalloc_launch_rejects_too_many_queues():
    launch = _native.Launch()
    launch.warps_per_cta = 24
    launch.n_ctas = 1
    launch.groups = launch.works = launch.ctas = launch.luts = 1
    launch.queues = 1025
    with pytest.raises(ValueError, match="at most 1024"):
        _native.decode_launch_noalloc(launch, 0)
