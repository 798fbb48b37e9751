"""GPU decoder host: prepares tile-decode launches and enqueues them.

Same protocol as neuralzip/gpu/decoder.py (CuPyDecoder): ``default_decoder()``
returns a process-wide decoder with ``prepare_group(device_index, group)``,
``prepare_batch(groups) -> PreparedBatch`` and ``decode_batch(prepared)``,
which launches on the torch current stream and returns the outputs
(decoder.py:121-208). ``_DECODER`` may be replaced (tests do), and
``shared_memory_bytes`` / ``KERNEL_PATH`` exist as in the reference.

What differs is the device side. There is no NVRTC compilation: the sm_100a
kernel is prebuilt in libnzb200.so and reached through the C ABI
(``nz_decode_launch``). One launch covers every group of one dtype,
whatever its codebook (singleton, mixed, long codes, raw), so a block needs
one launch per dtype instead of one per (layout, staging) combination. The
launch geometry is a list of (group, tile) works cut into CTAs that share a
decode table; ``staging_policy`` (warps per CTA, works per CTA of each
table) can be overridden the way the reference's tests override
``_staging``.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from neuralzip_b200 import _native

KERNEL_PATH = Path(__file__).resolve().parent.parent / "csrc" / "nz_decode.cu"
WARPS_PER_CTA = 24
# CTA widths the launch plan picks from, widest first (the kernel's
# instantiations: 24- and 16-warp CTAs fill an SM alone, 8- and 4-warp CTAs
# run two and three to an SM; narrower ones give each warp a larger copy of
# its tile's bitstream).
CTA_WIDTHS = (24, 16, 8, 4)
SM_COUNT_DEFAULT = 148
# Cost of a coded tile relative to a pair-coded bf16 tile (measured on
# config 2: fp16 bytes are singleton-coded, fewer bytes per lookup; fp32
# tiles move twice the bytes). A raw tile (no Huffman decode) costs about a
# quarter.
WORK_WEIGHT = {_native.LAYOUT_BF16: 1.0, _native.LAYOUT_FP16: 2.0, _native.LAYOUT_FP32: 2.0}
RAW_WORK_WEIGHT = 4


def shared_memory_bytes(warps_per_cta=WARPS_PER_CTA, max_elements=None):
    """Dynamic shared memory of one decode CTA (decode table + warp staging).

    ``max_elements`` is accepted for signature compatibility with the
    reference (decoder.py:53-54); the tile kernel's footprint does not grow
    with the group size."""
    del max_elements
    return _native.decode_smem_bytes(warps_per_cta)


def _layout_of(spec):
    return _native.layout_code(spec.element_size, spec.bit_reorder, spec.mantissa_bits, spec.exponent_bits,
                               spec.gpu_stream)


@dataclass(frozen=True)
class DeviceGroup:
    """Device addresses of one uploaded group (what a launch descriptor needs)."""

    spec: object            # DTypeSpec
    numel: int
    lut_index: int          # row in the decode-table tensor, or _native.RAW_LUT
    lut_ptr: int            # device address of that row (0 for raw)
    lut_words: int
    bits: int
    lens: int
    tile_off: int
    lanes: tuple            # 4 device addresses (0 where unused)
    out: int
    output: torch.Tensor = field(repr=False, compare=False)
    tile_words: int = 0     # largest per-tile bitstream copy (tile_copy_words)

    @property
    def tiles(self):
        return (self.numel + _native.TILE_ELEMS - 1) // _native.TILE_ELEMS


def tile_copy_words(tile_offsets, bit_length):
    """Largest shared-memory copy of one tile's bitstream, in words: from
    the 16-byte boundary at or below its first bit through the word 12 to
    15 past the word of its last bit (what the kernel copies)."""
    starts = np.asarray(tile_offsets, dtype=np.int64)
    if not len(starts):
        return 0
    ends = np.append(starts[1:], int(bit_length))
    return int(((((ends >> 5) + 16) & ~3) - ((starts >> 5) & ~3)).max())


@dataclass(frozen=True)
class PreparedBatch:
    descriptor_tensors: tuple = field(repr=False)
    device: torch.device
    layout: tuple
    warps_per_cta: int
    shared_memory: int
    kernel_grid: tuple
    launch: object = field(repr=False)
    outputs: tuple = field(repr=False)
    status: torch.Tensor = field(repr=False)
    works: int = 0
    elements: int = 0


class TileDecoder:
    """Host side of the sm_100a tile decode kernel."""

    # Whether the CTAs of one (layout, table) key share its works through a
    # queue counter in launch scratch (they then finish together: on config
    # 2 the bf16 launch takes 0.698 ms against 0.727 ms with a fixed range
    # per CTA), or each CTA takes a fixed range (no scratch).
    work_queues = True

    def __init__(self):
        self._sm_count = {}
        self._ctas_per_sm = {}
        self._copy_words = {}

    # Reference hook: the staging policy decides the launch geometry.
    def staging_policy(self, device_index, key_works, tile_words=0):
        """Launch geometry for a batch with ``key_works[key] = (tiles,
        layout, raw)`` per (layout, decode table): (warps per CTA,
        {key: CTAs}).

        Every CTA stages one table and runs one layout; its warps take the
        CTA's works in turn, so they get equal counts (+-1). Tiles are
        weighed by their cost relative to a pair-coded bf16 tile
        (WORK_WEIGHT, RAW_WORK_WEIGHT), and every resident CTA slot of one
        wave gets a share of the cost: a launch then ends when its busiest
        warps do, with no partial last wave and no idle SM. A launch with fewer tiles than one
        24-warp CTA per SM uses narrower CTAs so that every SM gets work
        (a 24-warp CTA fills an SM's shared memory with the 38 KB table and
        each warp's staging rows and tile-bitstream copy; 8- and 4-warp CTAs
        run two and three to an SM, 16 and 12 warps). Widths whose
        per-warp bitstream copy is smaller than the batch's largest tile
        (``tile_words``) are skipped: such a tile would be read from global
        memory, several times slower."""
        sms = self._sms(device_index)
        total = sum(n for n, _, _ in key_works.values())
        fits = [w for w in CTA_WIDTHS if tile_words <= self._tile_words(w)] or list(CTA_WIDTHS)
        nw = next((w for w in fits if total >= sms * w), fits[-1])
        slots = self._occupancy(device_index, nw) * sms

        def weight(layout, raw):
            """Cost of one tile relative to a pair-coded bf16 tile."""
            return WORK_WEIGHT[layout] * (1.0 / RAW_WORK_WEIGHT if raw else 1.0)

        # One CTA per key, then each free slot of the wave to the key whose
        # CTAs carry the most cost each (while it has a tile left for it):
        # every SM gets a share and the shares are as even as whole tiles
        # allow; a CTA's warps then take its works in turn (+-1 each).
        cost = {key: n * weight(layout, raw) for key, (n, layout, raw) in key_works.items()}
        alloc = {key: 1 for key in key_works}
        for _ in range(slots - len(alloc)):
            open_keys = [key for key in alloc if alloc[key] < key_works[key][0]]
            if not open_keys:
                break
            key = max(open_keys, key=lambda k: cost[k] / alloc[k])
            alloc[key] += 1
        return nw, alloc

    def _tile_words(self, nw):
        if nw not in self._copy_words:
            self._copy_words[nw] = _native.decode_tile_words(nw)
        return self._copy_words[nw]

    def _occupancy(self, device_index, nw):
        """Resident CTAs per SM (CUDA occupancy calculator; shared memory
        allows 1, 1, 2 and 3 CTAs of 24, 16, 8 and 4 warps on a B200)."""
        key = (device_index, nw)
        if key not in self._ctas_per_sm:
            fallback = {24: 1, 16: 1, 8: 2, 4: 3}[nw]
            try:
                with torch.cuda.device(device_index):
                    self._ctas_per_sm[key] = _native.decode_occupancy(nw) or fallback
            except (RuntimeError, AssertionError, TypeError):
                self._ctas_per_sm[key] = fallback
        return self._ctas_per_sm[key]

    def _sms(self, device_index):
        if device_index not in self._sm_count:
            try:
                self._sm_count[device_index] = torch.cuda.get_device_properties(device_index).multi_processor_count
            except (RuntimeError, AssertionError):
                self._sm_count[device_index] = SM_COUNT_DEFAULT
        return self._sm_count[device_index]

    def prepare_group(self, device_index, group):
        """Validates a GPUWeightGroup before any weight is removed
        (neuralzip/gpu/decoder.py:121-128): the dtype must have a tile
        kernel and the codebook a decode table."""
        _native.load()
        if _layout_of(group.encoded.dtype) is None:
            raise ValueError("The GPU decoder has no kernel for this dtype layout.")
        if group.codebook.max_bits and group.codebook.decode_lut is None:
            raise ValueError("The GPU codebook has no decode table.")
        return shared_memory_bytes()

    def prepare_batch(self, groups):
        """Builds the device descriptors of one launch over DeviceGroups of
        any mix of dtypes (neuralzip/gpu/decoder.py:130-191)."""
        groups = tuple(groups)
        if not groups:
            raise ValueError("A decode batch must contain at least one group.")
        device = groups[0].output.device
        if device.type != "cuda" or any(g.output.device != device for g in groups):
            raise ValueError("A decode batch must use one CUDA device.")
        layouts = [_layout_of(g.spec) for g in groups]
        if any(code is None for code in layouts):
            raise ValueError("The GPU decoder has no kernel for this dtype layout.")
        table = np.zeros(len(groups), dtype=_native.GROUP_DTYPE)
        for g in groups:
            if g.lut_index != _native.RAW_LUT and (g.bits % 16 or g.lut_ptr % 16):
                raise ValueError("Bitstreams and decode tables must be 16-byte aligned.")
        for i, g in enumerate(groups):
            table[i] = (g.bits, g.lens, g.tile_off, g.lanes, g.out, g.numel, g.lut_index)
        lut_ids = sorted({g.lut_index for g in groups if g.lut_index != _native.RAW_LUT})
        lut_slot = {lut: i for i, lut in enumerate(lut_ids)}
        lut_ptrs = np.array([next(g.lut_ptr for g in groups if g.lut_index == lut) for lut in lut_ids],
                            dtype=np.uint64)
        lut_words = {g.lut_index: g.lut_words for g in groups}
        for i, g in enumerate(groups):
            table[i]["lut"] = _native.RAW_LUT if g.lut_index == _native.RAW_LUT else lut_slot[g.lut_index]
        # Works sorted by (layout, decode table): each CTA stages one table
        # and runs one layout.
        keys = sorted({(layouts[i], g.lut_index) for i, g in enumerate(groups)})
        members = {key: [i for i, g in enumerate(groups) if (layouts[i], g.lut_index) == key] for key in keys}
        key_works = {key: (sum(groups[i].tiles for i in members[key]), key[0], key[1] == _native.RAW_LUT)
                     for key in keys}
        total_works = sum(n for n, _, _ in key_works.values())
        tile_words = max((g.tile_words for g in groups if g.lut_index != _native.RAW_LUT), default=0)
        nw, key_ctas = self.staging_policy(device.index, key_works, tile_words)
        works = np.zeros(total_works, dtype=_native.WORK_DTYPE)
        ctas = []
        cursor = 0
        for queue, key in enumerate(keys):
            layout, lut = key
            begin = cursor
            for i in members[key]:
                n = groups[i].tiles
                works["group"][cursor:cursor + n] = i
                works["tile"][cursor:cursor + n] = np.arange(n, dtype=np.uint32)
                cursor += n
            slot = _native.RAW_LUT if lut == _native.RAW_LUT else lut_slot[lut]
            words = 0 if lut == _native.RAW_LUT else lut_words[lut]
            n_ctas = max(1, int(key_ctas[key]))
            if self.work_queues:
                # The key's CTAs share its range through one queue counter.
                ctas.extend((slot, begin, cursor, words, layout, queue, 0) for _ in range(n_ctas))
            else:
                step = -(-(cursor - begin) // n_ctas)
                for start in range(begin, cursor, step):
                    ctas.append((slot, start, min(cursor, start + step), words, layout, 0, 0))
        cta_array = np.array(ctas, dtype=_native.CTA_DTYPE)
        if not len(lut_ptrs):
            lut_ptrs = np.zeros(1, dtype=np.uint64)
        tensors = tuple(
            torch.from_numpy(a.view(np.uint8).copy()).to(device)
            for a in (table, works, cta_array, lut_ptrs)
        )
        status = torch.zeros(1, dtype=torch.int32, device=device)
        launch = _native.Launch()
        launch.warps_per_cta = nw
        launch.groups, launch.works, launch.ctas, launch.luts = (t.data_ptr() for t in tensors)
        launch.status = status.data_ptr()
        launch.n_ctas = len(cta_array)
        if self.work_queues:
            # One counter per key plus the launch's finished-CTA count; the
            # kernel sets them back to zero at the end of each launch.
            scratch = torch.zeros(len(keys) + 1, dtype=torch.int32, device=device)
            tensors = tensors + (scratch,)
            launch.scratch, launch.queues = scratch.data_ptr(), len(keys)
        return PreparedBatch(
            descriptor_tensors=tensors, device=device, layout=tuple(sorted(set(layouts))), warps_per_cta=nw,
            shared_memory=shared_memory_bytes(nw), kernel_grid=(len(cta_array),), launch=launch,
            outputs=tuple(g.output for g in groups), status=status, works=total_works,
            elements=sum(g.numel for g in groups),
        )

    def decode_batches(self, batches, stream=None):
        """Enqueues several prepared batches (e.g. one per dtype of a block)
        as one step on `stream`: the largest alone on the stream, then the
        others side by side on the library's side streams, joined back
        (nz_decode_launch_many)."""
        batches = tuple(batches)
        if not batches:
            return ()
        if stream is None:
            stream = torch.cuda.current_stream(device=batches[0].device)
        if len(batches) == 1:
            _native.decode_launch(batches[0].launch, stream.cuda_stream)
        else:
            _native.decode_launch_many([b.launch for b in batches], stream.cuda_stream)
        return tuple(out for b in batches for out in b.outputs)

    def decode_batch(self, prepared, stream=None):
        """Enqueues the decode on `stream` (default: torch's current stream)."""
        if stream is None:
            stream = torch.cuda.current_stream(device=prepared.device)
        _native.decode_launch(prepared.launch, stream.cuda_stream)
        return prepared.outputs

    @staticmethod
    def check_status(prepared):
        """Raises if a launch of this batch reported an error: a corrupt
        decode table (2), an unknown element layout (3), a work-queue index
        out of range (4) or a decode-table copy that did not complete (5)."""
        code = int(prepared.status.item())
        if code:
            what = {2: "corrupt decode table", 3: "unknown element layout", 4: "work-queue index out of range",
                    5: "decode-table copy did not complete"}
            raise RuntimeError(f"The GPU decoder reported status {code} ({what.get(code, 'unknown error')}).")


_DECODER = TileDecoder()


def default_decoder():
    return _DECODER
