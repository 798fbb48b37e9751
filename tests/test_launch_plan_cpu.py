"""CPU checks of the decode launch plan (TileDecoder.staging_policy): the
CTA width it picks and how it spreads one wave of CTAs over the (layout,
decode table) keys of a launch. No GPU: the SM count and the resident CTAs
per SM are given, as a B200 reports them (148 SMs; 1, 1, 2, 3 CTAs of 24,
16, 8, 4 warps)."""

import pytest

from neuralzip_b200 import _native
from neuralzip_b200.gpu.decoder import TileDecoder

BF16, FP16, FP32 = _native.LAYOUT_BF16, _native.LAYOUT_FP16, _native.LAYOUT_FP32


def _decoder():
    d = TileDecoder()
    d._sm_count[0] = 148
    d._ctas_per_sm.update({(0, 24): 1, (0, 16): 1, (0, 8): 2, (0, 4): 3})
    return d


def _plan(key_tiles, tile_words=0):
    key_works = {key: (n, key[0], False) for key, n in key_tiles.items()}
    return _decoder().staging_policy(0, key_works, tile_words)


def test_config2_sized_launch_fills_every_sm_evenly():
    tiles = {(BF16, 0): 33000, (BF16, 1): 32500, (BF16, 2): 32800, (BF16, 3): 32772}
    nw, ctas = _plan(tiles, tile_words=900)
    assert nw == 24
    assert sum(ctas.values()) == 148
    per_cta = [tiles[k] / ctas[k] for k in tiles]
    assert max(per_cta) - min(per_cta) <= max(per_cta) / min(ctas.values())  # within one CTA's share


def test_tiles_larger_than_the_24_warp_copy_take_16_warp_ctas():
    assert _native.decode_tile_words(24) < 1300 <= _native.decode_tile_words(16)
    nw, ctas = _plan({(FP16, 0): 2048, (FP32, 1): 2048}, tile_words=1300)
    assert nw == 16 and sum(ctas.values()) == 148


def test_small_launches_narrow_their_ctas():
    nw, ctas = _plan({(BF16, 0): 600})  # fewer tiles than one 8-warp CTA per SM
    assert nw == 4 and sum(ctas.values()) == 148 * 3
    nw, ctas = _plan({(BF16, 0): 5})
    assert nw == 4 and ctas == {(BF16, 0): 5}  # never more CTAs than tiles


def test_more_keys_than_slots_get_one_cta_each():
    tiles = {(BF16, k): 10 for k in range(400)}  # 400 keys, 148 slots of 24 warps
    nw, ctas = _plan(tiles)
    assert nw == 24 and set(ctas.values()) == {1} and len(ctas) == 400


@pytest.mark.parametrize("weight_layout", [FP16, FP32])
def test_costlier_tiles_get_more_ctas(weight_layout):
    # fp16 and fp32 tiles weigh twice a bf16 tile: equal tile counts, twice the CTAs.
    nw, ctas = _plan({(BF16, 0): 14800, (weight_layout, 1): 14800})
    assert abs(ctas[(weight_layout, 1)] - 2 * ctas[(BF16, 0)]) <= 2


def _export(block_bytes):
    """A stand-in export: one bf16 group per block with `bytes` of output."""
    from types import SimpleNamespace

    groups = [SimpleNamespace(block_name=name, encoded=SimpleNamespace(numel=size // 2,
                                                                       dtype=SimpleNamespace(element_size=2)))
              for name, size in block_bytes.items()]
    return SimpleNamespace(block_order=tuple(block_bytes), groups=groups)


def test_auto_units_fill_small_blocks_up_to_the_floor():
    from neuralzip_b200.gpu.inference import AUTO_UNIT_BYTES, _plan_units

    layer = 30 << 20  # a Qwen2.5-0.5B decoder layer: 8 fit in 256 MiB
    export = _export({f"layers.{i}": layer for i in range(24)})
    units = _plan_units(export, "auto")
    assert [len(u) for u in units] == [8] * 3 and AUTO_UNIT_BYTES == 256 << 20
    assert [b for u in units for b in u] == list(export.block_order)


def test_auto_units_keep_the_largest_block_as_the_limit_when_larger():
    from neuralzip_b200.gpu.inference import _plan_units

    # Llama-3-8B: 436 MB layers and a 1.05 GB LM head: two layers a unit.
    blocks = {f"layers.{i}": 436 << 20 for i in range(4)}
    blocks["lm_head"] = 1050 << 20
    units = _plan_units(_export(blocks), "auto")
    assert units == [("layers.0", "layers.1"), ("layers.2", "layers.3"), ("lm_head",)]
    assert _plan_units(_export(blocks), 1) == [(b,) for b in blocks]
