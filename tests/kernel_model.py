"""Step-for-step CPU model of the tile decode kernel's lane loop.

Test helper: it runs the same per-lane algorithm as nz_tile_decode in
neuralzip_b200/csrc/nz_decode.cu over the decode table produced by the
product (nz_codebook_lut): 12-bit lookups of two-word entries (metadata
with the code length in bits 0..4 and eight times the byte count in bits
8..15, and up to four bytes), codes longer than 12 bits through the
canonical limit/offset/leaf tables or the suffix-tree walk, a one-word byte queue whose overflow is
rebuilt from the entry when a word is stored, 128-element staging rounds, and
only the staged prefix of the table (rounded up to 16 bytes) visible, so
table, staging and loop errors show up on a CPU. Expected bytes always come
from the oracle, never from this model.
"""

import numpy as np

LANE, LANES, TILE = 256, 32, 8192
ROUND = 128
LUT_ENTRIES = 4096
LUT_CANON = 2 * LUT_ENTRIES
LUT_TREE = LUT_CANON + 64 + 512
MASK64 = (1 << 64) - 1


class _Window:
    """hi:lo as one 64-bit integer; valid bits are the top `avail` bits."""

    def __init__(self, words, bitpos):
        # Same loads as the kernel: two words into the window and the next
        # one requested ahead, so an out-of-range read raises IndexError here.
        self.words = words
        p = bitpos >> 5
        sh = bitpos & 31
        self.buf = (((int(words[p]) << 32) | int(words[p + 1])) << sh) & MASK64
        self.avail = 64 - sh
        self.pf = int(words[p + 2])
        self.ptr = p + 3

    def consume(self, n):
        n &= 31
        self.buf = (self.buf << n) & MASK64
        self.avail -= n

    def top_up(self):
        if self.avail <= 32:
            self.buf |= (self.pf << 32) >> self.avail
            self.avail += 32
            self.pf = int(self.words[self.ptr])
            self.ptr += 1


def staged_table(lut, lut_words):
    """What a CTA holds in shared memory: the first lut_words words rounded
    up to 16 bytes, zeros after."""
    staged = np.zeros(len(lut), dtype=np.uint32)
    n = min(len(lut), (int(lut_words) + 3) // 4 * 4)
    staged[:n] = lut[:n]
    return staged


def decode_group(lut, bits, lens, tile_off, numel, lut_words=None):
    """Selected-lane bytes of one coded group, as the kernel computes them."""
    table = staged_table(np.asarray(lut, dtype=np.uint32), len(lut) if lut_words is None else lut_words)
    out = np.zeros(numel, dtype=np.uint8)
    for tile in range(len(tile_off)):
        lens_t = [int(x) for x in lens[tile * LANES:(tile + 1) * LANES]]
        for lane in range(LANES):
            first = (tile * LANES + lane) * LANE
            n_lane = min(LANE, numel - first) if first < numel else 0
            win = _Window(bits, int(tile_off[tile]) + sum(lens_t[:lane]))
            qa, qbits = 0, 0
            for r in range(LANE // ROUND):
                done = r * ROUND
                want = min(ROUND, n_lane - done) if n_lane > done else 0
                target = (want + 3) >> 2
                staged = bytearray()
                while len(staged) < 4 * target:
                    k = win.buf >> 52
                    e, x = int(table[2 * k]), int(table[2 * k + 1])
                    if (e & 0xFF00) == 0 and e >> 31:
                        win.consume(12)
                        node = (e >> 16) & 511
                        for _ in range(44):
                            win.top_up()
                            bit = win.buf >> 63
                            win.consume(1)
                            child = int(table[LUT_TREE + 2 * node + bit])
                            if child & 0xE0:
                                e = ((child >> 5) & 7) << 11
                                x = child >> 8
                                break
                            node = (child >> 8) & 511
                        else:
                            raise AssertionError("suffix walk exceeded 44 steps")
                    elif (e & 0xFF00) == 0:
                        # canonical long code: limits, rank offsets, leaf words
                        w32 = win.buf >> 32
                        length = max((e >> 16) & 31, 13)
                        while w32 > int(table[LUT_CANON + length]) and length < 31:
                            length += 1
                        assert w32 <= int(table[LUT_CANON + length]), "window beyond the last canonical limit"
                        rank = (int(table[LUT_CANON + 32 + length]) + (w32 >> (32 - length))) & 0xFFFFFFFF
                        assert rank < 512, "canonical rank out of range"
                        leaf = int(table[LUT_CANON + 64 + rank])
                        assert leaf & 0xE0, "empty canonical leaf"
                        win.consume(length)
                        e = ((leaf >> 5) & 7) << 11
                        x = leaf >> 8
                    win.consume(e)
                    win.top_up()
                    qa = (qa | (x << qbits)) & 0xFFFFFFFF
                    qn = qbits + (e >> 8)
                    assert qn < 64, "entry byte count out of range"
                    if qn >= 32:
                        staged += qa.to_bytes(4, "little")
                        qa = (x >> (32 - qbits)) if qbits else 0
                    qbits = qn & 31
                if want:
                    out[first + done:first + done + want] = np.frombuffer(bytes(staged), dtype=np.uint8)[:want]
            # Every word the lane read lies in the tile's shared-memory copy:
            # from the 16-byte boundary at or below the tile's first bit
            # through 12..15 words past the word of its last bit.
            start, end = int(tile_off[tile]), int(tile_off[tile]) + sum(lens_t)
            wa, wb = (start >> 5) & ~3, ((end >> 5) + 16) & ~3
            assert wa <= (int(tile_off[tile]) + sum(lens_t[:lane])) >> 5 and win.ptr <= wb, \
                f"lane {lane} of tile {tile} read word {win.ptr - 1} outside the copy [{wa}, {wb})"
    return out


def byte_perm(a, b, sel):
    """__byte_perm: byte i of the result is byte (sel >> 4i) & 7 of b:a."""
    src = (int(b) << 32) | int(a)
    return sum(((src >> (8 * ((sel >> (4 * i)) & 7))) & 0xFF) << (8 * i) for i in range(4))


def bsel(a, b, m):
    return (a & m) | (b & ~m & 0xFFFFFFFF)


def merge_bf16_words(raw, exp):
    """Two output words (4 bf16 elements) from 4 raw bytes (sign|mant7) and
    4 decoded exponent bytes, as the kernel's store8 forms them."""
    hi = bsel(raw, exp >> 1, 0x80808080)
    lo = bsel(raw, (exp << 7) & 0xFFFFFFFF, 0x7F7F7F7F)
    return byte_perm(lo, hi, 0x5140), byte_perm(lo, hi, 0x7362)


def merge_fp32_words(a, b, c, exp):
    """Four fp32 words from raw lanes a, b, c and decoded exponents (store4)."""
    hi = bsel(c, exp >> 1, 0x80808080)
    mid = bsel(c, (exp << 7) & 0xFFFFFFFF, 0x7F7F7F7F)
    t0, t1 = byte_perm(a, b, 0x5140), byte_perm(a, b, 0x7362)
    t2, t3 = byte_perm(mid, hi, 0x5140), byte_perm(mid, hi, 0x7362)
    return (byte_perm(t0, t2, 0x5410), byte_perm(t0, t2, 0x7632), byte_perm(t1, t3, 0x5410),
            byte_perm(t1, t3, 0x7632))
