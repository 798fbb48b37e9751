"""Step-for-step CPU model of the tile decode kernel's lane loop.

Test helper: it runs the same per-lane algorithm as nz_tile_decode in
neuralzip_b200/csrc/nz_decode.cu over the decode table produced by the
product (nz_codebook_lut): 12-bit lookups of two-word entries (metadata
whose low five bits are the shift amount, and up to four bytes), the suffix-tree walk for codes longer than 12
bits, a byte queue flushed as 32-bit words, 128-element staging rounds, and
only the staged prefix of the table (rounded up to 16 bytes) visible, so
table, staging and loop errors show up on a CPU. Expected bytes always come
from the oracle, never from this model.
"""

import numpy as np

LANE, LANES, TILE = 256, 32, 8192
ROUND = 128
LUT_ENTRIES = 4096
LUT_TREE = 2 * LUT_ENTRIES
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
            queue, qbits = 0, 0
            for r in range(LANE // ROUND):
                done = r * ROUND
                want = min(ROUND, n_lane - done) if n_lane > done else 0
                target = (want + 3) >> 2
                staged = bytearray()
                while len(staged) < 4 * target:
                    k = win.buf >> 52
                    e, x = int(table[2 * k]), int(table[2 * k + 1])
                    if (e & 0xE0) == 0:
                        win.consume(12)
                        node = (e >> 8) & 511
                        for _ in range(44):
                            win.top_up()
                            bit = win.buf >> 63
                            win.consume(1)
                            child = int(table[LUT_TREE + 2 * node + bit])
                            if child & 0xE0:
                                e = child & ~0x1F
                                x = e >> 8
                                break
                            node = (child >> 8) & 511
                        else:
                            raise AssertionError("suffix walk exceeded 44 steps")
                    win.consume(e)
                    win.top_up()
                    queue |= x << qbits
                    qbits += ((e >> 5) & 7) * 8
                    if qbits >= 32:
                        staged += (queue & 0xFFFFFFFF).to_bytes(4, "little")
                        queue >>= 32
                        qbits -= 32
                if want:
                    out[first + done:first + done + want] = np.frombuffer(bytes(staged), dtype=np.uint8)[:want]
    return out
