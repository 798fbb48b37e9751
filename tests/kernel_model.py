"""Step-for-step CPU model of the tile decode kernel's lane loop.

Test helper: it runs the same per-lane algorithm as nz_tile_decode in
neuralzip_b200/csrc/nz_decode.cu (12-bit multi-byte table lookups, the
suffix-tree walk for long codes, the byte queue flushed as 32-bit words,
64-element staging rounds) over the decode table produced by the product
(nz_codebook_lut), so table/loop logic errors show up on a CPU. The
expected bytes come from the oracle, never from this model.
"""

import numpy as np

LANE, LANES, TILE = 256, 32, 8192
ROUND = 64


class _Reader:
    def __init__(self, words, bitpos):
        self.words = words
        p = bitpos >> 5
        sh = bitpos & 31
        w = (int(words[p]) << 32) | int(words[p + 1])
        self.buf = (w << sh) & ((1 << 64) - 1)
        self.nvalid = 64 - sh
        self.ptr = p + 2

    def refill(self):
        self.buf |= int(self.words[self.ptr]) << (32 - self.nvalid)
        self.nvalid += 32
        self.ptr += 1

    def consume(self, n):
        self.buf = (self.buf << n) & ((1 << 64) - 1)
        self.nvalid -= n


def decode_group(lut, bits, lens, tile_off, numel):
    """Selected-lane bytes of one coded group, as the kernel computes them."""
    out = np.zeros(numel, dtype=np.uint8)
    n_tiles = len(tile_off)
    for tile in range(n_tiles):
        lens_t = [int(x) for x in lens[tile * LANES:(tile + 1) * LANES]]
        for lane in range(LANES):
            s = tile * LANES + lane
            first = s * LANE
            n_lane = min(LANE, numel - first) if first < numel else 0
            start = int(tile_off[tile]) + sum(lens_t[:lane])
            br = _Reader(bits, start)
            q, qn, pushed = 0, 0, 0
            staged = bytearray()
            for r in range(LANE // ROUND):
                done = r * ROUND
                want = min(ROUND, n_lane - done) if n_lane > done else 0
                target = (want + 3) >> 2
                wi = 0
                while wi < target:
                    if pushed < n_lane:
                        e = int(lut[br.buf >> 52])
                        nbits = (e >> 24) & 15
                        if (e >> 28) == 0:
                            br.consume(12)
                            node = e & 511
                            for _ in range(44):
                                if br.nvalid <= 32:
                                    br.refill()
                                bit = br.buf >> 63
                                br.consume(1)
                                child = int(lut[4096 + 2 * node + bit])
                                if child >> 28:
                                    e = child
                                    break
                                node = child & 511
                            else:
                                raise AssertionError("suffix walk exceeded 44 steps")
                            nbits = 0
                        nb = (e >> 28) & 3
                        q |= (e & 0xFFFFFF) << (8 * qn)
                        qn += nb
                        pushed += nb
                        br.consume(nbits)
                        if br.nvalid <= 32:
                            br.refill()
                    if qn >= 4 or pushed >= n_lane:
                        staged += (q & 0xFFFFFFFF).to_bytes(4, "little")
                        q >>= 32
                        qn = qn - 4 if qn >= 4 else 0
                        wi += 1
                if want:
                    out[first + done:first + done + want] = np.frombuffer(bytes(staged[-4 * target:]),
                                                                          dtype=np.uint8)[:want]
    return out
