/*
 * nz_oracle.c — CPU oracle for the NeuralZip decompression path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (neuralzip_b200/) loads
 * or calls this file; tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline use it as the checker. It restates, in plain C, the reference
 * algorithms of MartinEBravo/neuralzip (paths inside that project):
 *
 *   oz_mixed_codes      neuralzip/native/mixed_huffman.h:5-57 (make_mixed_table:
 *                       canonical codes sorted by (length, symbol), validation)
 *   oz_ref_lut          neuralzip/gpu/inference.py:28-75 (GPUCodebook.decode_lut)
 *   oz_ref_encode       neuralzip/native/gpu_layout.h:62-241 (encode_gpu_symbols,
 *                       encode_gpu_layout: MSB-first bitstream, 64-bit segment
 *                       restart gaps, 4 KiB block output positions)
 *   oz_ref_decode       neuralzip/gpu/cuda/decode.cu:177-381 (decode_batched:
 *                       count pass, block scan, write pass, staged merge)
 *   oz_mixed_frame_*    neuralzip/native/mixed_huffman.h:127-240 (CPU frames)
 *   oz_restore          neuralzip/native/common.h:198-257 (lane merge) and
 *                       neuralzip/dtypes.py:23-45 (reorder)
 *
 * and adds oz_tile_decode, an independent bit-by-bit reader of the B200 tile
 * layout (include/nz_b200.h) used to check the product packer on machines
 * without a GPU.
 *
 * Parity pins: the mixed codes, the reference GPU layout and the mixed
 * frames are checked byte for byte against the reference's own headers
 * compiled by oracle/Makefile into oracle/_ref/ (tests/test_oracle_pin.py)
 * and against tests/golden/ fixtures generated from them. Singleton (Huff0)
 * tables come from zstd, which the reference tree does not vendor: for those
 * the oracle takes code lengths and values as inputs and parity of the Huff0
 * header bytes themselves is unpinned.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OZ_OK 0
#define OZ_ERR 1

static int g_err_line = 0;
#define FAIL() do { g_err_line = __LINE__; return OZ_ERR; } while (0)

int oz_error_line(void) { return g_err_line; }

/* ---- canonical mixed codes (mixed_huffman.h:5-57) ---------------------- */

int oz_mixed_codes(const uint8_t* lengths, uint32_t nsym, uint64_t* codes) {
    uint32_t order[512];
    if (nsym > 512) FAIL();
    for (uint32_t i = 0; i < nsym; ++i) {
        if (lengths[i] == 0 || lengths[i] > 56) FAIL();
        order[i] = i;
    }
    /* insertion sort by (length, symbol) */
    for (uint32_t i = 1; i < nsym; ++i) {
        uint32_t v = order[i];
        int j = (int)i - 1;
        while (j >= 0 && lengths[order[j]] > lengths[v]) {
            order[j + 1] = order[j];
            --j;
        }
        order[j + 1] = v;
    }
    uint64_t code = 0;
    uint32_t previous = 0;
    for (uint32_t k = 0; k < nsym; ++k) {
        uint32_t s = order[k];
        uint32_t len = lengths[s];
        code <<= (len - previous);
        if (code >= ((uint64_t)1 << len)) FAIL();
        codes[s] = code;
        ++code;
        previous = len;
    }
    if (code != ((uint64_t)1 << previous)) FAIL();
    return OZ_OK;
}

/* ---- reference GPU LUT (inference.py:28-75) ---------------------------- */

/* lut_out capacity: 4096 + 2 * nodes; returns the number of entries in
 * *lut_len and max_bits in *max_bits_out. Entries are u32 for mixed tables
 * ((len << 24) | (nbytes << 16) | bytes_le) and u16-in-u32 for singleton
 * tables ((len << 8) | symbol). */
int oz_ref_lut(const uint8_t* lengths, const uint64_t* values, uint32_t nsym, const uint8_t* vocab,
               uint32_t vocab_size, uint32_t* lut_out, uint32_t cap, uint32_t* lut_len,
               uint32_t* max_bits_out) {
    uint32_t longest = 0;
    for (uint32_t s = 0; s < nsym; ++s)
        if (lengths[s] > longest) longest = lengths[s];
    if (longest > (vocab_size ? 56u : 12u)) FAIL();
    uint32_t max_bits = longest < 12 ? longest : 12;
    *max_bits_out = max_bits;
    if (!longest) {
        *lut_len = 0;
        return OZ_OK;
    }
    if (nsym != 256 + vocab_size / 2) FAIL();
    uint32_t size = 1u << max_bits;
    if (cap < size) FAIL();
    memset(lut_out, 0, sizeof(uint32_t) * size);
    /* binary tree of all codes when some code is longer than max_bits */
    uint32_t (*nodes)[2] = calloc(4096 + 64 * 512, sizeof(uint32_t[2]));
    uint32_t n_nodes = 1;
    for (uint32_t s = 0; s < nsym; ++s) {
        uint32_t len = lengths[s];
        if (!len) continue;
        uint32_t entry;
        if (vocab_size) {
            uint32_t nbytes = s >= 256 ? 2 : 1;
            uint32_t bytes = s >= 256 ? (uint32_t)(vocab[2 * (s - 256)] | (vocab[2 * (s - 256) + 1] << 8)) : s;
            entry = (len << 24) | (nbytes << 16) | bytes;
        } else {
            entry = (len << 8) | s;
        }
        if (longest <= max_bits) {
            uint32_t begin = (uint32_t)(values[s] << (max_bits - len));
            uint32_t span = 1u << (max_bits - len);
            for (uint32_t i = 0; i < span; ++i) lut_out[begin + i] = entry;
        } else {
            uint32_t node = 0;
            for (int bit = (int)len - 1; bit >= 0; --bit) {
                uint32_t branch = (uint32_t)((values[s] >> bit) & 1u);
                if (bit == 0) {
                    nodes[node][branch] = entry;
                } else {
                    if (!nodes[node][branch]) {
                        if (n_nodes >= 4096 + 64 * 512) { free(nodes); FAIL(); }
                        nodes[node][branch] = n_nodes++;
                    }
                    node = nodes[node][branch];
                }
            }
        }
    }
    uint32_t total = size;
    if (longest > max_bits) {
        for (uint32_t prefix = 0; prefix < size; ++prefix) {
            uint32_t node = 0;
            for (int bit = (int)max_bits - 1; bit >= 0; --bit) {
                node = nodes[node][(prefix >> bit) & 1u];
                if (node >> 24) break;
            }
            lut_out[prefix] = (node >> 24) ? node : size + 2 * node;
        }
        total = size + 2 * n_nodes;
        if (cap < total) { free(nodes); FAIL(); }
        for (uint32_t n = 0; n < n_nodes; ++n)
            for (int b = 0; b < 2; ++b) {
                uint32_t child = nodes[n][b];
                lut_out[size + 2 * n + b] = (child >> 24) ? child : size + 2 * child;
            }
    }
    free(nodes);
    for (uint32_t i = 0; i < size; ++i)
        if (!lut_out[i]) FAIL();
    *lut_len = total;
    return OZ_OK;
}

/* ---- lane split / reorder (gpu_layout.h:200-231, dtypes.py:23-45) ------ */

static uint32_t reorder_value(uint32_t v, uint32_t reorder, uint32_t mant, uint32_t expb) {
    if (!reorder) return v;
    uint32_t mant_mask = (1u << mant) - 1u, sign = 1u << mant, exp = ((1u << expb) - 1u) << (mant + 1u);
    return (v & mant_mask) | ((v >> expb) & sign) | ((v << 1u) & exp);
}

static uint32_t restore_value(uint32_t v, uint32_t reorder, uint32_t mant, uint32_t expb) {
    if (!reorder) return v;
    uint32_t mant_mask = (1u << mant) - 1u;
    uint32_t sign = 1u << (mant + expb), exp = ((1u << expb) - 1u) << mant;
    return (v & mant_mask) | ((v << expb) & sign) | ((v >> 1u) & exp);
}

static uint32_t load_elem(const uint8_t* raw, uint64_t i, uint32_t es) {
    uint32_t v = 0;
    for (uint32_t l = 0; l < es; ++l) v |= (uint32_t)raw[i * es + l] << (8 * l);
    return v;
}

/* Splits raw elements into byte lanes (all lanes, selected included). */
int oz_split(const uint8_t* raw, uint64_t numel, uint32_t es, uint32_t reorder, uint32_t mant,
             uint32_t expb, uint8_t** lanes) {
    for (uint64_t i = 0; i < numel; ++i) {
        uint32_t v = reorder_value(load_elem(raw, i, es), reorder, mant, expb);
        for (uint32_t l = 0; l < es; ++l)
            if (lanes[l]) lanes[l][i] = (uint8_t)(v >> (8 * l));
    }
    return OZ_OK;
}

/* Merge: byte lanes -> element words, undoing the reorder
 * (decode.cu:83-100 assemble_value; common.h:198-257). */
int oz_restore(uint8_t* const* lanes, uint64_t numel, uint32_t es, uint32_t reorder, uint32_t mant,
               uint32_t expb, uint8_t* out) {
    for (uint64_t i = 0; i < numel; ++i) {
        uint32_t v = 0;
        for (uint32_t l = 0; l < es; ++l) v |= (uint32_t)lanes[l][i] << (8 * l);
        v = restore_value(v, reorder, mant, expb);
        for (uint32_t l = 0; l < es; ++l) out[i * es + l] = (uint8_t)(v >> (8 * l));
    }
    return OZ_OK;
}

/* ---- reference GPU layout encode (gpu_layout.h:62-241) ----------------- */

typedef struct {
    const uint8_t* sym;      /* selected lane bytes */
    uint64_t numel;
    const uint16_t* pairs;   /* 65536-entry pair lookup or NULL */
} oz_reader;

static uint32_t read_token(const oz_reader* r, uint64_t index) {
    uint32_t symbol = r->sym[index];
    if (r->pairs && index + 1 < r->numel) {
        uint32_t pair = r->pairs[symbol | ((uint32_t)r->sym[index + 1] << 8)];
        if (pair) return pair;
    }
    return symbol;
}

/* Outputs: bitstream (cap bytes), gaps (raw u8 per segment, unpacked, cap
 * gap_cap), positions (cap pos_cap). Sizes are returned through pointers.
 * For singleton tables the caller packs gaps to nibbles with oz_pack_gaps. */
int oz_ref_encode(const uint8_t* sym, uint64_t numel, const uint8_t* lengths, const uint64_t* codes,
                  uint32_t nsym, const uint8_t* vocab, uint32_t vocab_size, uint8_t* bitstream,
                  uint64_t bit_cap, uint64_t* n_bytes, uint8_t* gaps, uint64_t gap_cap,
                  uint64_t* n_gaps, uint32_t* positions, uint64_t pos_cap, uint64_t* n_positions,
                  uint64_t* bit_length_out, uint32_t* max_bits_out) {
    if (numel > 0x7FFFFFFFull) FAIL();
    uint16_t* pairs = NULL;
    if (vocab_size) {
        pairs = calloc(65536, sizeof(uint16_t));
        for (uint32_t i = 0; i < vocab_size; i += 2)
            pairs[vocab[i] | (vocab[i + 1] << 8)] = (uint16_t)(256 + i / 2);
    }
    oz_reader r = {sym, numel, pairs};
    uint32_t max_bits = 0;
    for (uint32_t s = 0; s < nsym; ++s)
        if (lengths[s] > max_bits) max_bits = lengths[s];
    if (max_bits == 0 || max_bits > 56) { free(pairs); FAIL(); }
    int mixed = vocab_size != 0;
    uint64_t bit_length = 0;
    for (uint64_t i = 0; i < numel;) {
        uint32_t t = read_token(&r, i);
        if (t >= nsym || lengths[t] == 0) { free(pairs); FAIL(); }
        bit_length += lengths[t];
        i += t >= 256 ? 2 : 1;
    }
    uint64_t bytes = bit_length / 8 + (bit_length % 8 != 0);
    if (bytes > bit_cap) { free(pairs); FAIL(); }
    const uint64_t block_bytes = 8 * 512;
    uint64_t blocks = bytes / block_bytes + (bytes % block_bytes != 0);
    uint64_t gap_count = blocks * 512;
    uint64_t populated = bytes / 8 + (bytes % 8 != 0);
    if (gap_count > gap_cap || blocks + 1 > pos_cap) { free(pairs); FAIL(); }
    memset(gaps, 0, gap_count);
    memset(bitstream, 0, bytes);
    for (uint64_t b = 0; b <= blocks; ++b) positions[b] = (uint32_t)numel;
    uint64_t next_segment = 0, next_block = 0, offset = 0, start = 0, acc = 0;
    uint32_t pending = 0;
    for (uint64_t i = 0; i < numel;) {
        while (next_segment < populated && start >= next_segment * 64) {
            uint64_t gap = start - next_segment * 64;
            if (gap >= (mixed ? 256u : 16u)) { free(pairs); FAIL(); }
            gaps[next_segment++] = (uint8_t)gap;
        }
        while (next_block < blocks && start >= next_block * block_bytes * 8)
            positions[next_block++] = (uint32_t)i;
        uint32_t t = read_token(&r, i);
        uint32_t len = lengths[t];
        /* acc holds < 8 pending bits before each code; codes <= 56 bits */
        acc = (acc << len) | codes[t];
        pending += len;
        start += len;
        i += t >= 256 ? 2 : 1;
        while (pending >= 8) {
            pending -= 8;
            bitstream[offset++] = (uint8_t)((acc >> pending) & 0xFF);
            acc = pending ? (acc & (((uint64_t)1 << pending) - 1)) : 0;
        }
    }
    if (pending) bitstream[offset++] = (uint8_t)((acc << (8 - pending)) & 0xFF);
    while (next_segment < populated) {
        gaps[next_segment] = (uint8_t)(bit_length - next_segment * 64);
        ++next_segment;
    }
    free(pairs);
    *n_bytes = bytes;
    *n_gaps = gap_count;
    *n_positions = blocks + 1;
    *bit_length_out = bit_length;
    *max_bits_out = max_bits;
    return OZ_OK;
}

/* 4-bit gaps, even index in the high nibble (gpu_layout.h:49-59). */
int oz_pack_gaps(const uint8_t* gaps, uint64_t n, uint8_t* out) {
    memset(out, 0, n / 2 + (n % 2));
    for (uint64_t i = 0; i < n; ++i) out[i / 2] |= (uint8_t)(gaps[i] << ((i & 1) ? 0 : 4));
    return OZ_OK;
}

/* ---- reference GPU layout decode (decode.cu:177-381) ------------------- */

static uint32_t lut_decode(const uint32_t* lut, int mixed, uint64_t window, uint32_t max_bits,
                           uint32_t* nbits, uint32_t* count, uint32_t* bytes) {
    uint32_t index = (uint32_t)(window >> (64 - max_bits));
    uint32_t e = lut[index];
    if (mixed) {
        uint32_t depth = max_bits;
        while ((e >> 24) == 0) {
            uint32_t branch = (uint32_t)((window >> (63 - depth)) & 1u);
            e = lut[e + branch];
            ++depth;
            if (depth > 64) return 0;
        }
        *nbits = e >> 24;
        *count = (e >> 16) & 255u;
        *bytes = e & 0xFFFFu;
    } else {
        *nbits = (e >> 8) & 255u;
        *count = 1;
        *bytes = e & 255u;
    }
    return 1;
}

static uint64_t peek_bits(uint64_t high, uint64_t low, unsigned consumed) {
    return consumed ? (high << consumed) | (low >> (64u - consumed)) : high;
}

/* Decodes one group laid out by oz_ref_encode into `symbols` (numel
 * exponent bytes), mirroring the kernel's per-thread segments: symbols
 * starting in [gap, 64) of each 64-bit segment belong to its thread, the
 * block's threads scan their counts, and writes are clamped to the block's
 * [positions[b], positions[b+1]) range. gaps: one byte per segment
 * (unpacked). */
int oz_ref_decode(const uint32_t* lut, int mixed, uint32_t max_bits, const uint8_t* code,
                  uint64_t n_bytes, const uint8_t* gaps, const uint32_t* positions,
                  uint64_t numel, uint8_t* symbols) {
    if (max_bits == 0) {  /* raw group */
        memcpy(symbols, code, numel);
        return OZ_OK;
    }
    int long_codes = 0;
    (void)long_codes;
    uint64_t blocks = n_bytes / 4096 + (n_bytes % 4096 != 0);
    uint32_t counts[512];
    for (uint64_t b = 0; b < blocks; ++b) {
        uint32_t block_start = positions[b], block_end = positions[b + 1];
        for (uint32_t t = 0; t < 512; ++t) {
            uint64_t tid = b * 512 + t, offset = tid * 8;
            uint64_t high = 0, low = 0;
            for (int i = 0; i < 16; ++i) {
                uint64_t src = offset + i;
                uint64_t byte = src < n_bytes ? code[src] : 0;
                if (i < 8) high |= byte << (56 - 8 * i);
                else low |= byte << (56 - 8 * (i - 8));
            }
            unsigned consumed = offset < n_bytes ? gaps[tid] : 64u;
            uint32_t count = 0;
            while (consumed < 64) {
                uint32_t nb, c, by;
                if (!lut_decode(lut, mixed, peek_bits(high, low, consumed), max_bits, &nb, &c, &by)) FAIL();
                count += c;
                consumed += nb;
            }
            counts[t] = count;
        }
        uint32_t index = block_start;
        for (uint32_t t = 0; t < 512; ++t) {
            uint64_t tid = b * 512 + t, offset = tid * 8;
            uint64_t high = 0, low = 0;
            for (int i = 0; i < 16; ++i) {
                uint64_t src = offset + i;
                uint64_t byte = src < n_bytes ? code[src] : 0;
                if (i < 8) high |= byte << (56 - 8 * i);
                else low |= byte << (56 - 8 * (i - 8));
            }
            uint64_t end64 = (uint64_t)index + counts[t];
            uint32_t end = (uint32_t)(end64 < block_end ? end64 : block_end);
            unsigned consumed = gaps[tid < blocks * 512 ? tid : 0];
            uint32_t out = index;
            while (out < end) {
                uint32_t nb, c, by;
                if (!lut_decode(lut, mixed, peek_bits(high, low, consumed), max_bits, &nb, &c, &by)) FAIL();
                symbols[out++] = (uint8_t)(by & 255u);
                if (c == 2 && out < end) symbols[out++] = (uint8_t)(by >> 8);
                consumed += nb;
            }
            index += counts[t];
        }
    }
    (void)numel;
    return OZ_OK;
}

/* ---- mixed CPU frames (mixed_huffman.h:127-240) ------------------------ */

static void put_u32(uint8_t* p, uint32_t v) {
    for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i));
}

static uint32_t get_u32(const uint8_t* p) {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) v |= (uint32_t)p[i] << (8 * i);
    return v;
}

/* Returns the frame size in *out_size, or 0 when it does not fit `cap`
 * (the reference returns 0 in that case). */
int oz_mixed_frame_encode(const uint8_t* data, uint64_t size, const uint8_t* lengths,
                          const uint64_t* codes, const uint8_t* vocab, uint32_t vocab_size,
                          uint8_t* out, uint64_t cap, uint64_t* out_size) {
    *out_size = 0;
    uint16_t* pairs = calloc(65536, sizeof(uint16_t));
    for (uint32_t i = 0; i < vocab_size; i += 2) pairs[vocab[i] | (vocab[i + 1] << 8)] = (uint16_t)(256 + i / 2);
    if (cap <= 32) { free(pairs); return OZ_OK; }
    uint64_t cursor = 32, source = 0;
    for (unsigned lane = 0; lane < 4; ++lane) {
        uint64_t end = size * (lane + 1) / 4, tokens = 0, bits = 0;
        uint64_t buffer = 0;
        unsigned pending = 0;
        while (source < end) {
            uint32_t pair = source + 1 < size ? pairs[data[source] | ((uint32_t)data[source + 1] << 8)] : 0;
            uint32_t token = pair ? pair : data[source];
            source += pair ? 2 : 1;
            unsigned length = lengths[token];
            for (unsigned b = length; b-- > 0;) {
                buffer = (buffer << 1) | ((codes[token] >> b) & 1u);
                if (++pending == 8) {
                    if (cursor >= cap) { free(pairs); return OZ_OK; }
                    out[cursor++] = (uint8_t)buffer;
                    buffer = 0;
                    pending = 0;
                }
            }
            bits += length;
            ++tokens;
        }
        if (pending) {
            if (cursor >= cap) { free(pairs); return OZ_OK; }
            out[cursor++] = (uint8_t)(buffer << (8 - pending));
        }
        if (bits > 0xFFFFFFFFull || tokens > 0xFFFFFFFFull) { free(pairs); FAIL(); }
        put_u32(out + 8 * lane, (uint32_t)tokens);
        put_u32(out + 8 * lane + 4, (uint32_t)bits);
    }
    free(pairs);
    *out_size = cursor;
    return OZ_OK;
}

/* Bit-serial decoder of a mixed frame using the canonical code table. */
int oz_mixed_frame_decode(const uint8_t* data, uint64_t size, const uint8_t* lengths,
                          const uint64_t* codes, uint32_t nsym, const uint8_t* vocab, uint8_t* out,
                          uint64_t expected) {
    if (size < 32) FAIL();
    /* trie of the code */
    int32_t (*trie)[3] = calloc(64 * 512 + 2, sizeof(int32_t[3]));
    int32_t n = 1;
    trie[0][0] = trie[0][1] = -1;
    trie[0][2] = -1;
    for (uint32_t s = 0; s < nsym; ++s) {
        int32_t node = 0;
        for (int b = (int)lengths[s] - 1; b >= 0; --b) {
            int br = (int)((codes[s] >> b) & 1u);
            if (trie[node][br] < 0) {
                trie[node][br] = n;
                trie[n][0] = trie[n][1] = -1;
                trie[n][2] = -1;
                ++n;
            }
            node = trie[node][br];
        }
        trie[node][2] = (int32_t)s;
    }
    uint64_t cursor = 32, written = 0;
    for (unsigned lane = 0; lane < 4; ++lane) {
        uint32_t count = get_u32(data + 8 * lane);
        uint64_t bit_size = get_u32(data + 8 * lane + 4);
        uint64_t bytes = (bit_size + 7) / 8;
        if (bytes > size - cursor || count > expected - written) { free(trie); FAIL(); }
        const uint8_t* stream = data + cursor;
        uint64_t pos = 0;
        for (uint32_t i = 0; i < count; ++i) {
            int32_t node = 0;
            while (trie[node][2] < 0) {
                if (pos >= bit_size) { free(trie); FAIL(); }
                int bit = (stream[pos / 8] >> (7 - pos % 8)) & 1;
                ++pos;
                node = trie[node][bit];
                if (node < 0) { free(trie); FAIL(); }
            }
            uint32_t s = (uint32_t)trie[node][2];
            if (s < 256) {
                if (written >= expected) { free(trie); FAIL(); }
                out[written++] = (uint8_t)s;
            } else {
                if (written + 2 > expected) { free(trie); FAIL(); }
                out[written++] = vocab[2 * (s - 256)];
                out[written++] = vocab[2 * (s - 256) + 1];
            }
        }
        if (pos != bit_size) { free(trie); FAIL(); }
        cursor += bytes;
    }
    free(trie);
    if (cursor != size || written != expected) FAIL();
    return OZ_OK;
}

/* ---- B200 tile layout reader (include/nz_b200.h) ----------------------- */

/* Decodes the selected lane of one group packed in the tile layout into
 * `symbols` (numel bytes), bit by bit through a code trie; checks that each
 * sub-stream consumes exactly its stored length and that pairs do not
 * straddle sub-streams. */
int oz_tile_decode(const uint32_t* bits, uint64_t n_words, const uint16_t* lens,
                   const uint32_t* tile_off, uint64_t numel, const uint8_t* lengths,
                   const uint64_t* codes, uint32_t nsym, const uint8_t* vocab, uint8_t* symbols) {
    int32_t (*trie)[3] = calloc(64 * 512 + 2, sizeof(int32_t[3]));
    int32_t n = 1;
    trie[0][0] = trie[0][1] = trie[0][2] = -1;
    for (uint32_t s = 0; s < nsym; ++s) {
        if (!lengths[s]) continue;
        int32_t node = 0;
        for (int b = (int)lengths[s] - 1; b >= 0; --b) {
            int br = (int)((codes[s] >> b) & 1u);
            if (trie[node][br] < 0) {
                trie[node][br] = n;
                trie[n][0] = trie[n][1] = trie[n][2] = -1;
                ++n;
            }
            node = trie[node][br];
        }
        trie[node][2] = (int32_t)s;
    }
    const uint64_t lane_elems = 256, tile_lanes = 32;
    uint64_t subs = (numel + lane_elems * tile_lanes - 1) / (lane_elems * tile_lanes) * tile_lanes;
    uint64_t pos = 0;
    for (uint64_t s = 0; s < subs; ++s) {
        if (s % tile_lanes == 0 && tile_off[s / tile_lanes] != pos) { free(trie); FAIL(); }
        uint64_t begin = s * lane_elems < numel ? s * lane_elems : numel;
        uint64_t end = begin + lane_elems < numel ? begin + lane_elems : numel;
        uint64_t start = pos;
        for (uint64_t i = begin; i < end;) {
            int32_t node = 0;
            while (trie[node][2] < 0) {
                if (pos / 32 >= n_words) { free(trie); FAIL(); }
                int bit = (int)((bits[pos / 32] >> (31 - pos % 32)) & 1u);
                ++pos;
                node = trie[node][bit];
                if (node < 0) { free(trie); FAIL(); }
            }
            uint32_t t = (uint32_t)trie[node][2];
            if (t < 256) {
                symbols[i++] = (uint8_t)t;
            } else {
                if (i + 2 > end) { free(trie); FAIL(); }
                symbols[i++] = vocab[2 * (t - 256)];
                symbols[i++] = vocab[2 * (t - 256) + 1];
            }
        }
        if (pos - start != lens[s]) { free(trie); FAIL(); }
    }
    free(trie);
    return OZ_OK;
}
