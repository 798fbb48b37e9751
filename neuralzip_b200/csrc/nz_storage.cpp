// CPU storage codec pieces: token counting, mixed frames and Huff0 4-stream
// blocks. Setup uses the encoders to size both codebook options
// (neuralzip/setup.py:207-249); the storage format v2 save/load path uses
// encoders and decoders.
//
// Reference behaviour restated here (paths inside the reference project):
//   count_mixed_tokens      neuralzip/native/mixed_huffman.h:85-115
//   encode_mixed_block_into mixed_huffman.h:127-178: a 32-byte header of four
//                           (u32 tokens, u32 bits) pairs, then four MSB-first,
//                           byte-padded lanes split at source positions
//                           size * (lane + 1) / 4 without resetting the greedy
//                           parse; 0 when the frame does not fit `cap`.
//   decode_mixed_block_into mixed_huffman.h:180-240 (validation included).
//   encode/decode_huff0     zstd HUF_compress4X_usingCTable /
//                           HUF_decompress4X_usingDTable (codebooks.h:131-206),
//                           restated from RFC 8878 section 4.2.2: a 6-byte jump
//                           table of three little-endian u16 stream sizes, four
//                           segments of (size + 3) / 4 symbols (the last takes
//                           the rest), each a backward bitstream ending in a
//                           1-bit marker whose first-read bits are the first
//                           symbol's code. Byte parity with zstd's output is not
//                           pinned here (zstd is not vendored by the reference).

#include "nz_b200.h"
#include "nz_internal.h"

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace nz {
namespace {

// LSB-first bit sink used for backward (Huff0) streams.
struct BackwardWriter {
    uint8_t* out;
    uint64_t cap;
    uint64_t bytes = 0;
    uint64_t acc = 0;
    uint32_t n = 0;
    bool overflow = false;
    void add(uint64_t value, uint32_t bits) {  // bits <= 32
        acc |= value << n;
        n += bits;
        while (n >= 8) {
            if (out) {
                if (bytes >= cap) overflow = true;
                else out[bytes] = static_cast<uint8_t>(acc);
            }
            ++bytes;
            acc >>= 8;
            n -= 8;
        }
    }
    void close() {
        add(1, 1);
        if (n) {
            if (out) {
                if (bytes >= cap) overflow = true;
                else out[bytes] = static_cast<uint8_t>(acc);
            }
            ++bytes;
            acc = 0;
            n = 0;
        }
    }
};

}  // namespace

uint64_t mixed_encode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t cap) {
    if (cap <= 32) return 0;
    const bool pairs = !cb.pair_tokens.empty();
    uint64_t cursor = 32, source = 0;
    for (unsigned lane = 0; lane < 4; ++lane) {
        const uint64_t end = size * (lane + 1) / 4;
        uint64_t tokens = 0, bits = 0, acc = 0;
        uint32_t pending = 0;
        auto put_byte = [&](uint8_t b) -> bool {
            if (cursor >= cap) return false;
            if (out) out[cursor] = b;
            ++cursor;
            return true;
        };
        while (source < end) {
            uint32_t token = data[source];
            if (pairs && source + 1 < size) {
                const uint16_t pair = cb.pair_tokens[token | (static_cast<uint32_t>(data[source + 1]) << 8)];
                if (pair) token = pair;
            }
            source += token >= 256 ? 2 : 1;
            const uint32_t length = cb.lengths[token];
            if (!length) throw Error(NZ_ERUNTIME, "Symbol has no mixed codebook entry.");
            const uint64_t code = cb.codes[token];
            for (uint32_t done = 0; done < length;) {
                const uint32_t take = std::min<uint32_t>(length - done, 32);
                const uint64_t part = (code >> (length - done - take)) & ((uint64_t{1} << take) - 1);
                acc = (acc << take) | part;
                pending += take;
                done += take;
                while (pending >= 8) {
                    pending -= 8;
                    if (!put_byte(static_cast<uint8_t>(acc >> pending))) return 0;
                    acc &= pending ? ((uint64_t{1} << pending) - 1) : 0;
                }
            }
            bits += length;
            ++tokens;
        }
        if (pending && !put_byte(static_cast<uint8_t>(acc << (8 - pending)))) return 0;
        if (bits > 0xFFFFFFFFULL || tokens > 0xFFFFFFFFULL)
            throw Error(NZ_ERUNTIME, "Mixed frame exceeds uint32 limits.");
        if (out) {
            for (int i = 0; i < 4; ++i) {
                out[8 * lane + i] = static_cast<uint8_t>(tokens >> (8 * i));
                out[8 * lane + 4 + i] = static_cast<uint8_t>(bits >> (8 * i));
            }
        }
    }
    return cursor;
}

// Forward MSB-first window starting at bit `at` of `stream` (`bytes`
// long), zeros past the end. Codes are at most 56 bits, so one big-endian
// 8-byte load shifted by at most 7 bits holds every bit a token can read
// (the lowest `at & 7` bits of the window are left zero).
static inline uint64_t forward_window(const uint8_t* stream, uint64_t bytes, uint64_t at) {
    const uint64_t byte = at >> 3;
    uint64_t w = 0;
    if (byte + 8 <= bytes) {
        std::memcpy(&w, stream + byte, 8);
        w = __builtin_bswap64(w);
    } else {
        for (uint64_t i = 0; i < 8; ++i) w = (w << 8) | (byte + i < bytes ? stream[byte + i] : 0U);
    }
    return w << (at & 7U);
}

// One token from a 64-bit window: writes its bytes (<= 2) and returns its
// code length; 0 for an invalid prefix.
static inline uint32_t decode_token(const Codebook& cb, uint64_t w, uint32_t* bytes, uint32_t* count) {
    uint32_t e = cb.single[w >> 52];
    if ((e >> 16) & 3U) {
        *bytes = e & 0xFFFFU;
        *count = (e >> 16) & 3U;
        return e >> 20;
    }
    uint32_t node = e & (NZ_TREE_MAX_NODES - 1);
    for (uint32_t used = NZ_LUT_BITS; used < NZ_MAX_CODE_BITS; ++used) {
        const uint32_t child = cb.lut[NZ_LUT_TREE + 2 * node + ((w >> (63 - used)) & 1U)];
        if (child & 0xE0U) {
            *bytes = (child >> 8) & 0xFFFFU;
            *count = (child >> 5) & 7U;
            return used + 1;
        }
        node = (child >> 8) & (NZ_TREE_MAX_NODES - 1);
    }
    return 0;
}

void mixed_decode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t expected) {
    if (size < 32) throw Error(NZ_EVALUE, "Truncated mixed Huffman frame.");
    auto read_u32 = [](const uint8_t* p) {
        return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
               (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
    };
    // The frame's four lanes are independent bitstreams: each is decoded
    // into its own stretch of scratch (at most two bytes a token), the four
    // in lockstep (four dependency chains instead of one), and the stretches
    // are then copied out in lane order.
    struct Lane {
        const uint8_t* stream;
        uint64_t bytes, bits, pos, tokens, written;
        uint8_t* dst;
    } lanes[4];
    uint64_t cursor = 32, tokens_total = 0;
    for (unsigned k = 0; k < 4; ++k) {
        Lane& l = lanes[k];
        l.tokens = read_u32(data + 8 * k);
        l.bits = read_u32(data + 8 * k + 4);
        l.bytes = (l.bits + 7) / 8;
        if (l.bytes > size - cursor || l.tokens > expected - tokens_total)
            throw Error(NZ_EVALUE, "Mixed frame lengths exceed its payload.");
        l.stream = data + cursor;
        l.pos = l.written = 0;
        tokens_total += l.tokens;
        cursor += l.bytes;
    }
    if (cursor != size) throw Error(NZ_EVALUE, "Mixed decoded size mismatch.");
    thread_local std::vector<uint8_t> scratch;
    if (scratch.size() < 2 * tokens_total) scratch.resize(2 * tokens_total);
    uint64_t offset = 0;
    for (Lane& l : lanes) {
        l.dst = scratch.data() + offset;
        offset += 2 * l.tokens;
    }
    auto token = [&](Lane& l) {
        uint32_t value = 0, n = 0;
        const uint32_t length = decode_token(cb, forward_window(l.stream, l.bytes, l.pos), &value, &n);
        if (!length) throw Error(NZ_EVALUE, "Invalid mixed Huffman prefix.");
        if (l.pos + length > l.bits) throw Error(NZ_EVALUE, "Truncated mixed Huffman code.");
        l.dst[l.written] = static_cast<uint8_t>(value);
        l.dst[l.written + 1] = static_cast<uint8_t>(value >> 8);
        l.written += n;
        l.pos += length;
    };
    uint64_t together = lanes[0].tokens;
    for (const Lane& l : lanes) together = std::min(together, l.tokens);
    for (uint64_t i = 0; i < together; ++i) {
        token(lanes[0]);
        token(lanes[1]);
        token(lanes[2]);
        token(lanes[3]);
    }
    uint64_t written = 0;
    for (Lane& l : lanes) {
        for (uint64_t i = together; i < l.tokens; ++i) token(l);
        if (l.pos != l.bits) throw Error(NZ_EVALUE, "Mixed frame has unconsumed code bits.");
        if (l.bits % 8 && (l.stream[l.bytes - 1] & ((1U << (8 - l.bits % 8)) - 1)))
            throw Error(NZ_EVALUE, "Mixed frame has nonzero padding.");
        if (l.written > expected - written) throw Error(NZ_EVALUE, "Mixed expansion exceeds exponent count.");
        std::memcpy(out + written, l.dst, l.written);
        written += l.written;
    }
    if (written != expected) throw Error(NZ_EVALUE, "Mixed decoded size mismatch.");
}

uint64_t huff0_encode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t cap) {
    if (size == 0 || size > 128 * 1024 || cap < 6 + 1 + 1 + 1 + 8) return 0;
    for (uint64_t i = 0; i < size; ++i)
        if (!cb.lengths[data[i]]) return 0;
    const uint64_t segment = (size + 3) / 4;
    uint64_t total = 6;
    uint64_t sizes[4];
    for (int s = 0; s < 4; ++s) {
        const uint64_t begin = std::min<uint64_t>(size, segment * s);
        const uint64_t end = s == 3 ? size : std::min<uint64_t>(size, segment * (s + 1));
        if (begin >= end) return 0;
        uint8_t* dst = out ? out + total : nullptr;
        if (total >= cap) return 0;
        BackwardWriter w{dst, cap - total};
        for (uint64_t i = end; i-- > begin;) w.add(cb.codes[data[i]], cb.lengths[data[i]]);
        w.close();
        // A stream must leave 8 bytes of its capacity free (zstd's bit
        // stream refuses to write its last container otherwise).
        if (w.overflow || w.bytes + 8 > cap - total || w.bytes > 65535) return 0;
        sizes[s] = w.bytes;
        total += w.bytes;
    }
    if (out)
        for (int s = 0; s < 3; ++s) {
            out[2 * s] = static_cast<uint8_t>(sizes[s]);
            out[2 * s + 1] = static_cast<uint8_t>(sizes[s] >> 8);
        }
    return total;
}

// Blocks of four symbols of each of the four streams of a Huff0 block,
// from position k: every block reloads each stream's 64-bit container (at
// least 57 of its next bits, left-aligned; zeros below the stream's start)
// and decodes four symbols of at most 12 bits from it. The state lives in
// scalars (stores to the output bytes may alias anything else), and each
// stream's bits used by the call go to used[], for the caller to check
// against the `top` unread bits the streams held when the call started.
static inline __attribute__((always_inline)) void huff0_blocks_body(
    const uint32_t* single, const uint8_t* const* stream, const uint64_t* sizes, const int64_t* top,
    uint8_t* const* dst, uint64_t k, uint64_t run, uint64_t* used, uint32_t* bad) {
    auto load = [&](int s, uint64_t u) {
        const int64_t t = top[s] - static_cast<int64_t>(u);
        if (t <= 0) return uint64_t{0};
        const uint64_t last = static_cast<uint64_t>((t + 7) >> 3);
        const uint64_t start = last >= 8 ? last - 8 : 0;
        uint64_t w = 0;
        if (start + 8 <= sizes[s]) {
            std::memcpy(&w, stream[s] + start, 8);
        } else {
            for (uint64_t b = last; b-- > start;) w = (w << 8) | stream[s][b];
        }
        const int64_t have = t - static_cast<int64_t>(8 * start);
        return have >= 64 ? w : w << (64 - have);
    };
    uint64_t u0 = 0, u1 = 0, u2 = 0, u3 = 0;
    uint32_t invalid = 0;
    uint8_t* o0 = dst[0] + k;
    uint8_t* o1 = dst[1] + k;
    uint8_t* o2 = dst[2] + k;
    uint8_t* o3 = dst[3] + k;
    for (uint64_t r = 0; r < run; ++r) {
        uint64_t c0 = load(0, u0), c1 = load(1, u1), c2 = load(2, u2), c3 = load(3, u3);
        for (int j = 0; j < 4; ++j) {
            const uint32_t e0 = single[c0 >> 52], e1 = single[c1 >> 52];
            const uint32_t e2 = single[c2 >> 52], e3 = single[c3 >> 52];
            invalid |= ((e0 >> 16) & 3U) == 0 || ((e1 >> 16) & 3U) == 0 || ((e2 >> 16) & 3U) == 0 ||
                       ((e3 >> 16) & 3U) == 0;
            const uint32_t l0 = e0 >> 20, l1 = e1 >> 20, l2 = e2 >> 20, l3 = e3 >> 20;
            o0[4 * r + j] = static_cast<uint8_t>(e0);
            o1[4 * r + j] = static_cast<uint8_t>(e1);
            o2[4 * r + j] = static_cast<uint8_t>(e2);
            o3[4 * r + j] = static_cast<uint8_t>(e3);
            c0 <<= l0, c1 <<= l1, c2 <<= l2, c3 <<= l3;
            u0 += l0, u1 += l1, u2 += l2, u3 += l3;
        }
    }
    used[0] = u0, used[1] = u1, used[2] = u2, used[3] = u3;
    *bad |= invalid;
}

static void huff0_blocks_generic(const uint32_t* single, const uint8_t* const* stream, const uint64_t* sizes,
                                 const int64_t* top, uint8_t* const* dst, uint64_t k, uint64_t run, uint64_t* used,
                                 uint32_t* bad) {
    huff0_blocks_body(single, stream, sizes, top, dst, k, run, used, bad);
}

// The same with BMI2's shifts by any register (no round trip through CL).
__attribute__((target("bmi2"))) static void huff0_blocks_bmi2(const uint32_t* single, const uint8_t* const* stream,
                                                              const uint64_t* sizes, const int64_t* top,
                                                              uint8_t* const* dst, uint64_t k, uint64_t run,
                                                              uint64_t* used, uint32_t* bad) {
    huff0_blocks_body(single, stream, sizes, top, dst, k, run, used, bad);
}

static void huff0_blocks(const uint32_t* single, const uint8_t* const* stream, const uint64_t* sizes,
                         const int64_t* top, uint8_t* const* dst, uint64_t k, uint64_t run, uint64_t* used,
                         uint32_t* bad) {
    static const bool bmi2 = (__builtin_cpu_init(), __builtin_cpu_supports("bmi2") != 0);
    if (bmi2) huff0_blocks_bmi2(single, stream, sizes, top, dst, k, run, used, bad);
    else huff0_blocks_generic(single, stream, sizes, top, dst, k, run, used, bad);
}

void huff0_decode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t count) {
    if (size < 10) throw Error(NZ_EVALUE, "Truncated Huff0 block.");
    uint64_t sizes[4];
    uint64_t sum = 0;
    for (int s = 0; s < 3; ++s) {
        sizes[s] = static_cast<uint64_t>(data[2 * s]) | (static_cast<uint64_t>(data[2 * s + 1]) << 8);
        sum += sizes[s];
    }
    if (6 + sum >= size) throw Error(NZ_EVALUE, "Corrupt Huff0 jump table.");
    sizes[3] = size - 6 - sum;
    const uint64_t segment = (count + 3) / 4;
    const uint8_t* stream[4];
    int64_t top[4];
    uint64_t begin[4], end[4];
    const uint8_t* at = data + 6;
    for (int s = 0; s < 4; ++s) {
        const uint64_t n = sizes[s];
        if (n == 0 || at[n - 1] == 0) throw Error(NZ_EVALUE, "Corrupt Huff0 stream end.");
        stream[s] = at;
        top[s] = static_cast<int64_t>(8 * (n - 1) + (31 - __builtin_clz(at[n - 1])));
        begin[s] = std::min<uint64_t>(count, segment * s);
        end[s] = s == 3 ? count : std::min<uint64_t>(count, segment * (s + 1));
        at += n;
    }
    // The four streams are independent: decode them in lockstep (four
    // dependency chains instead of one) by huff0_blocks, then each stream's
    // last few symbols one at a time from a freshly loaded container.
    const uint32_t* single = cb.single.data();
    uint32_t bad = 0;
    uint64_t c[4];
    auto reload = [&](int s) {
        const int64_t t = top[s];
        if (t <= 0) {
            c[s] = 0;
            return;
        }
        const uint64_t last = static_cast<uint64_t>((t + 7) >> 3);  // bytes that hold unread bits
        const uint64_t start = last >= 8 ? last - 8 : 0;
        uint64_t w = 0;
        if (start + 8 <= sizes[s]) {
            std::memcpy(&w, stream[s] + start, 8);
        } else {
            for (uint64_t b = last; b-- > start;) w = (w << 8) | stream[s][b];
        }
        const int64_t have = t - static_cast<int64_t>(8 * start);  // valid low bits of w
        c[s] = have >= 64 ? w : w << (64 - have);
    };
    auto step = [&](int s, uint64_t i) {
        const uint32_t e = single[c[s] >> 52];
        const uint32_t length = e >> 20;
        bad |= static_cast<uint32_t>(!((e >> 16) & 3U)) | static_cast<uint32_t>(top[s] < static_cast<int64_t>(length));
        out[i] = static_cast<uint8_t>(e);
        c[s] <<= length;
        top[s] -= length;
    };
    uint64_t together = end[3] - begin[3];
    for (int s = 0; s < 3; ++s) together = std::min(together, end[s] - begin[s]);
    uint64_t k = 0;
    uint8_t* dst[4] = {out + begin[0], out + begin[1], out + begin[2], out + begin[3]};
    const uint64_t blocks = together / 4;
    for (uint64_t done = 0; done < blocks && !bad;) {
        // Up to 64 blocks of four symbols a stream between checks of the
        // bits used against the bits the streams held.
        const uint64_t run = std::min<uint64_t>(64, blocks - done);
        uint64_t used[4];
        huff0_blocks(single, stream, sizes, top, dst, k, run, used, &bad);
        for (int s = 0; s < 4; ++s) {
            top[s] -= static_cast<int64_t>(used[s]);
            bad |= static_cast<uint32_t>(top[s] < 0);
        }
        k += 4 * run;
        done += run;
    }
    for (int s = 0; s < 4 && !bad; ++s)
        for (uint64_t i = begin[s] + k; i < end[s] && !bad; ++i) {
            reload(s);
            step(s, i);
        }
    if (bad) throw Error(NZ_EVALUE, "Corrupt Huff0 stream.");
    for (int s = 0; s < 4; ++s)
        if (top[s] != 0) throw Error(NZ_EVALUE, "Huff0 stream has unconsumed bits.");
}

}  // namespace nz

using nz::Error;


namespace nz {

// Validation of one storage piece before any worker runs.
void check_piece(const nz_storage_piece& p) {
    check_dtype(p.dt);
    if (!p.lanes) throw Error(NZ_EVALUE, "A storage piece has no lanes.");
    if (p.count && !p.out) throw Error(NZ_EVALUE, "A storage piece has no output.");
    if (p.count > static_cast<uint64_t>(INT32_MAX))
        throw Error(NZ_EOVERFLOW, "A storage piece exceeds 2^31 elements.");
    for (uint32_t lane = 0; lane < p.dt.elem_size; ++lane) {
        const nz_storage_lane& l = p.lanes[lane];
        if (l.payload_size && !l.payload) throw Error(NZ_EVALUE, "A storage chunk has no payload.");
        if (l.mode == NZ_CHUNK_RAW) {
            if (l.payload_size != p.count) throw Error(NZ_EVALUE, "Raw payload size mismatch.");
        } else if (l.mode == NZ_CHUNK_HUFF0 || l.mode == NZ_CHUNK_MIXED) {
            if (!l.codebook) throw Error(NZ_EVALUE, "Compressed chunk needs a decode table.");
            if (l.mode == NZ_CHUNK_HUFF0 && p.count > 128 * 1024)
                throw Error(NZ_EVALUE, "Shared chunk exceeds Huff0's block limit.");
        } else {
            throw Error(NZ_EVALUE, "Unsupported decoded chunk mode.");
        }
    }
}

// Decodes every lane of one piece (raw lanes are read in place), then
// interleaves the lanes into element words and undoes the reorder of
// neuralzip/dtypes.py:23-45 (the sign moves back above the exponent).
void decode_piece(const nz_storage_piece& p) {
    const uint32_t es = p.dt.elem_size;
    const uint64_t n = p.count;
    if (n == 0) return;
    thread_local std::vector<uint8_t> scratch;
    if (scratch.size() < es * n) scratch.resize(es * n);
    const uint8_t* lane[4] = {nullptr, nullptr, nullptr, nullptr};
    for (uint32_t k = 0; k < es; ++k) {
        const nz_storage_lane& l = p.lanes[k];
        const Codebook* cb = reinterpret_cast<const Codebook*>(l.codebook);
        if (l.mode == NZ_CHUNK_RAW) {
            lane[k] = l.payload;
            continue;
        }
        uint8_t* dst = scratch.data() + k * n;
        if (l.mode == NZ_CHUNK_HUFF0) huff0_decode(*cb, l.payload, l.payload_size, dst, n);
        else mixed_decode(*cb, l.payload, l.payload_size, dst, n);
        lane[k] = dst;
    }
    const uint32_t mant = (1U << p.dt.mant_bits) - 1U;
    const uint32_t sign_stored = 1U << p.dt.mant_bits;
    const uint32_t exp_field = ((1U << p.dt.exp_bits) - 1U) << p.dt.mant_bits;
    const bool reorder = p.dt.reorder != 0;
    auto restore = [&](uint32_t v) {
        return reorder ? (v & mant) | ((v & sign_stored) << p.dt.exp_bits) | ((v >> 1) & exp_field) : v;
    };
    if (es == 2) {
        uint16_t* out = reinterpret_cast<uint16_t*>(p.out);
        for (uint64_t i = 0; i < n; ++i) {
            const uint16_t w = static_cast<uint16_t>(restore(lane[0][i] | (static_cast<uint32_t>(lane[1][i]) << 8)));
            std::memcpy(out + i, &w, 2);
        }
    } else {
        uint32_t* out = reinterpret_cast<uint32_t*>(p.out);
        for (uint64_t i = 0; i < n; ++i) {
            const uint32_t w = restore(lane[0][i] | (static_cast<uint32_t>(lane[1][i]) << 8) |
                                       (static_cast<uint32_t>(lane[2][i]) << 16) |
                                       (static_cast<uint32_t>(lane[3][i]) << 24));
            std::memcpy(out + i, &w, 4);
        }
    }
}

}  // namespace nz

namespace {

// Exponent counts of elements [begin, end), four interleaved tables.
template <typename Word>
void count_exponents(const uint8_t* raw, uint64_t begin, uint64_t end, uint32_t shift, uint32_t mask,
                     uint64_t (&local)[4][256]) {
    auto exponent = [&](uint64_t k) {
        Word v;
        std::memcpy(&v, raw + sizeof(Word) * k, sizeof(Word));
        return (static_cast<uint32_t>(v) >> shift) & mask;
    };
    uint64_t i = begin;
    for (; i + 4 <= end; i += 4) {
        ++local[0][exponent(i)];
        ++local[1][exponent(i + 1)];
        ++local[2][exponent(i + 2)];
        ++local[3][exponent(i + 3)];
    }
    for (; i < end; ++i) ++local[0][exponent(i)];
}

}  // namespace

extern "C" {

int nz_count_tokens(const uint8_t* data, uint64_t size, const uint8_t* vocab, uint32_t vocab_size,
                    uint64_t* counts) {
    NZ_GUARD({
        if ((size && !data) || !counts || (vocab_size && !vocab)) throw Error(NZ_EVALUE, "Null argument.");
        if (vocab_size % 2 || vocab_size > 2 * NZ_MAX_PAIRS) throw Error(NZ_EVALUE, "Invalid mixed pair vocabulary.");
        std::vector<uint16_t> lookup(vocab_size ? 65536 : 0, 0);
        for (uint32_t i = 0; i < vocab_size; i += 2) {
            const uint32_t pair = vocab[i] | (vocab[i + 1] << 8);
            if (lookup[pair]) throw Error(NZ_EVALUE, "Duplicate mixed pair definition.");
            lookup[pair] = static_cast<uint16_t>(256 + i / 2);
        }
        if (!vocab_size) {
            // Plain byte counts: independent blocks on the host's threads,
            // each into four interleaved local tables, added under a lock.
            constexpr uint64_t kBlock = uint64_t{1} << 22;
            std::mutex add;
            nz::run_jobs((size + kBlock - 1) / kBlock, 0, [&](uint64_t b) {
                uint64_t local[4][256] = {};
                const uint8_t* p = data + b * kBlock;
                const uint64_t n = std::min<uint64_t>(kBlock, size - b * kBlock);
                uint64_t i = 0;
                for (; i + 4 <= n; i += 4) {
                    ++local[0][p[i]];
                    ++local[1][p[i + 1]];
                    ++local[2][p[i + 2]];
                    ++local[3][p[i + 3]];
                }
                for (; i < n; ++i) ++local[0][p[i]];
                std::lock_guard<std::mutex> hold(add);
                for (uint32_t v = 0; v < 256; ++v) counts[v] += local[0][v] + local[1][v] + local[2][v] + local[3][v];
            });
            return NZ_OK;
        }
        // The greedy pair parse is sequential (a pair can start anywhere).
        for (uint64_t i = 0; i < size;) {
            const uint32_t pair = i + 1 < size ? lookup[data[i] | (data[i + 1] << 8)] : 0;
            ++counts[pair ? pair : data[i]];
            i += pair ? 2 : 1;
        }
    })
}

int nz_exponent_histograms(const uint8_t* raw, uint64_t numel, const nz_dtype* dt, uint64_t step,
                           uint64_t* histograms) {
    NZ_GUARD({
        if ((numel && !raw) || !dt || !histograms || step == 0) throw Error(NZ_EVALUE, "Null argument.");
        nz::check_dtype(*dt);
        const uint32_t mask = (1U << dt->exp_bits) - 1U;
        const uint32_t shift = dt->mant_bits;
        // Chunks are independent rows: they are counted on the host's
        // threads, each into four interleaved local tables (consecutive
        // elements rarely wait on the same counter) added into its row.
        const uint64_t chunks = (numel + step - 1) / step;
        nz::run_jobs(chunks, 0, [&](uint64_t chunk) {
            uint64_t local[4][256] = {};
            const uint64_t begin = chunk * step, end = std::min(numel, begin + step);
            if (dt->elem_size == 2) count_exponents<uint16_t>(raw, begin, end, shift, mask, local);
            else count_exponents<uint32_t>(raw, begin, end, shift, mask, local);
            uint64_t* h = histograms + chunk * 256;
            for (uint32_t b = 0; b < 256; ++b) h[b] += local[0][b] + local[1][b] + local[2][b] + local[3][b];
        });
    })
}

int nz_mixed_encode(const nz_codebook* codebook, const uint8_t* data, uint64_t size, uint8_t* out,
                    uint64_t cap, uint64_t* written) {
    NZ_GUARD({
        if (!codebook || !written || (size && !data)) throw Error(NZ_EVALUE, "Null argument.");
        *written = nz::mixed_encode(*reinterpret_cast<const nz::Codebook*>(codebook), data, size, out, cap);
    })
}

int nz_mixed_decode(const nz_codebook* codebook, const uint8_t* frame, uint64_t size, uint8_t* out,
                    uint64_t expected) {
    NZ_GUARD({
        if (!codebook || !frame || (expected && !out)) throw Error(NZ_EVALUE, "Null argument.");
        nz::mixed_decode(*reinterpret_cast<const nz::Codebook*>(codebook), frame, size, out, expected);
    })
}

int nz_huff0_encode(const nz_codebook* codebook, const uint8_t* data, uint64_t size, uint8_t* out,
                    uint64_t cap, uint64_t* written) {
    NZ_GUARD({
        if (!codebook || !written || (size && !data)) throw Error(NZ_EVALUE, "Null argument.");
        *written = nz::huff0_encode(*reinterpret_cast<const nz::Codebook*>(codebook), data, size, out, cap);
    })
}

int nz_storage_decode(const nz_storage_piece* pieces, uint64_t count, int32_t threads) {
    NZ_GUARD({
        if (count && !pieces) throw Error(NZ_EVALUE, "Null storage pieces.");
        for (uint64_t i = 0; i < count; ++i) nz::check_piece(pieces[i]);
        // Every piece decodes on its own; the first failure by piece index
        // is the one reported, whatever order the workers ran in.
        std::mutex lock;
        uint64_t failed_at = count;
        int failed_status = NZ_OK;
        std::string failed_message;
        const unsigned hw = std::thread::hardware_concurrency();
        const int workers = threads > 0 ? threads : static_cast<int>(std::min<unsigned>(hw ? hw : 1U, 16U));
        nz::run_jobs(count, workers, [&](uint64_t i) {
            try {
                nz::decode_piece(pieces[i]);
            } catch (const nz::Error& e) {
                std::lock_guard<std::mutex> hold(lock);
                if (i < failed_at) failed_at = i, failed_status = e.status, failed_message = e.what();
            } catch (const std::exception& e) {
                std::lock_guard<std::mutex> hold(lock);
                if (i < failed_at) failed_at = i, failed_status = NZ_ERUNTIME, failed_message = e.what();
            }
        });
        if (failed_at < count) throw Error(failed_status, failed_message);
    })
}

int nz_huff0_decode(const nz_codebook* codebook, const uint8_t* block, uint64_t size, uint8_t* out,
                    uint64_t count) {
    NZ_GUARD({
        if (!codebook || !block || (count && !out)) throw Error(NZ_EVALUE, "Null argument.");
        nz::huff0_decode(*reinterpret_cast<const nz::Codebook*>(codebook), block, size, out, count);
    })
}

}  // extern "C"
