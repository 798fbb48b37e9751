// Huff0 table headers and singleton code construction.
//
// The reference takes singleton (shared_huff0) tables from zstd's Huff0 at
// revision 5233c58e6ca0b1c4c6b353ad79649191ed195bdc (not vendored in the
// reference tree): HUF_buildCTable_wksp / HUF_writeCTable_wksp build and
// serialize a table (neuralzip/native/codebooks.h:20-39), HUF_readCTable
// reads it back and export_code_table_from_header turns it into code
// lengths and values (codebooks.h:60-68, 79-111). This file restates the
// published format instead, RFC 8878 section 4.2.1 ("Huffman Tree
// Description") with the FSE table description and bitstream of section
// 4.1.1:
//   * a header byte < 128 announces that many bytes of FSE-compressed
//     weights (accuracy log <= 6, two interleaved states), a byte >= 128
//     announces (byte - 127) weights stored as 4-bit nibbles;
//   * the weight of the last symbol is implied by completing the sum of
//     2^(weight-1) to a power of two, 2^max_bits;
//   * code length = max_bits + 1 - weight (weight 0: symbol absent), and
//     codes are handed out from the longest length to the shortest, in
//     symbol order within one length, counting up from zero.
// The table builder is a plain Huffman construction limited to 12 bits
// with the length-adjustment procedure of ITU-T T.81 Annex K.3; its lengths
// can differ from zstd's on ties, so header bytes are not claimed to be
// byte-identical with the reference's (the decoded GPU weights do not
// depend on which valid table is used).

#include "nz_b200.h"
#include "nz_internal.h"

#include <algorithm>
#include <cstring>
#include <numeric>
#include <vector>

namespace nz {
namespace {

constexpr uint32_t kHuffMaxBits = 12;      // HUF_TABLELOG_MAX
constexpr uint32_t kWeightAccuracyMax = 6;  // FSE accuracy log limit for weights
constexpr uint32_t kFseMinAccuracy = 5;

inline uint32_t highbit(uint32_t v) { return 31U - static_cast<uint32_t>(__builtin_clz(v)); }

// ---- FSE table description (RFC 8878 4.1.1) --------------------------------

struct ForwardBits {  // little-endian, least significant bit first
    const uint8_t* src;
    size_t size;
    size_t bitpos = 0;
    uint32_t peek(uint32_t n) const {
        uint32_t v = 0;
        for (uint32_t i = 0; i < n; ++i) {
            const size_t p = bitpos + i;
            const uint32_t bit = p / 8 < size ? (src[p / 8] >> (p % 8)) & 1U : 0U;
            v |= bit << i;
        }
        return v;
    }
    uint32_t read(uint32_t n) {
        const uint32_t v = peek(n);
        bitpos += n;
        return v;
    }
};

// Returns bytes consumed; norm[] gets -1 for "less than one" probabilities.
size_t read_ncount(const uint8_t* src, size_t size, uint32_t max_symbol, int16_t* norm,
                   uint32_t* max_symbol_used, uint32_t* accuracy_log) {
    if (size < 1) throw Error(NZ_EVALUE, "Truncated FSE table description.");
    ForwardBits in{src, size};
    const uint32_t al = in.read(4) + kFseMinAccuracy;
    if (al > kWeightAccuracyMax) throw Error(NZ_EVALUE, "FSE accuracy log too large for Huffman weights.");
    int32_t remaining = (1 << al) + 1;
    int32_t threshold = 1 << al;
    uint32_t nbits = al + 1;
    uint32_t symbol = 0;
    bool previous_zero = false;
    std::fill(norm, norm + max_symbol + 1, 0);
    for (;;) {
        if (previous_zero) {
            uint32_t flag = in.read(2);
            while (flag == 3) {
                symbol += 3;
                flag = in.read(2);
            }
            symbol += flag;
            if (symbol > max_symbol) throw Error(NZ_EVALUE, "FSE table describes too many symbols.");
        }
        const int32_t max = (2 * threshold - 1) - remaining;
        int32_t value;
        const uint32_t low = in.peek(nbits - 1);
        if (static_cast<int32_t>(low) < max) {
            value = static_cast<int32_t>(low);
            in.bitpos += nbits - 1;
        } else {
            value = static_cast<int32_t>(in.peek(nbits));
            if (value >= threshold) value -= max;
            in.bitpos += nbits;
        }
        const int32_t proba = value - 1;
        remaining -= proba < 0 ? -proba : proba;
        if (symbol > max_symbol) throw Error(NZ_EVALUE, "FSE table describes too many symbols.");
        norm[symbol++] = static_cast<int16_t>(proba);
        previous_zero = proba == 0;
        if (remaining < threshold) {
            if (remaining <= 1) break;
            nbits = highbit(static_cast<uint32_t>(remaining)) + 1;
            threshold = 1 << (nbits - 1);
        }
        if (symbol > max_symbol) break;
    }
    if (remaining != 1) throw Error(NZ_EVALUE, "Corrupt FSE table description.");
    *max_symbol_used = symbol - 1;
    *accuracy_log = al;
    const size_t used = (in.bitpos + 7) / 8;
    if (used > size) throw Error(NZ_EVALUE, "Truncated FSE table description.");
    return used;
}

struct FseState {
    uint8_t symbol;
    uint8_t nbits;
    uint16_t base;
};

std::vector<FseState> build_fse_table(const int16_t* norm, uint32_t max_symbol, uint32_t al) {
    const uint32_t size = 1U << al;
    std::vector<FseState> table(size);
    std::vector<uint32_t> next(max_symbol + 1);
    uint32_t high = size - 1;
    for (uint32_t s = 0; s <= max_symbol; ++s) {
        if (norm[s] == -1) {
            table[high--].symbol = static_cast<uint8_t>(s);
            next[s] = 1;
        } else {
            next[s] = static_cast<uint32_t>(norm[s]);
        }
    }
    const uint32_t step = (size >> 1) + (size >> 3) + 3;
    const uint32_t mask = size - 1;
    uint32_t pos = 0;
    for (uint32_t s = 0; s <= max_symbol; ++s) {
        for (int i = 0; i < norm[s]; ++i) {
            table[pos].symbol = static_cast<uint8_t>(s);
            do {
                pos = (pos + step) & mask;
            } while (pos > high);
        }
    }
    if (pos != 0) throw Error(NZ_EVALUE, "Corrupt FSE table description.");
    for (uint32_t u = 0; u < size; ++u) {
        const uint32_t s = table[u].symbol;
        const uint32_t ns = next[s]++;
        const uint32_t nb = al - highbit(ns);
        table[u].nbits = static_cast<uint8_t>(nb);
        table[u].base = static_cast<uint16_t>((ns << nb) - size);
    }
    return table;
}

// Backward FSE bitstream: bits are read from the highest bit below the end
// marker of the last byte towards bit 0 of the first byte; reads past the
// start yield zeros and count as overflow.
struct BackwardBits {
    const uint8_t* src;
    size_t size;
    int64_t total = 0;    // real bits below the marker
    int64_t consumed = 0;
    void init() {
        if (size == 0 || src[size - 1] == 0) throw Error(NZ_EVALUE, "Corrupt FSE bitstream end.");
        total = static_cast<int64_t>(8 * (size - 1) + highbit(src[size - 1]));
    }
    uint32_t read(uint32_t n) {
        uint32_t v = 0;
        for (uint32_t i = 0; i < n; ++i) {
            const int64_t p = total - consumed - 1 - static_cast<int64_t>(i);
            const uint32_t bit = p >= 0 ? (src[p / 8] >> (p % 8)) & 1U : 0U;
            v = (v << 1) | bit;
        }
        consumed += n;
        return v;
    }
    bool overflow() const { return consumed > total; }
};

size_t decode_weights_fse(const uint8_t* src, size_t size, uint8_t* weights, size_t cap) {
    int16_t norm[kHuffMaxBits + 1];
    uint32_t max_symbol = 0, al = 0;
    const size_t nc = read_ncount(src, size, kHuffMaxBits, norm, &max_symbol, &al);
    const std::vector<FseState> table = build_fse_table(norm, max_symbol, al);
    BackwardBits in{src + nc, size - nc};
    in.init();
    uint32_t s1 = in.read(al);
    uint32_t s2 = in.read(al);
    size_t n = 0;
    auto emit = [&](uint32_t state) {
        if (n >= cap) throw Error(NZ_EVALUE, "Too many Huffman weights.");
        weights[n++] = table[state].symbol;
    };
    auto update = [&](uint32_t& state) { state = table[state].base + in.read(table[state].nbits); };
    for (;;) {
        emit(s1);
        update(s1);
        if (in.overflow()) {
            emit(s2);
            break;
        }
        emit(s2);
        update(s2);
        if (in.overflow()) {
            emit(s1);
            break;
        }
    }
    return n;
}

// ---- FSE encoding of weights (own encoder for the same format) -------------

struct BitSink {  // forward, LSB first
    std::vector<uint8_t> bytes;
    uint64_t bitpos = 0;
    void put(uint32_t value, uint32_t n) {
        for (uint32_t i = 0; i < n; ++i) {
            if (bitpos / 8 >= bytes.size()) bytes.push_back(0);
            bytes[bitpos / 8] |= static_cast<uint8_t>(((value >> i) & 1U) << (bitpos % 8));
            ++bitpos;
        }
    }
};

std::vector<uint8_t> write_ncount(const int16_t* norm, uint32_t max_symbol, uint32_t al) {
    BitSink out;
    out.put(al - kFseMinAccuracy, 4);
    int32_t remaining = (1 << al) + 1;
    int32_t threshold = 1 << al;
    uint32_t nbits = al + 1;
    uint32_t symbol = 0;
    bool previous_zero = false;
    while (symbol <= max_symbol && remaining > 1) {
        if (previous_zero) {
            uint32_t start = symbol;
            while (symbol <= max_symbol && norm[symbol] == 0) ++symbol;
            if (symbol > max_symbol) throw Error(NZ_ERUNTIME, "Invalid FSE distribution.");
            while (symbol >= start + 3) {
                out.put(3, 2);
                start += 3;
            }
            out.put(symbol - start, 2);
        }
        int32_t count = norm[symbol++];
        const int32_t max = (2 * threshold - 1) - remaining;
        remaining -= count < 0 ? -count : count;
        ++count;
        if (count >= threshold) count += max;
        out.put(static_cast<uint32_t>(count), nbits - (count < max ? 1U : 0U));
        previous_zero = count == 1;
        if (remaining < 1) throw Error(NZ_ERUNTIME, "Invalid FSE distribution.");
        while (remaining < threshold) {
            --nbits;
            threshold >>= 1;
        }
    }
    if (remaining != 1) throw Error(NZ_ERUNTIME, "Invalid FSE distribution.");
    return out.bytes;
}

// Normalizes weight counts to 2^al with every present symbol >= 1.
void normalize(const uint32_t* counts, uint32_t max_symbol, uint32_t total, uint32_t al,
               int16_t* norm) {
    const int32_t target = 1 << al;
    int32_t sum = 0;
    uint32_t largest = 0;
    for (uint32_t s = 0; s <= max_symbol; ++s) {
        if (!counts[s]) {
            norm[s] = 0;
            continue;
        }
        const uint64_t scaled = (static_cast<uint64_t>(counts[s]) * target + total / 2) / total;
        norm[s] = static_cast<int16_t>(std::max<uint64_t>(1, scaled));
        sum += norm[s];
        if (counts[s] > counts[largest] || !counts[largest]) largest = s;
    }
    // Move the rounding error onto the largest entries, keeping each >= 1.
    while (sum != target) {
        uint32_t pick = largest;
        if (sum > target) {
            int16_t best = 1;
            for (uint32_t s = 0; s <= max_symbol; ++s)
                if (norm[s] > best) best = norm[s], pick = s;
            if (best <= 1) throw Error(NZ_ERUNTIME, "Weights cannot be normalized.");
            --norm[pick];
            --sum;
        } else {
            ++norm[pick];
            ++sum;
        }
    }
}

// Encodes `weights` (decode order) with two interleaved tANS states so that
// the RFC 8878 decoding loop above yields exactly these n weights.
std::vector<uint8_t> encode_weights_fse(const uint8_t* weights, size_t n) {
    if (n < 2) throw Error(NZ_ERUNTIME, "Too few Huffman weights for FSE.");
    uint32_t counts[kHuffMaxBits + 1] = {};
    uint32_t max_symbol = 0;
    for (size_t i = 0; i < n; ++i) {
        ++counts[weights[i]];
        max_symbol = std::max<uint32_t>(max_symbol, weights[i]);
    }
    uint32_t distinct = 0;
    for (uint32_t c : counts) distinct += c ? 1 : 0;
    if (distinct < 2) throw Error(NZ_ERUNTIME, "A single weight value cannot be FSE-coded.");
    const uint32_t al = kWeightAccuracyMax;
    int16_t norm[kHuffMaxBits + 1];
    normalize(counts, max_symbol, static_cast<uint32_t>(n), al, norm);
    std::vector<uint8_t> out = write_ncount(norm, max_symbol, al);
    const std::vector<FseState> table = build_fse_table(norm, max_symbol, al);
    const uint32_t size = 1U << al;
    std::vector<std::vector<uint32_t>> states(max_symbol + 1);
    for (uint32_t u = 0; u < size; ++u) states[table[u].symbol].push_back(u);
    // Final state of each stream: one whose update reads >= 1 bit, so the
    // decoder overflows right after it.
    auto final_state = [&](uint32_t symbol) {
        for (uint32_t u : states[symbol])
            if (table[u].nbits > 0) return u;
        throw Error(NZ_ERUNTIME, "Weights cannot be FSE-coded.");
    };
    auto previous = [&](uint32_t symbol, uint32_t d, uint32_t* bits, uint32_t* nb) {
        for (uint32_t u : states[symbol]) {
            const uint32_t lo = table[u].base, span = 1U << table[u].nbits;
            if (d >= lo && d < lo + span) {
                *bits = d - lo;
                *nb = table[u].nbits;
                return u;
            }
        }
        throw Error(NZ_ERUNTIME, "FSE state search failed.");
    };
    // Stream of index i: i even -> state 1, i odd -> state 2.
    std::vector<std::pair<uint32_t, uint32_t>> update(n, {0, 0});  // (bits, nb) read after symbol i
    uint32_t d[2] = {0, 0};
    bool started[2] = {false, false};
    for (size_t k = n; k-- > 0;) {
        const int st = static_cast<int>(k & 1U);
        if (!started[st]) {
            d[st] = final_state(weights[k]);
            started[st] = true;
            continue;
        }
        uint32_t bits = 0, nb = 0;
        d[st] = previous(weights[k], d[st], &bits, &nb);
        update[k] = {bits, nb};
    }
    // Bits in decoding order: state 1, state 2, then the updates.
    std::vector<uint8_t> seq;
    auto push = [&](uint32_t v, uint32_t nb) {
        for (uint32_t i = nb; i-- > 0;) seq.push_back(static_cast<uint8_t>((v >> i) & 1U));
    };
    push(d[0], al);
    push(d[1], al);
    for (size_t k = 0; k + 2 < n; ++k) push(update[k].first, update[k].second);
    // Stream integer X = 1 << T | B with B's first-read bit most significant.
    const size_t t = seq.size();
    std::vector<uint8_t> stream((t + 1 + 7) / 8, 0);
    for (size_t i = 0; i < t; ++i) {
        const size_t p = t - 1 - i;
        stream[p / 8] |= static_cast<uint8_t>(seq[i] << (p % 8));
    }
    stream[t / 8] |= static_cast<uint8_t>(1U << (t % 8));
    out.insert(out.end(), stream.begin(), stream.end());
    return out;
}

// ---- Huffman lengths ----------------------------------------------------------

void limit_lengths(std::vector<uint32_t>& bl_count, uint32_t max_bits) {
    // ITU-T T.81 Annex K.3 (Figure K.3, "Adjust_BITS").
    for (uint32_t i = static_cast<uint32_t>(bl_count.size()) - 1; i > max_bits; --i) {
        while (bl_count[i] > 0) {
            uint32_t j = i - 2;
            while (bl_count[j] == 0) --j;
            bl_count[i] -= 2;
            bl_count[i - 1] += 1;
            bl_count[j + 1] += 2;
            bl_count[j] -= 1;
        }
    }
}

}  // namespace

void huffman_lengths(const uint64_t* counts, uint32_t nsym, uint32_t max_bits, uint8_t* lengths) {
    std::vector<uint32_t> present;
    for (uint32_t s = 0; s < nsym; ++s) {
        lengths[s] = 0;
        if (counts[s]) present.push_back(s);
    }
    if (present.size() < 2) throw Error(NZ_ERUNTIME, "Huff0 requires at least two symbols.");
    if (present.size() > (size_t{1} << max_bits))
        throw Error(NZ_ERUNTIME, "Huff0 max_bits cannot represent every observed symbol.");
    // Most frequent first; ties by symbol.
    std::sort(present.begin(), present.end(), [&](uint32_t a, uint32_t b) {
        return counts[a] != counts[b] ? counts[a] > counts[b] : a < b;
    });
    // Two-queue Huffman over leaves sorted by increasing weight.
    const size_t m = present.size();
    std::vector<uint64_t> weight(2 * m);
    std::vector<int32_t> parent(2 * m, -1);
    for (size_t i = 0; i < m; ++i) weight[i] = counts[present[m - 1 - i]];
    size_t leaf = 0, inner = m, inner_end = m;
    auto take = [&]() -> size_t {
        if (leaf < m && (inner == inner_end || weight[leaf] <= weight[inner])) return leaf++;
        return inner++;
    };
    for (size_t k = 0; k + 1 < m; ++k) {
        const size_t a = take(), b = take();
        weight[inner_end] = weight[a] + weight[b];
        parent[a] = parent[b] = static_cast<int32_t>(inner_end);
        ++inner_end;
    }
    std::vector<uint32_t> depth(inner_end, 0);
    for (size_t i = inner_end - 1; i-- > 0;) depth[i] = depth[static_cast<size_t>(parent[i])] + 1;
    uint32_t deepest = 0;
    for (size_t i = 0; i < m; ++i) deepest = std::max(deepest, depth[i]);
    std::vector<uint32_t> bl_count(std::max(deepest, max_bits) + 1, 0);
    for (size_t i = 0; i < m; ++i) ++bl_count[depth[i]];
    limit_lengths(bl_count, max_bits);
    // Shortest lengths to the most frequent symbols.
    size_t next = 0;
    for (uint32_t len = 1; len <= max_bits; ++len)
        for (uint32_t c = 0; c < bl_count[len]; ++c) lengths[present[next++]] = static_cast<uint8_t>(len);
}

size_t read_huff0_header(const uint8_t* src, size_t size, Huff0Table* table) {
    if (size < 1) throw Error(NZ_EVALUE, "Huff0 codebook header is empty.");
    uint8_t weights[256] = {};
    size_t n = 0, used = 0;
    const uint32_t head = src[0];
    if (head >= 128) {
        n = head - 127;
        used = 1 + (n + 1) / 2;
        if (used > size) throw Error(NZ_EVALUE, "Truncated Huff0 header.");
        for (size_t i = 0; i < n; ++i) {
            const uint8_t b = src[1 + i / 2];
            weights[i] = (i & 1) ? (b & 15U) : (b >> 4);
        }
    } else {
        if (head == 0 || 1 + head > size) throw Error(NZ_EVALUE, "Truncated Huff0 header.");
        n = decode_weights_fse(src + 1, head, weights, 255);
        used = 1 + head;
    }
    if (n == 0 || n > 255) throw Error(NZ_EVALUE, "Corrupt Huff0 header.");
    uint32_t total = 0;
    uint32_t rank[kHuffMaxBits + 2] = {};
    for (size_t i = 0; i < n; ++i) {
        if (weights[i] > kHuffMaxBits) throw Error(NZ_EVALUE, "Corrupt Huff0 header.");
        ++rank[weights[i]];
        total += (1U << weights[i]) >> 1;
    }
    if (total == 0) throw Error(NZ_EVALUE, "Corrupt Huff0 header.");
    const uint32_t table_log = highbit(total) + 1;
    if (table_log > kHuffMaxBits) throw Error(NZ_EVALUE, "Huff0 table log too large.");
    const uint32_t rest = (1U << table_log) - total;
    const uint32_t last = highbit(rest) + 1;
    if ((1U << highbit(rest)) != rest) throw Error(NZ_EVALUE, "Corrupt Huff0 header.");
    weights[n] = static_cast<uint8_t>(last);
    ++rank[last];
    if (rank[1] < 2 || (rank[1] & 1U)) throw Error(NZ_EVALUE, "Corrupt Huff0 header.");
    table->nsym = static_cast<uint32_t>(n + 1);
    table->table_log = table_log;
    std::memset(table->lengths, 0, sizeof(table->lengths));
    std::memset(table->values, 0, sizeof(table->values));
    uint32_t per_len[kHuffMaxBits + 2] = {};
    for (uint32_t s = 0; s < table->nsym; ++s) {
        const uint32_t w = weights[s];
        table->lengths[s] = static_cast<uint8_t>(w ? table_log + 1 - w : 0);
        ++per_len[table->lengths[s]];
    }
    // First code of each length, from the longest down: the running value is
    // halved whenever the length drops by one.
    uint32_t start[kHuffMaxBits + 2] = {};
    uint32_t code = 0;
    for (uint32_t len = table_log; len > 0; --len) {
        start[len] = code;
        code += per_len[len];
        code >>= 1;
    }
    for (uint32_t s = 0; s < table->nsym; ++s) {
        const uint32_t len = table->lengths[s];
        if (len) table->values[s] = static_cast<uint16_t>(start[len]++);
    }
    return used;
}

std::vector<uint8_t> write_huff0_header(const uint8_t* lengths, uint32_t nsym) {
    uint32_t last = 0, longest = 0;
    for (uint32_t s = 0; s < nsym; ++s) {
        if (lengths[s]) last = s;
        longest = std::max<uint32_t>(longest, lengths[s]);
    }
    if (longest == 0 || longest > kHuffMaxBits) throw Error(NZ_ERUNTIME, "Invalid Huff0 code lengths.");
    uint64_t kraft = 0;
    for (uint32_t s = 0; s < nsym; ++s)
        if (lengths[s]) kraft += uint64_t{1} << (longest - lengths[s]);
    if (kraft != (uint64_t{1} << longest)) throw Error(NZ_ERUNTIME, "Huff0 code lengths are incomplete.");
    std::vector<uint8_t> weights(last);
    for (uint32_t s = 0; s < last; ++s)
        weights[s] = static_cast<uint8_t>(lengths[s] ? longest + 1 - lengths[s] : 0);
    std::vector<uint8_t> header;
    try {
        const std::vector<uint8_t> fse = encode_weights_fse(weights.data(), weights.size());
        if (fse.size() > 1 && fse.size() < 128 && fse.size() < last / 2) {
            header.push_back(static_cast<uint8_t>(fse.size()));
            header.insert(header.end(), fse.begin(), fse.end());
            return header;
        }
    } catch (const Error&) {
    }
    if (last > 128) throw Error(NZ_ERUNTIME, "Huff0 cannot serialize this table.");
    header.push_back(static_cast<uint8_t>(127 + last));
    for (uint32_t s = 0; s < last; s += 2) {
        const uint8_t hi = weights[s];
        const uint8_t lo = s + 1 < last ? weights[s + 1] : 0;
        header.push_back(static_cast<uint8_t>((hi << 4) | lo));
    }
    return header;
}

}  // namespace nz

using nz::Error;

extern "C" {

int nz_export_code_table(const uint8_t* header, size_t header_size, const uint8_t* vocab,
                         size_t vocab_size, uint32_t max_bits, uint8_t* lengths_out,
                         uint64_t* values_out, uint32_t cap, uint32_t* nsym_out,
                         uint32_t* longest_out) {
    NZ_GUARD({
        if (!header || !lengths_out || !values_out || !nsym_out || !longest_out ||
            (vocab_size && !vocab))
            throw Error(NZ_EVALUE, "Null argument.");
        if (max_bits == 0 || max_bits > NZ_MAX_CODE_BITS)
            throw Error(NZ_EVALUE, "max_bits must be in [1, 56].");
        uint32_t longest = 0, nsym = 0;
        if (header_size >= 4 && std::memcmp(header, "NZM1", 4) == 0) {
            // neuralzip/native/mixed_huffman.h:5-57
            if (!(header_size >= 260 && header_size <= 514 && vocab_size == 2 * (header_size - 260)))
                throw Error(NZ_ERUNTIME, "Mixed table must contain 256 singletons and at most 254 pairs.");
            nsym = static_cast<uint32_t>(header_size - 4);
            if (cap < nsym) throw Error(NZ_EVALUE, "Output buffers are too small.");
            std::vector<uint16_t> pairs;
            for (size_t i = 0; i < vocab_size; i += 2)
                pairs.push_back(static_cast<uint16_t>(vocab[i] | (vocab[i + 1] << 8)));
            std::sort(pairs.begin(), pairs.end());
            if (std::adjacent_find(pairs.begin(), pairs.end()) != pairs.end())
                throw Error(NZ_ERUNTIME, "Duplicate mixed pair definition.");
            const std::vector<uint64_t> codes = nz::canonical_mixed_codes(header + 4, nsym);
            for (uint32_t s = 0; s < nsym; ++s) {
                lengths_out[s] = header[4 + s];
                values_out[s] = codes[s];
                longest = std::max<uint32_t>(longest, header[4 + s]);
            }
        } else {
            // neuralzip/native/codebooks.h:79-111 via RFC 8878 4.2.1.
            if (vocab_size) throw Error(NZ_ERUNTIME, "GPU export requires a singleton Huff0 table.");
            nz::Huff0Table table;
            nz::read_huff0_header(header, header_size, &table);
            if (table.table_log > NZ_MAX_SINGLETON_BITS)
                throw Error(NZ_ERUNTIME, "Huff0 codebook exceeds the requested max_bits limit.");
            nsym = 256;
            if (cap < nsym) throw Error(NZ_EVALUE, "Output buffers are too small.");
            for (uint32_t s = 0; s < 256; ++s) {
                lengths_out[s] = table.lengths[s];
                values_out[s] = table.values[s];
                longest = std::max<uint32_t>(longest, table.lengths[s]);
            }
        }
        if (longest > max_bits)
            throw Error(NZ_ERUNTIME, "GPU codebook exceeds the requested max_bits limit.");
        *nsym_out = nsym;
        *longest_out = longest;
    })
}

int nz_huff0_build(const uint64_t* counts, uint32_t max_bits, uint8_t* header_out, size_t cap,
                   size_t* size_out, uint8_t* lengths_out) {
    NZ_GUARD({
        if (!counts || !header_out || !size_out) throw Error(NZ_EVALUE, "Null argument.");
        if (max_bits < 1 || max_bits > 12) throw Error(NZ_EVALUE, "max_bits must be in [1, 12].");
        uint8_t lengths[256];
        nz::huffman_lengths(counts, 256, max_bits, lengths);
        // A 1-bit code beside 12-bit codes has weight 12. zstd's decoder
        // reads that weight from 4-bit direct weights but rejects it in
        // FSE-coded weights (measured with libzstd 1.5.5; its weight
        // decoder takes weights up to 11 there), so such a table is built
        // with 11 bits instead and stays readable by zstd's Huff0.
        uint32_t shortest = 255, longest = 0;
        for (uint32_t s = 0; s < 256; ++s)
            if (lengths[s]) {
                shortest = std::min<uint32_t>(shortest, lengths[s]);
                longest = std::max<uint32_t>(longest, lengths[s]);
            }
        if (longest == 12 && shortest == 1) nz::huffman_lengths(counts, 256, 11, lengths);
        const std::vector<uint8_t> header = nz::write_huff0_header(lengths, 256);
        if (header.size() > cap) throw Error(NZ_EVALUE, "Header buffer is too small.");
        std::memcpy(header_out, header.data(), header.size());
        *size_out = header.size();
        if (lengths_out) std::memcpy(lengths_out, lengths, 256);
    })
}

int nz_huff0_read(const uint8_t* header, size_t size, uint8_t* lengths_out, uint16_t* values_out,
                  uint32_t* table_log, size_t* consumed) {
    NZ_GUARD({
        if (!header || !lengths_out) throw Error(NZ_EVALUE, "Null argument.");
        nz::Huff0Table table;
        const size_t used = nz::read_huff0_header(header, size, &table);
        std::memcpy(lengths_out, table.lengths, 256);
        if (values_out) std::memcpy(values_out, table.values, sizeof(table.values));
        if (table_log) *table_log = table.table_log;
        if (consumed) *consumed = used;
    })
}

}  // extern "C"
