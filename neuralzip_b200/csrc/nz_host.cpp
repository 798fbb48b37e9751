// Host half of libnzb200: codebooks, decode tables and the tile-layout packer.
//
// Reference behaviour this file re-implements (paths inside the reference
// project):
//   * canonical mixed codes and their validation:
//     neuralzip/native/mixed_huffman.h:5-57 (make_mixed_table);
//   * singleton code export from a Huff0 header:
//     neuralzip/native/codebooks.h:79-111 and gpu_layout.h:7-17, restated
//     from RFC 8878 section 4.2.1 in nz_huff0.cpp;
//   * the lane split / reorder of encode_gpu_layout:
//     neuralzip/native/gpu_layout.h:185-241;
//   * the greedy pair parse: gpu_layout.h:232-239, mixed_huffman.h:85-94.
// The GPU layout itself is new (see nz_b200.h): independent 256-element
// sub-streams per warp lane instead of 64-bit segments with restart gaps.

#include "nz_b200.h"
#include "nz_internal.h"

#include <algorithm>
#include <functional>
#include <atomic>
#include <cstring>
#include <exception>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

namespace nz {

thread_local std::string g_last_error;

int fail(int status, const std::string& message) {
    g_last_error = message;
    return status;
}

// ---------------------------------------------------------------------------
// Codebook

namespace {

struct TrieNode {
    int child[2] = {-1, -1};
    int symbol = -1;
    int suffix = -1;  // index in the suffix tree (internal nodes at depth >= 12)
};

}  // namespace

void Codebook::build(const uint8_t* in_lengths, const uint64_t* in_values,
                     uint32_t in_nsym, const uint8_t* in_vocab,
                     uint32_t vocab_size) {
    if (vocab_size % 2 != 0 || vocab_size > 2 * NZ_MAX_PAIRS)
        throw Error(NZ_EVALUE, "Invalid mixed pair vocabulary.");
    if (in_nsym != 256 + vocab_size / 2)
        throw Error(NZ_EVALUE, "The GPU alphabet does not match its pair vocabulary.");
    nsym = in_nsym;
    lengths.assign(in_lengths, in_lengths + nsym);
    vocab.clear();
    for (uint32_t i = 0; i < vocab_size; i += 2)
        vocab.push_back(static_cast<uint16_t>(in_vocab[i] | (in_vocab[i + 1] << 8)));
    {
        std::vector<uint16_t> sorted = vocab;
        std::sort(sorted.begin(), sorted.end());
        if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end())
            throw Error(NZ_EVALUE, "Duplicate mixed pair definition.");
    }
    longest = 0;
    for (uint8_t length : lengths) longest = std::max<uint32_t>(longest, length);
    const uint32_t limit = vocab.empty() ? NZ_MAX_SINGLETON_BITS : NZ_MAX_CODE_BITS;
    if (longest > limit)
        throw Error(NZ_EVALUE, "The GPU codebook exceeds its decoder's code-length limit.");
    if (longest == 0)
        throw Error(NZ_EVALUE, "A GPU codebook needs at least one coded symbol.");
    if (in_values != nullptr) {
        codes.assign(in_values, in_values + nsym);
    } else {
        codes = canonical_mixed_codes(lengths.data(), nsym);
    }
    for (uint32_t s = 0; s < nsym; ++s) {
        if (lengths[s] && lengths[s] < 64 && (codes[s] >> lengths[s]) != 0)
            throw Error(NZ_EVALUE, "A code value does not fit its code length.");
    }
    pair_tokens.assign(vocab.empty() ? 0 : 65536, 0);
    for (size_t i = 0; i < vocab.size(); ++i)
        pair_tokens[vocab[i]] = static_cast<uint16_t>(256 + i);
    build_lut();
}

// Canonical code assignment of make_mixed_table: symbols ordered by
// (length, symbol), codes counting up from zero and shifted left whenever
// the length grows (neuralzip/native/mixed_huffman.h:22-57).
std::vector<uint64_t> canonical_mixed_codes(const uint8_t* lengths, uint32_t nsym) {
    std::vector<uint32_t> order(nsym);
    for (uint32_t i = 0; i < nsym; ++i) {
        if (lengths[i] == 0 || lengths[i] > NZ_MAX_CODE_BITS)
            throw Error(NZ_ERUNTIME, "Mixed code lengths must be in [1, 56].");
        order[i] = i;
    }
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        return lengths[a] < lengths[b];
    });
    std::vector<uint64_t> codes(nsym, 0);
    uint64_t code = 0;
    uint32_t previous = 0;
    for (uint32_t symbol : order) {
        const uint32_t length = lengths[symbol];
        code <<= (length - previous);
        if (code >= (uint64_t{1} << length))
            throw Error(NZ_ERUNTIME, "Oversubscribed mixed Huffman table.");
        codes[symbol] = code;
        ++code;
        previous = length;
    }
    if (code != (uint64_t{1} << previous))
        throw Error(NZ_ERUNTIME, "Incomplete mixed Huffman table.");
    return codes;
}

// Multi-symbol decode table: NZ_LUT_ENTRIES entries of two words, then the
// canonical long-code tables, then the suffix tree. Entry for a 12-bit
// window (word 0 / word 1):
//   w0 bits 0..4   window bits the decoded tokens consume (1..12)
//   w0 bits 5..7   zero
//   w0 bits 8..15  eight times the number of decoded bytes (8..32), the
//                  amount the kernel's byte queue grows by
//   w1             up to four decoded bytes (first byte lowest)
// A window whose first code is longer than 12 bits instead has zero in
// bits 0..15 of w0, and in bits 16..31 either
//   * the shortest code length under that 12-bit prefix (bit 31 clear):
//     the code is then found by comparing the 32-bit window with the
//     canonical limits at NZ_LUT_CANON (words 0..31: the largest
//     left-justified window of each length, words 32..63: rank offset of
//     each length, words 64..: the leaf word of each long code in code
//     order); used when every long code is at most 31 bits and the long
//     codes are numbered in canonical order (consecutive values per length,
//     lengths growing with the value); or
//   * bit 31 set and the index of the trie node reached after 12 bits in
//     bits 16..30: the kernel walks the suffix tree at word NZ_LUT_TREE,
//     two words per node (child for bit 0, child for bit 1).
// A leaf word has its byte count in bits 5..7 and its bytes in bits 8..23;
// any other tree child holds the next node index in bits 8..31.
void Codebook::build_lut() {
    std::vector<TrieNode> trie(1);
    for (uint32_t s = 0; s < nsym; ++s) {
        const uint32_t length = lengths[s];
        if (!length) continue;
        int node = 0;
        for (int bit = static_cast<int>(length) - 1; bit >= 0; --bit) {
            if (trie[node].symbol >= 0)
                throw Error(NZ_EVALUE, "Huffman prefix collision.");
            const int branch = static_cast<int>((codes[s] >> bit) & 1U);
            if (trie[node].child[branch] < 0) {
                trie[node].child[branch] = static_cast<int>(trie.size());
                trie.emplace_back();
            }
            node = trie[node].child[branch];
        }
        if (trie[node].symbol >= 0 || trie[node].child[0] >= 0 || trie[node].child[1] >= 0)
            throw Error(NZ_EVALUE, "Huffman prefix collision.");
        trie[node].symbol = static_cast<int>(s);
    }
    // Number the internal nodes at depth >= 12 (breadth first from depth 12).
    std::vector<int> frontier{0};
    for (uint32_t depth = 0; depth < NZ_LUT_BITS && !frontier.empty(); ++depth) {
        std::vector<int> next;
        for (int node : frontier) {
            if (trie[node].symbol >= 0) continue;
            for (int b = 0; b < 2; ++b)
                if (trie[node].child[b] >= 0) next.push_back(trie[node].child[b]);
        }
        frontier.swap(next);
    }
    tree_nodes = 0;
    std::vector<int> queue;
    for (int node : frontier)
        if (trie[node].symbol < 0) queue.push_back(node);
    for (size_t head = 0; head < queue.size(); ++head) {
        const int node = queue[head];
        trie[node].suffix = static_cast<int>(tree_nodes++);
        for (int b = 0; b < 2; ++b) {
            const int child = trie[node].child[b];
            if (child >= 0 && trie[child].symbol < 0) queue.push_back(child);
        }
    }
    if (tree_nodes > NZ_TREE_MAX_NODES)
        throw Error(NZ_EVALUE, "The Huffman codebook needs too many long-code nodes.");

    auto token_bytes = [&](int symbol, uint32_t* value) -> uint32_t {
        if (symbol < 256) {
            *value = static_cast<uint32_t>(symbol);
            return 1;
        }
        *value = vocab[static_cast<size_t>(symbol - 256)];
        return 2;
    };

    single.assign(NZ_LUT_ENTRIES, 0);
    for (uint32_t prefix = 0; prefix < NZ_LUT_ENTRIES; ++prefix) {
        int node = 0;
        uint32_t depth = 0;
        while (trie[node].symbol < 0 && depth < NZ_LUT_BITS) {
            node = trie[node].child[(prefix >> (NZ_LUT_BITS - 1 - depth)) & 1U];
            ++depth;
            if (node < 0) throw Error(NZ_EVALUE, "The Huffman codebook does not cover every prefix.");
        }
        if (trie[node].symbol >= 0) {
            uint32_t value = 0;
            const uint32_t count = token_bytes(trie[node].symbol, &value);
            single[prefix] = value | (count << 16) | (depth << 20);
        } else {
            single[prefix] = static_cast<uint32_t>(trie[node].suffix);
        }
    }

    lut.assign(NZ_LUT_WORDS, 0);
    // Canonical long-code tables: codes longer than 12 bits, in the order of
    // their left-justified values.
    std::vector<uint32_t> long_syms;
    for (uint32_t s = 0; s < nsym; ++s)
        if (lengths[s] > NZ_LUT_BITS) long_syms.push_back(s);
    auto left = [&](uint32_t s) { return codes[s] << (64 - lengths[s]); };
    std::sort(long_syms.begin(), long_syms.end(), [&](uint32_t a, uint32_t b) { return left(a) < left(b); });
    bool canonical = !long_syms.empty() && longest <= NZ_CANON_MAX_BITS && long_syms.size() <= NZ_CANON_TOKENS;
    for (size_t i = 1; canonical && i < long_syms.size(); ++i) {
        const uint32_t a = long_syms[i - 1], b = long_syms[i];
        if (lengths[b] < lengths[a] || (lengths[b] == lengths[a] && codes[b] != codes[a] + 1)) canonical = false;
    }
    std::vector<uint32_t> shortest_under(NZ_LUT_ENTRIES, 0);
    if (canonical) {
        uint32_t* limit = lut.data() + NZ_LUT_CANON;
        uint32_t* offset = limit + 32;
        uint32_t* token = limit + 64;
        // limit[L]: the largest 32-bit window decoded by a code of length <= L
        // (the next code's left-justified start minus one).
        for (uint32_t L = 0; L < 32; ++L) limit[L] = 0xFFFFFFFFU;
        for (size_t i = 0; i < long_syms.size(); ++i) {
            const uint32_t s = long_syms[i], L = lengths[s];
            const uint32_t prefix = static_cast<uint32_t>(codes[s] >> (L - NZ_LUT_BITS));
            if (!shortest_under[prefix] || L < shortest_under[prefix]) shortest_under[prefix] = L;
            if (i == 0 || lengths[long_syms[i - 1]] != L)
                offset[L] = static_cast<uint32_t>(i) - static_cast<uint32_t>(codes[s]);
            if (i + 1 < long_syms.size() && lengths[long_syms[i + 1]] != L) {
                const uint32_t next_start = static_cast<uint32_t>(left(long_syms[i + 1]) >> 32);
                for (uint32_t k = L; k < lengths[long_syms[i + 1]]; ++k) limit[k] = next_start - 1U;
            }
            uint32_t value = 0;
            const uint32_t count = token_bytes(static_cast<int>(s), &value);
            token[i] = (value << 8) | (count << 5);
        }
    }
    for (uint32_t prefix = 0; prefix < NZ_LUT_ENTRIES; ++prefix) {
        uint32_t pos = 0, nbytes = 0, bytes = 0;
        uint32_t meta = 0;
        while (pos < NZ_LUT_BITS) {
            int node = 0;
            uint32_t depth = 0;
            while (trie[node].symbol < 0 && pos + depth < NZ_LUT_BITS) {
                const uint32_t bit = (prefix >> (NZ_LUT_BITS - 1 - (pos + depth))) & 1U;
                node = trie[node].child[bit];
                ++depth;
                if (node < 0)
                    throw Error(NZ_EVALUE, "The Huffman codebook does not cover every prefix.");
            }
            if (trie[node].symbol < 0) {
                if (pos == 0)
                    meta = canonical ? shortest_under[prefix] << 16
                                     : 0x80000000U | (static_cast<uint32_t>(trie[node].suffix) << 16);
                break;
            }
            uint32_t value = 0;
            const uint32_t count = token_bytes(trie[node].symbol, &value);
            if (nbytes + count > 4) break;
            bytes |= value << (8 * nbytes);
            nbytes += count;
            pos += depth;
        }
        if (nbytes) meta = pos | ((8U * nbytes) << 8);
        lut[2 * prefix] = meta;
        lut[2 * prefix + 1] = bytes;
    }
    // Suffix tree below depth 12.
    for (size_t i = 0; i < trie.size(); ++i) {
        const TrieNode& node = trie[i];
        if (node.suffix < 0) continue;
        for (int b = 0; b < 2; ++b) {
            const int child = node.child[b];
            if (child < 0)
                throw Error(NZ_EVALUE, "The Huffman codebook does not cover every prefix.");
            uint32_t word;
            if (trie[child].symbol >= 0) {
                uint32_t value = 0;
                const uint32_t count = token_bytes(trie[child].symbol, &value);
                const uint32_t length = lengths[static_cast<size_t>(trie[child].symbol)];
                (void)length;
                word = (value << 8) | (count << 5);
            } else {
                word = static_cast<uint32_t>(trie[child].suffix) << 8;
            }
            lut[NZ_LUT_TREE + 2 * static_cast<uint32_t>(node.suffix) + b] = word;
        }
    }
    table_words = long_syms.empty() ? NZ_LUT_CANON
                  : canonical       ? NZ_LUT_TREE
                                    : NZ_LUT_TREE + 2 * tree_nodes;
}

// ---------------------------------------------------------------------------
// Lane split (neuralzip/native/gpu_layout.h:200-231)

namespace {

struct LaneMasks {
    uint32_t mant, sign, exp;
};

inline LaneMasks masks_of(const nz_dtype& dt) {
    return {(1U << dt.mant_bits) - 1U, 1U << dt.mant_bits,
            ((1U << dt.exp_bits) - 1U) << (dt.mant_bits + 1U)};
}

// One byte lane of the reordered elements: a loop per lane, with nothing
// but the element's load, reorder and shift in it, so that it vectorizes.
template <unsigned E>
void split_one(const uint8_t* __restrict__ raw, uint64_t numel, const nz_dtype& dt, const LaneMasks& m,
               unsigned lane, uint8_t* __restrict__ out) {
    const unsigned shift = 8U * lane;
    if (!dt.reorder) {
        for (uint64_t i = 0; i < numel; ++i) out[i] = raw[i * E + lane];
        return;
    }
    // Elements are read at their own width (a 2-byte copy into a 32-bit
    // word does not vectorize).
    using Word = typename std::conditional<E == 2, uint16_t, uint32_t>::type;
    const Word mant = static_cast<Word>(m.mant), sign = static_cast<Word>(m.sign), exp = static_cast<Word>(m.exp);
    const unsigned exp_bits = dt.exp_bits;
    for (uint64_t i = 0; i < numel; ++i) {
        Word value;
        std::memcpy(&value, raw + i * E, E);
        const Word v = static_cast<Word>((value & mant) | ((value >> exp_bits) & sign) |
                                         (static_cast<Word>(value << 1U) & exp));
        out[i] = static_cast<uint8_t>(v >> shift);
    }
}

// Extracts the selected lane into `symbols` and the other lanes into
// lanes[lane] (when non-null).
template <unsigned E>
void split(const uint8_t* raw, uint64_t numel, const nz_dtype& dt, uint8_t* symbols,
           uint8_t* const* lanes) {
    const LaneMasks m = masks_of(dt);
    for (unsigned lane = 0; lane < E; ++lane) {
        uint8_t* out = lane == dt.stream_id ? symbols : (lanes ? lanes[lane] : nullptr);
        if (out) split_one<E>(raw, numel, dt, m, lane, out);
    }
}

void split_lanes(const uint8_t* raw, uint64_t numel, const nz_dtype& dt, uint8_t* symbols,
                 uint8_t* const* lanes) {
    if (dt.elem_size == 2) split<2>(raw, numel, dt, symbols, lanes);
    else split<4>(raw, numel, dt, symbols, lanes);
}

// MSB-first bit writer into 32-bit words (bit 31 of a word is earliest).
struct BitWriter {
    uint32_t* words;
    uint64_t cap;
    uint64_t used = 0;
    uint64_t acc = 0;
    uint32_t pending = 0;
    uint64_t bits = 0;

    void put32(uint64_t value, uint32_t length) {  // length <= 32
        acc = (acc << length) | value;
        pending += length;
        bits += length;
        if (pending >= 32) {
            pending -= 32;
            if (used >= cap) throw Error(NZ_EOVERFLOW, "Tile bitstream exceeds its buffer.");
            words[used++] = static_cast<uint32_t>(acc >> pending);
            acc &= (pending ? ((uint64_t{1} << pending) - 1U) : 0U);
        }
    }
    void put(uint64_t code, uint32_t length) {
        if (length > 32) {
            put32(code >> 32, length - 32);
            put32(code & 0xFFFFFFFFULL, 32);
        } else {
            put32(code, length);
        }
    }
    void finish(uint64_t pad_words) {
        if (pending) {
            if (used >= cap) throw Error(NZ_EOVERFLOW, "Tile bitstream exceeds its buffer.");
            words[used++] = static_cast<uint32_t>(acc << (32 - pending));
            acc = 0;
            pending = 0;
        }
        uint64_t target = used + pad_words;
        target = (target + 3U) & ~uint64_t{3};
        if (target > cap) throw Error(NZ_EOVERFLOW, "Tile bitstream exceeds its buffer.");
        while (used < target) words[used++] = 0;
    }
};

}  // namespace

void check_dtype(const nz_dtype& dt) {
    if (dt.elem_size != 2 && dt.elem_size != 4)
        throw Error(NZ_EVALUE, "GPU element_size must be 2 or 4.");
    if (!(dt.mant_bits < 8U * dt.elem_size && dt.exp_bits > 0 && dt.exp_bits < 8U * dt.elem_size &&
          dt.mant_bits + dt.exp_bits + 1U == 8U * dt.elem_size))
        throw Error(NZ_EVALUE, "Sign, exponent and mantissa fields must fill the element.");
    if (dt.stream_id >= dt.elem_size) throw Error(NZ_EVALUE, "GPU stream_id is out of range.");
}

void pack_bound(uint64_t numel, uint32_t longest, uint64_t* bits_words, uint64_t* lens_count,
                uint64_t* tiles) {
    const uint64_t t = (numel + NZ_TILE_ELEMS - 1) / NZ_TILE_ELEMS;
    const uint64_t total_bits = numel * static_cast<uint64_t>(longest);
    *tiles = t;
    *lens_count = t * NZ_TILE_LANES;
    *bits_words = ((total_bits + 31) / 32 + NZ_BITS_PAD_WORDS + 3) & ~uint64_t{3};
}

void pack_chunk(const Codebook& cb, const uint8_t* raw, uint64_t numel, const nz_dtype& dt,
                uint32_t* bits, uint64_t bits_cap, uint16_t* lens, uint64_t lens_cap,
                uint32_t* tile_off, uint64_t tiles_cap, uint8_t* const* lanes,
                uint64_t* bit_length, uint64_t* words_used) {
    check_dtype(dt);
    if (numel > static_cast<uint64_t>(INT32_MAX))
        throw Error(NZ_EOVERFLOW, "Element count exceeds the int32 CUDA decoder ABI limit.");
    uint64_t need_words, need_lens, need_tiles;
    pack_bound(numel, cb.longest, &need_words, &need_lens, &need_tiles);
    if (lens_cap < need_lens || tiles_cap < need_tiles)
        throw Error(NZ_EVALUE, "Tile metadata buffers are too small.");
    thread_local std::vector<uint8_t> symbols;
    symbols.resize(numel);
    split_lanes(raw, numel, dt, symbols.data(), lanes);

    BitWriter out{bits, bits_cap};
    const bool pairs = !cb.pair_tokens.empty();
    const uint64_t lanes_total = need_lens;
    for (uint64_t s = 0; s < lanes_total; ++s) {
        if (s % NZ_TILE_LANES == 0) {
            if (out.bits > 0xFFFFFFFFULL)
                throw Error(NZ_EOVERFLOW, "A group bitstream exceeds 2^32 bits.");
            tile_off[s / NZ_TILE_LANES] = static_cast<uint32_t>(out.bits);
        }
        const uint64_t begin = std::min<uint64_t>(s * NZ_LANE_ELEMS, numel);
        const uint64_t end = std::min<uint64_t>(begin + NZ_LANE_ELEMS, numel);
        const uint64_t start_bits = out.bits;
        for (uint64_t i = begin; i < end;) {
            uint32_t token = symbols[i];
            if (pairs && i + 1 < end) {
                const uint16_t pair = cb.pair_tokens[token | (static_cast<uint32_t>(symbols[i + 1]) << 8)];
                if (pair) token = pair;
            }
            const uint32_t length = cb.lengths[token];
            if (length == 0)
                throw Error(NZ_ERUNTIME, "Symbol " + std::to_string(token) + " at index " +
                                             std::to_string(i) + " has no codebook entry.");
            out.put(cb.codes[token], length);
            i += token >= 256 ? 2 : 1;
        }
        lens[s] = static_cast<uint16_t>(out.bits - start_bits);
    }
    if (out.bits > 0xFFFFFFFFULL) throw Error(NZ_EOVERFLOW, "A group bitstream exceeds 2^32 bits.");
    *bit_length = out.bits;
    out.finish(NZ_BITS_PAD_WORDS);
    *words_used = out.used;
}

void run_jobs(uint64_t count, int threads, const std::function<void(uint64_t)>& job) {
    if (count == 0) return;
    unsigned hw = std::thread::hardware_concurrency();
    uint64_t workers = threads > 0 ? static_cast<uint64_t>(threads) : (hw ? hw : 1);
    workers = std::max<uint64_t>(1, std::min<uint64_t>(workers, count));
    std::atomic<uint64_t> next{0};
    auto worker = [&]() {
        for (;;) {
            const uint64_t i = next.fetch_add(1, std::memory_order_relaxed);
            if (i >= count) return;
            job(i);
        }
    };
    if (workers == 1) {
        worker();
        return;
    }
    std::vector<std::thread> pool;
    pool.reserve(workers - 1);
    for (uint64_t w = 1; w < workers; ++w) pool.emplace_back(worker);
    worker();
    for (auto& t : pool) t.join();
}

}  // namespace nz

// ---------------------------------------------------------------------------
// C ABI

using nz::Error;
using nz::fail;


extern "C" {

int nz_last_error(char* buf, size_t cap) {
    if (!buf || cap == 0) return NZ_EVALUE;
    const std::string& m = nz::g_last_error;
    const size_t n = std::min(cap - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = 0;
    return NZ_OK;
}

int nz_abi_version(void) { return 4; }

int nz_codebook_create(const uint8_t* lengths, const uint64_t* values, uint32_t nsym,
                       const uint8_t* vocab, uint32_t vocab_size, nz_codebook** out) {
    NZ_GUARD({
        if (!lengths || !out || (vocab_size && !vocab))
            throw Error(NZ_EVALUE, "Null codebook argument.");
        auto* cb = new nz::Codebook();
        try {
            cb->build(lengths, values, nsym, vocab, vocab_size);
        } catch (...) {
            delete cb;
            throw;
        }
        *out = reinterpret_cast<nz_codebook*>(cb);
    })
}

int nz_codebook_destroy(nz_codebook* codebook) {
    delete reinterpret_cast<nz::Codebook*>(codebook);
    return NZ_OK;
}

int nz_codebook_info(const nz_codebook* codebook, uint32_t* longest, uint32_t* tree_nodes) {
    NZ_GUARD({
        if (!codebook) throw Error(NZ_EVALUE, "Null codebook.");
        const auto* cb = reinterpret_cast<const nz::Codebook*>(codebook);
        if (longest) *longest = cb->longest;
        if (tree_nodes) *tree_nodes = cb->tree_nodes;
    })
}

int nz_codebook_table_words(const nz_codebook* codebook, uint32_t* words) {
    NZ_GUARD({
        if (!codebook || !words) throw Error(NZ_EVALUE, "Null codebook argument.");
        *words = reinterpret_cast<const nz::Codebook*>(codebook)->table_words;
    })
}

int nz_codebook_lut(const nz_codebook* codebook, uint32_t* lut, uint32_t cap_words) {
    NZ_GUARD({
        if (!codebook || !lut) throw Error(NZ_EVALUE, "Null codebook argument.");
        if (cap_words < NZ_LUT_WORDS) throw Error(NZ_EVALUE, "LUT buffer is too small.");
        const auto* cb = reinterpret_cast<const nz::Codebook*>(codebook);
        std::memcpy(lut, cb->lut.data(), NZ_LUT_WORDS * sizeof(uint32_t));
    })
}

int nz_pack_bound(uint64_t numel, uint32_t longest, uint64_t* bits_words, uint64_t* lens_count,
                  uint64_t* tiles) {
    NZ_GUARD({
        if (!bits_words || !lens_count || !tiles) throw Error(NZ_EVALUE, "Null output.");
        if (longest == 0 || longest > NZ_MAX_CODE_BITS)
            throw Error(NZ_EVALUE, "GPU Huffman code length must be in [1, 56].");
        nz::pack_bound(numel, longest, bits_words, lens_count, tiles);
    })
}

int nz_pack_chunk(const nz_codebook* codebook, const uint8_t* raw, uint64_t numel,
                  const nz_dtype* dt, uint32_t* bits, uint64_t bits_cap_words, uint16_t* lens,
                  uint64_t lens_cap, uint32_t* tile_off, uint64_t tiles_cap,
                  uint8_t* const* lanes, uint64_t* bit_length_out, uint64_t* words_used_out) {
    NZ_GUARD({
        if (!codebook || !dt || !bits || !lens || !tile_off || !lanes || !bit_length_out ||
            !words_used_out || (numel && !raw))
            throw Error(NZ_EVALUE, "Null packer argument.");
        nz::pack_chunk(*reinterpret_cast<const nz::Codebook*>(codebook), raw, numel, *dt, bits,
                       bits_cap_words, lens, lens_cap, tile_off, tiles_cap, lanes,
                       bit_length_out, words_used_out);
    })
}

int nz_pack_many(nz_pack_job* jobs, uint64_t count, const nz_dtype* dt, int32_t threads) {
    NZ_GUARD({
        if ((count && !jobs) || !dt) throw Error(NZ_EVALUE, "Null packer argument.");
        nz::check_dtype(*dt);
        std::vector<std::string> errors(count);
        nz::run_jobs(count, threads, [&](uint64_t i) {
            nz_pack_job& job = jobs[i];
            job.status = NZ_OK;
            try {
                if (!job.codebook) throw Error(NZ_EVALUE, "Null codebook in pack job.");
                nz::pack_chunk(*reinterpret_cast<const nz::Codebook*>(job.codebook), job.raw,
                               job.numel, *dt, job.bits, job.bits_cap_words, job.lens,
                               job.lens_cap, job.tile_off, job.tiles_cap, job.lanes,
                               &job.bit_length, &job.words_used);
            } catch (const Error& e) {
                job.status = e.status;
                errors[i] = e.what();
            } catch (const std::exception& e) {
                job.status = NZ_ERUNTIME;
                errors[i] = e.what();
            }
        });
        for (uint64_t i = 0; i < count; ++i)
            if (jobs[i].status != NZ_OK) throw Error(jobs[i].status, errors[i]);
    })
}

int nz_split_lanes(const uint8_t* raw, uint64_t numel, const nz_dtype* dt, uint8_t* const* lanes) {
    NZ_GUARD({
        if (!dt || !lanes || (numel && !raw)) throw Error(NZ_EVALUE, "Null argument.");
        nz::check_dtype(*dt);
        if (!lanes[dt->stream_id]) throw Error(NZ_EVALUE, "The selected lane's buffer is null.");
        // Large inputs are split in blocks on the host's threads.
        constexpr uint64_t kBlock = uint64_t{1} << 20;
        const uint64_t blocks = (numel + kBlock - 1) / kBlock;
        nz::run_jobs(blocks, 0, [&](uint64_t b) {
            const uint64_t first = b * kBlock, n = std::min<uint64_t>(kBlock, numel - first);
            uint8_t* part[4] = {nullptr, nullptr, nullptr, nullptr};
            for (uint32_t lane = 0; lane < dt->elem_size; ++lane)
                part[lane] = lanes[lane] ? lanes[lane] + first : nullptr;
            nz::split_lanes(raw + first * dt->elem_size, n, *dt, part[dt->stream_id], part);
        });
    })
}

}  // extern "C"
