// Internal declarations shared by the host translation units of libnzb200.
#pragma once

#include "nz_b200.h"

#include <cstdint>
#include <functional>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

namespace nz {

// Error carrying an nz_status; the C ABI turns it into a return code and a
// thread-local message.
struct Error : std::runtime_error {
    int status;
    Error(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

int fail(int status, const std::string& message);

struct Codebook {
    uint32_t nsym = 0;
    uint32_t longest = 0;
    uint32_t tree_nodes = 0;
    uint32_t table_words = 0;  // leading lut words the kernel reads
    std::vector<uint8_t> lengths;
    std::vector<uint64_t> codes;
    std::vector<uint16_t> vocab;        // pair k -> first | second << 8
    std::vector<uint16_t> pair_tokens;  // (first | second << 8) -> 256 + k, 0 = none
    std::vector<uint32_t> lut;          // NZ_LUT_WORDS words (tile kernel table)
    // Host single-token table for the CPU codecs: for a 12-bit window,
    // bytes (bits 0..15) | byte count << 16 | code length << 20, or a
    // suffix-tree node index with a zero byte count for longer codes.
    std::vector<uint32_t> single;

    void build(const uint8_t* lengths, const uint64_t* values, uint32_t nsym,
               const uint8_t* vocab, uint32_t vocab_size);
    void build_lut();
};

std::vector<uint64_t> canonical_mixed_codes(const uint8_t* lengths, uint32_t nsym);

void check_dtype(const nz_dtype& dt);
void pack_bound(uint64_t numel, uint32_t longest, uint64_t* bits_words, uint64_t* lens_count,
                uint64_t* tiles);
void pack_chunk(const Codebook& cb, const uint8_t* raw, uint64_t numel, const nz_dtype& dt,
                uint32_t* bits, uint64_t bits_cap, uint16_t* lens, uint64_t lens_cap,
                uint32_t* tile_off, uint64_t tiles_cap, uint8_t* const* lanes,
                uint64_t* bit_length, uint64_t* words_used);
uint64_t mixed_encode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t cap);
void mixed_decode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t expected);
uint64_t huff0_encode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t cap);
void huff0_decode(const Codebook& cb, const uint8_t* data, uint64_t size, uint8_t* out, uint64_t count);

void run_jobs(uint64_t count, int threads, const std::function<void(uint64_t)>& job);

// Huff0 table headers (RFC 8878 section 4.2.1): weights -> code lengths and
// the canonical values the format prescribes.
struct Huff0Table {
    uint32_t table_log = 0;
    uint32_t nsym = 0;  // symbols described (max symbol value + 1)
    uint8_t lengths[256] = {};
    uint16_t values[256] = {};
};
// Parses a header; returns the number of header bytes consumed.
size_t read_huff0_header(const uint8_t* src, size_t size, Huff0Table* table);
// Serializes code lengths (<= 12 bits, complete code) as a Huff0 header.
std::vector<uint8_t> write_huff0_header(const uint8_t* lengths, uint32_t nsym);
// Length-limited Huffman code lengths for a 256-bin histogram.
void huffman_lengths(const uint64_t* counts, uint32_t nsym, uint32_t max_bits, uint8_t* lengths);

}  // namespace nz

// Body of a C-ABI entry point: runs the statements, returns NZ_OK, and turns
// exceptions into a status code plus the thread-local message.
#define NZ_GUARD(...)                                        \
    try {                                                    \
        __VA_ARGS__;                                         \
        return NZ_OK;                                        \
    } catch (const nz::Error& e) {                           \
        return nz::fail(e.status, e.what());                 \
    } catch (const std::bad_alloc&) {                        \
        return nz::fail(NZ_ERUNTIME, "Out of host memory."); \
    } catch (const std::exception& e) {                      \
        return nz::fail(NZ_ERUNTIME, e.what());              \
    }
