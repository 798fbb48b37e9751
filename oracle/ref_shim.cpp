// C entry points over the reference's own native code, compiled from the
// reference sources where they lie (oracle/Makefile passes their directory
// with -I). TEST INFRASTRUCTURE ONLY: tests pin the oracle restatement
// against these functions, and bench.py's reference arm times the
// reference's own CPU decode of mixed chunks through ref_decode_chunks.
//
// Reference code reached from here (paths inside the reference project):
//   make_mixed_table            neuralzip/native/mixed_huffman.h:5-83
//   encode_gpu_layout           neuralzip/native/gpu_layout.h:185-241
//   encode/decode_mixed_block   neuralzip/native/mixed_huffman.h:127-240
//   restore_mixed_stream_chunk  neuralzip/native/common.h:198-257
//   run_parallel_jobs           neuralzip/native/common.h:134-185
#include "ref_stub.hpp"

namespace {
namespace nb = stub_nb;
#include "common.h"
#include "mixed_huffman.h"

struct StubExportedTable {
    std::array<std::uint8_t, 256> code_lengths{};
    std::array<std::uint16_t, 256> code_values{};
};
// Huff0 headers need zstd, which the reference tree does not vendor.
StubExportedTable export_code_table_from_header(const std::uint8_t*, Py_ssize_t, unsigned) {
    throw std::runtime_error("Huff0 headers are unavailable in this build.");
}

#include "gpu_layout.h"

thread_local std::string g_error;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

std::shared_ptr<MixedHuffmanTable> explicit_table(const std::uint8_t* lengths,
                                                  const std::uint64_t* codes, std::uint32_t nsym,
                                                  const std::uint8_t* vocab, std::size_t vsize) {
    auto table = std::make_shared<MixedHuffmanTable>();
    table->lengths.assign(lengths, lengths + nsym);
    table->codes.assign(codes, codes + nsym);
    if (vsize) {
        table->pair_tokens.assign(65536, 0);
        for (std::size_t i = 0; i < vsize; i += 2) {
            const auto pair = static_cast<std::uint16_t>(vocab[i] | (vocab[i + 1] << 8));
            table->pair_tokens[pair] = static_cast<std::uint16_t>(256 + i / 2);
            table->vocabulary.push_back(pair);
        }
    }
    return table;
}

}  // namespace

extern "C" {

int ref_last_error(char* buf, std::size_t cap) {
    const std::size_t n = std::min(cap - 1, g_error.size());
    std::memcpy(buf, g_error.data(), n);
    buf[n] = 0;
    return 0;
}

// Canonical codes of a mixed header ("NZM1" + lengths) with its vocab.
int ref_mixed_codes(const std::uint8_t* header, std::size_t size, const std::uint8_t* vocab,
                    std::size_t vsize, std::uint64_t* codes_out) {
    return guarded([&] {
        auto table = make_mixed_table(header, size, vocab, vsize, true);
        std::copy(table->codes.begin(), table->codes.end(), codes_out);
    });
}

// The reference GPU layout of one chunk. Buffers must be large enough
// (bitstream: numel * 7 bytes; gaps: ceil(bytes / 4096) * 512; positions:
// blocks + 1; raw lanes: numel each, NULL for the selected lane).
int ref_gpu_layout(const std::uint8_t* raw, std::size_t numel, unsigned elem_size, int reorder,
                   unsigned mant, unsigned expb, unsigned stream_id, const std::uint8_t* lengths,
                   const std::uint64_t* codes, std::uint32_t nsym, const std::uint8_t* vocab,
                   std::size_t vsize, std::uint8_t* bitstream, std::size_t* n_bytes,
                   std::uint8_t* gaps, std::size_t* n_gaps, std::uint32_t* positions,
                   std::size_t* n_positions, std::uint64_t* bit_length, unsigned* max_bits,
                   std::uint8_t** raw_lanes) {
    return guarded([&] {
        auto table = explicit_table(lengths, codes, nsym, vocab, vsize);
        const bool aligned = reorder && expb == 8 && stream_id == elem_size - 1U;
        GPULayoutEncoding enc;
        if (elem_size == 2)
            enc = aligned ? encode_gpu_layout<2, true>(raw, numel, *table, stream_id, reorder, mant, expb)
                          : encode_gpu_layout<2, false>(raw, numel, *table, stream_id, reorder, mant, expb);
        else
            enc = aligned ? encode_gpu_layout<4, true>(raw, numel, *table, stream_id, reorder, mant, expb)
                          : encode_gpu_layout<4, false>(raw, numel, *table, stream_id, reorder, mant, expb);
        std::memcpy(bitstream, enc.symbols.bitstream.data(), enc.symbols.bitstream.size());
        *n_bytes = enc.symbols.bitstream.size();
        std::memcpy(gaps, enc.symbols.packed_gaps.data(), enc.symbols.packed_gaps.size());
        *n_gaps = enc.symbols.packed_gaps.size();
        std::copy(enc.symbols.output_positions.begin(), enc.symbols.output_positions.end(), positions);
        *n_positions = enc.symbols.output_positions.size();
        *bit_length = enc.symbols.bit_length;
        *max_bits = enc.symbols.max_bits;
        for (unsigned lane = 0; lane < elem_size; ++lane)
            if (lane != stream_id && raw_lanes[lane])
                std::memcpy(raw_lanes[lane], enc.raw_streams[lane].data(), numel);
    });
}

int ref_mixed_encode(const std::uint8_t* data, std::size_t size, const std::uint8_t* header,
                     std::size_t hsize, const std::uint8_t* vocab, std::size_t vsize,
                     std::uint8_t* out, std::size_t cap, std::size_t* out_size) {
    return guarded([&] {
        auto table = make_mixed_table(header, hsize, vocab, vsize, true);
        *out_size = encode_mixed_block_into(data, size, *table, out, cap);
    });
}

int ref_mixed_decode(const std::uint8_t* data, std::size_t size, const std::uint8_t* header,
                     std::size_t hsize, const std::uint8_t* vocab, std::size_t vsize,
                     std::uint8_t* out, std::size_t expected) {
    return guarded([&] {
        auto table = make_mixed_table(header, hsize, vocab, vsize, false);
        decode_mixed_block_into(data, size, *table, out, expected);
    });
}

// A decode table made once (make_mixed_table with encoding = false).
void* ref_mixed_decodebook(const std::uint8_t* header, std::size_t hsize, const std::uint8_t* vocab,
                           std::size_t vsize) {
    try {
        return new std::shared_ptr<const MixedHuffmanTable>(
            make_mixed_table(header, hsize, vocab, vsize, false));
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

void ref_mixed_decodebook_free(void* book) {
    delete static_cast<std::shared_ptr<const MixedHuffmanTable>*>(book);
}

// The reference's CPU decode path for a batch of mixed-coded chunks
// (decode_queue.h semantics): each job decodes one selected-lane frame with
// decode_mixed_block_into and merges the lanes with
// restore_mixed_stream_chunk, on run_parallel_jobs' pool.
struct RefChunk {
    const std::uint8_t* payload;
    std::uint64_t payload_size;
    void* book;                      // from ref_mixed_decodebook
    const std::uint8_t* lanes[4];    // raw lanes; the selected entry is ignored
    std::uint8_t* out;               // numel * elem_size bytes
    std::uint64_t numel;
    std::uint32_t elem_size;
    std::uint32_t reorder;
    std::uint32_t stream_id;
    std::uint32_t pad;
};

int ref_decode_chunks(const RefChunk* chunks, std::size_t count, int threads) {
    std::vector<std::string> errors(count);
    std::size_t total = 0;
    for (std::size_t i = 0; i < count; ++i) total += chunks[i].numel * chunks[i].elem_size;
    run_parallel_jobs(count, total, threads, [&](std::size_t i) {
        const RefChunk& c = chunks[i];
        try {
            thread_local std::vector<std::uint8_t> scratch;
            scratch.resize(c.numel);
            const auto& table = **static_cast<std::shared_ptr<const MixedHuffmanTable>*>(c.book);
            decode_mixed_block_into(c.payload, c.payload_size, table, scratch.data(), c.numel);
            std::array<const std::uint8_t*, 4> lanes{};
            for (unsigned l = 0; l < c.elem_size; ++l)
                lanes[l] = l == c.stream_id ? scratch.data() : c.lanes[l];
            MixedStreamDecodeTensor request;
            request.element_size = static_cast<int>(c.elem_size);
            request.bit_reorder = c.reorder != 0;
            request.output_data = c.out;
            restore_mixed_stream_chunk(request, lanes, 0, c.numel);
        } catch (const std::exception& e) {
            errors[i] = e.what();
        }
    });
    for (const auto& e : errors)
        if (!e.empty()) {
            g_error = e;
            return 1;
        }
    return 0;
}

}  // extern "C"
