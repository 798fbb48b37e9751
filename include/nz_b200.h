/*
 * nz_b200.h — C ABI of the B200-native NeuralZip decompression path.
 *
 * One shared library (libnzb200.so) exports every symbol declared here. All
 * signatures use plain pointers, sizes and fixed-layout structs; no torch or
 * Python types cross the boundary. Every entry point returns an int status
 * (NZ_OK = 0); on failure a thread-local message is available through
 * nz_last_error(). The status maps onto the exception classes the reference
 * raises for the same conditions (neuralzip/native/common.h:59-63 `require<>`
 * plus nanobind's translation): NZ_EVALUE -> ValueError, NZ_ETYPE ->
 * TypeError, NZ_EOVERFLOW -> OverflowError, NZ_ERUNTIME -> RuntimeError.
 *
 * Layout produced by the packer and consumed by the decode kernel
 * ("tile layout"): a group is one source chunk of one tensor's selected byte
 * lane (neuralzip/gpu/inference.py:302-330). Its elements are cut into
 * sub-streams of NZ_LANE_ELEMS consecutive elements; NZ_TILE_LANES
 * sub-streams form one tile, decoded by one warp (one sub-stream per lane).
 * Sub-streams are Huffman bitstreams packed back to back, MSB-first, stored
 * as 32-bit words whose bit 31 is the earliest bit. `lens[s]` holds the bit
 * length of sub-stream s and `tile_off[t]` the bit offset of tile t's first
 * sub-stream; a lane finds its start with a warp scan of its tile's lens.
 * A pair token never straddles two sub-streams. The bitstream starts on a
 * 16-byte boundary and ends with at least NZ_BITS_PAD_WORDS zero words (a
 * lane reads up to three words past its sub-stream). The non-selected byte lanes are
 * stored raw, one byte per element, 16-byte aligned.
 */
#ifndef NZ_B200_H
#define NZ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NZ_LANE_ELEMS 256u
#define NZ_TILE_LANES 32u
#define NZ_TILE_ELEMS (NZ_LANE_ELEMS * NZ_TILE_LANES)
#define NZ_LUT_BITS 12u
#define NZ_LUT_ENTRIES (1u << NZ_LUT_BITS)
#define NZ_TREE_MAX_NODES 512u
/* Decode-table layout (words): NZ_LUT_ENTRIES two-word entries, the
 * canonical long-code tables (limits, rank offsets, tokens) at
 * NZ_LUT_CANON, then the binary suffix tree at NZ_LUT_TREE. */
#define NZ_LUT_CANON (2u * NZ_LUT_ENTRIES)
#define NZ_CANON_MAX_BITS 31u
#define NZ_CANON_TOKENS 512u
#define NZ_CANON_WORDS (64u + NZ_CANON_TOKENS)
#define NZ_LUT_TREE (NZ_LUT_CANON + NZ_CANON_WORDS)
#define NZ_LUT_WORDS (NZ_LUT_TREE + 2u * NZ_TREE_MAX_NODES)
#define NZ_MAX_CODE_BITS 56u
#define NZ_MAX_SINGLETON_BITS 12u
#define NZ_MAX_PAIRS 254u
#define NZ_BITS_PAD_WORDS 16u
#define NZ_RAW_LUT 0xFFFFFFFFu

enum nz_status {
    NZ_OK = 0,
    NZ_EVALUE = 1,
    NZ_ETYPE = 2,
    NZ_EOVERFLOW = 3,
    NZ_ERUNTIME = 4,
    NZ_ECUDA = 5
};

/* Byte-lane layout of one floating format; mirrors DTypeSpec
 * (neuralzip/dtypes.py:8-50) and the packer arguments of encode_gpu_tensor
 * (neuralzip/native/binding_helpers.h:125-195). */
typedef struct nz_dtype {
    uint32_t elem_size;  /* 2 or 4 */
    uint32_t reorder;    /* 1: sign moved below the exponent (bf16, fp32) */
    uint32_t mant_bits;  /* 7 bf16, 10 fp16, 23 fp32 */
    uint32_t exp_bits;   /* 8 bf16/fp32, 5 fp16 */
    uint32_t stream_id;  /* byte lane holding the Huffman-coded symbols */
} nz_dtype;

/* Opaque host codebook: canonical codes, pair lookup and decode table. */
typedef struct nz_codebook nz_codebook;

/* ---- host: codebooks -------------------------------------------------- */

/* Replaces export_code_table (neuralzip/native/binding_helpers.h:103-123,
 * module.cpp:57-62). `header` is either a mixed table ("NZM1" + 256..510
 * code lengths, neuralzip/native/mixed_huffman.h:5-83) or a Huff0 table
 * header (RFC 8878 section 4.2.1). Writes one length and one canonical
 * code value per symbol (cap >= 256 + vocab_size / 2). */
int nz_export_code_table(const uint8_t* header, size_t header_size,
                         const uint8_t* vocab, size_t vocab_size,
                         uint32_t max_bits, uint8_t* lengths_out,
                         uint64_t* values_out, uint32_t cap,
                         uint32_t* nsym_out, uint32_t* longest_out);

/* Builds a codebook from explicit per-symbol code lengths and values (the
 * GPUCodebook inputs, neuralzip/gpu/inference.py:20-27). `values` may be
 * NULL, in which case canonical mixed-table codes are assigned
 * (mixed_huffman.h:5-83 semantics). nsym = 256 + vocab_size / 2. */
int nz_codebook_create(const uint8_t* lengths, const uint64_t* values,
                       uint32_t nsym, const uint8_t* vocab,
                       uint32_t vocab_size, nz_codebook** out);
int nz_codebook_destroy(nz_codebook* codebook);
/* Longest code length and the number of suffix-tree nodes. */
int nz_codebook_info(const nz_codebook* codebook, uint32_t* longest,
                     uint32_t* tree_nodes);
/* Decode table of the tile kernel (replaces GPUCodebook.decode_lut,
 * neuralzip/gpu/inference.py:28-75). Writes NZ_LUT_WORDS words. */
int nz_codebook_lut(const nz_codebook* codebook, uint32_t* lut,
                    uint32_t cap_words);
/* Leading words of that table the kernel reads (and stages): the entries,
 * plus the long-code tables when some code is longer than 12 bits. Part of
 * GPUCodebook.decode_lut's size (neuralzip/gpu/inference.py:52-72). */
int nz_codebook_table_words(const nz_codebook* codebook, uint32_t* words);

/* Setup-time singleton tables (replaces build_codebook_from_counts ->
 * HUF_buildCTable_wksp + HUF_writeCTable_wksp, neuralzip/native/
 * codebooks.h:20-39, binding_helpers.h:68-90): Huffman code lengths limited
 * to max_bits (<= 12) for a 256-bin histogram, serialized as an RFC 8878
 * Huff0 header. lengths_out (256 bytes) may be NULL. */
int nz_huff0_build(const uint64_t* counts, uint32_t max_bits, uint8_t* header_out,
                   size_t cap, size_t* size_out, uint8_t* lengths_out);
/* Reads a Huff0 header (replaces HUF_readCTable, codebooks.h:60-68):
 * 256 code lengths, canonical values (may be NULL), table log and the
 * number of header bytes consumed. */
int nz_huff0_read(const uint8_t* header, size_t size, uint8_t* lengths_out,
                  uint16_t* values_out, uint32_t* table_log, size_t* consumed);

/* ---- host: packer ----------------------------------------------------- */

/* Capacities for nz_pack_chunk: bitstream words (padding included),
 * lens entries and tile count for `numel` elements whose longest code is
 * `longest` bits. */
int nz_pack_bound(uint64_t numel, uint32_t longest, uint64_t* bits_words,
                  uint64_t* lens_count, uint64_t* tiles);

/* Replaces encode_gpu_tensor / encode_gpu_layout
 * (neuralzip/native/binding_helpers.h:125-195, gpu_layout.h:62-241).
 * Splits `raw` (numel elements of dt->elem_size bytes) into byte lanes,
 * writes the non-selected lanes to lanes[lane] (entries for the selected
 * lane are ignored and may be NULL) and Huffman-codes the selected lane
 * into the tile layout. Thread-safe; releases nothing it did not take. */
int nz_pack_chunk(const nz_codebook* codebook, const uint8_t* raw,
                  uint64_t numel, const nz_dtype* dt, uint32_t* bits,
                  uint64_t bits_cap_words, uint16_t* lens,
                  uint64_t lens_cap, uint32_t* tile_off, uint64_t tiles_cap,
                  uint8_t* const* lanes, uint64_t* bit_length_out,
                  uint64_t* words_used_out);

/* Many chunks on a host thread pool (replaces the per-chunk Python loop of
 * neuralzip/gpu/inference.py:308-330). Job i packs raws[i] with
 * codebooks[i] into its own caller buffers; threads = 0 uses every core. */
typedef struct nz_pack_job {
    const nz_codebook* codebook;
    const uint8_t* raw;
    uint64_t numel;
    uint32_t* bits;
    uint64_t bits_cap_words;
    uint16_t* lens;
    uint64_t lens_cap;
    uint32_t* tile_off;
    uint64_t tiles_cap;
    uint8_t* lanes[4];
    uint64_t bit_length;  /* out */
    uint64_t words_used;  /* out */
    int32_t status;       /* out */
    int32_t pad;
} nz_pack_job;
int nz_pack_many(nz_pack_job* jobs, uint64_t count, const nz_dtype* dt,
                 int32_t threads);

/* Raw fragment (no codebook, neuralzip/gpu/inference.py:319-324): applies
 * the reorder and writes every byte lane, the selected one included; a
 * NULL entry of lanes[] other than the selected lane's skips that lane.
 * Large inputs are split on the host's threads. */
int nz_split_lanes(const uint8_t* raw, uint64_t numel, const nz_dtype* dt,
                   uint8_t* const* lanes);

/* ---- host: CPU storage codec (storage format v2 payloads) ----------- */

/* Greedy pair parse counts (neuralzip/native/mixed_huffman.h:85-115):
 * counts[token] += occurrences; counts has 256 + vocab_size / 2 entries. */
int nz_count_tokens(const uint8_t* data, uint64_t size, const uint8_t* vocab,
                    uint32_t vocab_size, uint64_t* counts);
/* Exponent-field histograms (256 bins) of consecutive `step`-element chunks
 * of raw elements, added into histograms[chunk * 256 + exponent]; the
 * per-chunk distributions setup clusters (neuralzip/setup.py:91-141). */
int nz_exponent_histograms(const uint8_t* raw, uint64_t numel, const nz_dtype* dt,
                           uint64_t step, uint64_t* histograms);
/* Setup-time clustering of chunk exponent distributions (restates the
 * rule of neuralzip/setup.py:91-141): chunk i (in checkpoint order, a
 * normalized `bins`-bin distribution of weight weights[i]) joins the
 * nearest cluster of its class by base-2 Jensen-Shannon distance (ties: the
 * earliest) when that distance is <= threshold or forced[i] is set, else it
 * opens a cluster; share = 0 opens one cluster per chunk. Centroids are
 * weight-averaged and updated after each assignment. Writes assign[count],
 * the centroids (cap_clusters x bins) and the cluster count. */
int nz_cluster_chunks(const double* distributions, const double* weights,
                      const int32_t* classes, const uint8_t* forced,
                      uint64_t count, uint32_t bins, double threshold,
                      int32_t share, uint32_t* assign, double* centroids,
                      uint64_t cap_clusters, uint64_t* n_clusters);
/* Mixed frame (mixed_huffman.h:127-178). *written = 0 when the frame does
 * not fit `cap`; out may be NULL to measure only. */
int nz_mixed_encode(const nz_codebook* codebook, const uint8_t* data,
                    uint64_t size, uint8_t* out, uint64_t cap, uint64_t* written);
/* Inverse of nz_mixed_encode with the validation of mixed_huffman.h:180-240. */
int nz_mixed_decode(const nz_codebook* codebook, const uint8_t* frame,
                    uint64_t size, uint8_t* out, uint64_t expected);
/* Huff0 4-stream block of a singleton codebook (RFC 8878 section 4.2.2;
 * replaces HUF_compress4X_usingCTable, codebooks.h:131-141). *written = 0
 * when it does not fit; out may be NULL to measure only. */
int nz_huff0_encode(const nz_codebook* codebook, const uint8_t* data,
                    uint64_t size, uint8_t* out, uint64_t cap, uint64_t* written);
/* Replaces HUF_decompress4X_usingDTable (codebooks.h:156-206). */
int nz_huff0_decode(const nz_codebook* codebook, const uint8_t* block,
                    uint64_t size, uint8_t* out, uint64_t count);

/* Storage v2 decode on the host cores. Replaces the reference's CPU decode
 * queue, decompress_mixed_streams_many (neuralzip/native/decode_queue.h:
 * 1-113: per chunk, decode each byte lane, then restore_mixed_stream_chunk,
 * common.h:198-257, merges the lanes and undoes the sign/exponent reorder)
 * and its worker pool (common.h:134-185). One piece is one source chunk of
 * one tensor: `count` elements whose byte lanes are `lanes[0 ..
 * dt.elem_size)` in lane order, each raw (payload_size == count), a Huff0
 * 4-stream block (count <= 128 KiB) or a mixed frame, decoded with its
 * codebook (NULL for raw). The piece's element bytes are written to `out`.
 * Pieces run on `threads` workers (0: the host cores, at most 16, as the
 * reference's pool). A corrupt or inconsistent piece makes the call fail
 * with the message of the lowest failing piece; other pieces may have been
 * written. */
#define NZ_CHUNK_RAW 0u
#define NZ_CHUNK_HUFF0 1u
#define NZ_CHUNK_MIXED 2u
typedef struct nz_storage_lane {
    const uint8_t* payload;
    uint64_t payload_size;
    const nz_codebook* codebook;
    uint32_t mode;       /* NZ_CHUNK_* */
    uint32_t reserved;   /* zero */
} nz_storage_lane;
typedef struct nz_storage_piece {
    const nz_storage_lane* lanes;
    uint8_t* out;
    uint64_t count;
    nz_dtype dt;         /* elem_size, reorder, mant_bits, exp_bits (stream_id unused) */
    uint32_t reserved;   /* zero */
} nz_storage_piece;
int nz_storage_decode(const nz_storage_piece* pieces, uint64_t count, int32_t threads);

/* ---- device: decode --------------------------------------------------- */

/* One group of a decode launch (device-resident array). Pointers are
 * device addresses. lut == NZ_RAW_LUT marks a raw group whose selected
 * lane is lanes[stream_id]. */
typedef struct nz_group {
    uint64_t bits;       /* const uint32_t*: tile-layout bitstream */
    uint64_t lens;       /* const uint16_t*: bit length per sub-stream */
    uint64_t tile_off;   /* const uint32_t*: bit offset per tile */
    uint64_t lanes[4];   /* const uint8_t*: byte lanes by lane index */
    uint64_t out;        /* element words */
    uint32_t numel;
    uint32_t lut;
} nz_group;

/* One tile of work: (group index, tile index within the group). */
typedef struct nz_work {
    uint32_t group;
    uint32_t tile;
} nz_work;

/* Element layouts the decode kernel writes (nz_cta.layout): bf16 (sign
 * moved under the exponent, byte 1 coded), fp16 (no reorder, byte 1 coded)
 * and fp32 (sign moved, byte 3 coded); neuralzip/dtypes.py:23-83. */
#define NZ_LAYOUT_BF16 0u
#define NZ_LAYOUT_FP16 1u
#define NZ_LAYOUT_FP32 2u

/* One CTA: a contiguous range of works sharing one decode table and one
 * element layout. With launch scratch (nz_launch.scratch), the CTAs that
 * name the same queue share their range: each warp claims the range's
 * next work from the queue's counter, so those CTAs finish together. */
typedef struct nz_cta {
    uint32_t lut;        /* index into luts, or NZ_RAW_LUT */
    uint32_t begin;
    uint32_t end;
    uint16_t lut_words;  /* words of the table to stage (<= NZ_LUT_WORDS) */
    uint16_t layout;     /* NZ_LAYOUT_* of every group of the range */
    uint32_t queue;      /* counter index in the launch scratch (< queues) */
    uint32_t reserved;   /* zero */
} nz_cta;

/* Replaces CuPyDecoder.decode_batch (neuralzip/gpu/decoder.py:193-208) and
 * the kernel launch of decode_batched (neuralzip/gpu/cuda/decode.cu:323).
 * One launch decodes groups of any mix of layouts (each CTA names its
 * own). All arrays are device-resident; `luts` is a device array of device
 * pointers to NZ_LUT_WORDS-word tables, each 16-byte aligned (a CTA
 * stages its table with one bulk copy). `status` (device int32) receives a
 * nonzero code if a corrupt table made a lane give up (2), a CTA named an
 * unknown layout (3) or, in a queue launch, a queue index not below
 * `queues` (4), or if a table copy did not complete within the kernel's
 * bounded wait (5; that CTA decodes nothing); it is only written on
 * error. Asynchronous on
 * `cuda_stream` (a cudaStream_t, NULL = legacy default stream).
 * warps_per_cta: 4, 8, 16 or 24 (0 = default, 8); 24-warp CTAs fill an SM
 * alone, 8- and 4-warp CTAs run two and three to an SM. */
typedef struct nz_launch {
    uint32_t warps_per_cta;
    uint32_t n_ctas;
    uint64_t groups;   /* const nz_group* */
    uint64_t works;    /* const nz_work* */
    uint64_t ctas;     /* const nz_cta* */
    uint64_t luts;     /* const uint64_t* */
    uint64_t status;   /* int32_t* */
    /* uint32_t[queues + 1], zero before the first launch that uses it; the
     * launch's last CTA sets it back to zero. 0: no queues, each CTA
     * decodes its own range (also when queues is 0). Launches that share
     * scratch must not overlap on the GPU. */
    uint64_t scratch;
    uint32_t queues;
    uint32_t reserved; /* zero */
} nz_launch;
int nz_decode_launch(const nz_launch* launch, void* cuda_stream);

/* nz_decode_launch with work queues whose counters live in this library's
 * own device memory, for callers that cannot allocate device memory: a
 * plugin inside a serving process whose memory pool has reserved all of
 * HBM, or a host path that must not call cudaMalloc because it may
 * synchronize the device. It allocates nothing; the caller still passes
 * every input and output. launch->scratch is ignored and launch->queues
 * must be at most 1024 (NZ_EVALUE otherwise; 0 gives the fixed-range
 * launch); the CTAs name their queues as for nz_decode_launch. The counters (4 KB per GPU that loads the
 * library, held until the process exits) are looked up and cleared by the
 * first call on each device, which should therefore come before any stream
 * capture; each launch's last CTA sets them back to zero. All calls on
 * one GPU share them, so calls that overlap on that GPU (streams with no
 * order between them) race and must not be issued. No counterpart in the
 * reference, whose decoder allocates its own buffers
 * (neuralzip/gpu/decoder.py). */
int nz_decode_launch_noalloc(const nz_launch* launch, void* cuda_stream);

/* Several launches (e.g. one per dtype of a block) as one step on
 * `cuda_stream`: the launch with the most warps goes first on that stream,
 * the others are enqueued at once on low-priority side streams of this
 * library (their CTAs take SMs as the first launch's CTAs finish, and run
 * side by side), and the stream waits for all of them. No reference
 * counterpart (the reference launches each layout in turn,
 * neuralzip/gpu/inference.py:491-493). */
int nz_decode_launch_many(const nz_launch* launches, uint32_t count,
                          void* cuda_stream);
/* Resident CTAs per SM of the decode kernel at warps_per_cta (the CUDA
 * occupancy calculator on the current device; no reference counterpart:
 * the reference sizes its grid per group, decoder.py:89-119). */
int nz_decode_occupancy(uint32_t warps_per_cta, uint32_t* ctas_per_sm);
/* Dynamic shared memory one CTA of nz_decode_launch uses. */
int nz_decode_smem_bytes(uint32_t warps_per_cta, uint32_t* bytes);
/* Words of a tile's bitstream a warp copies into shared memory at
 * warps_per_cta (956, 1960, 1332, 1292 for 24, 16, 8, 4 warps): from the
 * 16-byte boundary at or below the tile's first bit through at least 12
 * words past the word of its last one. A larger tile is read from global
 * memory,
 * slower. No reference counterpart (decode.cu reads global memory). */
int nz_decode_tile_words(uint32_t warps_per_cta, uint32_t* words);

/* ---- host: decode schedule ----------------------------------------------- */

/* The runtime's per-block decode as one C call per forward pre-hook.
 * Replaces NeuralZipRuntime._decode_block / _install's hooks
 * (neuralzip/gpu/inference.py:476-493), which decode each block on the
 * current stream right before it runs; the schedule adds units of
 * consecutive blocks per launch and, with depth > 1, an overlapped decode
 * on `side_stream` into depth rotating workspace slots (unit u uses slot
 * u % depth), ordered against the compute stream by CUDA events only.
 * `launches` holds the nz_launch descriptors of all units, unit u owning
 * [unit_first[u], unit_first[u + 1]); the device arrays they point to must
 * outlive the schedule. Create it with the device of the launches current.
 * A schedule is not thread-safe: one forward at a time. */
typedef struct nz_schedule nz_schedule;
int nz_schedule_create(const nz_launch* launches, const uint32_t* unit_first,
                       uint32_t n_units, uint32_t depth, void* side_stream,
                       nz_schedule** out);
int nz_schedule_destroy(nz_schedule* schedule);
/* Forward pre-hook of a block of `unit` (is_head: its first block): waits
 * for the unit's side-stream decode, or decodes the unit on compute_stream
 * when none is pending and the slot does not hold it (always for a head);
 * a head then starts the side-stream decode of the following units whose
 * slots are free. */
int nz_schedule_enter(nz_schedule* schedule, uint32_t unit, uint32_t is_head,
                      void* compute_stream);
/* Decodes a whole unit on `stream` after every pending side decode. */
int nz_schedule_decode_unit(nz_schedule* schedule, uint32_t unit, void* stream);
/* Makes `stream` wait for every pending side decode. */
int nz_schedule_drain(nz_schedule* schedule, void* stream);
/* Records what a unit's slot holds after a decode done outside the
 * schedule: the whole unit (whole = 1) or only part of it (0). */
int nz_schedule_mark(nz_schedule* schedule, uint32_t unit, uint32_t whole);

/* ---- errors ------------------------------------------------------------ */

/* Copies the calling thread's last error message (NUL-terminated). */
int nz_last_error(char* buf, size_t cap);
/* ABI version of this header, for loaders. */
int nz_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NZ_B200_H */
