// Device half of libnzb200: the tile decode kernel for sm_100a.
//
// Replaces decode_batched and its helpers (neuralzip/gpu/cuda/decode.cu:
// 32-381). What it computes is the same: for every group, the selected byte
// lane is Huffman-decoded (singleton or pair tokens, codes up to 56 bits),
// merged with the raw byte lanes, the sign/exponent reorder of
// neuralzip/dtypes.py:23-45 is undone, and the element words are written
// (decode.cu:83-127). How it computes it is different:
//   * one warp decodes one tile of 32 independent 256-element sub-streams,
//     one per lane; a lane finds its start bit with a warp scan of the
//     stored sub-stream lengths, so there is no counting pass, no block
//     prefix scan and no __syncthreads in the decode loop (the reference
//     decodes every segment twice and scans with two block barriers,
//     decode.cu:129-175, 207-255);
//   * the warp copies its tile's bitstream into shared memory (cp.async)
//     and its lanes refill their bit windows from there (the reference's
//     threads read their segments from global memory);
//   * the decode table lives in shared memory (staged once per CTA) and one
//     8-byte lookup of the 12-bit window yields up to four output bytes (two
//     pair tokens); codes of 13..31 bits are resolved from canonical limits
//     in the same table, longer ones through a suffix tree
//     (decode.cu:41-60 reads its table through __ldg, one token per probe,
//     and walks long codes bit by bit);
//   * decoded bytes are staged per warp, 128 elements per lane at a time,
//     and merged with the raw lanes through 8-byte loads and 16-byte stores
//     that are contiguous across the warp (decode.cu:83-100 loads and
//     stores one element at a time);
//   * one CTA per SM (24 warps); the CTAs of one decode table can share its
//     tiles through an atomic work queue, so that they finish together
//     (the reference launches one grid per group layout, sized per group).

#include "nz_b200.h"
#include "nz_internal.h"

#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

namespace {

constexpr uint32_t kRoundElems = 128;                      // per lane per staging round
constexpr uint32_t kRounds = NZ_LANE_ELEMS / kRoundElems;  // 2
constexpr uint32_t kStageStride = kRoundElems / 4 + 1;     // words per staged row (odd: no conflicts)
constexpr uint32_t kStageWordsPerWarp = NZ_TILE_LANES * kStageStride;
// A CTA's shared memory holds the decode table, per warp the staging rows
// plus a copy of the warp's current tile bitstream, and the mbarrier the
// table copy completes on (kBarWords). CTAs of 24 and 16 warps run one to
// an SM, of 8 and 4 warps two and three; each width gets the largest
// bitstream copy (a multiple of four words) that keeps that many CTAs
// resident: 956, 1960, 1332 and 1292 words.
constexpr uint32_t kSmemPerSm = 233472;     // 228 KB
constexpr uint32_t kSmemPerBlock = 232448;  // 227 KB opt-in limit
constexpr uint32_t kSmemReserved = 1024;    // per resident CTA
constexpr uint32_t kBarWords = 4;           // one 8-byte mbarrier, kept 16-byte aligned
__host__ __device__ constexpr uint32_t ctas_per_sm(uint32_t nw) { return nw >= 16 ? 1U : (nw >= 8 ? 2U : 3U); }
__host__ __device__ constexpr uint32_t bit_buf_words(uint32_t nw) {
    return (((kSmemPerSm / ctas_per_sm(nw) - kSmemReserved < kSmemPerBlock
                  ? kSmemPerSm / ctas_per_sm(nw) - kSmemReserved
                  : kSmemPerBlock) /
                 4U -
             NZ_LUT_WORDS - kBarWords) /
                nw -
            kStageWordsPerWarp) &
           ~3U;
}
__host__ __device__ constexpr uint32_t warp_words(uint32_t nw) { return kStageWordsPerWarp + bit_buf_words(nw); }
static_assert(bit_buf_words(24) == 956 && bit_buf_words(16) == 1960 && bit_buf_words(8) == 1332 &&
                  bit_buf_words(4) == 1292,
              "bitstream copy per warp");
constexpr uint32_t kLanesPerRow = kRoundElems / 8;          // merge: 8 elements per lane
constexpr uint32_t kRowsPerPass = 32 / kLanesPerRow;
constexpr uint32_t kMergePasses = NZ_TILE_LANES / kRowsPerPass;
constexpr uint32_t kTreeMask = NZ_TREE_MAX_NODES - 1;
constexpr uint32_t kMaxTreeDepth = NZ_MAX_CODE_BITS - NZ_LUT_BITS;
constexpr int32_t kStatusCorruptTable = 2;

// Polls of a bounded mbarrier wait: far beyond any copy's latency (each
// poll may also suspend the thread for a while), yet finite.
constexpr uint32_t kMaxBarrierPolls = 1U << 22;
constexpr int32_t kStatusCopyTimeout = 5;

__device__ __forceinline__ void mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One thread: copies `bytes` (a multiple of 16, both addresses 16-byte
// aligned) from this GPU's global memory into this CTA's shared memory with
// the bulk-copy (TMA) engine; the copy completes on `bar`. No multicast.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Waits for phase `parity` of `bar`; false after kMaxBarrierPolls polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMaxBarrierPolls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Streaming 8-byte load of a raw lane: read once, kept out of L1.
__device__ __forceinline__ uint2 ldg_u2(const void* p) {
    uint2 v;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// Asks L2 to fetch [p, p + bytes) ahead of use; p is 16-byte aligned and
// bytes is rounded down to a multiple of 16 (a hint: nothing is written).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    bytes &= ~15U;
    if (bytes)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Streaming 16-byte store of decoded elements (evict-first in L2: they are
// not read again by this kernel, and L2 keeps the prefetched inputs instead).
__device__ __forceinline__ void stg_u4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// MSB-first window over 32-bit words (bit 31 earliest). The valid bits are
// the top `avail` bits of hi:lo and everything below them is zero. The next
// word is requested one refill ahead (pf). kShared: the words come from the
// warp's shared-memory copy of its tile (32-bit addresses, ld.shared);
// otherwise from global memory, for a tile larger than that copy. Lanes
// refill at different lookups, and a load's register is tracked for the
// whole warp, so a refill waits for the load other lanes issued just
// before; from shared memory that wait is short. The refill stays a
// branch: a form without one reads pf on every lookup and so waits for its
// load there. All shifts are 32-bit funnel shifts.
template <bool kShared>
struct Window {
    uint32_t hi, lo, avail, pf;
    uint32_t saddr;        // shared: byte address of the next word
    const uint32_t* gsrc;  // global: the next word
    __device__ __forceinline__ uint32_t next() {
        if constexpr (kShared) {
            uint32_t v;
            asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(saddr));
            saddr += 4U;
            return v;
        } else {
            return __ldg(gsrc++);
        }
    }
    // sbase / gbase: shared byte address / global address of the word that
    // holds bit 0 of `bitpos`'s numbering (the other one is unused).
    __device__ __forceinline__ void init(uint32_t sbase, const uint32_t* gbase, uint32_t bitpos) {
        if constexpr (kShared) saddr = sbase + 4U * (bitpos >> 5);
        else gsrc = gbase + (bitpos >> 5);
        const uint32_t sh = bitpos & 31U;
        const uint32_t w0 = next(), w1 = next();
        pf = next();
        hi = __funnelshift_l(w1, w0, sh);
        lo = w1 << sh;
        avail = 64U - sh;
    }
    // Drops n & 31 bits (a table entry's code length is its low five bits).
    __device__ __forceinline__ void consume(uint32_t n) {
        hi = __funnelshift_l(lo, hi, n);
        lo = __funnelshift_l(0U, lo, n);
        avail -= n & 31U;
    }
    // Appends the next word when at most 32 bits remain.
    __device__ __forceinline__ void top_up() {
        if (avail <= 32U) {
            hi |= __funnelshift_rc(pf, 0U, avail);
            lo = __funnelshift_rc(0U, pf, avail);
            avail += 32U;
            pf = next();
        }
    }
};

// Code longer than 12 bits: consume the 12-bit prefix, then walk the suffix
// tree one bit at a time (at most 44 steps). Returns a leaf word (byte
// count in bits 5..7, bytes in 8..23). A table that exceeds the depth sets
// *status and yields one zero byte, so the lane still finishes.
template <typename W>
__device__ __forceinline__ uint32_t walk_long(const uint32_t* __restrict__ table, uint32_t marker, W& w,
                                              int32_t* status) {
    w.consume(NZ_LUT_BITS);
    uint32_t node = (marker >> 16) & kTreeMask;
    uint32_t leaf = 0;
    for (uint32_t d = 0; d < kMaxTreeDepth; ++d) {
        w.top_up();
        const uint32_t bit = w.hi >> 31;
        w.consume(1);
        const uint32_t child = table[NZ_LUT_TREE + 2U * node + bit];
        if (child & 0xE0U) {
            leaf = child;
            break;
        }
        node = (child >> 8) & kTreeMask;
    }
    if (!leaf) {
        if (status) *status = kStatusCorruptTable;
        leaf = 1U << 5;
    }
    return leaf;
}

// Code longer than 12 bits (the entry has no bytes). With canonical
// long-code tables (marker bit 31 clear) the code's length is the first one,
// from the shortest under this 12-bit prefix up, whose limit the 32-bit
// window does not exceed, and its rank in code order is the window's top L
// bits plus that length's offset: a couple of shared-memory reads instead
// of one tree step per bit. Otherwise the suffix tree is walked. Returns a
// leaf word; a table that does not resolve the window sets *status and
// yields one zero byte.
template <typename W>
__device__ __forceinline__ uint32_t decode_long(const uint32_t* __restrict__ table, uint32_t marker, W& w,
                                                int32_t* status) {
    if (marker & 0x80000000U) return walk_long(table, marker, w, status);
    const uint32_t* canon = table + NZ_LUT_CANON;
    const uint32_t win = w.hi;  // at least 33 valid bits: the whole code
    uint32_t len = max((marker >> 16) & 31U, NZ_LUT_BITS + 1U);
    while (win > canon[len] && len < NZ_CANON_MAX_BITS) ++len;
    const uint32_t rank = canon[32U + len] + (win >> (32U - len));
    uint32_t leaf = canon[64U + min(rank, NZ_CANON_TOKENS - 1U)];
    w.consume(len);
    if (win > canon[len] || (leaf & 0xE0U) == 0U) {
        if (status) *status = kStatusCorruptTable;
        leaf = 1U << 5;
    }
    return leaf;
}

// Bitwise select: bits of a where m is set, bits of b elsewhere (one LOP3).
__device__ __forceinline__ uint32_t bsel(uint32_t a, uint32_t b, uint32_t m) { return (a & m) | (b & ~m); }

// Element assembly (undoes DTypeSpec.reorder_bytes, neuralzip/dtypes.py:
// 23-45; the reference kernel's assemble_value, decode.cu:83-100). The
// reorder is undone on four elements at once, byte-wise: for bf16 the raw
// byte is sign|mant7 and the decoded byte the exponent, so the element's
// high byte is sign|exp[7:1] and its low byte exp[0]|mant7; fp32 does the
// same on its third byte.
template <int ES, bool REORDER>
struct Layout;

// bf16 (REORDER) and fp16: lane 0 raw, lane 1 decoded.
template <bool REORDER>
struct Layout<2, REORDER> {
    static constexpr int kSel = 1;
    static constexpr int kRawLanes = 1;
    // 8 elements from raw bytes r[0] (lane 0) and decoded bytes x0, x1.
    __device__ __forceinline__ static void store8(uint8_t* out, uint32_t e, const uint2* r, uint32_t x0,
                                                  uint32_t x1) {
        uint32_t l0 = r[0].x, h0 = x0, l1 = r[0].y, h1 = x1;
        if (REORDER) {
            h0 = bsel(r[0].x, x0 >> 1, 0x80808080U);
            l0 = bsel(r[0].x, x0 << 7, 0x7F7F7F7FU);
            h1 = bsel(r[0].y, x1 >> 1, 0x80808080U);
            l1 = bsel(r[0].y, x1 << 7, 0x7F7F7F7FU);
        }
        stg_u4(out + 2ull * e, __byte_perm(l0, h0, 0x5140), __byte_perm(l0, h0, 0x7362),
               __byte_perm(l1, h1, 0x5140), __byte_perm(l1, h1, 0x7362));
    }
    __device__ __forceinline__ static void store1(uint8_t* out, const uint8_t* const* lanes, uint32_t e,
                                                  uint32_t x) {
        uint32_t v = static_cast<uint32_t>(lanes[0][e]) | (x << 8);
        if (REORDER) v = (v & 0x7FU) | ((v >> 1) & 0x7F80U) | ((v << 8) & 0x8000U);
        reinterpret_cast<uint16_t*>(out)[e] = static_cast<uint16_t>(v);
    }
};

// fp32: lanes 0..2 raw, lane 3 decoded.
template <>
struct Layout<4, true> {
    static constexpr int kSel = 3;
    static constexpr int kRawLanes = 3;
    // Four elements from byte lanes a, b (raw), c (raw sign|mant[22:16]) and
    // x (exponents): undo the reorder on c/x, then a 4x4 byte transpose.
    __device__ __forceinline__ static void store4(uint8_t* o, uint32_t a, uint32_t b, uint32_t c, uint32_t x) {
        const uint32_t hi = bsel(c, x >> 1, 0x80808080U);
        const uint32_t mid = bsel(c, x << 7, 0x7F7F7F7FU);
        const uint32_t t0 = __byte_perm(a, b, 0x5140), t1 = __byte_perm(a, b, 0x7362);
        const uint32_t t2 = __byte_perm(mid, hi, 0x5140), t3 = __byte_perm(mid, hi, 0x7362);
        stg_u4(o, __byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632), __byte_perm(t1, t3, 0x5410),
               __byte_perm(t1, t3, 0x7632));
    }
    __device__ __forceinline__ static void store8(uint8_t* out, uint32_t e, const uint2* r, uint32_t x0,
                                                  uint32_t x1) {
        uint8_t* o = out + 4ull * e;
        store4(o, r[0].x, r[1].x, r[2].x, x0);
        store4(o + 16, r[0].y, r[1].y, r[2].y, x1);
    }
    __device__ __forceinline__ static void store1(uint8_t* out, const uint8_t* const* lanes, uint32_t e,
                                                  uint32_t x) {
        const uint32_t v = static_cast<uint32_t>(lanes[0][e]) | (static_cast<uint32_t>(lanes[1][e]) << 8) |
                           (static_cast<uint32_t>(lanes[2][e]) << 16) | (x << 24);
        reinterpret_cast<uint32_t*>(out)[e] =
            (v & 0x007FFFFFU) | ((v >> 1) & 0x7F800000U) | ((v << 8) & 0x80000000U);
    }
};

// Scalar tail: elements e .. min(e + 8, numel) with decoded bytes x0 | x1.
template <int ES, bool REORDER>
__device__ __forceinline__ void merge_tail(uint8_t* out, const uint8_t* const* lanes, uint32_t e, uint32_t numel,
                                           uint32_t x0, uint32_t x1) {
    const uint32_t n = min(8U, numel - e);
    for (uint32_t j = 0; j < n; ++j) {
        const uint32_t x = ((j < 4 ? x0 : x1) >> (8U * (j & 3U))) & 0xFFU;
        Layout<ES, REORDER>::store1(out, lanes, e + j, x);
    }
}

// Raw-lane bytes of one merge group: kGroup passes of 8 elements per lane.
template <int ES, bool REORDER>
struct MergeGroup {
    static constexpr uint32_t kGroup = ES == 4 ? 2 : 4;
    uint2 raw[kGroup][Layout<ES, REORDER>::kRawLanes];

    // Loads group g of a staging round; every element is inside the group
    // and every lane 16-byte aligned (interior tiles only).
    __device__ __forceinline__ void load(const uint8_t* const* lanes, uint32_t base, uint32_t g, uint32_t lane) {
#pragma unroll
        for (uint32_t k = 0; k < kGroup; ++k) {
            const uint32_t rrow = (g * kGroup + k) * kRowsPerPass + lane / kLanesPerRow;
            const uint32_t ex = base + rrow * NZ_LANE_ELEMS + (lane % kLanesPerRow) * 8U;
#pragma unroll
            for (int l = 0; l < Layout<ES, REORDER>::kRawLanes; ++l) raw[k][l] = ldg_u2(lanes[l] + ex);
        }
    }
    __device__ __forceinline__ void store(uint8_t* out, const uint32_t* stage, uint32_t base, uint32_t g,
                                          uint32_t lane) const {
#pragma unroll
        for (uint32_t k = 0; k < kGroup; ++k) {
            const uint32_t rrow = (g * kGroup + k) * kRowsPerPass + lane / kLanesPerRow;
            const uint32_t col = (lane % kLanesPerRow) * 8U;
            const uint32_t* src = stage + rrow * kStageStride + (col >> 2);
            Layout<ES, REORDER>::store8(out, base + rrow * NZ_LANE_ELEMS + col, raw[k], src[0], src[1]);
        }
    }
};

// The works [begin, end) of one CTA, taken in turn by its NW warps, for
// one element layout. `table` is the CTA's decode table; while `table_bar`
// (the shared address of its copy's mbarrier, 0 when the CTA has no table)
// is nonzero the copy may still be in flight, and each warp waits for it
// just before its first lookup.
template <int ES, bool REORDER, int NW, bool kQueue>
__device__ __forceinline__ void decode_works(const nz_group* __restrict__ groups,
                                             const nz_work* __restrict__ works, uint32_t begin,
                                             uint32_t end, const uint32_t* __restrict__ table,
                                             uint32_t table_bar, uint32_t* stage, int32_t* __restrict__ status,
                                             uint32_t* __restrict__ queue) {
    constexpr uint32_t kBitBufWords = bit_buf_words(NW);
    using L = Layout<ES, REORDER>;
    using G = MergeGroup<ES, REORDER>;
    constexpr uint32_t kGroups = kMergePasses / G::kGroup;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31U;
    const uint2* table2 = reinterpret_cast<const uint2*>(table);
    // The warp's first coded tile waits for the table (every lane, and
    // the warp agrees on the outcome). A copy that did not arrive within
    // the bounded wait sets status 5, and the warp decodes nothing more.
    bool table_pending = table_bar != 0U;
    auto table_arrived = [&]() {
        if (!table_pending) return true;
        table_pending = false;
        if (__all_sync(0xFFFFFFFFU, mbar_wait(table_bar, 0U))) return true;
        if (lane == 0 && status) *status = kStatusCopyTimeout;
        return false;
    };
    // Without a queue the warps take the CTA's works in turn. With one, each
    // warp claims the next work of the range shared by the queue's CTAs
    // (lane 0, one atomic per work), the next claim issued halfway through
    // the current work so that the atomic's round trip is hidden.
    uint32_t w = begin + warp;
    if constexpr (kQueue) {
        uint32_t first = 0;
        if (lane == 0) first = atomicAdd(queue, 1U);
        w = begin + __shfl_sync(0xFFFFFFFFU, first, 0);
    }
    while (w < end) {
        uint32_t claim = 0;    // lane 0: the next claimed index
        bool claimed = false;  // warp-uniform
        auto claim_next = [&]() {
            if constexpr (kQueue) {
                if (!claimed) {
                    if (lane == 0) claim = atomicAdd(queue, 1U);
                    claimed = true;
                }
            }
        };
        const nz_work item = works[w];
        const nz_group& g = groups[item.group];
        const uint32_t numel = g.numel;
        uint8_t* out = reinterpret_cast<uint8_t*>(g.out);
        const uint8_t* lanes[4];
#pragma unroll
        for (int l = 0; l < 4; ++l) lanes[l] = reinterpret_cast<const uint8_t*>(g.lanes[l]);
        uint64_t align = g.out;
#pragma unroll
        for (int l = 0; l < L::kRawLanes; ++l) align |= g.lanes[l];
        const bool vec_ok = (align & 15U) == 0;
        const uint32_t tile_base = item.tile * NZ_TILE_ELEMS;

        if (g.lut == NZ_RAW_LUT) {
            claim_next();
            // Raw fragment: the selected lane is stored as bytes.
            const uint8_t* sel = lanes[L::kSel];
            const bool sel_ok = vec_ok && (reinterpret_cast<uint64_t>(sel) & 15U) == 0;
            for (uint32_t it = 0; it < NZ_TILE_ELEMS / 256; ++it) {
                const uint32_t e = tile_base + it * 256U + lane * 8U;
                if (e >= numel) break;
                if (sel_ok && e + 8U <= numel) {
                    const uint2 x = ldg_u2(sel + e);  // 8-byte aligned: sel_ok
                    uint2 r[L::kRawLanes];
#pragma unroll
                    for (int l = 0; l < L::kRawLanes; ++l) r[l] = ldg_u2(lanes[l] + e);
                    L::store8(out, e, r, x.x, x.y);
                } else {
                    uint32_t x0 = 0, x1 = 0;
                    const uint32_t n = min(8U, numel - e);
                    for (uint32_t j = 0; j < n; ++j) {
                        const uint32_t b = sel[e + j];
                        if (j < 4) x0 |= b << (8U * j);
                        else x1 |= b << (8U * (j - 4U));
                    }
                    merge_tail<ES, REORDER>(out, lanes, e, numel, x0, x1);
                }
            }
            w = kQueue ? begin + __shfl_sync(0xFFFFFFFFU, claim, 0) : w + NW;
            continue;
        }

        // Coded tile: lane `lane` owns sub-stream s.
        const uint32_t s = item.tile * NZ_TILE_LANES + lane;
        const uint32_t first = s * NZ_LANE_ELEMS;
        const uint32_t n_lane = first < numel ? min(NZ_LANE_ELEMS, numel - first) : 0U;
        // Every element of an interior tile is inside the group and every
        // lane 16-byte aligned: its merges need no bounds checks, and each
        // round's first raw loads are issued before the round's decode.
        const bool interior = vec_ok && tile_base + NZ_TILE_ELEMS <= numel;
        const uint32_t len = reinterpret_cast<const uint16_t*>(g.lens)[s];
        uint32_t incl = len;
#pragma unroll
        for (uint32_t d = 1; d < 32; d <<= 1) {
            const uint32_t v = __shfl_up_sync(0xFFFFFFFFU, incl, d);
            if (lane >= d) incl += v;
        }
        // The tile's bits and raw lanes go to L2 now: the refills and the
        // merges then wait for L2, not DRAM. The bit range is widened to
        // 16-byte bounds, which stay inside the stream and its zero pad; a
        // raw lane's ragged end (< 16 bytes) is left to the loads.
        const uint32_t tile_bits = __shfl_sync(0xFFFFFFFFU, incl, 31);
        const uint32_t bit0 = reinterpret_cast<const uint32_t*>(g.tile_off)[item.tile];
        if (lane == 0) {
            const uint32_t w0 = (bit0 >> 5) & ~3U;
            const uint32_t w1 = ((bit0 + tile_bits + 127U) >> 7) << 2;
            prefetch_l2(reinterpret_cast<const uint32_t*>(g.bits) + w0, (w1 - w0) * 4U);
            if (vec_ok) {
                const uint32_t n = min(NZ_TILE_ELEMS, numel - tile_base);
#pragma unroll
                for (int l = 0; l < L::kRawLanes; ++l) prefetch_l2(lanes[l] + tile_base, n);
            }
        }
        // Byte queue: `qbits` bits (0, 8, 16 or 24) of decoded bytes wait in
        // qa between lookups. A lookup's bytes that do not fit in qa are not
        // kept: when qa fills up it is stored and rebuilt from the entry.
        uint32_t qa = 0, qbits = 0;
        uint32_t* row = stage + lane * kStageStride;

        // The tile's rounds, over a window on shared or global memory (two
        // instantiations, so that each reads its words with its own loads).
        auto rounds = [&](auto& win) {
            for (uint32_t r = 0; r < kRounds; ++r) {
                const uint32_t done = r * kRoundElems;
                if (__all_sync(0xFFFFFFFFU, n_lane <= done)) break;
                const uint32_t base = tile_base + done;
                // bf16/fp16 keep two groups of raw bytes in flight; fp32 (three
                // raw lanes) loads each group just before it merges, within the
                // register budget of 64 (8-warp CTAs) to 80 (24-warp CTAs).
                constexpr bool kAhead = ES == 2;
                G raw[2];
                if (kAhead && interior) raw[0].load(lanes, base, 0, lane);
                if (r + 1 == kRounds) claim_next();
                const uint32_t want = n_lane > done ? min(kRoundElems, n_lane - done) : 0U;
                const uint32_t target = (want + 3U) >> 2;
                for (uint32_t wi = 0; wi < target;) {
                    const uint2 entry = table2[win.hi >> (32 - NZ_LUT_BITS)];
                    uint32_t e = entry.x, x = entry.y;
                    if ((e & 0xFF00U) == 0U) {
                        const uint32_t leaf = decode_long(table, e, win, status);
                        e = ((leaf >> 5) & 7U) << 11;
                        x = leaf >> 8;
                    }
                    win.consume(e);
                    win.top_up();
                    qa |= x << qbits;
                    const uint32_t qn = qbits + (e >> 8);  // < 64
                    if (qn >= 32U) {
                        row[wi++] = qa;
                        qa = __funnelshift_l(x, 0U, qbits);
                    }
                    qbits = qn & 31U;
                }
                __syncwarp();
                if (interior) {
                    // Merge the 32 staged rows, kLanesPerRow lanes per row and 8
                    // elements per lane; each group's raw loads are in flight
                    // while the previous group merges.
#pragma unroll
                    for (uint32_t gi = 0; gi < kGroups; ++gi) {
                        if (kAhead) {
                            if (gi + 1 < kGroups) raw[(gi + 1) & 1U].load(lanes, base, gi + 1, lane);
                        } else {
                            raw[0].load(lanes, base, gi, lane);
                        }
                        raw[kAhead ? (gi & 1U) : 0U].store(out, stage, base, gi, lane);
                    }
                } else {
                    const uint32_t col = (lane % kLanesPerRow) * 8U;
#pragma unroll
                    for (uint32_t p0 = 0; p0 < kMergePasses; p0 += G::kGroup) {
                        uint2 raw[G::kGroup][L::kRawLanes];
                        uint32_t ex[G::kGroup];
                        bool full[G::kGroup];
#pragma unroll
                        for (uint32_t k = 0; k < G::kGroup; ++k) {
                            const uint32_t rrow = (p0 + k) * kRowsPerPass + lane / kLanesPerRow;
                            ex[k] = base + rrow * NZ_LANE_ELEMS + col;
                            full[k] = vec_ok && ex[k] + 8U <= numel;
                            if (full[k]) {
#pragma unroll
                                for (int l = 0; l < L::kRawLanes; ++l) raw[k][l] = ldg_u2(lanes[l] + ex[k]);
                            }
                        }
#pragma unroll
                        for (uint32_t k = 0; k < G::kGroup; ++k) {
                            const uint32_t rrow = (p0 + k) * kRowsPerPass + lane / kLanesPerRow;
                            const uint32_t* src = stage + rrow * kStageStride + (col >> 2);
                            const uint32_t x0 = src[0], x1 = src[1];
                            if (full[k]) L::store8(out, ex[k], raw[k], x0, x1);
                            else if (ex[k] < numel) merge_tail<ES, REORDER>(out, lanes, ex[k], numel, x0, x1);
                        }
                    }
                }
                __syncwarp();
            }
        };
        {
            // The tile's bits are copied into the warp's buffer when they
            // fit: from the 16-byte boundary at or below the first bit
            // through 12 to 15 words past the word of the last bit, inside
            // the stream's zero pad of at least 16 words. Lanes read past
            // their last bit: the window's read-ahead (3 words), and, for a
            // ragged last sub-stream, up to 3 lookups of bits that are not
            // its own (at most 3 x 56 bits) until its staged word is full;
            // at most 9 words in all, so every read stays in the copy.
            const uint32_t* gbits = reinterpret_cast<const uint32_t*>(g.bits);
            const uint32_t wa = (bit0 >> 5) & ~3U;
            const uint32_t wb = (((bit0 + tile_bits) >> 5) + 16U) & ~3U;
            if (wb - wa <= kBitBufWords) {
                uint32_t* buf = stage + kStageWordsPerWarp;
                const uint32_t sbuf = static_cast<uint32_t>(__cvta_generic_to_shared(buf));
#pragma unroll
                for (uint32_t k = 0; k < (kBitBufWords + 127U) / 128U; ++k) {
                    const uint32_t i = lane * 4U + k * 128U;
                    if (i < wb - wa)
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sbuf + 4U * i),
                                     "l"(gbits + wa + i)
                                     : "memory");
                }
                asm volatile("cp.async.wait_all;" ::: "memory");
                __syncwarp();
                if (!table_arrived()) return;
                Window<true> win;
                win.init(sbuf - 4U * wa, nullptr, bit0 + incl - len);
                rounds(win);
            } else {
                if (!table_arrived()) return;
                Window<false> win;
                win.init(0U, gbits, bit0 + incl - len);
                rounds(win);
            }
        }
        claim_next();  // a tile that ended before its last round
        w = kQueue ? begin + __shfl_sync(0xFFFFFFFFU, claim, 0) : w + NW;
    }
}

constexpr int32_t kStatusBadLayout = 3;
constexpr int32_t kStatusBadQueue = 4;

// One launch covers CTAs of every element layout: each CTA stages its
// decode table and runs the body of its layout (uniform per CTA, so the
// switch does not diverge).
// kQueue: the launch has work-queue scratch (its CTAs share ranges);
// fixed ranges and queues are separate kernels, so that neither path
// carries the other's registers.
template <int NW, bool kQueue>
__global__ void __launch_bounds__(NW * 32, ctas_per_sm(NW))
    nz_tile_decode(const nz_group* __restrict__ groups, const nz_work* __restrict__ works,
                   const nz_cta* __restrict__ ctas, const uint64_t* __restrict__ luts,
                   int32_t* __restrict__ status, uint32_t* __restrict__ scratch, uint32_t queues) {
    extern __shared__ __align__(16) uint32_t smem[];
    uint32_t* table = smem;
    uint32_t* stage = smem + NZ_LUT_WORDS + (threadIdx.x >> 5) * warp_words(NW);

    const nz_cta cta = ctas[blockIdx.x];
    // A queue launch's CTA whose queue index is out of range sets status 4
    // and decodes nothing (as a CTA with an unknown layout).
    const bool bad_queue = kQueue && cta.queue >= queues;
    uint32_t* queue = kQueue && !bad_queue ? scratch + cta.queue : nullptr;
    // The decode table (its leading table words, rounded up to 16 bytes)
    // arrives by one bulk copy issued by thread 0. The warps do not wait for
    // it here: each claims its first tile, reads its records and copies its
    // bitstream while the table is in flight, and waits for the table just
    // before its first lookup. Thread 0 waits for the copy (bounded) before
    // the CTA ends, so that no copy into this CTA's shared memory outlives
    // it; a copy that never arrives sets status 5.
    uint32_t bar = 0;
    if (cta.lut != NZ_RAW_LUT) {
        bar = static_cast<uint32_t>(__cvta_generic_to_shared(smem + NZ_LUT_WORDS + NW * warp_words(NW)));
        if (threadIdx.x == 0) mbar_init(bar);
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t n4 = (min(static_cast<uint32_t>(cta.lut_words), NZ_LUT_WORDS) + 3U) / 4U;
            bulk_load(static_cast<uint32_t>(__cvta_generic_to_shared(table)),
                      reinterpret_cast<const void*>(luts[cta.lut]), n4 * 16U, bar);
        }
    }
    switch (bad_queue ? 0xFFFFU : cta.layout) {
        case NZ_LAYOUT_BF16:
            decode_works<2, true, NW, kQueue>(groups, works, cta.begin, cta.end, table, bar, stage, status, queue);
            break;
        case NZ_LAYOUT_FP16:
            decode_works<2, false, NW, kQueue>(groups, works, cta.begin, cta.end, table, bar, stage, status, queue);
            break;
        case NZ_LAYOUT_FP32:
            decode_works<4, true, NW, kQueue>(groups, works, cta.begin, cta.end, table, bar, stage, status, queue);
            break;
        default:
            if (threadIdx.x == 0 && status) *status = bad_queue ? kStatusBadQueue : kStatusBadLayout;
    }
    if (bar && threadIdx.x == 0 && !mbar_wait(bar, 0U) && status) *status = kStatusCopyTimeout;
    if constexpr (kQueue) {
        // The launch's last CTA to finish sets the queue counters back to
        // zero for the next launch that uses this scratch.
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(scratch + queues, 1U) == gridDim.x - 1U) {
                for (uint32_t q = 0; q < queues; ++q) scratch[q] = 0U;
                scratch[queues] = 0U;
                __threadfence();
            }
        }
    }
}

template <int NW>
constexpr size_t smem_bytes() {
    return (NZ_LUT_WORDS + NW * warp_words(NW) + kBarWords) * sizeof(uint32_t);
}

// Opts the instantiation into its dynamic shared memory on the current
// device. The attribute belongs to the device's context, so it is set once
// per device (a process may launch on several GPUs).
template <int NW, bool kQueue>
cudaError_t ensure_smem_attribute() {
    static std::mutex lock;
    static std::vector<char> done;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> hold(lock);
    if (done.size() <= static_cast<size_t>(device)) done.resize(device + 1, 0);
    if (!done[device]) {
        err = cudaFuncSetAttribute(nz_tile_decode<NW, kQueue>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem_bytes<NW>()));
        if (err != cudaSuccess) return err;
        done[device] = 1;
    }
    return cudaSuccess;
}

template <int NW, bool kQueue>
cudaError_t launch_kernel(const nz_launch& l, cudaStream_t stream) {
    const cudaError_t attr_err = ensure_smem_attribute<NW, kQueue>();
    if (attr_err != cudaSuccess) return attr_err;
    nz_tile_decode<NW, kQueue><<<l.n_ctas, NW * 32, smem_bytes<NW>(), stream>>>(
        reinterpret_cast<const nz_group*>(l.groups), reinterpret_cast<const nz_work*>(l.works),
        reinterpret_cast<const nz_cta*>(l.ctas), reinterpret_cast<const uint64_t*>(l.luts),
        reinterpret_cast<int32_t*>(l.status), reinterpret_cast<uint32_t*>(l.scratch), l.queues);
    return cudaGetLastError();
}

template <int NW>
cudaError_t launch_one(const nz_launch& l, cudaStream_t stream) {
    // Queues only with scratch and at least one queue; else fixed ranges.
    return l.scratch && l.queues ? launch_kernel<NW, true>(l, stream) : launch_kernel<NW, false>(l, stream);
}

cudaError_t launch_nw(const nz_launch& l, cudaStream_t stream) {
    switch (l.warps_per_cta) {
        case 4: return launch_one<4>(l, stream);
        case 16: return launch_one<16>(l, stream);
        case 24: return launch_one<24>(l, stream);
        default: return launch_one<8>(l, stream);
    }
}

template <int NW>
cudaError_t occupancy_one(int* ctas) {
    const cudaError_t err = ensure_smem_attribute<NW, false>();
    if (err != cudaSuccess) return err;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas, nz_tile_decode<NW, false>, NW * 32,
                                                         smem_bytes<NW>());
}

// Side streams of nz_decode_launch_many, per device, created on first use
// and kept for the life of the process (with their fork/join events).
struct AuxStreams {
    std::mutex lock;
    std::vector<cudaStream_t> streams;
    std::vector<cudaEvent_t> join;
    cudaEvent_t fork = nullptr;
};

int aux_streams(uint32_t needed, AuxStreams** out) {
    static std::mutex registry_lock;
    static std::vector<AuxStreams*> per_device;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return nz::fail(NZ_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
    AuxStreams* aux;
    {
        std::lock_guard<std::mutex> hold(registry_lock);
        if (per_device.size() <= static_cast<size_t>(device)) per_device.resize(device + 1, nullptr);
        if (!per_device[device]) per_device[device] = new AuxStreams();
        aux = per_device[device];
    }
    std::lock_guard<std::mutex> hold(aux->lock);
    if (!aux->fork) {
        err = cudaEventCreateWithFlags(&aux->fork, cudaEventDisableTiming);
        if (err != cudaSuccess) return nz::fail(NZ_ECUDA, std::string("cudaEventCreate: ") + cudaGetErrorString(err));
    }
    while (aux->streams.size() < needed) {
        cudaStream_t s = nullptr;
        cudaEvent_t e = nullptr;
        // Lowest priority: when more CTAs wait than SMs are free, the
        // caller stream's launch is served first.
        int least = 0, greatest = 0;
        err = cudaDeviceGetStreamPriorityRange(&least, &greatest);
        if (err == cudaSuccess) err = cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, least);
        if (err == cudaSuccess) err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
        if (err != cudaSuccess) return nz::fail(NZ_ECUDA, std::string("aux stream: ") + cudaGetErrorString(err));
        aux->streams.push_back(s);
        aux->join.push_back(e);
    }
    *out = aux;
    return NZ_OK;
}

// Work-queue counters of nz_decode_launch_noalloc, in the library's own
// device memory: every GPU that loads this library holds this array until
// the process exits. kNoAllocQueues counters plus the finished-CTA count.
constexpr uint32_t kNoAllocQueues = 1024;
static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocQueues + 1];

// Device address of g_noalloc_scratch on the current device, looked up (and
// the counters cleared) on the first call per device. In host code the
// array's name is only a host-side stand-in, never a device address.
int noalloc_scratch(uint32_t** out) {
    static std::mutex lock;
    static std::vector<uint32_t*> per_device;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return nz::fail(NZ_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
    std::lock_guard<std::mutex> hold(lock);
    if (per_device.size() <= static_cast<size_t>(device)) per_device.resize(device + 1, nullptr);
    if (!per_device[device]) {
        uint32_t* ptr = nullptr;
        err = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_scratch);
        if (err != cudaSuccess)
            return nz::fail(NZ_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(err));
        err = cudaMemset(ptr, 0, sizeof(g_noalloc_scratch));
        if (err == cudaSuccess) err = cudaDeviceSynchronize();
        if (err != cudaSuccess) return nz::fail(NZ_ECUDA, std::string("cudaMemset: ") + cudaGetErrorString(err));
        per_device[device] = ptr;
    }
    *out = per_device[device];
    return NZ_OK;
}

}  // namespace

extern "C" {

int nz_decode_smem_bytes(uint32_t warps_per_cta, uint32_t* bytes) {
    if (!bytes) return nz::fail(NZ_EVALUE, "Null output.");
    const uint32_t nw = warps_per_cta == 0 ? 8U : warps_per_cta;
    *bytes = (NZ_LUT_WORDS + nw * warp_words(nw) + kBarWords) * static_cast<uint32_t>(sizeof(uint32_t));
    return NZ_OK;
}

int nz_decode_tile_words(uint32_t warps_per_cta, uint32_t* words) {
    if (!words) return nz::fail(NZ_EVALUE, "Null output.");
    const uint32_t nw = warps_per_cta == 0 ? 8U : warps_per_cta;
    if (nw != 4 && nw != 8 && nw != 16 && nw != 24)
        return nz::fail(NZ_EVALUE, "warps_per_cta must be 4, 8, 16 or 24.");
    *words = bit_buf_words(nw);
    return NZ_OK;
}

int nz_decode_occupancy(uint32_t warps_per_cta, uint32_t* ctas_per_sm) {
    if (!ctas_per_sm) return nz::fail(NZ_EVALUE, "Null argument.");
    int ctas = 0;
    cudaError_t err;
    switch (warps_per_cta) {
        case 4: err = occupancy_one<4>(&ctas); break;
        case 0:
        case 8: err = occupancy_one<8>(&ctas); break;
        case 16: err = occupancy_one<16>(&ctas); break;
        case 24: err = occupancy_one<24>(&ctas); break;
        default: return nz::fail(NZ_EVALUE, "warps_per_cta must be 4, 8, 16 or 24.");
    }
    if (err != cudaSuccess)
        return nz::fail(NZ_ECUDA, std::string("CUDA occupancy query failed: ") + cudaGetErrorString(err));
    *ctas_per_sm = static_cast<uint32_t>(ctas);
    return NZ_OK;
}

int nz_decode_launch_many(const nz_launch* launches, uint32_t count, void* cuda_stream) {
    if (count == 0) return NZ_OK;
    if (!launches) return nz::fail(NZ_EVALUE, "Null launch descriptors.");
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
    // The launch with the most warps goes first, on the caller's stream, and
    // fills every SM; the others are enqueued at once on low-priority side
    // streams, so their CTAs take SMs as the first launch's CTAs finish (its
    // tail) and run side by side, small launches being latency-bound. The
    // caller's stream then waits for all of them.
    uint32_t main = 0;
    for (uint32_t i = 1; i < count; ++i)
        if (launches[i].n_ctas * launches[i].warps_per_cta > launches[main].n_ctas * launches[main].warps_per_cta)
            main = i;
    if (count == 1) return nz_decode_launch(&launches[0], cuda_stream);
    AuxStreams* aux = nullptr;
    int rc = aux_streams(count - 1, &aux);
    if (rc != NZ_OK) return rc;
    std::lock_guard<std::mutex> hold(aux->lock);
    cudaError_t err = cudaEventRecord(aux->fork, stream);
    if (err != cudaSuccess) return nz::fail(NZ_ECUDA, std::string("cudaEventRecord: ") + cudaGetErrorString(err));
    rc = nz_decode_launch(&launches[main], cuda_stream);
    if (rc != NZ_OK) return rc;
    uint32_t k = 0;
    for (uint32_t i = 0; i < count; ++i) {
        if (i == main) continue;
        cudaStream_t side = aux->streams[k];
        err = cudaStreamWaitEvent(side, aux->fork, 0);
        if (err != cudaSuccess)
            return nz::fail(NZ_ECUDA, std::string("cudaStreamWaitEvent: ") + cudaGetErrorString(err));
        rc = nz_decode_launch(&launches[i], side);
        if (rc != NZ_OK) return rc;
        err = cudaEventRecord(aux->join[k], side);
        if (err == cudaSuccess) err = cudaStreamWaitEvent(stream, aux->join[k], 0);
        if (err != cudaSuccess) return nz::fail(NZ_ECUDA, std::string("stream join: ") + cudaGetErrorString(err));
        ++k;
    }
    return NZ_OK;
}

int nz_decode_launch_noalloc(const nz_launch* launch, void* cuda_stream) {
    if (!launch) return nz::fail(NZ_EVALUE, "Null launch descriptor.");
    if (launch->queues > kNoAllocQueues)
        return nz::fail(NZ_EVALUE, "nz_decode_launch_noalloc takes at most 1024 work queues.");
    if (launch->n_ctas == 0) return NZ_OK;
    uint32_t* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != NZ_OK) return rc;
    nz_launch l = *launch;
    l.scratch = reinterpret_cast<uint64_t>(scratch);
    return nz_decode_launch(&l, cuda_stream);
}

int nz_decode_launch(const nz_launch* launch, void* cuda_stream) {
    if (!launch) return nz::fail(NZ_EVALUE, "Null launch descriptor.");
    const nz_launch& l = *launch;
    if (l.n_ctas == 0) return NZ_OK;
    if (!l.groups || !l.works || !l.ctas || !l.luts)
        return nz::fail(NZ_EVALUE, "Null device descriptor array.");
    if (l.warps_per_cta != 0 && l.warps_per_cta != 4 && l.warps_per_cta != 8 &&
        l.warps_per_cta != 16 && l.warps_per_cta != 24)
        return nz::fail(NZ_EVALUE, "warps_per_cta must be 4, 8, 16 or 24.");
    const cudaError_t err = launch_nw(l, reinterpret_cast<cudaStream_t>(cuda_stream));
    if (err != cudaSuccess)
        return nz::fail(NZ_ECUDA, std::string("CUDA launch failed: ") + cudaGetErrorString(err));
    return NZ_OK;
}

}  // extern "C"
