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
//   * the decode table lives in shared memory (staged once per CTA) and one
//     lookup of the 12-bit window yields up to three output bytes; codes of
//     13..56 bits continue through a suffix tree in the same table
//     (decode.cu:41-60 reads its table through __ldg, one token per probe);
//   * decoded bytes are staged per warp, 64 elements per lane at a time, and
//     merged with the raw lanes through 8-byte loads and 16-byte stores that
//     are contiguous across the warp (decode.cu:83-100 loads and stores one
//     element at a time).

#include "nz_b200.h"
#include "nz_internal.h"

#include <cuda_runtime.h>

#include <mutex>
#include <string>

namespace {

constexpr uint32_t kRoundElems = 64;                       // per lane per staging round
constexpr uint32_t kRounds = NZ_LANE_ELEMS / kRoundElems;  // 4
constexpr uint32_t kStageStride = kRoundElems / 4 + 1;     // words per staged row
constexpr uint32_t kStageWordsPerWarp = NZ_TILE_LANES * kStageStride;
constexpr uint32_t kTreeMask = NZ_TREE_MAX_NODES - 1;
constexpr uint32_t kMaxTreeDepth = NZ_MAX_CODE_BITS - NZ_LUT_BITS;
constexpr int32_t kStatusCorruptTable = 2;

__device__ __forceinline__ uint32_t ldg_u32(const uint32_t* p) { return __ldg(p); }

__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void stg_u4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

// MSB-first reader over 32-bit words (bit 31 earliest) with one word of
// prefetch; `buf` holds `nvalid` valid bits left-aligned.
struct BitReader {
    uint64_t buf;
    uint32_t nvalid;
    uint32_t pf;
    const uint32_t* ptr;

    __device__ __forceinline__ void init(const uint32_t* words, uint32_t bitpos) {
        const uint32_t* p = words + (bitpos >> 5);
        const uint32_t sh = bitpos & 31U;
        const uint64_t w = (static_cast<uint64_t>(ldg_u32(p)) << 32) | ldg_u32(p + 1);
        buf = w << sh;
        nvalid = 64U - sh;
        ptr = p + 2;
        pf = ldg_u32(ptr);
    }
    // Precondition: nvalid <= 32.
    __device__ __forceinline__ void refill() {
        buf |= static_cast<uint64_t>(pf) << (32U - nvalid);
        nvalid += 32U;
        ++ptr;
        pf = ldg_u32(ptr);
    }
    __device__ __forceinline__ void consume(uint32_t n) {
        buf <<= n;
        nvalid -= n;
    }
};

// Walks the suffix tree for a code longer than 12 bits. `marker` is the LUT
// entry (node index reached after the first 12 bits). Returns a leaf entry
// (bytes | count << 28). The depth is bounded by 44; a table that exceeds
// it sets *status and yields one zero byte so the lane still terminates.
__device__ __forceinline__ uint32_t walk_long(const uint32_t* __restrict__ table, uint32_t marker,
                                            BitReader& br, int32_t* status) {
    br.consume(NZ_LUT_BITS);
    uint32_t node = marker & kTreeMask;
    for (uint32_t d = 0; d < kMaxTreeDepth; ++d) {
        if (br.nvalid <= 32U) br.refill();
        const uint32_t bit = static_cast<uint32_t>(br.buf >> 63);
        br.consume(1);
        const uint32_t child = table[NZ_LUT_ENTRIES + 2U * node + bit];
        if (child >> 28) return child;
        node = child & kTreeMask;
    }
    if (status) *status = kStatusCorruptTable;
    return 1U << 28;
}

// Element assembly (undoes DTypeSpec.reorder_bytes, neuralzip/dtypes.py:
// 23-45; the reference kernel's assemble_value, decode.cu:83-100).
template <int ES, bool REORDER>
struct Layout;

// bf16 (REORDER) and fp16: lane 0 raw, lane 1 decoded.
template <bool REORDER>
struct Layout<2, REORDER> {
    static constexpr int kSel = 1;
    // Two elements: raw bytes r (low 16 bits used), decoded bytes x.
    __device__ __forceinline__ static uint32_t pair(uint32_t r, uint32_t x, uint32_t sel) {
        const uint32_t t = __byte_perm(r, x, sel);
        if (!REORDER) return t;
        return (t & 0x007F007FU) | ((t >> 1) & 0x7F807F80U) | ((t << 8) & 0x80008000U);
    }
    __device__ __forceinline__ static void store8(uint8_t* out, const uint8_t* const* lanes,
                                                  uint32_t e, uint32_t x0, uint32_t x1) {
        const uint2 r = ldg_stream_u2(lanes[0] + e);
        stg_u4(out + 2ull * e, pair(r.x, x0, 0x5140), pair(r.x, x0, 0x7362),
               pair(r.y, x1, 0x5140), pair(r.y, x1, 0x7362));
    }
    __device__ __forceinline__ static void store1(uint8_t* out, const uint8_t* const* lanes,
                                                  uint32_t e, uint32_t x) {
        uint32_t v = static_cast<uint32_t>(lanes[0][e]) | (x << 8);
        if (REORDER) v = (v & 0x7FU) | ((v >> 1) & 0x7F80U) | ((v << 8) & 0x8000U);
        reinterpret_cast<uint16_t*>(out)[e] = static_cast<uint16_t>(v);
    }
};

// fp32: lanes 0..2 raw, lane 3 decoded.
template <>
struct Layout<4, true> {
    static constexpr int kSel = 3;
    __device__ __forceinline__ static uint32_t fix(uint32_t v) {
        return (v & 0x007FFFFFU) | ((v >> 1) & 0x7F800000U) | ((v << 8) & 0x80000000U);
    }
    __device__ __forceinline__ static uint32_t word(uint32_t l0, uint32_t l1, uint32_t l2,
                                                    uint32_t x, uint32_t i) {
        const uint32_t lo = __byte_perm(l0, l1, i | ((i + 4U) << 4));
        const uint32_t hi = __byte_perm(l2, x, i | ((i + 4U) << 4));
        return fix(__byte_perm(lo, hi, 0x5410));
    }
    __device__ __forceinline__ static void store8(uint8_t* out, const uint8_t* const* lanes,
                                                  uint32_t e, uint32_t x0, uint32_t x1) {
        const uint2 a = ldg_stream_u2(lanes[0] + e);
        const uint2 b = ldg_stream_u2(lanes[1] + e);
        const uint2 c = ldg_stream_u2(lanes[2] + e);
        uint8_t* o = out + 4ull * e;
        stg_u4(o, word(a.x, b.x, c.x, x0, 0), word(a.x, b.x, c.x, x0, 1),
               word(a.x, b.x, c.x, x0, 2), word(a.x, b.x, c.x, x0, 3));
        stg_u4(o + 16, word(a.y, b.y, c.y, x1, 0), word(a.y, b.y, c.y, x1, 1),
               word(a.y, b.y, c.y, x1, 2), word(a.y, b.y, c.y, x1, 3));
    }
    __device__ __forceinline__ static void store1(uint8_t* out, const uint8_t* const* lanes,
                                                  uint32_t e, uint32_t x) {
        const uint32_t v = static_cast<uint32_t>(lanes[0][e]) |
                           (static_cast<uint32_t>(lanes[1][e]) << 8) |
                           (static_cast<uint32_t>(lanes[2][e]) << 16) | (x << 24);
        reinterpret_cast<uint32_t*>(out)[e] = fix(v);
    }
};

// Merges 8 consecutive elements starting at e (< numel) whose decoded
// bytes are x0 (elements e..e+3) and x1 (e+4..e+7).
template <int ES, bool REORDER>
__device__ __forceinline__ void merge8(uint8_t* out, const uint8_t* const* lanes, bool vec_ok,
                                       uint32_t e, uint32_t numel, uint32_t x0, uint32_t x1) {
    using L = Layout<ES, REORDER>;
    if (vec_ok && e + 8U <= numel) {
        L::store8(out, lanes, e, x0, x1);
        return;
    }
    const uint32_t n = min(8U, numel - e);
    for (uint32_t j = 0; j < n; ++j) {
        const uint32_t x = ((j < 4 ? x0 : x1) >> (8U * (j & 3U))) & 0xFFU;
        L::store1(out, lanes, e + j, x);
    }
}

template <int ES, bool REORDER, int NW>
__global__ void __launch_bounds__(NW * 32, (NW >= 16 ? 2 : (NW >= 8 ? 4 : 8)))
    nz_tile_decode(const nz_group* __restrict__ groups, const nz_work* __restrict__ works,
                   const nz_cta* __restrict__ ctas, const uint64_t* __restrict__ luts,
                   int32_t* __restrict__ status) {
    extern __shared__ __align__(16) uint32_t smem[];
    uint32_t* table = smem;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31U;
    uint32_t* stage = smem + NZ_LUT_WORDS + warp * kStageWordsPerWarp;

    const nz_cta cta = ctas[blockIdx.x];
    const bool coded = cta.lut != NZ_RAW_LUT;
    if (coded) {
        const uint4* src = reinterpret_cast<const uint4*>(luts[cta.lut]);
        uint4* dst = reinterpret_cast<uint4*>(table);
        const uint32_t n4 = (min(cta.lut_words, NZ_LUT_WORDS) + 3U) / 4U;  // tables hold NZ_LUT_WORDS
        for (uint32_t i = threadIdx.x; i < n4; i += NW * 32) dst[i] = __ldg(src + i);
    }
    __syncthreads();

    for (uint32_t w = cta.begin + warp; w < cta.end; w += NW) {
        const nz_work item = works[w];
        const nz_group& g = groups[item.group];
        const uint32_t numel = g.numel;
        uint8_t* out = reinterpret_cast<uint8_t*>(g.out);
        const uint8_t* lanes[4];
#pragma unroll
        for (int l = 0; l < 4; ++l) lanes[l] = reinterpret_cast<const uint8_t*>(g.lanes[l]);
        uint64_t align = g.out;
#pragma unroll
        for (int l = 0; l < ES; ++l)
            if (l != Layout<ES, REORDER>::kSel) align |= g.lanes[l];
        const bool vec_ok = (align & 15U) == 0;
        const uint32_t tile_base = item.tile * NZ_TILE_ELEMS;

        if (g.lut == NZ_RAW_LUT) {
            // Raw fragment: the selected lane is stored as bytes.
            const uint8_t* sel = lanes[Layout<ES, REORDER>::kSel];
            const bool sel_ok = vec_ok && (reinterpret_cast<uint64_t>(sel) & 7U) == 0;
            for (uint32_t it = 0; it < NZ_TILE_ELEMS / 256; ++it) {
                const uint32_t e = tile_base + it * 256U + lane * 8U;
                if (e >= numel) break;
                uint32_t x0, x1;
                if (sel_ok && e + 8U <= numel) {
                    const uint2 x = ldg_stream_u2(sel + e);
                    x0 = x.x;
                    x1 = x.y;
                } else {
                    x0 = x1 = 0;
                    const uint32_t n = min(8U, numel - e);
                    for (uint32_t j = 0; j < n; ++j) {
                        const uint32_t b = sel[e + j];
                        if (j < 4) x0 |= b << (8U * j);
                        else x1 |= b << (8U * (j - 4U));
                    }
                }
                merge8<ES, REORDER>(out, lanes, sel_ok, e, numel, x0, x1);
            }
            continue;
        }

        // Coded tile: lane `lane` owns sub-stream s.
        const uint32_t s = item.tile * NZ_TILE_LANES + lane;
        const uint32_t first = s * NZ_LANE_ELEMS;
        const uint32_t n_lane = first < numel ? min(NZ_LANE_ELEMS, numel - first) : 0U;
        const uint32_t len = reinterpret_cast<const uint16_t*>(g.lens)[s];
        uint32_t incl = len;
#pragma unroll
        for (uint32_t d = 1; d < 32; d <<= 1) {
            const uint32_t v = __shfl_up_sync(0xFFFFFFFFU, incl, d);
            if (lane >= d) incl += v;
        }
        const uint32_t start = reinterpret_cast<const uint32_t*>(g.tile_off)[item.tile] + incl - len;
        BitReader br;
        br.init(reinterpret_cast<const uint32_t*>(g.bits), start);
        uint64_t q = 0;
        uint32_t qn = 0, pushed = 0;
        uint32_t* row = stage + lane * kStageStride;

        for (uint32_t r = 0; r < kRounds; ++r) {
            const uint32_t done = r * kRoundElems;
            if (__all_sync(0xFFFFFFFFU, n_lane <= done)) break;
            const uint32_t want = n_lane > done ? min(kRoundElems, n_lane - done) : 0U;
            const uint32_t target = (want + 3U) >> 2;
            for (uint32_t wi = 0; wi < target;) {
                if (pushed < n_lane) {
                    uint32_t e = table[static_cast<uint32_t>(br.buf >> (64 - NZ_LUT_BITS))];
                    uint32_t nbits = (e >> 24) & 15U;
                    if ((e >> 28) == 0) {
                        e = walk_long(table, e, br, status);
                        nbits = 0;
                    }
                    const uint32_t nb = (e >> 28) & 3U;
                    q |= static_cast<uint64_t>(e & 0xFFFFFFU) << (8U * qn);
                    qn += nb;
                    pushed += nb;
                    br.consume(nbits);
                    if (br.nvalid <= 32U) br.refill();
                }
                if (qn >= 4U || pushed >= n_lane) {
                    row[wi++] = static_cast<uint32_t>(q);
                    q >>= 32;
                    qn = qn >= 4U ? qn - 4U : 0U;
                }
            }
            __syncwarp();
            // Merge the 32 staged rows: 8 lanes per row, 8 elements per lane.
#pragma unroll 2
            for (uint32_t it = 0; it < NZ_TILE_LANES / 4; ++it) {
                const uint32_t rrow = it * 4U + (lane >> 3);
                const uint32_t col = (lane & 7U) * 8U;
                const uint32_t e = tile_base + rrow * NZ_LANE_ELEMS + done + col;
                if (e < numel) {
                    const uint32_t* src = stage + rrow * kStageStride + (col >> 2);
                    merge8<ES, REORDER>(out, lanes, vec_ok, e, numel, src[0], src[1]);
                }
            }
            __syncwarp();
        }
    }
}

template <int ES, bool REORDER, int NW>
cudaError_t launch_one(const nz_launch& l, cudaStream_t stream) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    const size_t smem = (NZ_LUT_WORDS + NW * kStageWordsPerWarp) * sizeof(uint32_t);
    std::call_once(once, [&]() {
        attr_err = cudaFuncSetAttribute(nz_tile_decode<ES, REORDER, NW>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem));
    });
    if (attr_err != cudaSuccess) return attr_err;
    nz_tile_decode<ES, REORDER, NW><<<l.n_ctas, NW * 32, smem, stream>>>(
        reinterpret_cast<const nz_group*>(l.groups), reinterpret_cast<const nz_work*>(l.works),
        reinterpret_cast<const nz_cta*>(l.ctas), reinterpret_cast<const uint64_t*>(l.luts),
        reinterpret_cast<int32_t*>(l.status));
    return cudaGetLastError();
}

template <int ES, bool REORDER>
cudaError_t launch_nw(const nz_launch& l, cudaStream_t stream) {
    switch (l.warps_per_cta) {
        case 4: return launch_one<ES, REORDER, 4>(l, stream);
        case 16: return launch_one<ES, REORDER, 16>(l, stream);
        default: return launch_one<ES, REORDER, 8>(l, stream);
    }
}

}  // namespace

extern "C" {

int nz_decode_smem_bytes(uint32_t warps_per_cta, uint32_t* bytes) {
    if (!bytes) return nz::fail(NZ_EVALUE, "Null output.");
    const uint32_t nw = warps_per_cta == 0 ? 8U : warps_per_cta;
    *bytes = (NZ_LUT_WORDS + nw * kStageWordsPerWarp) * static_cast<uint32_t>(sizeof(uint32_t));
    return NZ_OK;
}

int nz_decode_launch(const nz_launch* launch, void* cuda_stream) {
    if (!launch) return nz::fail(NZ_EVALUE, "Null launch descriptor.");
    const nz_launch& l = *launch;
    if (l.n_ctas == 0) return NZ_OK;
    if (!l.groups || !l.works || !l.ctas || !l.luts)
        return nz::fail(NZ_EVALUE, "Null device descriptor array.");
    if (l.warps_per_cta != 0 && l.warps_per_cta != 4 && l.warps_per_cta != 8 &&
        l.warps_per_cta != 16)
        return nz::fail(NZ_EVALUE, "warps_per_cta must be 4, 8 or 16.");
    const nz_dtype& d = l.dtype;
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
    cudaError_t err;
    if (d.elem_size == 2 && d.stream_id == 1 && d.reorder && d.mant_bits == 7 && d.exp_bits == 8)
        err = launch_nw<2, true>(l, stream);
    else if (d.elem_size == 2 && d.stream_id == 1 && !d.reorder && d.mant_bits == 10 &&
             d.exp_bits == 5)
        err = launch_nw<2, false>(l, stream);
    else if (d.elem_size == 4 && d.stream_id == 3 && d.reorder && d.mant_bits == 23 &&
             d.exp_bits == 8)
        err = launch_nw<4, true>(l, stream);
    else
        return nz::fail(NZ_EVALUE, "Unsupported GPU layout (bf16, fp16 and fp32 are decoded).");
    if (err != cudaSuccess)
        return nz::fail(NZ_ECUDA, std::string("CUDA launch failed: ") + cudaGetErrorString(err));
    return NZ_OK;
}

}  // extern "C"
