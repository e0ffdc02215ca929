// Fused index-resident per-sample LoRA forward (shrink + expand, decode fused in).
//
// Replaces the two Triton launches of lithe/kernels/shared.py:36-157 (shrink decodes A
// tiles and writes y_lo; expand decodes B tiles per M-tile and writes a fresh delta),
// the separate "delta * scaling" pass (shared.py:261-262) and the caller's "out + delta"
// pass (lithe/kernels/layers.py:131, lithe/serve.py:97).  One persistent launch per linear
// (calls with at most kSmallM token rows per sample take sgmv_small_kernel further down):
//
//   work unit  = (sample b, 64-token tile); CTA i owns a contiguous range of units.
//   per unit   = d_in/64 "x chunks" (64x64 bf16 activation tiles, 128B swizzle)
//              + d_out/64 "out chunks" (64x64 bf16 base-output tiles; the updated values go
//                back with coalesced 16-byte stores straight from registers).
//   stage      = two adjacent chunks of one unit, fetched by ONE TMA operation through a
//                "chunked" 3-D view of the array (64 columns, rows, chunks; the chunk stride,
//                128 B, is the outer dimension), so each op moves 16 KB.  On B200 the op count
//                matters: streaming 8 KB boxes from one CTA per SM topped out near 33-37 GB/s
//                per SM, 16 KB boxes reach ~42 GB/s (6.2 TB/s over 148 SMs).
//   warps      = 8 consumer warps in 2 groups that take alternate pipeline positions (each
//                group has 4 warps of 16 tokens; the groups add their partial x.A^T sums
//                through shared memory before the expand), and kFeed feeder warps that take
//                every kFeed-th position: each issues its positions' TMA loads (one lane) and
//                decodes their factor chunks (the whole warp) while the loads are in flight.
//   pipeline   = kStages shared-memory stages; each stage holds two 8 KB chunk tiles and the
//                two 512 B decoded factor chunks that go with them; full barrier = TMA bytes +
//                the feeder's arrival, empty barrier = one arrival per warp of the group.
//
// Decoded factors.  The codeword c_k has period 16 (device_common.cuh), so
//   A_j[r, 64c + t] = a_{r,c}[t & 15]     (16 values per (rank row, 64-column chunk))
//   B_j[o, r]       = w_G[r_eff]          with 4 consecutive-in-pattern rows identical
// and a decoded chunk is 16 rows x 16 values (512 B of bf16) for both sides.
//
// Shrink (per x chunk, per consumer warp): h[16 x 16] += x[16 x 64] . A_chunk^T with
// 8 mma.m16n8k16.  The reduction index inside each 32-column window is permuted so that
// every thread reads its activations as one 16-byte vector per row; the A fragment uses
// the same permutation (both are a bijection of the window's 32 columns).
// Expand (per out chunk): the 64 output columns of a chunk are 16 distinct "logical"
// columns repeated 4 times, so delta = h . B^T is 2 mma.m16n8k16 (n = 16 logical
// columns, k = 16 ranks) and each thread adds its 2 results to 8 output values per row.
// The stage is released as soon as the tile is in registers; the stores need no proxy fence.
//
// Shrink-only forms (the prep of lithe_lora_gemm's fused expand; SgmvParams::h_out set):
//   lithe_lora_prep      x tiles only, h = bf16(w . s . x . A^T) stored after the shrink.
//   lithe_lora_prep_ws   the same with the CTAs taking equal runs of the (unit, x stage)
//                        sequence (SgmvParams::split): a unit may be shared by neighbouring
//                        CTAs, each storing its fp32 partial h in a workspace that the B-decode
//                        launch after it adds up in CTA order (split_combine).
//   lithe_lora_prep_multi  kT (<= 4) linears reading the same x, staged form: their decoded A
//                        chunks come from a workspace (prep_multi_decode_kernel) next to each
//                        x tile, and the consumers accumulate kT h's from one read of x.
#include <mutex>

#include "device_common.cuh"
#include "host_common.h"

namespace lithe {

constexpr int kBM = 64;                 // tokens per work unit
constexpr int kChunk = 64;              // columns per chunk
constexpr int kGroupWarps = 4;                    // consumer warps per group (16 token rows each)
constexpr int kGroups = 2;                        // consumer groups; group g takes positions pos % 2 == g
constexpr int kConsumerWarps = kGroupWarps * kGroups;
constexpr int kDecodeWarps = 4;                   // feeder warps of the fused form (they also decode)
constexpr int kFeedStaged = 4;                    // feeder warps of the staged form (loads only)
constexpr int kFirstFeedWarp = kConsumerWarps;
constexpr int kStageChunks = 2;                   // 64-column chunks per stage (one TMA operation)
constexpr int kStages = 8;
constexpr int kTileBytes = kBM * kChunk * 2;      // 8192, one chunk
constexpr int kFactBytes = 16 * 16 * 2;           // 512, one chunk's decoded factor
constexpr int kStageBytes = kStageChunks * kTileBytes;
constexpr int kStageFactBytes = kStageChunks * kFactBytes;
constexpr int kLutFloats = 2 * LITHE_MAX_LEVELS * 16;
constexpr int kXchgFloats = kConsumerWarps * 32 * 8;   // partial h of every consumer thread (one buffer)
constexpr int kMaxTargets = 4;                    // linears sharing x in one lithe_lora_prep_multi call

struct SgmvParams {
    IndexView ia, ib;
    const int32_t* ids;
    const float* weights;
    int32_t* err;
    int64_t n_slots;
    int32_t m, d_in, d_out;
    int32_t n_mtiles, n_xchunks, n_ochunks, total_units;
    int32_t accumulate;
    int32_t out_pairs;          // 1: out tiles come as chunk pairs from a chunked map (d_out % 64 == 0)
    int32_t a_blocks_per_row;   // d_in / 64
    int32_t b_blocks;           // d_out * rank / 64
    float scaling;
    void* out;                  // x's 16-bit type, or fp32 when out_f32
    int32_t out_f32;            // delta-only form (accumulate == 0) writing fp32
    const uint8_t* ws;          // staged mode: decoded factor chunks, (batch, n_chunks, 512 B)
    int32_t n_chunks;           // n_xchunks + n_ochunks (per-sample stride of ws, in chunks)
    __nv_bfloat16* h_out;       // shrink-only mode (lithe_lora_prep): h rows (batch * m, 16), else null
    // Shrink-only mode with a workspace: the CTAs take equal runs of x stages rather than of
    // units, so a unit may be shared by neighbouring CTAs; each stores its fp32 partial h of a
    // shared unit in the workspace, and the B-decode kernel that follows adds them up.
    int32_t split;              // 0, or the stages of every unit (ceil(n_xchunks / 2))
    int32_t split_grid;         // CTAs of the split shrink launch
    int64_t split_total;        // total_units * split
    float* split_part;          // [2 * CTA + (first unit of the CTA ? 0 : 1)][64 rows][16] partial h
    // lithe_lora_prep_multi: n_targets linears that read the same x.  The staged shrink reads
    // target t's A chunk c of sample b from ws + ((b * n_xchunks + c) * n_targets + t) * 512.
    int32_t n_targets;
    IndexView ia_t[kMaxTargets], ib_t[kMaxTargets];
    int32_t d_out_t[kMaxTargets], b_blocks_t[kMaxTargets], n_ochunks_t[kMaxTargets];
    float scaling_t[kMaxTargets];
    __nv_bfloat16* h_t[kMaxTargets];
    __nv_bfloat16* bdec_t[kMaxTargets];
    float lut[2][LITHE_MAX_LEVELS][16];
};

struct Unit {
    int b, mt;
    int64_t slot;
    bool active;
    int nx, no;     // x chunks, out chunks
    int sx, so;     // stages they take: ceil(nx / 2), ceil(no / 2)
};

// The slot ids and weights of the samples a CTA's unit range touches, read once into shared
// memory at kernel start, so that no role waits on a global load when it moves to its next
// unit (those dependent loads stalled the pipeline at every unit boundary).  Samples beyond
// the first kUnitCache of the range (only when units are tiny) are read from global memory.
constexpr int kUnitCache = 128;
struct UnitCache {
    int32_t b0, n;
    int32_t slot[kUnitCache];
    float weight[kUnitCache];
};

__device__ __forceinline__ void fill_unit_cache(UnitCache* uc, const SgmvParams& p, int u_begin, int u_end, int tid,
                                                int nthreads) {
    const int b0 = u_begin / p.n_mtiles;
    const int nb = u_end > u_begin ? (u_end - 1) / p.n_mtiles - b0 + 1 : 0;
    const int n = nb < kUnitCache ? nb : kUnitCache;
    if (tid == 0) {
        uc->b0 = b0;
        uc->n = n;
    }
    for (int i = tid; i < n; i += nthreads) {
        uc->slot[i] = __ldg(p.ids + b0 + i);
        uc->weight[i] = p.weights ? __ldg(p.weights + b0 + i) : 1.0f;
    }
}

__device__ __forceinline__ Unit unit_at(const SgmvParams& p, const UnitCache* uc, int u) {
    Unit r;
    r.b = u / p.n_mtiles;
    r.mt = u - r.b * p.n_mtiles;
    const int i = r.b - uc->b0;
    const int32_t sid = i < uc->n ? uc->slot[i] : __ldg(p.ids + r.b);
    r.slot = sid;
    r.active = sid >= 0 && static_cast<int64_t>(sid) < p.n_slots;
    r.nx = r.active ? p.n_xchunks : 0;
    r.no = (r.active || !p.accumulate) ? p.n_ochunks : 0;
    r.sx = (r.nx + kStageChunks - 1) / kStageChunks;
    r.so = (r.no + kStageChunks - 1) / kStageChunks;
    return r;
}

// Dynamic shared memory of sgmv_index_kernel with kT targets' factor chunks per stage.
constexpr size_t smem_bytes(int kT) {
    return 1024 /*alignment slack*/ + kStages * (kStageBytes + kT * kStageFactBytes) + sizeof(DecodeTables) +
           2 * kXchgFloats * sizeof(float) + (2 * kStages + 2) * sizeof(uint64_t) + kLutFloats * sizeof(float) +
           sizeof(UnitCache) + 16;
}
constexpr size_t kSmemBytes = smem_bytes(1);
static_assert(smem_bytes(kMaxTargets) <= 227 * 1024, "shared memory of the 4-target shrink");

__device__ __forceinline__ float unit_weight(const SgmvParams& p, const UnitCache* uc, int b) {
    const int i = b - uc->b0;
    return i < uc->n ? uc->weight[i] : (p.weights ? __ldg(p.weights + b) : 1.0f);
}

// Split mode: every unit counts p.split stages (unrouted ones too), the stages of all units
// form one sequence of T = p.split_total, and CTA c of the G = p.split_grid runs its stages
// [c T / G, (c + 1) T / G).
__device__ __forceinline__ int64_t split_begin(const SgmvParams& p, int c) {
    return static_cast<int64_t>(c) * p.split_total / p.split_grid;
}
// The CTA whose run holds stage t.
__device__ __forceinline__ int split_owner(const SgmvParams& p, int64_t t) {
    return static_cast<int>(((t + 1) * p.split_grid - 1) / p.split_total);
}
// Where CTA c stores its partial h of unit u (u is its first or its last unit).
__device__ __forceinline__ float* split_piece(const SgmvParams& p, int c, int u) {
    const int first_unit = static_cast<int>(split_begin(p, c) / p.split);
    return p.split_part + static_cast<int64_t>(2 * c + (u == first_unit ? 0 : 1)) * (kBM * 16);
}

// The stages [q0, q1) of unit u that this CTA runs, given its run [tb, te) of the stage
// sequence (split mode); without split every unit of the CTA's range is whole.  A unit without
// x stages (an unrouted sample) is run whole by the CTA holding its first stage and skipped
// by the others.
struct Span {
    int q0, q1;
    int mode;
};
constexpr int kWhole = 0, kPart = 1, kSkip = 2;

__device__ __forceinline__ Span span_of(const SgmvParams& p, const Unit& un, int u, int64_t tb, int64_t te) {
    const int n = un.sx + un.so;
    if (!p.split) return Span{0, n, kWhole};
    const int64_t s0 = static_cast<int64_t>(u) * p.split;
    const int q0 = tb > s0 ? static_cast<int>(tb - s0) : 0;
    const int q1 = te < s0 + p.split ? static_cast<int>(te - s0) : p.split;
    if (q0 == 0 && q1 == p.split) return Span{0, n, kWhole};
    if (un.sx != p.split) return q0 == 0 ? Span{0, n, kWhole} : Span{0, 0, kSkip};
    return Span{q0, q1, kPart};
}

__device__ __forceinline__ uint4 lds128(const uint8_t* a) { return *reinterpret_cast<const uint4*>(a); }
__device__ __forceinline__ void sts128(uint8_t* a, uint4 v) { *reinterpret_cast<uint4*>(a) = v; }

// 16-bit pair word + (dlo, dhi) in fp32, rounded to nearest even
template <bool kF16>
__device__ __forceinline__ uint32_t add_x2(uint32_t w, float dlo, float dhi) {
    return Act<kF16>::pack(Act<kF16>::lo(w) + dlo, Act<kF16>::hi(w) + dhi);
}

// ---------------------------------------------------------------------------------------
// Factor chunks (decoded by the feeder warps)
// ---------------------------------------------------------------------------------------
// Issue the index loads of the block this lane decodes in chunk c of a unit (A chunk
// c < nx, else B chunk c - nx).  Returns false when the lane's values are structurally zero
// (rank rows >= kRank, or past the last B block); then nothing is loaded.
template <int kRank>
__device__ __forceinline__ bool chunk_fetch_v(const IndexView& ia, const IndexView& ib, int a_blocks_per_row,
                                              int b_blocks, const Unit& un, int c, int lane,
                                              RawIndices<LITHE_MAX_LEVELS>& raw) {
    const int row = lane >> 1;          // A: rank row r; B: logical column n
    const int half = lane & 1;
    if (c < un.nx) {
        if (row >= kRank) return false;
        fetch_raw<LITHE_MAX_LEVELS>(ia, un.slot, static_cast<int64_t>(row) * a_blocks_per_row + c, raw);
        return true;
    }
    constexpr int kPer = 16 / kRank;
    const int G = (16 * (c - un.nx) + row) / kPer;
    if (G >= b_blocks || 8 * half >= kRank) return false;
    fetch_raw<LITHE_MAX_LEVELS>(ib, un.slot, G, raw);
    return true;
}

template <int kRank>
__device__ __forceinline__ bool chunk_fetch(const SgmvParams& p, const Unit& un, int c, int lane,
                                            RawIndices<LITHE_MAX_LEVELS>& raw) {
    return chunk_fetch_v<kRank>(p.ia, p.ib, p.a_blocks_per_row, p.b_blocks, un, c, lane, raw);
}

__device__ __forceinline__ void decode_values(const SgmvParams& p, const DecodeTables* tab, const float* lut_s,
                                              int side, const uint32_t* k, uint32_t half, float v[8]) {
    if (p.ia.levels <= 3) decode_eight_fast(tab, side, k, half, v);
    else decode_eight<LITHE_MAX_LEVELS>(lut_s + side * LITHE_MAX_LEVELS * 16, k, p.ia.levels, half, v);
}

// A chunk: rows r = 0..15 (rows >= kRank are zero), values u = 0..15 in natural order.
// Lane (r = lane/2, half = lane&1) writes bytes [r*32 + half*16, +16).
// B chunk: 16 logical columns n, each a 16-rank vector stored with the rank order
// [0,1,8,9, 2,3,10,11, 4,5,12,13, 6,7,14,15] so that an mma B fragment is one 8-byte read.
// Logical column N = 16j + n covers the output columns of block G = N / per, pattern
// offset e = N % per (per = 16/kRank): B[o, r] = w_G[kRank*e + r].
template <int kRank, bool kF16>
__device__ __forceinline__ void decode_chunk(const SgmvParams& p, const DecodeTables* tab, const float* lut_s,
                                             const Unit& un, int c, bool live, const uint32_t* k, uint8_t* fact,
                                             int lane) {
    using T = Act<kF16>;
    const int row = lane >> 1;
    const uint32_t half = lane & 1;
    if (c < un.nx) {
        uint4 q = make_uint4(0, 0, 0, 0);
        if (live) {
            float v[8];
            decode_values(p, tab, lut_s, 0, k, half, v);
            q = make_uint4(T::pack(v[0], v[1]), T::pack(v[2], v[3]), T::pack(v[4], v[5]), T::pack(v[6], v[7]));
        }
        sts128(fact + row * 32 + half * 16, q);
        return;
    }
    constexpr int kPer = 16 / kRank;
    float val[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) val[i] = 0.f;
    if (live) {
        const int e = (16 * (c - un.nx) + row) % kPer;
        const int u0 = kRank * e + 8 * static_cast<int>(half);   // first pattern position needed
        float v[8];
        decode_values(p, tab, lut_s, 1, k, static_cast<uint32_t>(u0 >> 3), v);
        if constexpr (kRank == 16) {
#pragma unroll
            for (int i = 0; i < 8; ++i) val[i] = v[i];
        } else {
            const int off = u0 & 7;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (8 * static_cast<int>(half) + i < kRank) val[i] = v[(off + i) & 7];
        }
    }
    uint32_t* dst = reinterpret_cast<uint32_t*>(fact + row * 32);
#pragma unroll
    for (int i = 0; i < 8; i += 2) dst[(i >> 1) * 2 + half] = T::pack(val[i], val[i + 1]);
}

// The chunks of stage q of a unit, in the unit's chunk numbering (x chunks 0 .. nx-1, then
// out chunks nx .. nx+no-1): the first one and how many (1 or 2).
__device__ __forceinline__ void stage_chunks(const Unit& un, int q, int& c0, int& n) {
    if (q < un.sx) {
        c0 = kStageChunks * q;
        n = un.nx - c0 < kStageChunks ? un.nx - c0 : kStageChunks;
    } else {
        const int j0 = kStageChunks * (q - un.sx);
        c0 = un.nx + j0;
        n = un.no - j0 < kStageChunks ? un.no - j0 : kStageChunks;
    }
}

// Lane 0 of a feeder: the TMA load(s) of stage q's tiles into dst.  x chunks and, when
// d_out % 64 == 0, out chunks come as one 16 KB op from the chunked maps (a missing second
// chunk past the end reads as zeros); ragged out chunks come one 8 KB op each from a
// per-chunk map.  Returns the bytes the loads deliver.
__device__ __forceinline__ uint32_t load_stage_tiles(const SgmvParams& p, const CUtensorMap* tmx,
                                                     const CUtensorMap* tmo, const Unit& un, int q, uint8_t* dst,
                                                     uint64_t* bar, bool expect) {
    int c0, n;
    stage_chunks(un, q, c0, n);
    const int row = un.b * p.m + un.mt * kBM;
    const bool pair = q < un.sx || p.out_pairs;
    const uint32_t bytes = pair ? static_cast<uint32_t>(kStageBytes) : static_cast<uint32_t>(n * kTileBytes);
    if (expect) mbar_expect_tx(bar, bytes);
    if (q < un.sx) {
        tma_load_3d(dst, tmx, bar, 0, row, c0);
    } else if (pair) {
        tma_load_3d(dst, tmo, bar, 0, row, c0 - un.nx);
    } else {
        for (int k = 0; k < n; ++k) tma_load_3d(dst + k * kTileBytes, tmo, bar, (c0 - un.nx + k) * kChunk, row, 0);
    }
    return bytes;
}

// Feeder warp d (of kFeed) owns every pipeline position pos with pos % kFeed == d.  For each
// one it waits until the stage is free, issues the stage's TMA load from lane 0 (the x tiles
// of x chunks; the base-output tiles of out chunks when accumulating) and then, in the fused
// form, decodes the stage's factor chunks while the load is in flight and arrives on the
// stage's full barrier.  The staged form bulk-copies the chunks decode_chunks_kernel wrote
// instead.  The index words of a warp's next stage are fetched before it waits for the
// current one, so their load latency overlaps the wait and the decode.
// Why several feeder warps: on B200 a CTA whose TMA loads all come from one thread streams
// 8 KB boxes at about 20-25 GB/s per SM however deep its pipeline is; with the loads issued by
// four to eight warps the same stream reaches 33-37 GB/s per SM (measured with a streaming
// probe, 57344 x 3072 bf16, one CTA per SM).
// Returns one past the last position this warp issued (all of them have arrived).
template <int kRank, bool kStaged, int kFeed, bool kF16, int kT>
__device__ uint32_t run_feeder(int d, int lane, const SgmvParams& p, const UnitCache* uc, const CUtensorMap* tmx,
                               const CUtensorMap* tmo, uint8_t* tiles, uint8_t* facts, const DecodeTables* tab,
                               const float* lut_s, uint64_t* full, uint64_t* empty, volatile int* abort, int u_begin,
                               int u_end, int64_t hb, int64_t he) {
    int u = u_begin, q = 0;          // cursor: unit, stage within the unit
    uint32_t pos = 0;                // pipeline position of (u, q)
    Unit un;
    Span sp{0, 0, kWhole};
    // Move to the next position owned by this warp (the current one when first == true).
    auto seek = [&](bool first) {
        bool fresh = first;          // entering unit u
        if (!first) {
            ++q;
            ++pos;
        }
        while (u < u_end) {
            if (fresh) {
                un = unit_at(p, uc, u);
                sp = span_of(p, un, u, hb, he);
                q = sp.q0;
                fresh = false;
            }
            if (q < sp.q1) {
                const int skip = (d - static_cast<int>(pos % kFeed) + kFeed) % kFeed;
                if (q + skip < sp.q1) {
                    q += skip;
                    pos += skip;
                    return true;
                }
                pos += sp.q1 - q;
            }
            ++u;
            fresh = true;
        }
        return false;
    };
    uint32_t issued = 0;
    bool have = seek(true);
    RawIndices<LITHE_MAX_LEVELS> raw_next[kStageChunks];
    bool live_next[kStageChunks];
    auto fetch_next = [&]() {
        int c0 = 0, n = 0;
        if (have && un.active) stage_chunks(un, q, c0, n);
#pragma unroll
        for (int k = 0; k < kStageChunks; ++k)
            live_next[k] = k < n && chunk_fetch<kRank>(p, un, c0 + k, lane, raw_next[k]);
    };
    if constexpr (!kStaged) fetch_next();
    while (have) {
        const Unit cur = un;
        const int cq = q;
        const uint32_t cpos = pos;
        RawIndices<LITHE_MAX_LEVELS> raw[kStageChunks];
        bool live[kStageChunks];
#pragma unroll
        for (int k = 0; k < kStageChunks; ++k) {
            raw[k] = raw_next[k];
            live[k] = live_next[k];
        }
        have = seek(false);
        // loads of the next stage go out now and are unpacked only one iteration later
        if constexpr (!kStaged) fetch_next();

        const uint32_t s = cpos % kStages, ph = (cpos / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort, p.err)) return issued;
        const bool tile = cq < cur.sx || p.accumulate;
        uint8_t* dst = tiles + s * kStageBytes;
        uint8_t* fdst = facts + s * (kT * kStageFactBytes);
        int c0, n;
        stage_chunks(cur, cq, c0, n);
        if constexpr (kStaged) {
            if (lane == 0) {
                const uint32_t fbytes = cur.active ? static_cast<uint32_t>(n * kT * kFactBytes) : 0u;
                if (!tile && fbytes == 0) {
                    mbar_arrive(&full[s]);
                } else {
                    if (tile) load_stage_tiles(p, tmx, tmo, cur, cq, dst, &full[s], true);
                    if (fbytes) {
                        mbar_expect_tx(&full[s], fbytes);
                        bulk_load_1d(fdst, p.ws + (static_cast<int64_t>(cur.b) * p.n_chunks + c0) * kT * kFactBytes,
                                     fbytes, &full[s]);
                    }
                    mbar_arrive(&full[s]);
                }
            }
        } else {
            if (lane == 0 && tile) load_stage_tiles(p, tmx, tmo, cur, cq, dst, &full[s], true);
            if (cur.active) {
#pragma unroll
                for (int k = 0; k < kStageChunks; ++k) {
                    if (k < n) {
                        uint32_t kk[LITHE_MAX_LEVELS] = {0, 0, 0, 0};
                        if (live[k]) finish_raw<LITHE_MAX_LEVELS>(c0 + k < cur.nx ? p.ia : p.ib, raw[k], kk, p.err);
                        decode_chunk<kRank, kF16>(p, tab, lut_s, cur, c0 + k, live[k], kk, fdst + k * kFactBytes,
                                                  lane);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
        issued = cpos + 1;
    }
    return issued;
}

// ---------------------------------------------------------------------------------------
// Consumer warps
// ---------------------------------------------------------------------------------------
// Add the two expand results (c0 -> logical column 2t, c1 -> 2t+1 of n8 tile q) to the 8
// contiguous output values a thread owns per row (ranks 16 and 8).
template <int kRank, bool kF16>
__device__ __forceinline__ uint4 add_delta8(uint4 v, float c0, float c1) {
    if constexpr (kRank == 16) {   // columns: c0 c0 c0 c0 c1 c1 c1 c1
        v.x = add_x2<kF16>(v.x, c0, c0);
        v.y = add_x2<kF16>(v.y, c0, c0);
        v.z = add_x2<kF16>(v.z, c1, c1);
        v.w = add_x2<kF16>(v.w, c1, c1);
    } else {                       // columns: c0 c1 c0 c1 ...
        v.x = add_x2<kF16>(v.x, c0, c1);
        v.y = add_x2<kF16>(v.y, c0, c1);
        v.z = add_x2<kF16>(v.z, c0, c1);
        v.w = add_x2<kF16>(v.w, c0, c1);
    }
    return v;
}

// The fp32 delta of one out chunk (rows row0 and row0 + 8, the thread's 8 columns per n8 tile qq):
// the same column pattern as add_delta8 and the small-rank path, written as fp32.
template <int kRank>
__device__ __forceinline__ void store_delta_f32(float* out_b, const SgmvParams& p, int row0, int col0, int t4,
                                                const float (&d)[2][4]) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        const int row = row0 + 8 * hr;
        if (row >= p.m) continue;
        float* orow = out_b + static_cast<int64_t>(row) * p.d_out;
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
            const float c0 = d[qq][2 * hr], c1 = d[qq][2 * hr + 1];
            if constexpr (kRank >= 8) {
                const int col = col0 + 32 * qq + 8 * t4;
                if (col >= p.d_out) continue;
                const float4 a = kRank == 16 ? make_float4(c0, c0, c0, c0) : make_float4(c0, c1, c0, c1);
                const float4 b = kRank == 16 ? make_float4(c1, c1, c1, c1) : make_float4(c0, c1, c0, c1);
                __stcs(reinterpret_cast<float4*>(orow + col), a);
                __stcs(reinterpret_cast<float4*>(orow + col + 4), b);
            } else {
                constexpr int kPer = 16 / kRank;
                const int nl = 8 * qq + 2 * t4;
                const int base = (nl / kPer) * (4 * kPer) + (nl % kPer);
#pragma unroll
                for (int pp = 0; pp < 4; ++pp) {
                    const int col = col0 + base + pp * kPer;
                    if (col < p.d_out) *reinterpret_cast<float2*>(orow + col) = make_float2(c0, c1);
                }
            }
        }
    }
}

template <int kRank, bool kF16, int kT>
__device__ void run_consumer(int w, int lane, const SgmvParams& p, const UnitCache* uc, uint8_t* tiles,
                             const uint8_t* facts, uint64_t* full, uint64_t* empty, float* xchg, uint64_t* xbar,
                             volatile int* abort, int u_begin, int u_end, int64_t hb, int64_t he) {
    const int grp = w / kGroupWarps;     // this warp's group: positions pos % kGroups == grp
    const int wr = w % kGroupWarps;      // row block within the tile
    const int g = lane >> 2, t4 = lane & 3;
    // Fragment row g holds token row gr = sigma(g): a quarter-warp (g = 2q, 2q+1) then reads
    // token rows q and q + 4, whose 128-byte swizzles (16-byte unit ^= row & 7) differ in bit
    // 2, so its eight 16-byte reads hit eight different bank groups (rows 2q, 2q+1 would share
    // four and conflict 2-way).  Rank / logical-column indices stay on g.
    const int gr = (g >> 1) | ((g & 1) << 2);
    const int r0 = 16 * wr + gr;         // rows r0 and r0 + 8 of the 64-token tile
    uint32_t n_xchg = 0;                 // exchanges done (buffer = n_xchg & 1, phase = (n_xchg >> 1) & 1)
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    const bool accum = p.accumulate != 0;
    uint32_t pos = 0;
    for (int u = u_begin; u < u_end; ++u) {
        const Unit un = unit_at(p, uc, u);
        const Span sp = span_of(p, un, u, hb, he);
        if (sp.mode == kSkip) continue;
        if (w == 0 && lane == 0 && !un.active && un.slot >= p.n_slots && p.err) atomicOr(p.err, LITHE_DEVERR_SLOT);
        if (un.nx + un.no == 0) {
            if (p.h_out && grp == 0) {              // unrouted sample: its h rows are zero
#pragma unroll
                for (int t = 0; t < kT; ++t)
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int row = un.mt * kBM + r0 + 8 * hr;
                        if (row < p.m) {
                            __nv_bfloat16* hb_t = kT == 1 ? p.h_out : p.h_t[t];
                            uint32_t* hrow = reinterpret_cast<uint32_t*>(hb_t + (static_cast<int64_t>(un.b) * p.m + row) * 16);
                            hrow[t4] = 0u;
                            hrow[4 + t4] = 0u;
                        }
                    }
            }
            continue;
        }
        // per target, four independent accumulation chains: [rank half][32-column window]
        float acc[kT][2][2][4];
#pragma unroll
        for (int i = 0; i < 16 * kT; ++i) (&acc[0][0][0][0])[i] = 0.f;
        const int qx_end = sp.q1 < un.sx ? sp.q1 : un.sx;       // split spans hold x stages only
        for (int q = sp.q0; q < qx_end; ++q, ++pos) {
            if (static_cast<int>(pos % kGroups) != grp) continue;
            const uint32_t s = pos % kStages, ph = (pos / kStages) & 1u;
            if (!mbar_wait(&full[s], ph, abort, p.err)) return;
#pragma unroll
            for (int k = 0; k < kStageChunks; ++k) {
                if (kStageChunks * q + k >= un.nx) break;
                const uint8_t* tile = tiles + s * kStageBytes + k * kTileBytes;
                // the targets' factor chunks of chunk k: kT consecutive 512-byte blocks
                const uint8_t* fa = facts + s * (kT * kStageFactBytes) + k * kT * kFactBytes;
                const uint8_t* ra = tile + r0 * 128;
                const uint8_t* rb = ra + 8 * 128;
                uint4 f0[kT], f1[kT];
#pragma unroll
                for (int t = 0; t < kT; ++t) {
                    f0[t] = lds128(fa + t * kFactBytes + g * 32 + (t4 & 1) * 16);
                    f1[t] = lds128(fa + t * kFactBytes + (g + 8) * 32 + (t4 & 1) * 16);
                }
#pragma unroll
                for (int win = 0; win < 2; ++win) {
                    const uint4 xa = lds128(ra + (((4 * win + t4) ^ gr) << 4));
                    const uint4 xb = lds128(rb + (((4 * win + t4) ^ gr) << 4));
                    const uint32_t a0[4] = {xa.x, xb.x, xa.y, xb.y};
                    const uint32_t a1[4] = {xa.z, xb.z, xa.w, xb.w};
#pragma unroll
                    for (int t = 0; t < kT; ++t) {
                        Act<kF16>::mma(acc[t][0][win], a0, f0[t].x, f0[t].y, acc[t][0][win]);
                        Act<kF16>::mma(acc[t][1][win], a0, f1[t].x, f1[t].y, acc[t][1][win]);
                        Act<kF16>::mma(acc[t][0][win], a1, f0[t].z, f0[t].w, acc[t][0][win]);
                        Act<kF16>::mma(acc[t][1][win], a1, f1[t].z, f1[t].w, acc[t][1][win]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // The two groups each saw half of the x chunks: add the partner warp's partial h
        // (same rows, other group) through shared memory.  The exchange buffer and its
        // mbarrier alternate between two copies by unit, so one barrier per unit suffices: a
        // warp rewrites copy k only at exchange k + 2, after every warp has arrived at
        // exchange k + 1, which each does only after reading its partner's values of
        // exchange k.  (fp32 addition commutes, so both partners form the same sum.)
        // (With several targets, one exchange per target.)
        const int row0 = un.mt * kBM + r0;                   // token rows row0 and row0 + 8
        uint32_t ha[4];
        bool unit_done = false;
#pragma unroll
        for (int t = 0; t < kT; ++t) {
            float part[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                part[i] = acc[t][0][0][i] + acc[t][0][1][i];
                part[4 + i] = acc[t][1][0][i] + acc[t][1][1][i];
            }
            {
                float* buf = xchg + (n_xchg & 1u) * kXchgFloats;
                uint64_t* bar = &xbar[n_xchg & 1u];
                float4* mine = reinterpret_cast<float4*>(buf + (w * 32 + lane) * 8);
                mine[0] = make_float4(part[0], part[1], part[2], part[3]);
                mine[1] = make_float4(part[4], part[5], part[6], part[7]);
                __syncwarp();
                if (lane == 0) mbar_arrive(bar);
                if (!mbar_wait(bar, (n_xchg >> 1) & 1u, abort, p.err)) return;
                const int partner = (w + kGroupWarps) % kConsumerWarps;
                const float4* other = reinterpret_cast<const float4*>(buf + (partner * 32 + lane) * 8);
                const float4 o0 = other[0], o1 = other[1];
                part[0] += o0.x; part[1] += o0.y; part[2] += o0.z; part[3] += o0.w;
                part[4] += o1.x; part[5] += o1.y; part[6] += o1.z; part[7] += o1.w;
                ++n_xchg;
            }
            if (sp.mode == kPart) {
                // A unit shared with neighbouring CTAs (split shrink, one target): group 0 stores
                // this CTA's fp32 partial h of it (rows r0, r0 + 8; ranks 2 t4, 2 t4 + 1 and
                // 8 + 2 t4, 9 + 2 t4), for the B-decode kernel to add up.
                if (grp == 0) {
                    float* piece = split_piece(p, static_cast<int>(blockIdx.x), u);
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        float* row = piece + (r0 + 8 * hr) * 16;
                        __stcg(reinterpret_cast<float2*>(row + 2 * t4), make_float2(part[2 * hr], part[2 * hr + 1]));
                        __stcg(reinterpret_cast<float2*>(row + 8 + 2 * t4),
                               make_float2(part[4 + 2 * hr], part[5 + 2 * hr]));
                    }
                }
                unit_done = true;
                continue;
            }
            const float sc = (kT == 1 ? p.scaling : p.scaling_t[t]) * unit_weight(p, uc, un.b);
            float h0[4], h1[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                h0[i] = part[i] * sc;
                h1[i] = part[4 + i] * sc;
            }
            ha[0] = Act<kF16>::pack(h0[0], h0[1]);
            ha[1] = Act<kF16>::pack(h0[2], h0[3]);
            ha[2] = Act<kF16>::pack(h1[0], h1[1]);
            ha[3] = Act<kF16>::pack(h1[2], h1[3]);
            if (p.h_out) {
                // shrink-only: store h (ranks 2 t4, 2 t4 + 1 and 8 + 2 t4, 9 + 2 t4 of rows row0, row0 + 8)
                if (grp == 0) {
                    __nv_bfloat16* h_base = kT == 1 ? p.h_out : p.h_t[t];
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int row = row0 + 8 * hr;
                        if (row < p.m) {
                            uint32_t* hrow = reinterpret_cast<uint32_t*>(h_base + (static_cast<int64_t>(un.b) * p.m + row) * 16);
                            hrow[t4] = ha[hr];
                            hrow[4 + t4] = ha[2 + hr];
                        }
                    }
                }
                unit_done = true;
            }
        }
        if (unit_done) continue;
        if constexpr (kT > 1) continue;      // several targets: shrink-only
        uint16_t* out_b = static_cast<uint16_t*>(p.out) + static_cast<int64_t>(un.b) * p.m * p.d_out;
        float* outf_b = static_cast<float*>(p.out) + static_cast<int64_t>(un.b) * p.m * p.d_out;
        for (int q = 0; q < un.so; ++q, ++pos) {
            if (static_cast<int>(pos % kGroups) != grp) continue;
            const uint32_t s = pos % kStages, ph = (pos / kStages) & 1u;
            if (!mbar_wait(&full[s], ph, abort, p.err)) return;
            const int n = un.no - kStageChunks * q < kStageChunks ? un.no - kStageChunks * q : kStageChunks;
#pragma unroll
            for (int k = 0; k < kStageChunks; ++k) {
                if (k >= n) break;
                const bool release = k == n - 1;      // the stage is free once its last tile is in registers
                const int j = kStageChunks * q + k;
                const uint8_t* tile = tiles + s * kStageBytes + k * kTileBytes;
                float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                if (un.active) {
                    const uint8_t* fb = facts + s * kStageFactBytes + k * kFactBytes;
                    const uint2 b0 = *reinterpret_cast<const uint2*>(fb + g * 32 + t4 * 8);
                    const uint2 b1 = *reinterpret_cast<const uint2*>(fb + (g + 8) * 32 + t4 * 8);
                    Act<kF16>::mma(d[0], ha, b0.x, b0.y, zero);
                    Act<kF16>::mma(d[1], ha, b1.x, b1.y, zero);
                }
                const int col0 = j * kChunk;
                if (p.out_f32) {
                    // delta-only form with an fp32 output: nothing is read from the tile
                    if (release) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[s]);
                    }
                    store_delta_f32<kRank>(outf_b, p, row0, col0, t4, d);
                    continue;
                }
                if constexpr (kRank >= 8) {
                    uint4 v[2][2];          // [n8 tile q][row half]
#pragma unroll
                    for (int qq = 0; qq < 2; ++qq)
#pragma unroll
                        for (int hr = 0; hr < 2; ++hr) {
                            const uint4 o = accum ? lds128(tile + (r0 + 8 * hr) * 128 + ((((qq << 2) + t4) ^ gr) << 4))
                                                  : make_uint4(0, 0, 0, 0);
                            v[qq][hr] = add_delta8<kRank, kF16>(o, d[qq][2 * hr], d[qq][2 * hr + 1]);
                        }
                    if (release) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[s]);
                    }
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int row = row0 + 8 * hr;
                        if (row < p.m) {
#pragma unroll
                            for (int qq = 0; qq < 2; ++qq) {
                                const int col = col0 + 32 * qq + 8 * t4;
                                if (col < p.d_out)   // streaming store: out is not re-read by this launch
                                    __stcs(reinterpret_cast<uint4*>(out_b + static_cast<int64_t>(row) * p.d_out + col),
                                           v[qq][hr]);
                            }
                        }
                    }
                } else {
                    constexpr int kPer = 16 / kRank;        // logical columns per block
                    uint32_t v[2][2][4];                    // [qq][row half][pp]
#pragma unroll
                    for (int qq = 0; qq < 2; ++qq) {
                        const int nl = 8 * qq + 2 * t4;     // local logical column of c0
                        const int base = (nl / kPer) * (4 * kPer) + (nl % kPer);
#pragma unroll
                        for (int hr = 0; hr < 2; ++hr)
#pragma unroll
                            for (int pp = 0; pp < 4; ++pp) {
                                const int col = base + pp * kPer;   // even: c0 at col, c1 at col + 1
                                const uint32_t o = accum ? *reinterpret_cast<const uint32_t*>(
                                                               tile + (r0 + 8 * hr) * 128 + (((col >> 3) ^ gr) << 4) +
                                                               (col & 7) * 2)
                                                         : 0u;
                                v[qq][hr][pp] = add_x2<kF16>(o, d[qq][2 * hr], d[qq][2 * hr + 1]);
                            }
                    }
                    if (release) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[s]);
                    }
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int row = row0 + 8 * hr;
                        if (row < p.m) {
#pragma unroll
                            for (int qq = 0; qq < 2; ++qq) {
                                const int nl = 8 * qq + 2 * t4;
                                const int base = (nl / kPer) * (4 * kPer) + (nl % kPer);
#pragma unroll
                                for (int pp = 0; pp < 4; ++pp) {
                                    const int col = col0 + base + pp * kPer;
                                    if (col < p.d_out)
                                        *reinterpret_cast<uint32_t*>(out_b + static_cast<int64_t>(row) * p.d_out + col) =
                                            v[qq][hr][pp];
                                }
                            }
                        }
                    }
                }
            }
        }
    }
}

template <int kRank, bool kStaged, int kFeed, bool kF16, int kT = 1>
__global__ void __launch_bounds__(32 * (kConsumerWarps + kFeed), 1)
    sgmv_index_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmo_ld,
                      const __grid_constant__ SgmvParams p) {
    // Every pipeline wait is a parity wait, which is only correct when the waiter is at most
    // one phase ahead of the barrier.  That holds when the warp (or group) waiting for position
    // pos also owned position pos - kStages on the same stage, i.e. when the owners' counts
    // divide kStages; otherwise two feeders could share a stage in different phases.
    static_assert(kStages % kFeed == 0, "each feeder warp must own whole stages");
    static_assert(kStages % kGroups == 0, "each consumer group must own whole stages");
    // several targets only in the staged shrink (their factor chunks come decoded)
    static_assert(kT == 1 || (kStaged && kRank == 16 && kT <= kMaxTargets), "multi-target form");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* tiles = base;
    uint8_t* facts = tiles + kStages * kStageBytes;
    DecodeTables* tab = reinterpret_cast<DecodeTables*>(facts + kStages * kT * kStageFactBytes);
    float* xchg = reinterpret_cast<float*>(tab + 1);                       // 2 x kXchgFloats
    uint64_t* full = reinterpret_cast<uint64_t*>(xchg + 2 * kXchgFloats);
    uint64_t* empty = full + kStages;
    uint64_t* xbar = empty + kStages;
    float* lut_s = reinterpret_cast<float*>(xbar + 2);
    UnitCache* uc = reinterpret_cast<UnitCache*>(lut_s + kLutFloats);
    volatile int* abort = reinterpret_cast<volatile int*>(uc + 1);

    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);                 // the owning feeder's arrival (+ the TMA bytes)
            mbar_init(&empty[s], kGroupWarps);      // one arrival per warp of the consuming group
        }
        mbar_init(&xbar[0], kConsumerWarps);
        mbar_init(&xbar[1], kConsumerWarps);
        *abort = 0;
        fence_mbar_init();
    }
    // Units [u_begin, u_end); with split, the CTA's share is the stages [hb, he) and its first
    // and last unit may be shared with the neighbouring CTAs.
    int u_begin, u_end;
    int64_t hb = 0, he = 0;
    if (p.split) {
        hb = split_begin(p, blockIdx.x);
        he = split_begin(p, blockIdx.x + 1);
        u_begin = static_cast<int>(hb / p.split);
        u_end = he > hb ? static_cast<int>((he - 1) / p.split) + 1 : u_begin;
    } else {
        u_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.total_units / gridDim.x);
        u_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.total_units / gridDim.x);
    }
    fill_unit_cache(uc, p, u_begin, u_end, tid, blockDim.x);
    if constexpr (!kStaged) {
        for (int i = tid; i < kLutFloats; i += blockDim.x) lut_s[i] = (&p.lut[0][0][0])[i];
        build_decode_tables(tab, &p.lut[0][0][0], p.ia.levels, tid, blockDim.x);
    }
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31;

    uint32_t issued = 0;
    if (warp < kConsumerWarps) {
        run_consumer<kRank, kF16, kT>(warp, lane, p, uc, tiles, facts, full, empty, xchg, xbar, abort, u_begin, u_end, hb,
                                  he);
    } else {
        if (lane == 0) {
            prefetch_tmap(&tmx);
            prefetch_tmap(&tmo_ld);
        }
        issued = run_feeder<kRank, kStaged, kFeed, kF16, kT>(warp - kFirstFeedWarp, lane, p, uc, &tmx, &tmo_ld, tiles,
                                                                 facts,
                                                   tab, lut_s, full, empty, abort, u_begin, u_end, hb, he);
    }
    __syncthreads();
    // After an aborted pipeline, let every feeder's last TMA loads land before the block's
    // shared memory is released (bounded: loads complete in microseconds).  Each of its
    // issued positions has its arrival, so the full barrier completes once the bytes are in.
    if (*abort && warp >= kFirstFeedWarp && lane == 0) {
        const uint32_t d = static_cast<uint32_t>(warp - kFirstFeedWarp);
        const uint64_t t0 = global_timer_ns();
        const uint32_t first = issued > static_cast<uint32_t>(kStages) ? issued - kStages : 0u;
        for (uint32_t q = first; q < issued; ++q) {
            if (q % kFeed != d) continue;
            const uint32_t s = q % kStages, ph = (q / kStages) & 1u;
            while (!mbar_try_wait(&full[s], ph) && global_timer_ns() - t0 < 20000000ull) {
            }
        }
    }
}

// Staged mode, phase 1: decode every routed sample's factor chunks once into the workspace,
// in the exact 512-byte layout the decoder warps write into a stage (decode_chunk).  One warp
// per (sample, chunk); every CTA builds the decode tables once and grid-strides.
template <int kRank, bool kF16>
__global__ void __launch_bounds__(256) decode_chunks_kernel(const __grid_constant__ SgmvParams p, uint8_t* ws,
                                                            int32_t batch) {
    __shared__ DecodeTables tab;
    __shared__ float lut_s[kLutFloats];
    for (int i = threadIdx.x; i < kLutFloats; i += blockDim.x) lut_s[i] = (&p.lut[0][0][0])[i];
    build_decode_tables(&tab, &p.lut[0][0][0], p.ia.levels, threadIdx.x, blockDim.x);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t total = static_cast<int64_t>(batch) * p.n_chunks;
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
        const int b = static_cast<int>(w / p.n_chunks);
        const int c = static_cast<int>(w - static_cast<int64_t>(b) * p.n_chunks);
        const int32_t sid = __ldg(p.ids + b);
        if (sid < 0 || static_cast<int64_t>(sid) >= p.n_slots) continue;   // no factors needed
        Unit un;
        un.b = b;
        un.mt = 0;
        un.slot = sid;
        un.active = true;
        un.nx = p.n_xchunks;
        un.no = p.n_ochunks;
        RawIndices<LITHE_MAX_LEVELS> raw;
        const bool live = chunk_fetch<kRank>(p, un, c, lane, raw);
        uint32_t k[LITHE_MAX_LEVELS] = {0, 0, 0, 0};
        if (live) finish_raw<LITHE_MAX_LEVELS>(c < un.nx ? p.ia : p.ib, raw, k, p.err);
        decode_chunk<kRank, kF16>(p, &tab, lut_s, un, c, live, k, ws + w * kFactBytes, lane);
    }
}

// One 64-column chunk j of sample b's B factor (view ib, b_blocks blocks, d_out rows) decoded
// into bdec (batch, d_out, 16) bf16 by one warp; zero for an unrouted sample.
__device__ __forceinline__ void bdec_chunk(const SgmvParams& p, const IndexView& ib, int b_blocks, int d_out,
                                           __nv_bfloat16* bdec, int b, int j, const DecodeTables* tab,
                                           const float* lut_s, int lane) {
    const uint32_t half = lane & 1;
    const int32_t sid = __ldg(p.ids + b);
    Unit un;
    un.b = b;
    un.mt = 0;
    un.slot = sid;
    un.active = sid >= 0 && static_cast<int64_t>(sid) < p.n_slots;
    un.nx = 0;                        // chunk j of the B side
    un.no = (d_out + kChunk - 1) / kChunk;
    RawIndices<LITHE_MAX_LEVELS> raw;
    const bool live = un.active && chunk_fetch_v<16>(p.ia, ib, p.a_blocks_per_row, b_blocks, un, j, lane, raw);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (live) {
        uint32_t k[LITHE_MAX_LEVELS] = {0, 0, 0, 0};
        finish_raw<LITHE_MAX_LEVELS>(ib, raw, k, p.err);
        decode_values(p, tab, lut_s, 1, k, half, v);
    }
    const int G = 16 * j + (lane >> 1);
    if (4 * G < d_out) {
        const uint4 q = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                                   pack_bf16x2(v[6], v[7]));
        __nv_bfloat16* dst = bdec + (static_cast<int64_t>(b) * d_out + 4 * G) * 16 + 8 * half;
#pragma unroll
        for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(dst + i * 16) = q;
    }
}

// The split shrink's shared units, finished by one warp per CTA boundary c (1 .. G-1) of that
// launch: the boundary that falls first inside a routed unit u adds the partial h of the
// CTAs c - 1 .. (owner of u's last stage) in CTA order, scales by w_b * scaling, rounds to
// bf16 and stores u's h rows -- the same sum whatever order the CTAs ran in.  Lane l takes
// rows 2l and 2l + 1 of the tile.
__device__ __forceinline__ void split_combine(const SgmvParams& p, int c, int lane) {
    const int64_t t = split_begin(p, c);
    if (t % p.split == 0) return;                               // the boundary is a unit edge
    const int u = static_cast<int>(t / p.split);
    const int64_t s0 = static_cast<int64_t>(u) * p.split;
    if (split_owner(p, s0) != c - 1) return;                   // an earlier boundary takes u
    const int b = u / p.n_mtiles, mt = u - b * p.n_mtiles;
    const int32_t sid = __ldg(p.ids + b);
    if (sid < 0 || static_cast<int64_t>(sid) >= p.n_slots) return;   // unrouted: run whole, not split
    const int c_hi = split_owner(p, s0 + p.split - 1);
    float acc[2][16];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 16; ++k) acc[r][k] = 0.f;
    for (int cc = c - 1; cc <= c_hi; ++cc) {
        const float* piece = split_piece(p, cc, u) + 2 * lane * 16;
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(piece + r * 16) + k);
                acc[r][4 * k] += v.x;
                acc[r][4 * k + 1] += v.y;
                acc[r][4 * k + 2] += v.z;
                acc[r][4 * k + 3] += v.w;
            }
    }
    const float sc = p.scaling * (p.weights ? __ldg(p.weights + b) : 1.0f);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = mt * kBM + 2 * lane + r;
        if (row >= p.m) continue;
        uint4* dst = reinterpret_cast<uint4*>(p.h_out + (static_cast<int64_t>(b) * p.m + row) * 16);
        dst[0] = make_uint4(pack_bf16x2(acc[r][0] * sc, acc[r][1] * sc), pack_bf16x2(acc[r][2] * sc, acc[r][3] * sc),
                            pack_bf16x2(acc[r][4] * sc, acc[r][5] * sc), pack_bf16x2(acc[r][6] * sc, acc[r][7] * sc));
        dst[1] = make_uint4(pack_bf16x2(acc[r][8] * sc, acc[r][9] * sc), pack_bf16x2(acc[r][10] * sc, acc[r][11] * sc),
                            pack_bf16x2(acc[r][12] * sc, acc[r][13] * sc),
                            pack_bf16x2(acc[r][14] * sc, acc[r][15] * sc));
    }
}

// lithe_lora_prep, B side: every sample's rank-16 B factor decoded into (batch, d_out, 16)
// bf16, row o = B[o, :] (the operand of the GEMM's fused expand).  For rank 16 a B block G
// holds four identical rows 4G .. 4G + 3, so one warp decodes a 64-column chunk (16 logical
// columns x 2 rank halves, the lanes of decode_chunk) and writes each 8-value half 4 times.
// The values are the fp32 level sums rounded to bf16, exactly as the expand path uses them.
// After a split shrink, warps past the decode work finish its shared units (split_combine).
__global__ void __launch_bounds__(256) decode_bdec_kernel(const __grid_constant__ SgmvParams p,
                                                          __nv_bfloat16* bdec, int32_t batch) {
    __shared__ DecodeTables tab;
    __shared__ float lut_s[kLutFloats];
    for (int i = threadIdx.x; i < kLutFloats; i += blockDim.x) lut_s[i] = (&p.lut[0][0][0])[i];
    build_decode_tables(&tab, &p.lut[0][0][0], p.ia.levels, threadIdx.x, blockDim.x);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t n_dec = bdec ? static_cast<int64_t>(batch) * p.n_ochunks : 0;
    const int64_t total = n_dec + (p.split ? p.split_grid - 1 : 0);
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
        if (w >= n_dec) {
            split_combine(p, static_cast<int>(w - n_dec) + 1, lane);
            continue;
        }
        const int b = static_cast<int>(w / p.n_ochunks);
        const int j = static_cast<int>(w - static_cast<int64_t>(b) * p.n_ochunks);
        bdec_chunk(p, p.ib, p.b_blocks, p.d_out, bdec, b, j, &tab, lut_s, lane);
    }
}

// lithe_lora_prep_multi, phase 1: every routed sample's A chunks of the n_targets linears,
// decoded once into ws in the staged shrink's layout (chunk c of target t of sample b at
// ((b * n_xchunks + c) * n_targets + t) * 512 bytes), and each target's b_dec where asked.
// One warp per (sample, chunk, target) or per (target, sample, out chunk).
__global__ void __launch_bounds__(256) prep_multi_decode_kernel(const __grid_constant__ SgmvParams p, uint8_t* ws,
                                                                int32_t batch) {
    __shared__ DecodeTables tab;
    __shared__ float lut_s[kLutFloats];
    for (int i = threadIdx.x; i < kLutFloats; i += blockDim.x) lut_s[i] = (&p.lut[0][0][0])[i];
    build_decode_tables(&tab, &p.lut[0][0][0], p.ia.levels, threadIdx.x, blockDim.x);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int nt = p.n_targets;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t n_a = static_cast<int64_t>(batch) * p.n_xchunks * nt;
    int64_t n_b[kMaxTargets];
    int64_t total = n_a;
    for (int t = 0; t < kMaxTargets; ++t) {
        n_b[t] = t < nt && p.bdec_t[t] ? static_cast<int64_t>(batch) * p.n_ochunks_t[t] : 0;
        total += n_b[t];
    }
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
        if (w < n_a) {
            const int b = static_cast<int>(w / (static_cast<int64_t>(p.n_xchunks) * nt));
            const int rem = static_cast<int>(w - static_cast<int64_t>(b) * p.n_xchunks * nt);
            const int c = rem / nt, t = rem - (rem / nt) * nt;
            const int32_t sid = __ldg(p.ids + b);
            if (sid < 0 || static_cast<int64_t>(sid) >= p.n_slots) continue;   // its h rows are zeroed
            Unit un;
            un.b = b;
            un.mt = 0;
            un.slot = sid;
            un.active = true;
            un.nx = p.n_xchunks;
            un.no = 0;
            RawIndices<LITHE_MAX_LEVELS> raw;
            const bool live = chunk_fetch_v<16>(p.ia_t[t], p.ib_t[t], p.a_blocks_per_row, p.b_blocks_t[t], un, c, lane,
                                                raw);
            uint32_t k[LITHE_MAX_LEVELS] = {0, 0, 0, 0};
            if (live) finish_raw<LITHE_MAX_LEVELS>(p.ia_t[t], raw, k, p.err);
            decode_chunk<16, false>(p, &tab, lut_s, un, c, live, k, ws + w * kFactBytes, lane);
            continue;
        }
        int64_t r = w - n_a;
        int t = 0;
        while (r >= n_b[t]) r -= n_b[t++];
        const int b = static_cast<int>(r / p.n_ochunks_t[t]);
        const int j = static_cast<int>(r - static_cast<int64_t>(b) * p.n_ochunks_t[t]);
        bdec_chunk(p, p.ib_t[t], p.b_blocks_t[t], p.d_out_t[t], p.bdec_t[t], b, j, &tab, lut_s, lane);
    }
}

template <int kRank, bool kStaged, bool kF16, int kFeed = kStaged ? kFeedStaged : kDecodeWarps>
static int32_t launch_rank(const CUtensorMap& tmx, const CUtensorMap& tmo_ld, const SgmvParams& p, int grid,
                           int device, int sms, int32_t batch, uint8_t* ws, cudaStream_t stream) {
    static bool configured[64] = {false};
    auto kern = sgmv_index_kernel<kRank, kStaged, kFeed, kF16>;
    if (!configured[device]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(sgmv_index_kernel)");
        configured[device] = true;
    }
    if constexpr (kStaged) {
        const int64_t warps_needed = static_cast<int64_t>(batch) * p.n_chunks;
        int64_t blocks = (warps_needed + 7) / 8;
        if (blocks > 2LL * sms) blocks = 2LL * sms;
        decode_chunks_kernel<kRank, kF16><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p, ws, batch);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "decode_chunks_kernel launch");
    }
    kern<<<grid, 32 * (kConsumerWarps + kFeed), kSmemBytes, stream>>>(tmx, tmo_ld, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "sgmv_index_kernel launch");
    return LITHE_OK;
}

// The staged shrink of kT targets (lithe_lora_prep_multi, phase 2).
template <int kT>
static int32_t launch_multi_shrink(const CUtensorMap& tmx, const SgmvParams& p, int grid, int device,
                                   cudaStream_t stream) {
    static bool configured[64] = {false};
    auto kern = sgmv_index_kernel<16, true, kFeedStaged, false, kT>;
    if (!configured[device]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem_bytes(kT)));
        if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(sgmv_index_kernel, targets)");
        configured[device] = true;
    }
    kern<<<grid, 32 * (kConsumerWarps + kFeedStaged), smem_bytes(kT), stream>>>(tmx, tmx, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "sgmv_index_kernel launch (targets)");
    return LITHE_OK;
}

// ---------------------------------------------------------------------------------------
// Small-m form: at most kSmallM token rows per sample (one decode step of a serving batch,
// or the per-sample modulation linears of a diffusion transformer).  A 64-token work unit
// of the persistent kernel would stream 64-row tiles for one live row and keep one CTA per
// sample busy through every chunk, so here the output columns are split over CTAs instead:
//   grid (n_split, batch); CTA (s, b) first forms h[i][r] = sum_k x[b,i,k] A[r,k] for all
//   rows of its sample (the A side is tiny and L2-resident, so every CTA of the sample
//   recomputes it), then adds scale * h . B^T to its share of the B blocks.
// Shrink: thread t owns rank row r = t % kRank and the 64-column chunks c = t / kRank + j *
// (256 / kRank); since A[r, 64c + u + 16q] = a_{r,c}[u], it folds the four 16-column quarters
// of each x chunk before the 16-term dot.  The partial sums are added in a fixed order
// (deterministic).  Decoded values are rounded to bf16 and h * scale to bf16, as in the
// tensor-core form; the expand and the add to out run in fp32.
// Expand: thread t owns B block G (64 values = 64/kRank output rows o, B[o, r] =
// v[(kRank*(o % (64/kRank)) + r) & 15]) and writes its rows for every token row of the sample.
// ---------------------------------------------------------------------------------------
constexpr int kSmallM = 8;
constexpr int kSmallThreads = 256;

template <bool kF16>
__device__ __forceinline__ void decode_block16(const float* lut_side, const uint32_t* k, int levels, float v[16]) {
    decode_eight<LITHE_MAX_LEVELS>(lut_side, k, levels, 0, v);
    decode_eight<LITHE_MAX_LEVELS>(lut_side, k, levels, 1, v + 8);
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = Act<kF16>::round(v[u]);
}

template <int kRank, int kM, bool kF16>
__global__ void __launch_bounds__(kSmallThreads) sgmv_small_kernel(const uint16_t* __restrict__ x,
                                                                   const __grid_constant__ SgmvParams p) {
    using T = Act<kF16>;
    constexpr int kCols = kSmallThreads / kRank;   // chunk stride of the shrink
    constexpr int kRowsPerBlock = 64 / kRank;      // output rows of one B block
    __shared__ float lut_s[kLutFloats];
    __shared__ float part_s[kM][kSmallThreads];
    __shared__ float h_s[kM][kRank];
    const int tid = threadIdx.x;
    const int b = blockIdx.y;
    const int m = p.m;
    const int32_t sid = __ldg(p.ids + b);
    const bool active = sid >= 0 && static_cast<int64_t>(sid) < p.n_slots;
    if (!active) {
        if (sid >= 0 && blockIdx.x == 0 && tid == 0 && p.err) atomicOr(p.err, LITHE_DEVERR_SLOT);
        if (p.accumulate) return;               // unrouted sample: out unchanged
    }
    for (int i = tid; i < kLutFloats; i += kSmallThreads) lut_s[i] = (&p.lut[0][0][0])[i];
    __syncthreads();

    // ---- shrink
    float acc[kM];
#pragma unroll
    for (int i = 0; i < kM; ++i) acc[i] = 0.f;
    const int r = tid % kRank;
    if (active) {
        for (int c = tid / kRank; c < p.n_xchunks; c += kCols) {
            uint32_t k[LITHE_MAX_LEVELS] = {0, 0, 0, 0};
            fetch_indices<LITHE_MAX_LEVELS>(p.ia, sid, static_cast<int64_t>(r) * p.a_blocks_per_row + c, k, p.err);
            float a[16];
            decode_block16<kF16>(lut_s, k, p.ia.levels, a);
#pragma unroll
            for (int i = 0; i < kM; ++i) {
                if (i < m) {
                    const uint4* xr = reinterpret_cast<const uint4*>(x + (static_cast<int64_t>(b) * m + i) * p.d_in +
                                                                     static_cast<int64_t>(kChunk) * c);
                    float f[16];
#pragma unroll
                    for (int u = 0; u < 16; ++u) f[u] = 0.f;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {        // 8 bf16 at columns 8q .. 8q + 7, u = 8 (q & 1) + j
                        const uint4 w = __ldg(xr + q);
                        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            f[8 * (q & 1) + 2 * j] += T::lo(ww[j]);
                            f[8 * (q & 1) + 2 * j + 1] += T::hi(ww[j]);
                        }
                    }
                    float s = 0.f;
#pragma unroll
                    for (int u = 0; u < 16; ++u) s = fmaf(a[u], f[u], s);
                    acc[i] += s;
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < kM; ++i) part_s[i][tid] = acc[i];
    __syncthreads();
    if (tid < kM * kRank) {
        const int i = tid / kRank, rr = tid % kRank;
        float s = 0.f;
        for (int c0 = 0; c0 < kCols; ++c0) s += part_s[i][rr + kRank * c0];
        const float sc = p.scaling * (p.weights ? __ldg(p.weights + b) : 1.0f);
        h_s[i][rr] = active ? T::round(s * sc) : 0.f;
    }
    __syncthreads();

    // ---- expand
    const float* lut_b = lut_s + LITHE_MAX_LEVELS * 16;
    for (int64_t G = static_cast<int64_t>(blockIdx.x) * kSmallThreads + tid; G < p.b_blocks;
         G += static_cast<int64_t>(gridDim.x) * kSmallThreads) {
        float v[16];
        if (active) {
            uint32_t k[LITHE_MAX_LEVELS] = {0, 0, 0, 0};
            fetch_indices<LITHE_MAX_LEVELS>(p.ib, sid, G, k, p.err);
            decode_block16<kF16>(lut_b, k, p.ia.levels, v);
        } else {
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < kM; ++i) {
            if (i < m) {
                const int64_t orow = (static_cast<int64_t>(b) * m + i) * p.d_out + G * kRowsPerBlock;
#pragma unroll
                for (int q0 = 0; q0 < kRowsPerBlock; q0 += 4) {   // 4 output rows = one 8-byte access
                    float d[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float s = 0.f;
#pragma unroll
                        for (int rr = 0; rr < kRank; ++rr) s = fmaf(h_s[i][rr], v[(kRank * (q0 + e) + rr) & 15], s);
                        d[e] = s;
                    }
                    if (p.out_f32) {      // delta-only form with an fp32 output
                        *reinterpret_cast<float4*>(static_cast<float*>(p.out) + orow + q0) =
                            make_float4(d[0], d[1], d[2], d[3]);
                        continue;
                    }
                    uint2* dst = reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + orow + q0);
                    uint2 o = make_uint2(0u, 0u);
                    if (p.accumulate) o = *dst;
                    *dst = make_uint2(add_x2<kF16>(o.x, d[0], d[1]), add_x2<kF16>(o.y, d[2], d[3]));
                }
            }
        }
    }
}

template <int kRank, bool kF16>
static int32_t launch_small_rank(const uint16_t* x, const SgmvParams& p, int32_t batch, int sms,
                                 cudaStream_t stream) {
    // one B block per thread, but no more CTAs per sample than fill ~2 waves of the SMs
    const int64_t per_sample = (static_cast<int64_t>(p.b_blocks) + kSmallThreads - 1) / kSmallThreads;
    const int64_t fill = (2LL * sms + batch - 1) / batch;
    const int64_t split = per_sample < fill ? per_sample : (fill < 1 ? 1 : fill);
    const dim3 grid(static_cast<unsigned>(split), static_cast<unsigned>(batch));
    if (p.m <= 1) sgmv_small_kernel<kRank, 1, kF16><<<grid, kSmallThreads, 0, stream>>>(x, p);
    else if (p.m <= 2) sgmv_small_kernel<kRank, 2, kF16><<<grid, kSmallThreads, 0, stream>>>(x, p);
    else if (p.m <= 4) sgmv_small_kernel<kRank, 4, kF16><<<grid, kSmallThreads, 0, stream>>>(x, p);
    else sgmv_small_kernel<kRank, kSmallM, kF16><<<grid, kSmallThreads, 0, stream>>>(x, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "sgmv_small_kernel launch");
    return LITHE_OK;
}

template <bool kF16>
static int32_t launch_small(const uint16_t* x, const SgmvParams& p, int32_t rank, int32_t batch, int sms,
                            cudaStream_t stream) {
    if (batch > 65535) return fail_unsupported("the small-m form takes at most 65535 samples, got %d", batch);
    switch (rank) {
        case 16: return launch_small_rank<16, kF16>(x, p, batch, sms, stream);
        case 8: return launch_small_rank<8, kF16>(x, p, batch, sms, stream);
        case 4: return launch_small_rank<4, kF16>(x, p, batch, sms, stream);
        case 2: return launch_small_rank<2, kF16>(x, p, batch, sms, stream);
        default: return launch_small_rank<1, kF16>(x, p, batch, sms, stream);
    }
}

static int32_t check_view(const lithe_index_view* v, const char* name) {
    if (!v) return fail_arg("%s is NULL", name);
    if (!v->base) return fail_arg("%s.base is NULL", name);
    if (v->format != LITHE_IDX_PACKED9 && v->format != LITHE_IDX_I16 && v->format != LITHE_IDX_I32)
        return fail_arg("%s.format %d is not a LITHE_IDX_* value", name, v->format);
    if (v->num_levels < 1 || v->num_levels > LITHE_MAX_LEVELS)
        return fail_unsupported("%s.num_levels must be in [1, %d], got %d", name, LITHE_MAX_LEVELS, v->num_levels);
    const int align = v->format == LITHE_IDX_PACKED9 ? 8 : (v->format == LITHE_IDX_I32 ? 4 : 2);
    if (reinterpret_cast<uintptr_t>(v->base) % align) return fail_arg("%s.base is misaligned", name);
    if (v->slot_stride < 0 || v->offset < 0 || v->level_stride < 0)
        return fail_arg("%s has a negative stride or offset", name);
    return LITHE_OK;
}

static IndexView to_view(const lithe_index_view* v) {
    IndexView r;
    r.base = v->base;
    r.format = v->format;
    r.levels = v->num_levels;
    r.slot_stride = v->slot_stride;
    r.offset = v->offset;
    r.level_stride = v->level_stride;
    return r;
}

}  // namespace lithe

namespace lithe {

int64_t sgmv_workspace_bytes(int32_t batch, int32_t d_in, int32_t d_out) {
    if (batch <= 0 || d_in <= 0 || d_out <= 0) return 0;
    return static_cast<int64_t>(batch) * (d_in / kChunk + (d_out + kChunk - 1) / kChunk) * kFactBytes;
}

// The split shrink (lithe_lora_prep_ws): per CTA two 64 x 16 fp32 partial-h pieces.  The grid
// is min(total stages, SMs).
constexpr int64_t kPrepPieceBytes = kBM * 16 * sizeof(float);
int64_t prep_split_grid(int32_t batch, int32_t m, int32_t d_in, int sms) {
    if (batch <= 0 || m <= 0 || d_in <= 0) return 0;
    const int64_t units = (static_cast<int64_t>(m) + kBM - 1) / kBM * batch;
    const int64_t stages = units * ((d_in / kChunk + kStageChunks - 1) / kStageChunks);
    return stages < sms ? stages : sms;
}
int64_t prep_split_bytes(int64_t grid) { return grid * 2 * kPrepPieceBytes; }

// Shared by the C entry points.  ws == nullptr: fused mode (decoder warps in the SGMV kernel);
// otherwise staged mode with ws_bytes >= sgmv_workspace_bytes(batch, d_in, d_out), or, with
// prep, the split shrink with ws_bytes >= prep_split_bytes(prep_split_grid(...)).
int32_t sgmv_index_impl(const void* x, void* out, int32_t accumulate, const lithe_index_view* idx_a,
                        const lithe_index_view* idx_b, int64_t n_slots, const int32_t* ids, const float* weights,
                        int32_t batch, int32_t m, int32_t d_in, int32_t d_out, int32_t rank, const float* lut,
                        float scaling, int32_t* err_flag, void* ws, int64_t ws_bytes, void* stream,
                        void* h_out = nullptr, void* bdec_out = nullptr, bool prep = false,
                        int32_t x_dtype = LITHE_DTYPE_BF16, int32_t out_dtype = LITHE_DTYPE_BF16) {
    if (batch < 0 || m < 0) return fail_arg("batch (%d) and m (%d) must be >= 0", batch, m);
    if (x_dtype != LITHE_DTYPE_BF16 && x_dtype != LITHE_DTYPE_F16)
        return fail_unsupported("x_dtype must be LITHE_DTYPE_BF16 or LITHE_DTYPE_F16, got %d", x_dtype);
    if (out_dtype != x_dtype && !(out_dtype == LITHE_DTYPE_F32 && !accumulate))
        return fail_unsupported("out_dtype must be x's dtype, or LITHE_DTYPE_F32 when accumulate == 0 (got x %d, "
                                "out %d, accumulate %d)", x_dtype, out_dtype, accumulate);
    if (prep && x_dtype != LITHE_DTYPE_BF16) return fail_unsupported("lithe_lora_prep takes bf16 activations");
    if (ws && out_dtype == LITHE_DTYPE_F32)
        return fail_unsupported("the staged form writes the activation dtype; use lithe_sgmv_index_typed");
    const bool f16 = x_dtype == LITHE_DTYPE_F16;
    if (rank != 1 && rank != 2 && rank != 4 && rank != 8 && rank != 16)
        return fail_unsupported("rank must be one of 1, 2, 4, 8, 16; got %d", rank);
    if (d_in <= 0 || d_in % 64) return fail_arg("d_in must be a positive multiple of 64, got %d", d_in);
    if (d_out <= 0 || d_out % 8) return fail_arg("d_out must be a positive multiple of 8, got %d", d_out);
    if ((static_cast<int64_t>(d_out) * rank) % 64)
        return fail_arg("d_out * rank must be a multiple of 64 (d_out=%d, rank=%d)", d_out, rank);
    int32_t rc = check_view(idx_a, "idx_a");
    if (rc != LITHE_OK) return rc;
    rc = check_view(idx_b, "idx_b");
    if (rc != LITHE_OK) return rc;
    if (idx_a->num_levels != idx_b->num_levels) return fail_arg("idx_a and idx_b have different num_levels");
    {
        const int64_t nb_a = static_cast<int64_t>(rank) * d_in / 64, nb_b = static_cast<int64_t>(d_out) * rank / 64;
        if ((idx_a->format == LITHE_IDX_PACKED9 && idx_a->offset + idx_a->num_levels * nb_a > 0xffffffffLL) ||
            (idx_b->format == LITHE_IDX_PACKED9 && idx_b->offset + idx_b->num_levels * nb_b > 0xffffffffLL))
            return fail_unsupported("packed stream positions of one slot must fit in 32 bits");
    }
    if (!lut) return fail_arg("lut is NULL");
    if (n_slots < 0) return fail_arg("n_slots must be >= 0");
    if (batch == 0 || m == 0) return LITHE_OK;
    if (prep) {
        if (rank != 16) return fail_unsupported("lithe_lora_prep supports rank 16, got %d", rank);
        if (!h_out && !bdec_out) return fail_arg("h and b_dec are both NULL");
        if (reinterpret_cast<uintptr_t>(h_out) % 16 || reinterpret_cast<uintptr_t>(bdec_out) % 16)
            return fail_arg("h and b_dec must be 16-byte aligned");
        out = h_out ? h_out : bdec_out;   // only used for the alignment check and an unused tensor map below
    }
    if (!x || !out || !ids) return fail_arg("x, out and ids must be non-NULL");
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return fail_arg("x and out must be 16-byte aligned");
    const int64_t n_mtiles = (static_cast<int64_t>(m) + kBM - 1) / kBM;
    if (n_mtiles * batch > 0x7fffffffLL || static_cast<int64_t>(m) * batch > 0x7fffffffLL)
        return fail_arg("batch * m exceeds 2^31");

    int device = 0, sms = 0;
    rc = current_device_sms(&device, &sms);
    if (rc != LITHE_OK) return rc;

    SgmvParams p{};
    p.ia = to_view(idx_a);
    p.ib = to_view(idx_b);
    p.ids = ids;
    p.weights = weights;
    p.err = err_flag;
    p.n_slots = n_slots;
    p.m = m;
    p.d_in = d_in;
    p.d_out = d_out;
    p.n_mtiles = static_cast<int32_t>(n_mtiles);
    p.n_xchunks = d_in / kChunk;
    p.n_ochunks = (d_out + kChunk - 1) / kChunk;
    p.total_units = static_cast<int32_t>(n_mtiles * batch);
    p.accumulate = accumulate ? 1 : 0;
    p.a_blocks_per_row = d_in / 64;
    p.b_blocks = static_cast<int32_t>(static_cast<int64_t>(d_out) * rank / 64);
    p.scaling = scaling;
    p.out = out;
    p.out_f32 = out_dtype == LITHE_DTYPE_F32 ? 1 : 0;
    expand_lut(lut, idx_a->num_levels, p.lut);

    p.n_chunks = p.n_xchunks + p.n_ochunks;
    p.ws = static_cast<const uint8_t*>(ws);
    p.h_out = nullptr;
    if (ws && !prep) {
        if (reinterpret_cast<uintptr_t>(ws) % 16) return fail_arg("workspace must be 16-byte aligned");
        const int64_t need = sgmv_workspace_bytes(batch, d_in, d_out);
        if (ws_bytes < need)
            return fail_arg("workspace holds %lld bytes, this call needs %lld", (long long)ws_bytes, (long long)need);
    }
    // A few token rows per sample (decode-time serving, modulation linears): the small-m form,
    // in every entry point (it needs no workspace, so the staged and fused modes agree).
    if (!prep && m <= kSmallM)
        return f16 ? launch_small<true>(static_cast<const uint16_t*>(x), p, rank, batch, sms,
                                        static_cast<cudaStream_t>(stream))
                   : launch_small<false>(static_cast<const uint16_t*>(x), p, rank, batch, sms,
                                                          static_cast<cudaStream_t>(stream));

    CUtensorMap tmx, tmo_ld;
    // Tensor maps over the flattened (batch * m) rows: measured on B200, a (d, m, batch) map
    // with a (64, 64, 1) box streams about 15% slower than a map over the same rows.  The
    // last tile of a sample may then read the next sample's first rows; those rows are never
    // stored (stores are bounded by the sample's own m), and rows past the tensor read zeros.
    // x and, when d_out % 64 == 0, out are read as chunk pairs through chunked maps (one
    // 16 KB TMA op per stage); a ragged d_out is read one 64-column chunk per op.
    const uint64_t rows_total = static_cast<uint64_t>(m) * batch;
    rc = encode_bf16_chunked(&tmx, x, d_in, rows_total, kBM, kStageChunks);
    if (rc != LITHE_OK) return rc;
    p.out_pairs = 0;
    if (prep) {
        tmo_ld = tmx;                 // no out tiles in shrink-only mode
    } else if (d_out % kChunk == 0) {
        rc = encode_bf16_chunked(&tmo_ld, out, d_out, rows_total, kBM, kStageChunks);
        if (rc != LITHE_OK) return rc;
        p.out_pairs = 1;
    } else {
        rc = encode_bf16_3d(&tmo_ld, out, d_out, rows_total, 1, kChunk, kBM);
        if (rc != LITHE_OK) return rc;
    }

    if (prep) {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        int64_t grid = p.total_units < sms ? p.total_units : sms;
        if (ws && h_out) {
            // split shrink: equal runs of x stages per CTA, partial h of shared units in ws
            grid = prep_split_grid(batch, m, d_in, sms);
            if (reinterpret_cast<uintptr_t>(ws) % 16) return fail_arg("workspace must be 16-byte aligned");
            const int64_t need = prep_split_bytes(grid);
            if (ws_bytes < need)
                return fail_arg("workspace holds %lld bytes, this call needs %lld", (long long)ws_bytes,
                                (long long)need);
            p.split = (p.n_xchunks + kStageChunks - 1) / kStageChunks;
            p.split_grid = static_cast<int32_t>(grid);
            p.split_total = static_cast<int64_t>(p.total_units) * p.split;
            p.split_part = static_cast<float*>(ws);
        }
        p.h_out = static_cast<__nv_bfloat16*>(h_out);
        // B side: every sample's decoded factor, (batch, d_out, 16), and after a split shrink
        // the shared units' h
        auto launch_bdec = [&]() -> int32_t {
            const int64_t warps_needed =
                (bdec_out ? static_cast<int64_t>(batch) * p.n_ochunks : 0) + (p.split ? p.split_grid - 1 : 0);
            if (warps_needed == 0) return LITHE_OK;
            int64_t blocks = (warps_needed + 7) / 8;
            if (blocks > 2LL * sms) blocks = 2LL * sms;
            decode_bdec_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(p, static_cast<__nv_bfloat16*>(bdec_out),
                                                                              batch);
            cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? LITHE_OK : fail_cuda(e, "decode_bdec_kernel launch");
        };
        if (!p.split) {
            rc = launch_bdec();
            if (rc != LITHE_OK || !h_out) return rc;
        }
        // A side: the fused kernel in shrink-only form (x tiles only, h stored after the shrink;
        // unrouted samples skip all work and their h rows are zeroed).  Every x tile needs an
        // A-chunk decode and no output tile is streamed, so the decode dominates: 8 feeder warps.
        SgmvParams ps = p;
        ps.n_ochunks = 0;
        ps.accumulate = 1;
        ps.n_chunks = ps.n_xchunks;
        ps.out = nullptr;
        rc = launch_rank<16, false, false, 2 * kDecodeWarps>(tmx, tmo_ld, ps, static_cast<int>(grid), device, sms,
                                                             batch, nullptr, s);
        if (rc != LITHE_OK || !p.split) return rc;
        return launch_bdec();
    }

    const int grid = static_cast<int>(p.total_units < sms ? p.total_units : sms);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t* w = static_cast<uint8_t*>(ws);
#define LITHE_LAUNCH(R)                                                                                     \
    if (ws) return f16 ? launch_rank<R, true, true>(tmx, tmo_ld, p, grid, device, sms, batch, w, s)               \
                       : launch_rank<R, true, false>(tmx, tmo_ld, p, grid, device, sms, batch, w, s);             \
    return f16 ? launch_rank<R, false, true>(tmx, tmo_ld, p, grid, device, sms, batch, w, s)                      \
               : launch_rank<R, false, false>(tmx, tmo_ld, p, grid, device, sms, batch, w, s)
    switch (rank) {
        case 16: LITHE_LAUNCH(16);
        case 8: LITHE_LAUNCH(8);
        case 4: LITHE_LAUNCH(4);
        case 2: LITHE_LAUNCH(2);
        default: LITHE_LAUNCH(1);
    }
#undef LITHE_LAUNCH
}

int64_t prep_multi_bytes(int32_t batch, int32_t d_in, int32_t n_targets) {
    if (batch <= 0 || d_in <= 0 || n_targets <= 0) return 0;
    return static_cast<int64_t>(batch) * (d_in / kChunk) * n_targets * kFactBytes;
}

// lithe_lora_prep_multi: n_targets rank-16 linears that read the same x.
int32_t prep_multi_impl(const void* x, int32_t n_targets, const lithe_index_view* idx_a,
                        const lithe_index_view* idx_b, const int32_t* d_out, int64_t n_slots, const int32_t* ids,
                        const float* weights, int32_t batch, int32_t m, int32_t d_in, int32_t rank, const float* lut,
                        const float* scaling, void* const* h, void* const* b_dec, int32_t* err_flag, void* ws,
                        int64_t ws_bytes, void* stream) {
    if (batch < 0 || m < 0) return fail_arg("batch (%d) and m (%d) must be >= 0", batch, m);
    if (n_targets < 1 || n_targets > kMaxTargets)
        return fail_unsupported("n_targets must be in [1, %d], got %d", kMaxTargets, n_targets);
    if (!idx_a || !idx_b || !d_out || !scaling || !h || !b_dec)
        return fail_arg("idx_a, idx_b, d_out, scaling, h and b_dec must be non-NULL arrays");
    if (rank != 16) return fail_unsupported("lithe_lora_prep_multi supports rank 16, got %d", rank);
    if (d_in <= 0 || d_in % 64) return fail_arg("d_in must be a positive multiple of 64, got %d", d_in);
    if (!lut) return fail_arg("lut is NULL");
    if (n_slots < 0) return fail_arg("n_slots must be >= 0");
    int32_t rc = LITHE_OK;
    for (int t = 0; t < n_targets; ++t) {
        if (d_out[t] <= 0 || d_out[t] % 8) return fail_arg("d_out[%d] must be a positive multiple of 8", t);
        rc = check_view(&idx_a[t], "idx_a");
        if (rc != LITHE_OK) return rc;
        rc = check_view(&idx_b[t], "idx_b");
        if (rc != LITHE_OK) return rc;
        if (idx_a[t].num_levels != idx_a[0].num_levels || idx_b[t].num_levels != idx_a[0].num_levels)
            return fail_arg("every view must have the same num_levels");
        const int64_t nb_a = 16LL * d_in / 64, nb_b = static_cast<int64_t>(d_out[t]) * 16 / 64;
        if ((idx_a[t].format == LITHE_IDX_PACKED9 && idx_a[t].offset + idx_a[t].num_levels * nb_a > 0xffffffffLL) ||
            (idx_b[t].format == LITHE_IDX_PACKED9 && idx_b[t].offset + idx_b[t].num_levels * nb_b > 0xffffffffLL))
            return fail_unsupported("packed stream positions of one slot must fit in 32 bits");
    }
    if (batch == 0 || m == 0) return LITHE_OK;
    if (!x || !ids) return fail_arg("x and ids must be non-NULL");
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail_arg("x must be 16-byte aligned");
    for (int t = 0; t < n_targets; ++t) {
        if (!h[t]) return fail_arg("h[%d] is NULL", t);
        if (reinterpret_cast<uintptr_t>(h[t]) % 16 || reinterpret_cast<uintptr_t>(b_dec[t]) % 16)
            return fail_arg("h[%d] and b_dec[%d] must be 16-byte aligned", t, t);
    }
    const int64_t n_mtiles = (static_cast<int64_t>(m) + kBM - 1) / kBM;
    if (n_mtiles * batch > 0x7fffffffLL || static_cast<int64_t>(m) * batch > 0x7fffffffLL)
        return fail_arg("batch * m exceeds 2^31");
    const int64_t need = prep_multi_bytes(batch, d_in, n_targets);
    if (!ws || reinterpret_cast<uintptr_t>(ws) % 16) return fail_arg("workspace must be non-NULL and 16-byte aligned");
    if (ws_bytes < need)
        return fail_arg("workspace holds %lld bytes, this call needs %lld", (long long)ws_bytes, (long long)need);

    int device = 0, sms = 0;
    rc = current_device_sms(&device, &sms);
    if (rc != LITHE_OK) return rc;

    SgmvParams p{};
    p.ia = to_view(&idx_a[0]);
    p.ib = to_view(&idx_b[0]);
    p.ids = ids;
    p.weights = weights;
    p.err = err_flag;
    p.n_slots = n_slots;
    p.m = m;
    p.d_in = d_in;
    p.d_out = d_out[0];
    p.n_mtiles = static_cast<int32_t>(n_mtiles);
    p.n_xchunks = d_in / kChunk;
    p.total_units = static_cast<int32_t>(n_mtiles * batch);
    p.a_blocks_per_row = d_in / 64;
    p.b_blocks = d_out[0] * 16 / 64;
    p.scaling = scaling[0];
    expand_lut(lut, idx_a[0].num_levels, p.lut);
    p.n_targets = n_targets;
    for (int t = 0; t < n_targets; ++t) {
        p.ia_t[t] = to_view(&idx_a[t]);
        p.ib_t[t] = to_view(&idx_b[t]);
        p.d_out_t[t] = d_out[t];
        p.b_blocks_t[t] = d_out[t] * 16 / 64;
        p.n_ochunks_t[t] = (d_out[t] + kChunk - 1) / kChunk;
        p.scaling_t[t] = scaling[t];
        p.h_t[t] = static_cast<__nv_bfloat16*>(h[t]);
        p.bdec_t[t] = static_cast<__nv_bfloat16*>(b_dec[t]);
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    {   // phase 1: the targets' A chunks into ws, and their b_dec
        int64_t warps_needed = static_cast<int64_t>(batch) * p.n_xchunks * n_targets;
        for (int t = 0; t < n_targets; ++t)
            if (b_dec[t]) warps_needed += static_cast<int64_t>(batch) * p.n_ochunks_t[t];
        int64_t blocks = (warps_needed + 7) / 8;
        if (blocks > 2LL * sms) blocks = 2LL * sms;
        prep_multi_decode_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(p, static_cast<uint8_t*>(ws), batch);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "prep_multi_decode_kernel launch");
    }
    // phase 2: the staged shrink, x read once for every target
    CUtensorMap tmx;
    rc = encode_bf16_chunked(&tmx, x, d_in, static_cast<uint64_t>(m) * batch, kBM, kStageChunks);
    if (rc != LITHE_OK) return rc;
    p.ws = static_cast<const uint8_t*>(ws);
    p.n_chunks = p.n_xchunks;
    p.n_ochunks = 0;
    p.accumulate = 1;                 // unrouted samples skip all work (their h rows are zeroed)
    p.h_out = p.h_t[0];
    const int grid = static_cast<int>(p.total_units < sms ? p.total_units : sms);
    switch (n_targets) {
        case 1: return launch_multi_shrink<1>(tmx, p, grid, device, s);
        case 2: return launch_multi_shrink<2>(tmx, p, grid, device, s);
        case 3: return launch_multi_shrink<3>(tmx, p, grid, device, s);
        default: return launch_multi_shrink<4>(tmx, p, grid, device, s);
    }
}

}  // namespace lithe

extern "C" int32_t lithe_sgmv_index(const void* x, void* out, int32_t accumulate, const lithe_index_view* idx_a,
                                    const lithe_index_view* idx_b, int64_t n_slots, const int32_t* ids,
                                    const float* weights, int32_t batch, int32_t m, int32_t d_in, int32_t d_out,
                                    int32_t rank, const float* lut, float scaling, int32_t* err_flag, void* stream) {
    lithe::clear_error();
    return lithe::sgmv_index_impl(x, out, accumulate, idx_a, idx_b, n_slots, ids, weights, batch, m, d_in, d_out,
                                  rank, lut, scaling, err_flag, nullptr, 0, stream);
}

extern "C" int32_t lithe_sgmv_index_typed(const void* x, void* out, int32_t accumulate,
                                          const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                                          int64_t n_slots, const int32_t* ids, const float* weights, int32_t batch,
                                          int32_t m, int32_t d_in, int32_t d_out, int32_t rank, const float* lut,
                                          float scaling, int32_t x_dtype, int32_t out_dtype, int32_t* err_flag,
                                          void* stream) {
    lithe::clear_error();
    return lithe::sgmv_index_impl(x, out, accumulate, idx_a, idx_b, n_slots, ids, weights, batch, m, d_in, d_out,
                                  rank, lut, scaling, err_flag, nullptr, 0, stream, nullptr, nullptr, false, x_dtype,
                                  out_dtype);
}

extern "C" int32_t lithe_lora_prep(const void* x, const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                                   int64_t n_slots, const int32_t* ids, const float* weights, int32_t batch, int32_t m,
                                   int32_t d_in, int32_t d_out, int32_t rank, const float* lut, float scaling, void* h,
                                   void* b_dec, int32_t* err_flag, void* stream) {
    lithe::clear_error();
    if (batch > 0 && m > 0 && !h && !b_dec) return lithe::fail_arg("h and b_dec are both NULL");
    return lithe::sgmv_index_impl(x, h ? h : b_dec, 1, idx_a, idx_b, n_slots, ids, weights, batch, m, d_in, d_out,
                                  rank, lut, scaling, err_flag, nullptr, 0, stream, h, b_dec, true);
}

extern "C" int32_t lithe_lora_prep_ws(const void* x, const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                                      int64_t n_slots, const int32_t* ids, const float* weights, int32_t batch,
                                      int32_t m, int32_t d_in, int32_t d_out, int32_t rank, const float* lut,
                                      float scaling, void* h, void* b_dec, int32_t* err_flag, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
    lithe::clear_error();
    if (batch > 0 && m > 0 && !h && !b_dec) return lithe::fail_arg("h and b_dec are both NULL");
    if (batch > 0 && m > 0 && h && !workspace) return lithe::fail_arg("workspace is NULL");
    return lithe::sgmv_index_impl(x, h ? h : b_dec, 1, idx_a, idx_b, n_slots, ids, weights, batch, m, d_in, d_out,
                                  rank, lut, scaling, err_flag, workspace, workspace_bytes, stream, h, b_dec, true);
}

extern "C" int64_t lithe_lora_prep_workspace_bytes(int32_t batch, int32_t m, int32_t d_in) {
    lithe::clear_error();
    int device = 0, sms = 0;
    const int32_t rc = lithe::current_device_sms(&device, &sms);
    if (rc != LITHE_OK) return rc;
    return lithe::prep_split_bytes(lithe::prep_split_grid(batch, m, d_in, sms));
}

extern "C" int64_t lithe_lora_prep_multi_workspace_bytes(int32_t batch, int32_t d_in, int32_t n_targets) {
    return lithe::prep_multi_bytes(batch, d_in, n_targets);
}

extern "C" int32_t lithe_lora_prep_multi(const void* x, int32_t n_targets, const lithe_index_view* idx_a,
                                         const lithe_index_view* idx_b, const int32_t* d_out, int64_t n_slots,
                                         const int32_t* ids, const float* weights, int32_t batch, int32_t m,
                                         int32_t d_in, int32_t rank, const float* lut, const float* scaling,
                                         void* const* h, void* const* b_dec, int32_t* err_flag, void* workspace,
                                         int64_t workspace_bytes, void* stream) {
    lithe::clear_error();
    return lithe::prep_multi_impl(x, n_targets, idx_a, idx_b, d_out, n_slots, ids, weights, batch, m, d_in, rank, lut,
                                  scaling, h, b_dec, err_flag, workspace, workspace_bytes, stream);
}

extern "C" int64_t lithe_sgmv_workspace_bytes(int32_t batch, int32_t d_in, int32_t d_out) {
    return lithe::sgmv_workspace_bytes(batch, d_in, d_out);
}

extern "C" int32_t lithe_sgmv_index_ws(const void* x, void* out, int32_t accumulate, const lithe_index_view* idx_a,
                                       const lithe_index_view* idx_b, int64_t n_slots, const int32_t* ids,
                                       const float* weights, int32_t batch, int32_t m, int32_t d_in, int32_t d_out,
                                       int32_t rank, const float* lut, float scaling, int32_t* err_flag,
                                       void* workspace, int64_t workspace_bytes, void* stream) {
    lithe::clear_error();
    if (batch > 0 && m > 0 && !workspace) return lithe::fail_arg("workspace is NULL");
    return lithe::sgmv_index_impl(x, out, accumulate, idx_a, idx_b, n_slots, ids, weights, batch, m, d_in, d_out,
                                  rank, lut, scaling, err_flag, workspace, workspace_bytes, stream);
}

// ---- lithe_sgmv_index_noalloc: the staged form over a static device workspace ----

namespace lithe {

// The workspace of lithe_sgmv_index_noalloc: one array per device, part of the module image,
// so calls never allocate.  256-byte alignment covers the 16-byte bulk-copy rule.
static __device__ __align__(256) uint8_t g_noalloc_ws[LITHE_NOALLOC_WS_BYTES];

// Device address of g_noalloc_ws in the current CUDA context.  The address belongs to the
// module image loaded into a context, so it is cached per context (keyed on the handle that
// cuCtxGetCurrent returns, looked up through the runtime's driver entry point) rather than per
// device ordinal: a context created after a reset of the device gets its own lookup.
static int32_t noalloc_workspace(void** ptr) {
    using CtxGetCurrent = CUresult (*)(CUcontext*);
    static std::mutex mu;
    static CtxGetCurrent get_ctx = nullptr;
    constexpr int kSlots = 64;
    static CUcontext ctx_of[kSlots] = {};
    static void* addr_of[kSlots] = {};
    static int used = 0;
    std::lock_guard<std::mutex> lock(mu);
    cudaError_t e = cudaSuccess;
    if (!get_ctx) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess) return fail_cuda(e, "cudaGetDriverEntryPoint(cuCtxGetCurrent)");
        if (q != cudaDriverEntryPointSuccess || !fn) return fail_unsupported("driver does not export cuCtxGetCurrent");
        get_ctx = reinterpret_cast<CtxGetCurrent>(fn);
    }
    CUcontext ctx = nullptr;
    if (get_ctx(&ctx) != CUDA_SUCCESS) return fail_arg("cuCtxGetCurrent failed");
    for (int i = 0; ctx && i < used; ++i) {
        if (ctx_of[i] == ctx) {
            *ptr = addr_of[i];
            return LITHE_OK;
        }
    }
    // also makes the device's primary context current when no context was current yet
    void* a = nullptr;
    e = cudaGetSymbolAddress(&a, g_noalloc_ws);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(noalloc workspace)");
    if (!a) return fail_arg("cudaGetSymbolAddress returned NULL for the noalloc workspace");
    if (!ctx && (get_ctx(&ctx) != CUDA_SUCCESS || !ctx)) return fail_arg("no current CUDA context");
    const int slot = used < kSlots ? used++ : static_cast<int>(reinterpret_cast<uintptr_t>(ctx) % kSlots);
    ctx_of[slot] = ctx;
    addr_of[slot] = a;
    *ptr = a;
    return LITHE_OK;
}

}  // namespace lithe

extern "C" int32_t lithe_sgmv_index_noalloc(const void* x, void* out, int32_t accumulate,
                                            const lithe_index_view* idx_a, const lithe_index_view* idx_b,
                                            int64_t n_slots, const int32_t* ids, const float* weights,
                                            int32_t batch, int32_t m, int32_t d_in, int32_t d_out, int32_t rank,
                                            const float* lut, float scaling, int32_t* err_flag, void* stream) {
    lithe::clear_error();
    if (batch <= 0 || m <= 0)   // validated and, when empty, a no-op, exactly as lithe_sgmv_index
        return lithe::sgmv_index_impl(x, out, accumulate, idx_a, idx_b, n_slots, ids, weights, batch, m, d_in,
                                      d_out, rank, lut, scaling, err_flag, nullptr, 0, stream);
    const int64_t need = lithe::sgmv_workspace_bytes(batch, d_in, d_out);
    if (need > LITHE_NOALLOC_WS_BYTES)
        return lithe::fail_unsupported(
            "lithe_sgmv_index_noalloc: batch %d x (d_in %d, d_out %d) needs %lld workspace bytes, the built-in "
            "workspace holds %lld; use lithe_sgmv_index or lithe_sgmv_index_ws",
            batch, d_in, d_out, (long long)need, (long long)LITHE_NOALLOC_WS_BYTES);
    void* ws = nullptr;
    const int32_t rc = lithe::noalloc_workspace(&ws);
    if (rc != LITHE_OK) return rc;
    return lithe::sgmv_index_impl(x, out, accumulate, idx_a, idx_b, n_slots, ids, weights, batch, m, d_in, d_out,
                                  rank, lut, scaling, err_flag, ws, LITHE_NOALLOC_WS_BYTES, stream);
}
