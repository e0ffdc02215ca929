// Device-side packing of a raw .lithe index stream into one packed bank slot.
//
// The reference makes an adapter resident on the host: fileio.load_lithe splits the LZMA
// payload into per-module (L, n_blocks) uint16 matrices (lithe/fileio.py:119-152),
// packed.flat_indices reorders them (block, level)-major and pack_indices packs 7 x 9 bits per
// uint64 with numpy (lithe/kernels/packed.py:38-52,125-143); only the packed words go to the
// GPU.  Here the raw payload itself is copied to the device and this kernel does the reorder
// and the packing, writing straight into the bank slot.
//
//   raw      the payload exactly as stored: every module's A matrix (header order), then every
//            module's B matrix; each (L, n) row-major uint16.
//   segments one entry per (module, side) in packed order: the segment's packed blocks
//            [first_block, first_block + n_blocks) take raw[raw_offset + l*n_blocks + j].
//   words    word w holds stream positions 7w..7w+6 (position = block * L + level) at bits
//            9k..9k+8; bit 63 and the positions past the end are zero.
//
// The kernel moves 2 B of raw stream in and 8/7 B of packed words out per index (HBM-bound);
// the blocks of a word that no segment covers are written as zero and flagged.
#include "device_common.cuh"
#include "host_common.h"

namespace lithe {

struct PackParams {
    const uint16_t* raw;                 // payload of blockIdx.y at raw + blockIdx.y * raw_stride
    int64_t n_raw;                       // indices in the raw stream (= L * total blocks)
    const lithe_pack_segment* segs;
    int32_t n_segs;
    int32_t levels;
    uint64_t* words;
    int64_t n_words;
    int32_t* err;
    int64_t raw_stride;                  // batch: elements between payloads
    int64_t slot_stride;                 // batch: words between bank slots
    const int32_t* slot_ids;             // batch: slot of payload y (nullptr: slot y)
    int64_t n_slots;
};

// Largest s with segs[s].first_block <= g, or -1.
__device__ __forceinline__ int find_segment(const lithe_pack_segment* segs, int n, int64_t g) {
    int lo = 0, hi = n - 1, found = -1;
    while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(&segs[mid].first_block) <= g) {
            found = mid;
            lo = mid + 1;
        } else {
            hi = mid - 1;
        }
    }
    return found;
}

constexpr int kPackThreads = 256;
constexpr int kSegCache = 32;           // segments a CTA keeps in shared memory
constexpr int kGroupBlocks = 7;         // 7 blocks x L levels = exactly L packed words
constexpr int kGroupsPerThread = 1;     // measured best: 2 or 4 raise registers and lower occupancy more than they gain
constexpr int kGroupsPerCta = kPackThreads * kGroupsPerThread;

// Segment entry (first, n, src) of block g, searched from cache slot c upward; false if no
// segment covers g.  Past the cache the table is walked in global memory (bounded by n_segs).
struct SegCache {
    int s0, nc;
    int64_t first[kSegCache], n[kSegCache], src[kSegCache];
};

__device__ __forceinline__ bool lookup(const SegCache& sc, const PackParams& p, int64_t g, int& c, int64_t& first,
                                       int64_t& n, int64_t& src) {
    while (c < sc.nc && g >= sc.first[c] + sc.n[c]) ++c;
    if (c < sc.nc) {
        first = sc.first[c];
        n = sc.n[c];
        src = sc.src[c];
        return g >= first;
    }
    if (sc.s0 < 0) return false;
    int e = sc.s0 + sc.nc;
    while (e + 1 < p.n_segs && __ldg(&p.segs[e + 1].first_block) <= g) ++e;
    if (e >= p.n_segs) return false;
    first = __ldg(&p.segs[e].first_block);
    n = __ldg(&p.segs[e].n_blocks);
    src = __ldg(&p.segs[e].raw_offset);
    return g >= first && g < first + n;
}

// A thread packs kGroupsPerThread groups of 7 consecutive blocks (groups t + 256 i of its CTA,
// so every store instruction of a warp is coalesced).  A group's 7 x L indices are exactly
// packed words L*G .. L*G + L - 1, so the (block, level) -> (word, bit) map is a compile-time
// constant for each L and no index needs a division.  When a group lies inside one segment
// (all but the groups at module boundaries), its L level rows are 7 consecutive values each.
// All 7 x L x kGroupsPerThread loads are issued before any value is used; groups that
// straddle a segment boundary, or the stream end, look every block up on their own.
template <int L>
__global__ void __launch_bounds__(kPackThreads) pack_raw_kernel(const __grid_constant__ PackParams pp) {
    __shared__ SegCache sc;
    // payload blockIdx.y -> its bank slot (a single payload: y = 0, slot stride 0)
    PackParams p = pp;
    if (blockIdx.y > 0 || p.slot_ids) {
        const int64_t slot = p.slot_ids ? static_cast<int64_t>(__ldg(p.slot_ids + blockIdx.y)) : blockIdx.y;
        if (slot < 0 || slot >= p.n_slots) {
            if (blockIdx.x == 0 && threadIdx.x == 0 && p.err) atomicOr(p.err, LITHE_DEVERR_SLOT);
            return;
        }
        p.raw += blockIdx.y * p.raw_stride;
        p.words += slot * p.slot_stride;
    }
    const int64_t n_blocks_total = p.n_raw / L;
    const int64_t g_cta = static_cast<int64_t>(blockIdx.x) * kGroupsPerCta * kGroupBlocks;
    if (threadIdx.x == 0) sc.s0 = -1;
    __syncthreads();
#pragma unroll 4
    for (int e = threadIdx.x; e < p.n_segs; e += kPackThreads) {
        const int64_t f = __ldg(&p.segs[e].first_block);
        const int64_t fn = e + 1 < p.n_segs ? __ldg(&p.segs[e + 1].first_block) : INT64_MAX;
        if (f <= g_cta && g_cta < fn) sc.s0 = e;                  // at most one e satisfies this
    }
    __syncthreads();
    if (threadIdx.x < kSegCache) {
        const int e = sc.s0 + static_cast<int>(threadIdx.x);
        if (sc.s0 >= 0 && e < p.n_segs) {
            sc.first[threadIdx.x] = __ldg(&p.segs[e].first_block);
            sc.n[threadIdx.x] = __ldg(&p.segs[e].n_blocks);
            sc.src[threadIdx.x] = __ldg(&p.segs[e].raw_offset);
        }
        if (threadIdx.x == 0) sc.nc = sc.s0 < 0 ? 0 : min(kSegCache, p.n_segs - sc.s0);
    }
    __syncthreads();

    // Phase 1: all loads of the thread's kGroupsPerThread groups (group t + 256 i of the CTA).
    uint32_t v[kGroupsPerThread][kGroupBlocks][L];
    uint32_t bad = 0;
    int c = 0;                                   // cache cursor: groups are visited in block order
#pragma unroll
    for (int i = 0; i < kGroupsPerThread; ++i) {
        const int64_t g0 = g_cta + (static_cast<int64_t>(threadIdx.x) + i * kPackThreads) * kGroupBlocks;
#pragma unroll
        for (int b = 0; b < kGroupBlocks; ++b)
#pragma unroll
            for (int l = 0; l < L; ++l) v[i][b][l] = 0;
        if (g0 >= n_blocks_total) continue;
        int64_t first = 0, n = 0, src = 0;
        const bool found = lookup(sc, p, g0, c, first, n, src);
        const int64_t lo = src + (g0 - first), hi = lo + static_cast<int64_t>(L - 1) * n + (kGroupBlocks - 1);
        if (found && g0 + kGroupBlocks <= first + n && lo >= 0 && hi < p.n_raw) {
            // fast path: one segment, L rows of 7 consecutive values (every address checked above)
            const uint16_t* row = p.raw + lo;
#pragma unroll
            for (int l = 0; l < L; ++l)
#pragma unroll
                for (int b = 0; b < kGroupBlocks; ++b) v[i][b][l] = __ldg(row + static_cast<int64_t>(l) * n + b);
        } else {
            int cc = c;
#pragma unroll
            for (int b = 0; b < kGroupBlocks; ++b) {
                const int64_t g = g0 + b;
                bool ok = g < n_blocks_total;
                if (ok) ok = lookup(sc, p, g, cc, first, n, src);
#pragma unroll
                for (int l = 0; l < L; ++l) {
                    const int64_t at = src + static_cast<int64_t>(l) * n + (g - first);
                    if (ok && at >= 0 && at < p.n_raw) {
                        v[i][b][l] = __ldg(p.raw + at);
                    } else if (g < n_blocks_total) {
                        bad |= LITHE_DEVERR_INDEX;          // block not covered by the segment table
                    }
                }
            }
        }
    }
    // Phase 2: check, pack, store (word L*G + k of group G; consecutive threads, consecutive groups).
#pragma unroll
    for (int i = 0; i < kGroupsPerThread; ++i) {
        const int64_t g0 = g_cta + (static_cast<int64_t>(threadIdx.x) + i * kPackThreads) * kGroupBlocks;
        if (g0 >= n_blocks_total) continue;
        uint64_t word[L];
#pragma unroll
        for (int k = 0; k < L; ++k) word[k] = 0;
#pragma unroll
        for (int b = 0; b < kGroupBlocks; ++b)
#pragma unroll
            for (int l = 0; l < L; ++l) {
                uint32_t x = v[i][b][l];
                if (x > 511u) {
                    bad |= LITHE_DEVERR_INDEX;
                    x &= 511u;
                }
                const int q = b * L + l;                               // position inside the group
                word[q / 7] |= static_cast<uint64_t>(x) << (9 * (q % 7));
            }
        const int64_t w0 = (g0 / kGroupBlocks) * L;
#pragma unroll
        for (int k = 0; k < L; ++k)
            if (w0 + k < p.n_words) p.words[w0 + k] = word[k];
    }
    if (bad && p.err) atomicOr(p.err, static_cast<int32_t>(bad));
}

}  // namespace lithe

namespace lithe {

static int32_t pack_raw_launch(PackParams& p, int32_t num_levels, unsigned n_payloads, cudaStream_t s) {
    const int64_t groups = (p.n_raw / num_levels + kGroupBlocks - 1) / kGroupBlocks;
    const dim3 grid(static_cast<unsigned>((groups + kGroupsPerCta - 1) / kGroupsPerCta), n_payloads);
    switch (num_levels) {
        case 1: pack_raw_kernel<1><<<grid, kPackThreads, 0, s>>>(p); break;
        case 2: pack_raw_kernel<2><<<grid, kPackThreads, 0, s>>>(p); break;
        case 3: pack_raw_kernel<3><<<grid, kPackThreads, 0, s>>>(p); break;
        default: pack_raw_kernel<4><<<grid, kPackThreads, 0, s>>>(p); break;
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "pack_raw_kernel launch");
    return LITHE_OK;
}

static int32_t pack_raw_check(const uint16_t* raw, int64_t n_raw, const lithe_pack_segment* segments,
                              int32_t n_segments, int32_t num_levels, const uint64_t* words, int64_t n_words) {
    if (n_raw < 0) return fail_arg("n_raw must be >= 0");
    if (num_levels < 1 || num_levels > LITHE_MAX_LEVELS)
        return fail_unsupported("num_levels must be in [1, %d], got %d", LITHE_MAX_LEVELS, num_levels);
    if (n_raw % num_levels) return fail_arg("n_raw (%lld) is not a multiple of num_levels", (long long)n_raw);
    const int64_t need = (n_raw + 6) / 7;
    if (n_words != need)
        return fail_arg("n_words must be ceil(n_raw / 7) = %lld, got %lld", (long long)need, (long long)n_words);
    if (n_raw == 0) return LITHE_OK;
    if (n_raw > 0x7fffffffLL) return fail_unsupported("one payload must hold fewer than 2^31 indices");
    if (!raw || !words || !segments) return fail_arg("raw, segments and words must be non-NULL");
    if (n_segments < 1) return fail_arg("n_segments must be >= 1");
    if (reinterpret_cast<uintptr_t>(raw) % 2 || reinterpret_cast<uintptr_t>(words) % 8 ||
        reinterpret_cast<uintptr_t>(segments) % 8)
        return fail_arg("raw, segments or words is misaligned");
    return LITHE_OK;
}

}  // namespace lithe

extern "C" int32_t lithe_pack_raw(const uint16_t* raw, int64_t n_raw, const lithe_pack_segment* segments,
                                  int32_t n_segments, int32_t num_levels, uint64_t* words, int64_t n_words,
                                  int32_t* err_flag, void* stream) {
    using namespace lithe;
    clear_error();
    int32_t rc = pack_raw_check(raw, n_raw, segments, n_segments, num_levels, words, n_words);
    if (rc != LITHE_OK || n_raw == 0) return rc;
    int device = 0, sms = 0;
    rc = current_device_sms(&device, &sms);
    if (rc != LITHE_OK) return rc;
    PackParams p{};
    p.raw = raw;
    p.n_raw = n_raw;
    p.segs = segments;
    p.n_segs = n_segments;
    p.levels = num_levels;
    p.words = words;
    p.n_words = n_words;
    p.err = err_flag;
    p.n_slots = 1;
    return pack_raw_launch(p, num_levels, 1, static_cast<cudaStream_t>(stream));
}

extern "C" int32_t lithe_pack_raw_batch(const uint16_t* raw, int64_t raw_stride, int32_t n_payloads, int64_t n_raw,
                                        const lithe_pack_segment* segments, int32_t n_segments, int32_t num_levels,
                                        uint64_t* bank, int64_t slot_stride, int64_t n_slots, const int32_t* slot_ids,
                                        int64_t n_words, int32_t* err_flag, void* stream) {
    using namespace lithe;
    clear_error();
    if (n_payloads < 0) return fail_arg("n_payloads must be >= 0");
    int32_t rc = pack_raw_check(raw, n_raw, segments, n_segments, num_levels, bank, n_words);
    if (rc != LITHE_OK || n_raw == 0 || n_payloads == 0) return rc;
    if (n_payloads > 65535) return fail_unsupported("at most 65535 payloads per call");
    if (raw_stride < n_raw || raw_stride % 8) return fail_arg("raw_stride must be >= n_raw and a multiple of 8");
    if (slot_stride < n_words || n_slots < 1) return fail_arg("slot_stride must be >= n_words and n_slots >= 1");
    if (!slot_ids && n_payloads > n_slots) return fail_arg("without slot_ids, n_payloads must be <= n_slots");
    int device = 0, sms = 0;
    rc = current_device_sms(&device, &sms);
    if (rc != LITHE_OK) return rc;
    PackParams p{};
    p.raw = raw;
    p.n_raw = n_raw;
    p.segs = segments;
    p.n_segs = n_segments;
    p.levels = num_levels;
    p.words = bank;
    p.n_words = n_words;
    p.err = err_flag;
    p.raw_stride = raw_stride;
    p.slot_stride = slot_stride;
    p.slot_ids = slot_ids;
    p.n_slots = n_slots;
    return pack_raw_launch(p, num_levels, static_cast<unsigned>(n_payloads), static_cast<cudaStream_t>(stream));
}
