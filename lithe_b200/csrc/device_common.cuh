// Device helpers shared by the LITHE sm_100a kernels: inline-PTX wrappers for mbarrier,
// TMA (cp.async.bulk.tensor) and warp MMA, plus the procedural twin-Hadamard decode.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>

#include "lithe_b200.h"

namespace lithe {

// ---------------------------------------------------------------------------------------
// Codebook: c_k[t] = (2*popc((k ^ P(t)) & 511) - 9) / 3, P(t) bit q = parity(t & q), q < 9
// (lithe/codebook.py:35-69).  q < 9 only touches bits 0..3 of t, so c_k has period 16 in t,
// and P is linear over GF(2): P(8h + i) = P(8h) ^ P(i) with P(8) = 256.
// ---------------------------------------------------------------------------------------
__host__ __device__ constexpr uint32_t hadamard_pattern(uint32_t t) {
    uint32_t p = 0;
    for (uint32_t q = 0; q < 9; ++q) {
        uint32_t v = t & q, par = 0;
        while (v) { par ^= (v & 1u); v >>= 1; }
        p |= par << q;
    }
    return p;
}
static_assert(hadamard_pattern(1) == 170 && hadamard_pattern(8) == 256 &&
              hadamard_pattern(15) == 406 && hadamard_pattern(16) == 0,
              "Sylvester-Hadamard row pattern");

// Decoded values of one 64-value block at the 8 positions u = 8*half + i (i = 0..7)
// (every t with t & 15 == u has the same value).  lut: [level][16] fp32 in shared memory,
// k[l]: the block's 9-bit index at level l.  Levels are summed 0,1,..,L-1 in fp32, the
// order of lithe/quant.py:77-80, so the result is bit-identical to the reference decode.
// This is the general form (any number of levels); decode_eight_fast below is the form the
// kernels use for L <= 3.
template <int kMaxLevels>
__device__ __forceinline__ void decode_eight(const float* __restrict__ lut, const uint32_t* k,
                                             int levels, uint32_t half, float v[8]) {
    constexpr uint32_t kP[8] = {0u, 170u, 204u, 102u, 240u, 90u, 60u, 150u};   // hadamard_pattern(0..7)
#pragma unroll
    for (int l = 0; l < kMaxLevels; ++l) {
        if (l < levels) {
            const uint32_t kk = k[l] ^ (half << 8);
            const float* row = lut + l * 16;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float c = row[__popc(kk ^ kP[i])];
                v[i] = (l == 0) ? c : v[i] + c;
            }
        }
    }
}
static_assert(hadamard_pattern(0) == 0 && hadamard_pattern(1) == 170 && hadamard_pattern(2) == 204 &&
              hadamard_pattern(3) == 102 && hadamard_pattern(4) == 240 && hadamard_pattern(5) == 90 &&
              hadamard_pattern(6) == 60 && hadamard_pattern(7) == 150, "decode_eight pattern table");

// Shared-memory tables of the fast decode (built once per CTA by build_decode_tables).
//
// With u = 8h + i, bit 0 of P(u) is 0, bit 8 is h and bits 1..7 are Q(i) = P(i) >> 1, so
//   n(k, u) = popc((k ^ P(u)) & 511) = (k & 1) + (((k >> 8) & 1) ^ h) + popc(((k >> 1) & 127) ^ Q(i)).
// pc[l][m] packs, for m = (k >> 1) & 127, the eight terms popc(m ^ Q(i)) as 16-bit fields
// already scaled by 4 * {100, 10, 1}[l]; adding the three levels' words gives, field by
// field, the byte offset of entry n0*100 + n1*10 + n2 of lut3, which holds the fp32 sum
// (lut[0][n0] + lut[1][n1]) + lut[2][n2] -- the reference's summation order.
struct DecodeTables {
    uint4 pc[3][128];
    float lut3[2][1000];
};

__device__ __forceinline__ void build_decode_tables(DecodeTables* t, const float* lut /*[2][4][16]*/,
                                                    int levels, int tid, int nthreads) {
    constexpr uint32_t kQ[8] = {0u, 85u, 102u, 51u, 120u, 45u, 30u, 75u};
    for (int e = tid; e < 3 * 128; e += nthreads) {
        const int l = e >> 7;
        const uint32_t m = static_cast<uint32_t>(e & 127);
        const uint32_t scale = l == 0 ? 400u : (l == 1 ? 40u : 4u);
        uint32_t f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = scale * static_cast<uint32_t>(__popc(m ^ kQ[i]));
        t->pc[l][m] = make_uint4(f[0] | (f[1] << 16), f[2] | (f[3] << 16), f[4] | (f[5] << 16), f[6] | (f[7] << 16));
    }
    for (int e = tid; e < 2000; e += nthreads) {
        const int side = e >= 1000;
        const int r = e - side * 1000;
        const float* L = lut + side * 64;
        float v = L[r / 100];
        if (levels > 1) v = __fadd_rn(v, L[16 + (r / 10) % 10]);
        if (levels > 2) v = __fadd_rn(v, L[32 + r % 10]);
        t->lut3[side][r] = v;
    }
}
static_assert((hadamard_pattern(1) >> 1) == 85 && (hadamard_pattern(2) >> 1) == 102 &&
              (hadamard_pattern(3) >> 1) == 51 && (hadamard_pattern(4) >> 1) == 120 &&
              (hadamard_pattern(5) >> 1) == 45 && (hadamard_pattern(6) >> 1) == 30 &&
              (hadamard_pattern(7) >> 1) == 75, "pc table patterns");

// Fast decode for L <= 3 (indices of absent levels must be 0): the 8 values of one half
// block, bit-identical to decode_eight.
__device__ __forceinline__ void decode_eight_fast(const DecodeTables* __restrict__ t, int side, const uint32_t* k,
                                                  uint32_t half, float v[8]) {
    uint32_t base = 0;
    uint4 f[3];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
        const uint32_t scale = l == 0 ? 400u : (l == 1 ? 40u : 4u);
        base += scale * ((k[l] & 1u) + (((k[l] >> 8) & 1u) ^ half));
        f[l] = t->pc[l][(k[l] >> 1) & 127u];
    }
    const uint32_t bb = base | (base << 16);
    const char* lut = reinterpret_cast<const char*>(t->lut3[side]);
    const uint32_t w[4] = {f[0].x + f[1].x + f[2].x + bb, f[0].y + f[1].y + f[2].y + bb,
                           f[0].z + f[1].z + f[2].z + bb, f[0].w + f[1].w + f[2].w + bb};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[2 * j] = *reinterpret_cast<const float*>(lut + (w[j] & 0xffffu));
        v[2 * j + 1] = *reinterpret_cast<const float*>(lut + (w[j] >> 16));
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// fp32 views of the two bf16 halves of a 32-bit word (exact)
__device__ __forceinline__ float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ---------------------------------------------------------------------------------------
// Index bank reads.  PACKED9: stream position p in word p/7 at bit 9*(p%7)
// (lithe/kernels/packed.py:38-52,171-177).  I16 / I32: level-major (slot, level, block).
// Out-of-range integers in the I16/I32 banks are masked to 9 bits and reported.
// ---------------------------------------------------------------------------------------
struct IndexView {
    const void* base;
    int32_t format;
    int32_t levels;
    int64_t slot_stride;
    int64_t offset;
    int64_t level_stride;
};

__device__ __forceinline__ uint64_t ldg_nc_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.global.nc.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}

// Raw index words of one block, loaded but not yet unpacked.  Splitting the load
// (fetch_raw) from the unpacking (finish_raw) lets a caller issue the loads one step ahead
// and use them a step later, so the load latency overlaps other work.
template <int kMaxLevels>
struct RawIndices {
    uint64_t a, b;          // PACKED9: the word holding the block's first index, and the next one
    int32_t q[kMaxLevels];  // I16 / I32: the raw integers
    uint32_t r0;            // PACKED9: field of the first index in word a
};

template <int kMaxLevels>
__device__ __forceinline__ void fetch_raw(const IndexView& v, int64_t slot, int64_t blk, RawIndices<kMaxLevels>& r) {
    if (v.format == LITHE_IDX_PACKED9) {
        // positions inside one slot fit in 32 bits (checked on the host)
        const uint64_t* w = static_cast<const uint64_t*>(v.base) + slot * v.slot_stride;
        const uint32_t p0 = static_cast<uint32_t>(v.offset) + static_cast<uint32_t>(v.levels) * static_cast<uint32_t>(blk);
        const uint32_t w0 = p0 / 7u;
        r.r0 = p0 - 7u * w0;
        r.a = ldg_nc_u64(w + w0);
        // the block's last index may sit in the next word; read it only then (never past the stream)
        r.b = (r.r0 + static_cast<uint32_t>(v.levels) > 7u) ? ldg_nc_u64(w + w0 + 1) : 0ull;
    } else {
#pragma unroll
        for (int l = 0; l < kMaxLevels; ++l) {
            if (l < v.levels) {
                const int64_t e = slot * v.slot_stride + v.offset + l * v.level_stride + blk;
                r.q[l] = v.format == LITHE_IDX_I16 ? static_cast<int32_t>(__ldg(static_cast<const int16_t*>(v.base) + e))
                                                   : __ldg(static_cast<const int32_t*>(v.base) + e);
            } else {
                r.q[l] = 0;
            }
        }
    }
}

template <int kMaxLevels>
__device__ __forceinline__ void finish_raw(const IndexView& v, const RawIndices<kMaxLevels>& r,
                                           uint32_t k[kMaxLevels], int32_t* err) {
    if (v.format == LITHE_IDX_PACKED9) {
#pragma unroll
        for (int l = 0; l < kMaxLevels; ++l) {
            if (l < v.levels) {
                const uint32_t f = r.r0 + l;
                k[l] = static_cast<uint32_t>((f < 7u ? (r.a >> (9u * f)) : (r.b >> (9u * (f - 7u))))) & 511u;
            } else {
                k[l] = 0;
            }
        }
    } else {
        bool bad = false;
#pragma unroll
        for (int l = 0; l < kMaxLevels; ++l) {
            bad |= (r.q[l] < 0) | (r.q[l] > 511);
            k[l] = static_cast<uint32_t>(r.q[l]) & 511u;
        }
        if (bad && err) atomicOr(err, LITHE_DEVERR_INDEX);
    }
}

template <int kMaxLevels>
__device__ __forceinline__ void fetch_indices(const IndexView& v, int64_t slot, int64_t blk,
                                              uint32_t k[kMaxLevels], int32_t* err) {
    RawIndices<kMaxLevels> r;
    fetch_raw<kMaxLevels>(v, slot, blk, r);
    finish_raw<kMaxLevels>(v, r, k, err);
}

// ---------------------------------------------------------------------------------------
// Shared-memory, mbarrier and TMA wrappers (PTX ISA 8.x, sm_90+ forms valid on sm_100a)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Raise the expected transaction count of the current phase without arriving (the arrival
// comes later from the same thread, e.g. after it has written its own part of the stage).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Time limit of one pipeline wait.  A wait that runs out sets *abort (shared) and the
// device error word, and every other wait of the block then returns false as well.
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr uint32_t kWaitSpinLimit = 1u << 28;   // second bound, independent of the timer

// try_wait with a suspend-time hint: a waiting warp sleeps in hardware until the phase
// completes or the hint runs out, instead of spinning and taking issue slots from the warps
// that do the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

constexpr uint32_t kSuspendHintNs = 100000;     // one sleeping try_wait lasts at most ~0.1 ms

static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                   int32_t* err) {
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0; it < kWaitSpinLimit; ++it) {
        if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
        if (*abort) return false;
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
    }
    *abort = 1;
    if (err) atomicOr(err, LITHE_DEVERR_TIMEOUT);
    return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, abort, err);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 1-D bulk copy global -> shared (TMA engine, no multicast), completion counted on an mbarrier.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, fp32 accumulate
__device__ __forceinline__ void mma_bf16_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                               const float c[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9},"
        " {%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
          "f"(c[2]), "f"(c[3]));
}

// D = A(16x16 fp16, row) * B(16x8 fp16, col) + C, fp32 accumulate
__device__ __forceinline__ void mma_f16_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                              const float c[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9},"
        " {%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
          "f"(c[2]), "f"(c[3]));
}

// The 16-bit activation types the SGMV kernels compute in (kF16: fp16, else bf16): packing two
// fp32 values into a 32-bit word (round to nearest even), the two halves of a word as fp32
// (exact), one value rounded to the type, and the warp MMA on that type (fp32 accumulate).
template <bool kF16>
struct Act;

template <>
struct Act<false> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_bf16x2(lo, hi); }
    static __device__ __forceinline__ float lo(uint32_t w) { return bf16lo_to_f32(w); }
    static __device__ __forceinline__ float hi(uint32_t w) { return bf16hi_to_f32(w); }
    static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
    static __device__ __forceinline__ void mma(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                               const float c[4]) {
        mma_bf16_16816(d, a, b0, b1, c);
    }
};

template <>
struct Act<true> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float lo(uint32_t w) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
    }
    static __device__ __forceinline__ float hi(uint32_t w) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
    }
    static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
    static __device__ __forceinline__ void mma(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                               const float c[4]) {
        mma_f16_16816(d, a, b0, b1, c);
    }
};

}  // namespace lithe
