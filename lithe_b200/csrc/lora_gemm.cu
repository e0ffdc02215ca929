// Base linear with the per-sample LoRA expand applied inside the GEMM (tcgen05 + TMEM + TMA).
//
//   out[r, :] = x[r, :] . W^T + bias + h[r, :] . Bdec_{sample(r)}^T
//
// The reference computes the base linear (cuBLAS through nn.Linear) and then adds the LoRA
// delta in a second pass over the output (lithe/kernels/layers.py:131, lithe/serve.py:96-97);
// even a fused decode+SGMV kernel must read x again and read + write the whole output.
// Here the rank-16 expand is one extra tcgen05.mma (K = 16) into the tile's TMEM accumulator
// after the K loop, so the output is written once, by the GEMM, and the LoRA costs 16/K of the
// tile's MMA work plus a 12 KB operand load.  The shrink h = bf16(scale * x . A_j^T) and the
// decoded B factors come from lithe_lora_prep (sgmv_index.cu).
//
// One persistent CTA per SM, 128 x 256 output tiles (M x N), K in steps of 64:
//   warp 0       TMA producer: x tile (128 x 64) and W tile (256 x 64) per stage, 128-byte
//                swizzle; per output tile also the h tile (128 x 16) and the Bdec tile
//                (256 x 16) of the tile's sample, 32-byte swizzle.
//   warp 1       allocates 512 TMEM columns (two 128 x 256 fp32 accumulators) and issues
//                the MMAs from one lane: 4 x tcgen05.mma (M128 N256 K16) per stage, the
//                LoRA MMA, tcgen05.commit to the stage / accumulator barriers.
//   warps 2..5   epilogue: tcgen05.ld (warp w reads TMEM lanes 32 (w % 4) ...), + bias,
//                bf16, 16-byte stores; the next tile's K loop runs into the other accumulator.
// Every mbarrier wait is bounded (4 s, LITHE_DEVERR_TIMEOUT, shared abort flag); on abort
// the CTA waits (bounded) for its in-flight TMA loads and MMAs before TMEM is freed.
#include "device_common.cuh"
#include "host_common.h"

namespace lithe {
namespace lg {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 4;
constexpr int kABytes = BM * BK * 2;          // 16 KB
constexpr int kBBytes = BN * BK * 2;          // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kR = 16;                        // LoRA rank of the fused expand
constexpr int kHBytes = BM * kR * 2;          // 4 KB
constexpr int kBdBytes = BN * kR * 2;         // 8 KB
constexpr int kLoraBufs = 2;
constexpr int kLoraBytes = 12288;             // h + Bdec, padded to a 1 KB multiple
constexpr int kTmemCols = 2 * BN;             // two fp32 accumulators
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;

struct Barriers {
    uint64_t full[kStages], empty[kStages];
    uint64_t lfull[kLoraBufs], lempty[kLoraBufs];
    uint64_t tfull[2], tempty[2];
    uint64_t done;
    uint32_t tmem_base;
    int abort;
};

// Epilogue staging: each epilogue warp writes a 32-row x 32-column bf16 chunk (2 KB) to shared
// memory and stores it with one TMA operation; kEpiBufs buffers per warp.
constexpr int kEpiChunkBytes = 32 * 32 * 2;
constexpr int kEpiBufs = 1;
constexpr int kSmemData = kStages * kStageBytes + kLoraBufs * kLoraBytes;
constexpr int kEpiBytes = kEpiWarps * kEpiBufs * kEpiChunkBytes;
constexpr int kSmemBytes = kSmemData + kEpiBytes + static_cast<int>(sizeof(Barriers)) + 1024;   // + alignment slack

struct Params {
    const __nv_bfloat16* bias;    // (n) or nullptr
    __nv_bfloat16* out;           // (rows, n)
    int32_t* err;
    int32_t rows, n, k;
    int32_t m_tiles, n_tiles, total_tiles;
    int32_t rows_per_sample;      // LoRA: rows of one sample (multiple of BM)
    int32_t lora;                 // 1: apply the fused expand
};

// UMMA shared-memory descriptor, K-major, swizzled (sm_100 layout: start >> 4 in bits 0-13,
// leading byte offset 16 B, stride byte offset = 8 rows in bits 32-45, version 1 in bit 46,
// layout type in bits 61-63: 2 = 128-byte swizzle, 6 = 32-byte swizzle).
__device__ __forceinline__ uint64_t desc_k_major(uint32_t saddr, uint32_t row_bytes, uint64_t layout) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(((8u * row_bytes) >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= layout << 61;
    return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A and
// B (bits 7-9, 10-12 = 1), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                            (static_cast<uint32_t>(BM >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Tile order: groups of kGroupN N-tiles, M-blocks walked inside a group, so the ~148 tiles in
// flight at once cover ~18 M-blocks x 8 N-tiles (14 MB of x rows + 12.6 MB of W at K = 3072)
// instead of every N-tile of a wide W (row-major order re-streams all of W once per wave).
constexpr int kGroupN = 8;

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& m0, int& n0) {
    const int per_group = kGroupN * p.m_tiles;
    const int g = t / per_group;
    const int in = t - g * per_group;
    const int width = min(kGroupN, p.n_tiles - g * kGroupN);
    m0 = (in / width) * BM;
    n0 = (g * kGroupN + in % width) * BN;
}

// TMA store (no multicast) of a shared-memory box to the tensor map's box at (x, y), in the
// issuing thread's bulk group; rows past the tensor's end are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's bulk groups still read shared memory / are in flight.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// One 32-column chunk of the epilogue for a warp's 32 accumulator rows (lane = row): + bias,
// bf16, written into the warp's staging buffer with the 64-byte swizzle of the output tensor
// map (16-byte unit v of row r at unit v ^ ((r >> 1) & 3), so the warp's stores hit every bank
// once per quarter-warp), then stored by lane 0 with one TMA operation at (x, y).  A chunk
// leaves as whole 64-byte row segments instead of 32 rows' scattered 16-byte stores per
// instruction, which measured about 6% of the GEMM's energy under the power cap.  kBufs:
// staging buffers per warp; buffer n % kBufs is reused once the store two chunks back has
// read it.
template <int kBufs>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[32], const float (&bias)[32], uint8_t* bufs,
                                               uint32_t& n_st, int lane, const CUtensorMap* tm_out, int32_t x,
                                               int32_t y) {
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
        pk[j] = pack_bf16x2(__uint_as_float(r[2 * j]) + bias[2 * j], __uint_as_float(r[2 * j + 1]) + bias[2 * j + 1]);
    if (n_st >= static_cast<uint32_t>(kBufs)) {
        if (lane == 0) bulk_wait_group_read<kBufs - 1>();
        __syncwarp();
    }
    uint8_t* buf = bufs + (n_st % kBufs) * kEpiChunkBytes;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int v = 0; v < 4; ++v)
        *reinterpret_cast<uint4*>(buf + lane * 64 + ((v ^ sw) << 4)) =
            make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(tm_out, buf, x, y);
        bulk_commit_group();
    }
    ++n_st;
}

__global__ void __launch_bounds__(kThreads, 1)
    lora_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_bd,
                     const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    uint8_t* lora_base = smem + kStages * kStageBytes;
    uint8_t* epi_base = smem + kSmemData;                  // kEpiWarps x kEpiBufs staging chunks
    Barriers* bars = reinterpret_cast<Barriers*>(smem + kSmemData + kEpiBytes);
    volatile int* abort = &bars->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = p.k / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < kLoraBufs; ++b) {
            mbar_init(&bars->lfull[b], 1);
            mbar_init(&bars->lempty[b], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&bars->tfull[a], 1);
            mbar_init(&bars->tempty[a], kEpiWarps);
        }
        mbar_init(&bars->done, 1);
        bars->abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_x);
        prefetch_tmap(&tm_w);
        if (p.lora) {
            prefetch_tmap(&tm_h);
            prefetch_tmap(&tm_bd);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t q = 0, it = 0;
            for (int t = blockIdx.x; t < p.total_tiles && !*abort; t += gridDim.x, ++it) {
                int m0, n0;
                tile_coords(p, t, m0, n0);
                for (int kb = 0; kb < nk; ++kb, ++q) {
                    const uint32_t s = q % kStages, ph = (q / kStages) & 1u;
                    if (!mbar_wait(&bars->empty[s], ph ^ 1u, abort, p.err)) break;
                    mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
                    uint8_t* a = stage_base + s * kStageBytes;
                    tma_load_2d(a, &tm_x, &bars->full[s], kb * BK, m0);
                    tma_load_2d(a + kABytes, &tm_w, &bars->full[s], kb * BK, n0);
                }
                if (p.lora && !*abort) {
                    const uint32_t b = it % kLoraBufs, ph = (it / kLoraBufs) & 1u;
                    if (!mbar_wait(&bars->lempty[b], ph ^ 1u, abort, p.err)) break;
                    mbar_arrive_expect_tx(&bars->lfull[b], kHBytes + kBdBytes);
                    uint8_t* l = lora_base + b * kLoraBytes;
                    const int sample = m0 / p.rows_per_sample;
                    tma_load_2d(l, &tm_h, &bars->lfull[b], 0, m0);
                    tma_load_2d(l + kHBytes, &tm_bd, &bars->lfull[b], 0, sample * p.n + n0);
                }
            }
            // On abort, let the loads already issued land before the CTA's shared memory is released.
            if (*abort) {
                const uint64_t t0 = global_timer_ns();
                const uint32_t first = q > static_cast<uint32_t>(kStages) ? q - kStages : 0u;
                for (uint32_t r = first; r < q; ++r) {
                    const uint32_t s = r % kStages, ph = (r / kStages) & 1u;
                    while (!mbar_try_wait(&bars->full[s], ph) && global_timer_ns() - t0 < 20000000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t q = 0, it = 0;
            for (int t = blockIdx.x; t < p.total_tiles && !*abort; t += gridDim.x, ++it) {
                const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
                if (!mbar_wait(&bars->tempty[acc], aph ^ 1u, abort, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++q) {
                    const uint32_t s = q % kStages, ph = (q / kStages) & 1u;
                    if (!mbar_wait(&bars->full[s], ph, abort, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(stage_base + s * kStageBytes);
                    const uint64_t ad = desc_k_major(a, 128, 2), bd = desc_k_major(a + kABytes, 128, 2);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)   // +32 bytes along K inside the 128-byte swizzle atom
                        umma(d, ad + 2 * kk, bd + 2 * kk, (kb | kk) != 0);
                    umma_commit(&bars->empty[s]);
                }
                if (!ok) break;
                if (p.lora) {
                    const uint32_t b = it % kLoraBufs, ph = (it / kLoraBufs) & 1u;
                    if (!mbar_wait(&bars->lfull[b], ph, abort, p.err)) break;
                    tc_fence_after();
                    const uint32_t l = smem_u32(lora_base + b * kLoraBytes);
                    umma(d, desc_k_major(l, 32, 6), desc_k_major(l + kHBytes, 32, 6), 1u);
                    umma_commit(&bars->lempty[b]);
                }
                umma_commit(&bars->tfull[acc]);
            }
            umma_commit(&bars->done);        // arrives once every MMA issued above has completed
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int quarter = warp & 3;                 // TMEM lanes 32*quarter .. +31
        const int row_in_tile = quarter * 32 + lane;
        uint8_t* epi_bufs = epi_base + quarter * kEpiBufs * kEpiChunkBytes;
        uint32_t n_st = 0;                            // chunks this warp has stored
        uint32_t it = 0;
        for (int t = blockIdx.x; t < p.total_tiles && !*abort; t += gridDim.x, ++it) {
            int m0, n0;
            tile_coords(p, t, m0, n0);
            const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
            if (!mbar_wait(&bars->tfull[acc], aph, abort, p.err)) break;
            tc_fence_after();
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + c0, r);
                float bias[32];
                if (p.bias) {
                    const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n0 + c0);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const uint4 w = __ldg(bp + v);
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            bias[v * 8 + 2 * j] = bf16lo_to_f32(ws[j]);
                            bias[v * 8 + 2 * j + 1] = bf16hi_to_f32(ws[j]);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) bias[j] = 0.0f;
                }
                epilogue_chunk<kEpiBufs>(r, bias, epi_bufs, n_st, lane, &tm_out, n0 + c0, m0 + row_in_tile - lane);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->tempty[acc]);
        }
        if (lane == 0) bulk_wait_group_all();        // the last stores have read their staging chunks
        __syncwarp();
    }

    __syncthreads();
    if (warp == 1) {
        // every MMA this CTA issued has completed (bounded wait) before the columns are freed
        if (lane == 0) {
            const uint64_t t0 = global_timer_ns();
            while (!mbar_try_wait(&bars->done, 0) && global_timer_ns() - t0 < 100000000ull) {
            }
        }
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ------------------------------------------------------------------------------------------
// CTA-pair form (cluster of 2, tcgen05.mma.cta_group::2): a pair computes a 256 x 256 tile.
// CTA r of the pair streams x rows [m0 + 128 r, +128) and W rows [n0 + 128 r, +128) (32 KB a
// stage instead of 48, so a pair moves 64 KB per 256 x 256 x 64 step instead of 96 KB); the
// leader (rank 0) issues M256 N256 K16 MMAs that read both CTAs' shared memory and write
// rows 0-127 of the tile into its own TMEM and rows 128-255 into its peer's.
//   - both CTAs' TMA loads complete on the leader's full barrier (cta_group::2 form, the
//     leader's address from mapa); only the leader arms it, with both CTAs' bytes;
//   - the leader's commits go to the empty / accumulator-full / LoRA-empty barriers of both
//     CTAs (tcgen05.commit ... multicast::cluster, mask 0b11);
//   - both CTAs' epilogue warps arrive on the leader's accumulator-empty barrier (count 8);
//   - TMEM is allocated and freed by warp 1 of both CTAs together; a cluster barrier precedes
//     the free so that no CTA leaves while the pair's MMAs may still read its shared memory.
constexpr int kStages2 = 6;
constexpr int kHalf = 128;                               // rows of A and of B per CTA
constexpr int kABytes2 = kHalf * BK * 2;                 // 16 KB
constexpr int kStageBytes2 = 2 * kABytes2;               // A half + B half
constexpr int kHBytes2 = kHalf * kR * 2;                 // 4 KB
constexpr int kLoraBytes2 = 2 * kHBytes2;                // h half + Bdec half
constexpr int kSmemData2 = kStages2 * kStageBytes2 + kLoraBufs * kLoraBytes2;
constexpr int kEpiBufs2 = 2;
constexpr int kEpiBytes2 = kEpiWarps * kEpiBufs2 * kEpiChunkBytes;
constexpr uint32_t kIdesc2 = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                             (static_cast<uint32_t>(256 >> 4) << 24);

struct Barriers2 {
    uint64_t full[kStages2], empty[kStages2];
    uint64_t lfull[kLoraBufs], lempty[kLoraBufs];
    uint64_t tfull[2], tempty[2];
    uint64_t done;
    uint32_t tmem_base;
    int abort;
};
constexpr int kSmemBytes2 = kSmemData2 + kEpiBytes2 + static_cast<int>(sizeof(Barriers2)) + 1024;   // + alignment slack
static_assert(kSmemBytes2 <= 232448, "shared memory of the pair kernel");
static_assert(kSmemBytes <= 232448, "shared memory of the single-CTA kernel");

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar, int32_t x,
                                                 int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(leader_bar)
        : "memory");
}

__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc2), "r"(accumulate));
}

// Arrive on the barrier at this shared-memory offset in both CTAs of the pair once the MMAs
// issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}

__device__ __forceinline__ void umma_commit_pair_local(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void pair_tile_coords(const Params& p, int t, int& m0, int& n0) {
    const int per_group = kGroupN * p.m_tiles;
    const int g = t / per_group;
    const int in = t - g * per_group;
    const int width = min(kGroupN, p.n_tiles - g * kGroupN);
    m0 = (in / width) * (2 * kHalf);
    n0 = (g * kGroupN + in % width) * BN;
}

// Bounded pause used on the abort path, so loads already issued land before shared memory
// is released.
__device__ __forceinline__ void drain_pause() {
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 2000000ull) __nanosleep(10000);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    lora_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                          const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_bd,
                          const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    uint8_t* lora_base = smem + kStages2 * kStageBytes2;
    uint8_t* epi_base = smem + kSmemData2;                 // kEpiWarps x kEpiBufs2 staging chunks
    Barriers2* bars = reinterpret_cast<Barriers2*>(smem + kSmemData2 + kEpiBytes2);
    volatile int* abort = &bars->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int nk = p.k / BK;
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages2; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < kLoraBufs; ++b) {
            mbar_init(&bars->lfull[b], 1);
            mbar_init(&bars->lempty[b], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&bars->tfull[a], 1);
            mbar_init(&bars->tempty[a], 2 * kEpiWarps);
        }
        mbar_init(&bars->done, 1);
        bars->abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_x);
        prefetch_tmap(&tm_w);
        if (p.lora) {
            prefetch_tmap(&tm_h);
            prefetch_tmap(&tm_bd);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync();                      // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t q = 0, it = 0;
            for (int t = pair; t < p.total_tiles && !*abort; t += n_pairs, ++it) {
                int m0, n0;
                pair_tile_coords(p, t, m0, n0);
                for (int kb = 0; kb < nk; ++kb, ++q) {
                    const uint32_t s = q % kStages2, ph = (q / kStages2) & 1u;
                    if (!mbar_wait(&bars->empty[s], ph ^ 1u, abort, p.err)) break;
                    if (leader) mbar_arrive_expect_tx(&bars->full[s], 2 * kStageBytes2);
                    const uint32_t fb = map_to_rank(&bars->full[s], 0);
                    uint8_t* a = stage_base + s * kStageBytes2;
                    tma_load_2d_pair(a, &tm_x, fb, kb * BK, m0 + kHalf * static_cast<int>(rank));
                    tma_load_2d_pair(a + kABytes2, &tm_w, fb, kb * BK, n0 + kHalf * static_cast<int>(rank));
                }
                if (p.lora && !*abort) {
                    const uint32_t b = it % kLoraBufs, ph = (it / kLoraBufs) & 1u;
                    if (!mbar_wait(&bars->lempty[b], ph ^ 1u, abort, p.err)) break;
                    if (leader) mbar_arrive_expect_tx(&bars->lfull[b], 2 * kLoraBytes2);
                    const uint32_t fb = map_to_rank(&bars->lfull[b], 0);
                    uint8_t* l = lora_base + b * kLoraBytes2;
                    const int sample = m0 / p.rows_per_sample;
                    tma_load_2d_pair(l, &tm_h, fb, 0, m0 + kHalf * static_cast<int>(rank));
                    tma_load_2d_pair(l + kHBytes2, &tm_bd, fb, 0, sample * p.n + n0 + kHalf * static_cast<int>(rank));
                }
            }
            if (*abort) drain_pause();
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            uint32_t q = 0, it = 0;
            for (int t = pair; t < p.total_tiles && !*abort; t += n_pairs, ++it) {
                const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
                if (!mbar_wait(&bars->tempty[acc], aph ^ 1u, abort, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++q) {
                    const uint32_t s = q % kStages2, ph = (q / kStages2) & 1u;
                    if (!mbar_wait(&bars->full[s], ph, abort, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(stage_base + s * kStageBytes2);
                    const uint64_t ad = desc_k_major(a, 128, 2), bd = desc_k_major(a + kABytes2, 128, 2);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) umma_pair(d, ad + 2 * kk, bd + 2 * kk, (kb | kk) != 0);
                    umma_commit_pair(&bars->empty[s]);
                }
                if (!ok) break;
                if (p.lora) {
                    const uint32_t b = it % kLoraBufs, ph = (it / kLoraBufs) & 1u;
                    if (!mbar_wait(&bars->lfull[b], ph, abort, p.err)) break;
                    tc_fence_after();
                    const uint32_t l = smem_u32(lora_base + b * kLoraBytes2);
                    umma_pair(d, desc_k_major(l, 32, 6), desc_k_major(l + kHBytes2, 32, 6), 1u);
                    umma_commit_pair(&bars->lempty[b]);
                }
                umma_commit_pair(&bars->tfull[acc]);
            }
            umma_commit_pair_local(&bars->done);
        }
    } else {
        const int quarter = warp & 3;
        const int row_in_tile = static_cast<int>(rank) * kHalf + quarter * 32 + lane;
        uint8_t* epi_bufs = epi_base + quarter * kEpiBufs2 * kEpiChunkBytes;
        uint32_t n_st = 0;                            // chunks this warp has stored
        const uint32_t tempty0 = map_to_rank(&bars->tempty[0], 0), tempty1 = map_to_rank(&bars->tempty[1], 0);
        uint32_t it = 0;
        for (int t = pair; t < p.total_tiles && !*abort; t += n_pairs, ++it) {
            int m0, n0;
            pair_tile_coords(p, t, m0, n0);
            const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
            if (!mbar_wait(&bars->tfull[acc], aph, abort, p.err)) break;
            tc_fence_after();
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + c0, r);
                float bias[32];
                if (p.bias) {
                    const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n0 + c0);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const uint4 w = __ldg(bp + v);
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            bias[v * 8 + 2 * j] = bf16lo_to_f32(ws[j]);
                            bias[v * 8 + 2 * j + 1] = bf16hi_to_f32(ws[j]);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) bias[j] = 0.0f;
                }
                epilogue_chunk<kEpiBufs2>(r, bias, epi_bufs, n_st, lane, &tm_out, n0 + c0, m0 + row_in_tile - lane);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acc ? tempty1 : tempty0);
        }
        if (lane == 0) bulk_wait_group_all();        // the last stores have read their staging chunks
        __syncwarp();
    }

    __syncthreads();
    if (leader && warp == 1 && lane == 0) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bars->done, 0) && global_timer_ns() - t0 < 100000000ull) {
        }
    }
    tc_fence_before();
    cluster_sync();                      // the pair's MMAs are done before either CTA frees anything
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

}  // namespace lg
}  // namespace lithe

extern "C" int32_t lithe_lora_gemm(const void* x, const void* w, const void* bias, void* out, int32_t rows, int32_t n,
                                   int32_t k, const void* h, const void* b_dec, int32_t rows_per_sample, int32_t rank,
                                   int32_t* err_flag, void* stream) {
    using namespace lithe;
    using namespace lithe::lg;
    clear_error();
    if (rows < 0 || n <= 0 || k <= 0) return fail_arg("rows must be >= 0 and n, k > 0 (rows %d, n %d, k %d)", rows, n, k);
    if (n % BN) return fail_unsupported("n must be a multiple of %d, got %d", BN, n);
    if (k % BK) return fail_unsupported("k must be a multiple of %d, got %d", BK, k);
    const bool lora = h != nullptr;
    if (lora) {
        if (!b_dec) return fail_arg("b_dec is NULL while h is given");
        if (rank != kR) return fail_unsupported("the fused expand supports rank %d, got %d", kR, rank);
        if (rows_per_sample <= 0 || rows_per_sample % BM || rows % rows_per_sample)
            return fail_unsupported("rows per sample (%d) must be a positive multiple of %d dividing rows (%d)",
                                    rows_per_sample, BM, rows);
        if (reinterpret_cast<uintptr_t>(h) % 16 || reinterpret_cast<uintptr_t>(b_dec) % 16)
            return fail_arg("h and b_dec must be 16-byte aligned");
    }
    if (rows == 0) return LITHE_OK;
    if (!x || !w || !out) return fail_arg("x, w and out must be non-NULL");
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16 ||
        reinterpret_cast<uintptr_t>(out) % 16 || reinterpret_cast<uintptr_t>(bias) % 16)
        return fail_arg("x, w, out and bias must be 16-byte aligned");
    int device = 0, sms = 0;
    int32_t rc = current_device_sms(&device, &sms);
    if (rc != LITHE_OK) return rc;

    // CTA pairs (256 x 256 tiles) whenever a tile's rows belong to one sample; single CTAs
    // (128 x 256) for fewer than 256 rows or 128-row samples.
    const bool use_pair = rows >= 2 * kHalf && (!lora || rows_per_sample % (2 * kHalf) == 0) && sms >= 2;
    const uint32_t b_rows = use_pair ? kHalf : BN;
    CUtensorMap tm_x, tm_w, tm_h, tm_bd, tm_out;
    if ((rc = encode_bf16_2d(&tm_x, x, k, rows, BK, BM, 128)) != LITHE_OK) return rc;
    if ((rc = encode_bf16_2d(&tm_w, w, k, n, BK, b_rows, 128)) != LITHE_OK) return rc;
    // the epilogue's TMA stores: 32 x 32 boxes with the 64-byte swizzle of its staging chunks
    if ((rc = encode_bf16_2d(&tm_out, out, n, rows, 32, 32, 64)) != LITHE_OK) return rc;
    if (lora) {
        if ((rc = encode_bf16_2d(&tm_h, h, kR, rows, kR, BM, 32)) != LITHE_OK) return rc;
        if ((rc = encode_bf16_2d(&tm_bd, b_dec, kR, static_cast<uint64_t>(rows / rows_per_sample) * n, kR, b_rows,
                                 32)) != LITHE_OK)
            return rc;
    } else {
        tm_h = tm_x;
        tm_bd = tm_x;
    }
    Params p{};
    p.bias = static_cast<const __nv_bfloat16*>(bias);
    p.out = static_cast<__nv_bfloat16*>(out);
    p.err = err_flag;
    p.rows = rows;
    p.n = n;
    p.k = k;
    const int tile_rows = use_pair ? 2 * kHalf : BM;
    p.m_tiles = (rows + tile_rows - 1) / tile_rows;
    p.n_tiles = n / BN;
    const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
    if (tiles > 0x7fffffffLL) return fail_arg("too many tiles");
    p.total_tiles = static_cast<int32_t>(tiles);
    p.rows_per_sample = lora ? rows_per_sample : 0;
    p.lora = lora ? 1 : 0;

    static bool configured[64] = {false};
    if (device >= 64) return fail_unsupported("device ordinal %d", device);
    if (!configured[device]) {
        cudaError_t e = cudaFuncSetAttribute(lora_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(lora_gemm_kernel)");
        e = cudaFuncSetAttribute(lora_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes2);
        if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(lora_gemm_pair_kernel)");
        configured[device] = true;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (use_pair) {
        const int64_t pairs = tiles < sms / 2 ? tiles : sms / 2;
        lora_gemm_pair_kernel<<<static_cast<int>(2 * pairs), kThreads, kSmemBytes2, st>>>(tm_x, tm_w, tm_h, tm_bd,
                                                                                          tm_out, p);
    } else {
        const int grid = static_cast<int>(tiles < sms ? tiles : sms);
        lora_gemm_kernel<<<grid, kThreads, kSmemBytes, st>>>(tm_x, tm_w, tm_h, tm_bd, tm_out, p);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, use_pair ? "lora_gemm_pair_kernel launch" : "lora_gemm_kernel launch");
    return LITHE_OK;
}
