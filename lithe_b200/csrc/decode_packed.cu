// Whole-adapter decode of a packed 9-bit index stream into dense 64-value blocks.
//
// Replaces lithe/kernels/packed.py:151-177 (_decode_packed_kernel) and the loop that the
// hot-swap harness runs once per slot (serving/_common.py:241-244).  One thread owns one
// half of a block: it reads the block's L indices (one or two uint64 words, L1-cached),
// computes the 8 distinct values of its half procedurally (the codeword has period 16,
// so a 64-value block is 16 values repeated 4 times) and writes them to the 4 places
// they occur.  Output traffic dominates (128 B bf16 / 256 B fp32 per block against
// <= 4 B of indices), so the kernel is HBM-write bound.
#include "device_common.cuh"
#include "host_common.h"

namespace lithe {

struct DecodeParams {
    const uint64_t* bank;
    int64_t slot_stride;
    int64_t n_slots;
    const int32_t* slot_ids;   // nullptr: a single stream at bank
    int64_t n_blocks;
    const int8_t* sides;       // nullptr: every block is side A
    void* out;
    int32_t* err;
    int32_t levels;
    float lut[2][LITHE_MAX_LEVELS][16];
};

template <bool kF32>
__global__ void __launch_bounds__(256) decode_packed_kernel(const __grid_constant__ DecodeParams p) {
    __shared__ float lut_s[2][LITHE_MAX_LEVELS][16];
    __shared__ DecodeTables tab;
    for (int i = threadIdx.x; i < 2 * LITHE_MAX_LEVELS * 16; i += blockDim.x)
        (&lut_s[0][0][0])[i] = (&p.lut[0][0][0])[i];
    build_decode_tables(&tab, &p.lut[0][0][0], p.levels, threadIdx.x, blockDim.x);
    __syncthreads();

    const int64_t sel = blockIdx.y;
    int64_t slot = 0;
    if (p.slot_ids) {
        slot = p.slot_ids[sel];
        if (slot < 0 || slot >= p.n_slots) {
            if (blockIdx.x == 0 && threadIdx.x == 0 && p.err) atomicOr(p.err, LITHE_DEVERR_SLOT);
            return;
        }
    }
    IndexView view;
    view.base = p.bank;
    view.format = LITHE_IDX_PACKED9;
    view.levels = p.levels;
    view.slot_stride = p.slot_stride;
    view.offset = 0;
    view.level_stride = 0;

    const int64_t items = 2 * p.n_blocks;
    constexpr int kBlockBytes = kF32 ? 256 : 128;
    char* out = static_cast<char*>(p.out) + sel * p.n_blocks * kBlockBytes;
    if constexpr (kF32) {
        const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
        for (int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < items;
             item += stride) {
            const int64_t blk = item >> 1;
            const uint32_t half = static_cast<uint32_t>(item & 1);
            const int side = p.sides ? (p.sides[blk] != 0) : 0;
            uint32_t k[LITHE_MAX_LEVELS];
            fetch_indices<LITHE_MAX_LEVELS>(view, slot, blk, k, nullptr);
            float v[8];
            if (p.levels <= 3) decode_eight_fast(&tab, side, k, half, v);
            else decode_eight<LITHE_MAX_LEVELS>(&lut_s[side][0][0], k, p.levels, half, v);
            char* dst = out + blk * kBlockBytes;
            const float4 lo = make_float4(v[0], v[1], v[2], v[3]);
            const float4 hi = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                float4* d = reinterpret_cast<float4*>(dst + half * 32 + m * 64);
                d[0] = lo;
                d[1] = hi;
            }
        }
    } else {
        // bf16: a warp decodes 16 consecutive blocks (lane = one half block), then 4 shuffle
        // rounds give every lane the 16-byte piece it stores, so each store instruction writes
        // 4 whole blocks (512 contiguous bytes).  Piece q of a block holds values 8q .. 8q+7,
        // i.e. half (q & 1) of the 16-value pattern.  Writing each half block to its 4 places
        // from its own lane touched 16 blocks per store instruction and kept L1 saturated.
        const int lane = threadIdx.x & 31;
        const int64_t warp_id = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
        const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
        for (int64_t base = warp_id * 32; base < items; base += n_warps * 32) {
            const int64_t item = base + lane;
            uint32_t q[4] = {0u, 0u, 0u, 0u};
            if (item < items) {
                const int64_t blk = item >> 1;
                const uint32_t half = static_cast<uint32_t>(item & 1);
                const int side = p.sides ? (p.sides[blk] != 0) : 0;
                uint32_t k[LITHE_MAX_LEVELS];
                fetch_indices<LITHE_MAX_LEVELS>(view, slot, blk, k, nullptr);
                float v[8];
                if (p.levels <= 3) decode_eight_fast(&tab, side, k, half, v);
                else decode_eight<LITHE_MAX_LEVELS>(&lut_s[side][0][0], k, p.levels, half, v);
                q[0] = pack_bf16x2(v[0], v[1]);
                q[1] = pack_bf16x2(v[2], v[3]);
                q[2] = pack_bf16x2(v[4], v[5]);
                q[3] = pack_bf16x2(v[6], v[7]);
            }
            const int64_t blk0 = base >> 1;                 // first of the warp's 16 blocks
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int b = 4 * j + (lane >> 3);          // block of this lane's piece
                const int src = 2 * b + (lane & 1);         // lane that decoded its half
                uint4 w;
                w.x = __shfl_sync(0xffffffffu, q[0], src);
                w.y = __shfl_sync(0xffffffffu, q[1], src);
                w.z = __shfl_sync(0xffffffffu, q[2], src);
                w.w = __shfl_sync(0xffffffffu, q[3], src);
                if (blk0 + b < p.n_blocks)   // streaming store: the output is larger than L2 and not re-read here
                    __stcs(reinterpret_cast<uint4*>(out + (blk0 + b) * kBlockBytes + (lane & 7) * 16), w);
            }
        }
    }
}

static int32_t launch_decode(const DecodeParams& p, int32_t n_sel, int32_t out_dtype, void* stream) {
    const int64_t items = 2 * p.n_blocks;
    if (items == 0 || n_sel == 0) return LITHE_OK;
    int device = 0, sms = 0;
    int32_t rc = current_device_sms(&device, &sms);
    if (rc != LITHE_OK) return rc;
    // Each CTA first builds its 14 KB of decode tables, so CTAs must be long-lived: about 8
    // resident CTAs per SM in total over all selected slots, each grid-striding over its slot.
    const int threads = 256;
    int64_t blocks = (items + threads - 1) / threads;
    int64_t cap = (static_cast<int64_t>(sms) * 8 + n_sel - 1) / n_sel;
    if (cap < 1) cap = 1;
    if (blocks > cap) blocks = cap;
    dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(n_sel));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_dtype == LITHE_DTYPE_F32) decode_packed_kernel<true><<<grid, threads, 0, s>>>(p);
    else decode_packed_kernel<false><<<grid, threads, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "decode_packed_kernel launch");
    return LITHE_OK;
}

static int32_t check_common(int64_t n_blocks, int32_t levels, const float* lut, const void* out,
                            int32_t out_dtype) {
    if (n_blocks < 0) return fail_arg("n_blocks must be >= 0, got %lld", (long long)n_blocks);
    if (levels < 1 || levels > LITHE_MAX_LEVELS)
        return fail_unsupported("num_levels must be in [1, %d], got %d", LITHE_MAX_LEVELS, levels);
    if (!lut) return fail_arg("lut is NULL");
    if (n_blocks > 0 && !out) return fail_arg("out is NULL");
    if (reinterpret_cast<uintptr_t>(out) % 16) return fail_arg("out must be 16-byte aligned");
    if (out_dtype != LITHE_DTYPE_BF16 && out_dtype != LITHE_DTYPE_F32)
        return fail_arg("out_dtype must be LITHE_DTYPE_BF16 or LITHE_DTYPE_F32");
    return LITHE_OK;
}

}  // namespace lithe

extern "C" {

int32_t lithe_decode_packed(const uint64_t* words, int64_t n_blocks, int32_t num_levels,
                            const int8_t* sides, const float* lut, void* out, int32_t out_dtype,
                            void* stream) {
    using namespace lithe;
    clear_error();
    int32_t rc = check_common(n_blocks, num_levels, lut, out, out_dtype);
    if (rc != LITHE_OK) return rc;
    if (n_blocks > 0 && !words) return fail_arg("words is NULL");
    if (static_cast<int64_t>(num_levels) * n_blocks > 0xffffffffLL)
        return fail_unsupported("packed stream positions must fit in 32 bits");
    DecodeParams p{};
    p.bank = words;
    p.slot_stride = 0;
    p.n_slots = 1;
    p.slot_ids = nullptr;
    p.n_blocks = n_blocks;
    p.sides = sides;
    p.out = out;
    p.err = nullptr;
    p.levels = num_levels;
    expand_lut(lut, num_levels, p.lut);
    return launch_decode(p, 1, out_dtype, stream);
}

int32_t lithe_decode_packed_batch(const uint64_t* bank, int64_t slot_stride, int64_t n_slots,
                                  const int32_t* slot_ids, int32_t n_sel, int64_t n_blocks,
                                  int32_t num_levels, const int8_t* sides, const float* lut,
                                  void* out, int32_t out_dtype, int32_t* err_flag, void* stream) {
    using namespace lithe;
    clear_error();
    int32_t rc = check_common(n_blocks, num_levels, lut, out, out_dtype);
    if (rc != LITHE_OK) return rc;
    if (n_sel < 0 || n_sel > 65535) return fail_arg("n_sel must be in [0, 65535], got %d", n_sel);
    if (n_sel > 0 && (!bank || !slot_ids)) return fail_arg("bank and slot_ids must be non-NULL");
    const int64_t words_needed = (static_cast<int64_t>(num_levels) * n_blocks + 6) / 7;
    if (static_cast<int64_t>(num_levels) * n_blocks > 0xffffffffLL)
        return fail_unsupported("packed stream positions must fit in 32 bits");
    if (slot_stride < words_needed)
        return fail_arg("slot_stride %lld is smaller than the stream (%lld words)",
                        (long long)slot_stride, (long long)words_needed);
    DecodeParams p{};
    p.bank = bank;
    p.slot_stride = slot_stride;
    p.n_slots = n_slots;
    p.slot_ids = slot_ids;
    p.n_blocks = n_blocks;
    p.sides = sides;
    p.out = out;
    p.err = err_flag;
    p.levels = num_levels;
    expand_lut(lut, num_levels, p.lut);
    return launch_decode(p, n_sel, out_dtype, stream);
}

}  // extern "C"
