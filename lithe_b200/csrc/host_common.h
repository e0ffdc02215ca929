// Host helpers shared by the C-ABI entry points: per-thread error text, CUDA error
// mapping, per-device attribute cache and TMA tensor-map encoding through the driver
// entry point (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>

#include "lithe_b200.h"

namespace lithe {

void set_error(const char* fmt, ...);
int32_t fail_arg(const char* fmt, ...);
int32_t fail_unsupported(const char* fmt, ...);
int32_t fail_cuda(cudaError_t e, const char* what);
void clear_error();

// Current device and its SM count (cached per device).
int32_t current_device_sms(int* device, int* sms);

// Encode a rank-3 bf16 tensor map over a contiguous (d2, d1, d0) array with box
// (b0, b1, 1) and 128-byte swizzle.  Returns LITHE_OK or an error code.
int32_t encode_bf16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                       uint32_t b0, uint32_t b1);
// "Chunked" view of a row-major (rows, inner) bf16 array, inner a multiple of 64: dimensions
// (64 columns, rows, inner / 64 chunks) with the chunk stride (128 B) as the outer one, so one
// box (64, box_rows, chunks_per_box) fetches chunks_per_box adjacent 64-column chunks of
// box_rows rows, each laid out as its own 128-byte-swizzled tile, in one TMA operation.
int32_t encode_bf16_chunked(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows,
                            uint32_t chunks_per_box);
// 2-D bf16 tensor map (rows of `inner` elements), box (box_inner, box_rows), swizzle 0/32/64/128 B.
int32_t encode_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint32_t box_inner,
                       uint32_t box_rows, int swizzle_bytes);

// Fill the kernel-side lookup table lut_dev[side][level][16] from the host-side
// [2][levels][10] array of the C ABI.
void expand_lut(const float* lut, int levels, float out[2][LITHE_MAX_LEVELS][16]);

}  // namespace lithe
