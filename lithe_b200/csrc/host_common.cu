// Host helpers: error reporting, device attribute cache, tensor-map encoding.
#include "host_common.h"

#include <cudaTypedefs.h>

#include <cstdarg>
#include <mutex>

namespace lithe {

namespace {
thread_local char g_error[512] = {0};
constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices] = {0};
std::mutex g_mutex;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

void vset(const char* fmt, va_list ap) { vsnprintf(g_error, sizeof(g_error), fmt, ap); }
}  // namespace

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vset(fmt, ap);
    va_end(ap);
}

void clear_error() { g_error[0] = 0; }

int32_t fail_arg(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vset(fmt, ap);
    va_end(ap);
    return LITHE_ERR_ARG;
}

int32_t fail_unsupported(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vset(fmt, ap);
    va_end(ap);
    return LITHE_ERR_UNSUPPORTED;
}

int32_t fail_cuda(cudaError_t e, const char* what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return LITHE_ERR_CUDA;
}

int32_t current_device_sms(int* device, int* sms) {
    cudaError_t e = cudaGetDevice(device);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
    if (*device < 0 || *device >= kMaxDevices) return fail_unsupported("device ordinal %d", *device);
    int v = g_sms[*device];
    if (v == 0) {
        e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, *device);
        if (e != cudaSuccess) return fail_cuda(e, "cudaDeviceGetAttribute(SM count)");
        g_sms[*device] = v;
    }
    *sms = v;
    return LITHE_OK;
}

static int32_t get_encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess) return fail_cuda(e, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
        if (q != cudaDriverEntryPointSuccess || !fn)
            return fail_unsupported("driver does not export cuTensorMapEncodeTiled");
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    *out = g_encode;
    return LITHE_OK;
}

int32_t encode_bf16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                       uint32_t b0, uint32_t b1) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int32_t rc = get_encoder(&enc);
    if (rc != LITHE_OK) return rc;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};   // bytes, dims 1 and 2
    const cuuint32_t box[3] = {b0, b1, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail_arg("cuTensorMapEncodeTiled failed (CUresult %d) for dims (%llu,%llu,%llu) box (%u,%u)",
                        static_cast<int>(r), (unsigned long long)d0, (unsigned long long)d1,
                        (unsigned long long)d2, b0, b1);
    return LITHE_OK;
}

int32_t encode_bf16_chunked(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows,
                            uint32_t chunks_per_box) {
    if (inner % 64 != 0) return fail_arg("chunked tensor map: row length %llu is not a multiple of 64",
                                         (unsigned long long)inner);
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int32_t rc = get_encoder(&enc);
    if (rc != LITHE_OK) return rc;
    // element (c0, r, k) = base[r * inner + 64 * k + c0]: the chunk index is the outer dimension,
    // with a stride (128 B) smaller than the row stride; the three extents cover the array exactly
    const cuuint64_t dims[3] = {64, rows, inner / 64};
    const cuuint64_t strides[2] = {inner * 2, 128};
    const cuuint32_t box[3] = {64, box_rows, chunks_per_box};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail_arg("cuTensorMapEncodeTiled failed (CUresult %d) for a chunked map: row length %llu, rows %llu",
                        static_cast<int>(r), (unsigned long long)inner, (unsigned long long)rows);
    return LITHE_OK;
}

int32_t encode_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint32_t box_inner,
                       uint32_t box_rows, int swizzle_bytes) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int32_t rc = get_encoder(&enc);
    if (rc != LITHE_OK) return rc;
    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
    if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
    else if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
    else if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * 2};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail_arg("cuTensorMapEncodeTiled failed (CUresult %d) for dims (%llu,%llu) box (%u,%u)",
                        static_cast<int>(r), (unsigned long long)inner, (unsigned long long)rows, box_inner, box_rows);
    return LITHE_OK;
}

void expand_lut(const float* lut, int levels, float out[2][LITHE_MAX_LEVELS][16]) {
    for (int s = 0; s < 2; ++s)
        for (int l = 0; l < LITHE_MAX_LEVELS; ++l)
            for (int n = 0; n < 16; ++n)
                out[s][l][n] = (l < levels && n < 10) ? lut[(s * levels + l) * 10 + n] : 0.0f;
}

}  // namespace lithe

extern "C" {

int32_t lithe_abi_version(void) { return LITHE_ABI_VERSION; }

const char* lithe_last_error(void) { return lithe::g_error; }

}  // extern "C"
