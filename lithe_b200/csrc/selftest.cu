// Self-test of the bounded pipeline wait every LITHE kernel uses (mbar_wait in
// device_common.cuh): a kernel waits on an mbarrier that nothing ever arrives at.  The wait
// must end by itself after its time limit, set the CTA's abort flag and OR
// LITHE_DEVERR_TIMEOUT into the error word, and the kernel must return normally, leaving the
// CUDA context usable.  No fault, trap or unbounded wait is involved: this is how the failure
// path of the real kernels is exercised on the GPU.
#include "device_common.cuh"
#include "host_common.h"

namespace lithe {

__global__ void __launch_bounds__(32) wait_timeout_kernel(int32_t* err, int32_t* waited_ok) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);                     // expects one arrival that never comes
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait(&bar, 0u, &abort_flag, err);
        if (waited_ok) *waited_ok = ok ? 1 : 0;
        // complete the barrier's phase ourselves so nothing is left pending at exit
        mbar_arrive(&bar);
    }
}

}  // namespace lithe

extern "C" int32_t lithe_selftest_wait_timeout(int32_t* err_flag, int32_t* waited_ok, void* stream) {
    using namespace lithe;
    clear_error();
    if (!err_flag) return fail_arg("err_flag is NULL");
    wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(err_flag, waited_ok);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "wait_timeout_kernel launch");
    return LITHE_OK;
}
