// k3_wait_selftest: the bounded device-side wait that every pipelined kernel of this
// library uses (mbar_wait), run on its own against a barrier whose completion the test
// controls. The failure it shows is made on purpose and harmlessly: a barrier that nothing
// arrives at, so the wait runs out of time, records K3_ERR_TIMEOUT in the status word and
// returns -- no trap, no fault, and the context stays usable for the next call.
#include "k3_async.cuh"

namespace k3 {
namespace {

// mode 0: nobody arrives (the wait's limit runs out); 1: warp 1 arrives (the wait
// succeeds); 2: warp 1 raises the abort flag instead (the wait gives up without a
// timeout). result = {status word, wait returned true (1) or false (0), elapsed ns}.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int mode, int32_t* result) {
    __shared__ alignas(8) uint64_t bar;
    __shared__ volatile int abort_flag;
    __shared__ int status;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        status = K3_OK;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    if (warp == 0 && threadIdx.x == 0) {
        const uint64_t t0 = global_ns();
        const bool ok = mbar_wait(&bar, 0, &status, &abort_flag, limit_ns);
        const uint64_t t1 = global_ns();
        result[0] = status;
        result[1] = ok ? 1 : 0;
        result[2] = int32_t(t1 - t0 > 0x7fffffffull ? 0x7fffffffull : t1 - t0);
    } else if (warp == 1 && threadIdx.x == 32) {
        if (mode == 1) mbar_arrive(&bar);
        if (mode == 2) abort_flag = 1;
    }
    __syncthreads();
    // mode 0 and 2 leave the barrier's phase open; it dies with the CTA's shared memory
}

}  // namespace
}  // namespace k3

using namespace k3;

extern "C" K3_API int k3_wait_selftest(int64_t limit_ns, int mode, int32_t* result, void* stream) {
    if (!result) return fail(K3_ERR_INVALID, "k3_wait_selftest: result is NULL");
    if (mode < 0 || mode > 2) return fail(K3_ERR_INVALID, "k3_wait_selftest: mode must be 0, 1 or 2");
    if (limit_ns < 1000 || limit_ns > int64_t(kWaitLimitNs))
        return fail(K3_ERR_INVALID, "k3_wait_selftest: limit_ns must be 1e3..2e9");
    wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(uint64_t(limit_ns), mode, result);
    K3_CHECK_LAUNCH("wait_selftest_kernel");
    return K3_OK;
}
