// selftest.cu - the bounded wait every kernel of the library uses, exercised on its own.
//
// Every mbarrier wait in the kernels (read, prefill, fused decode, streaming select) goes
// through mbar_wait_bounded: it polls the barrier's phase and gives up after a limit of
// %globaltimer time, after which the kernel records LSA_ERR_TIMEOUT and leaves instead of
// hanging. lsa_wait_selftest runs that helper on a barrier of its own: with `arrive` != 0
// the barrier's phase completes and the wait returns at once (status 0); with `arrive` == 0
// nothing ever arrives, the wait runs out after `limit_ns` and the status word receives
// LSA_ERR_TIMEOUT - the failure path, taken without a fault or a hang.
#include "common.cuh"

namespace lsa {

__global__ void wait_selftest_kernel(int32_t* status, int64_t limit_ns, int arrive) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (arrive) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bar)) : "memory");
    const bool ok = mbar_wait_bounded(&bar, 0, (uint64_t)limit_ns);
    *status = ok ? LSA_OK : LSA_ERR_TIMEOUT;
}

}  // namespace lsa

extern "C" {

int lsa_wait_selftest(int32_t* status, int64_t limit_ns, int arrive, cudaStream_t stream) {
    if (status == nullptr || limit_ns <= 0 || limit_ns > 2000000000ll) return LSA_ERR_ARG;
    lsa::wait_selftest_kernel<<<1, 32, 0, stream>>>(status, limit_ns, arrive);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // extern "C"
