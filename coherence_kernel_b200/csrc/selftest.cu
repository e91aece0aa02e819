// selftest.cu -- the failure path of the bounded device waits, run without faulting anything.
//
// Every pipeline in this library (grouped GEMM, tensor-core matvecs, streaming matvec) waits on
// mbarriers through mbar_wait_bounded, which gives up after a time limit, records a code in an
// error word and returns false instead of spinning forever.  k_wait_selftest runs that routine on
// an mbarrier that nothing ever arrives on, with a caller-chosen short limit: the wait must give
// up, the code must land in the error word the host reads, and the kernel must return -- leaving
// the context usable for the next launch.  No copy or MMA is in flight while it waits.
#include "../../include/ck_b200.h"
#include "ck_common.cuh"

namespace {
__global__ void k_wait_selftest(uint64_t limit_ns, int *err, unsigned long long *waited_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        ck::mbar_init(&bar, 1);  // one arrival expected; none is ever made
        ck::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = ck::globaltimer_ns();
        const bool ok = ck::mbar_wait_bounded_ns(&bar, 0, err, 77, limit_ns);
        *waited_ns = ok ? 0ull : (unsigned long long)(ck::globaltimer_ns() - t0);
    }
}
}  // namespace

extern "C" int ck_wait_selftest(uint64_t limit_ns, int *err_dev, unsigned long long *waited_ns_dev, void *stream) {
    if (!err_dev || !waited_ns_dev || limit_ns == 0 || limit_ns > 2000000000ull) return CK_EARG;
    k_wait_selftest<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns, err_dev, waited_ns_dev);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
}
