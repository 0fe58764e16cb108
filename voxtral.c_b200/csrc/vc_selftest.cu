// vc_selftest.cu - exercises the bounded-wait error path of the kernels
// without faulting the GPU: a kernel waits on an mbarrier that nothing will
// ever complete, through the same bounded wait the tensor-core kernels use,
// and raises the launch's error word when the deadline passes.  The host
// reads the word as it does after every step and reports the timeout; the
// context stays usable.
#include "vc_common.cuh"
#include "vc_internal.h"
#include "vc_tc.cuh"

namespace vc {

using namespace tc;

__global__ void stuck_wait_kernel(unsigned *err, unsigned long long wait_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);   // one arrival expected; none will come
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const uint64_t deadline = globaltimer() + wait_ns;
    const bool ok = mbar_wait(&bar, 0u, deadline);
    if (!ok && threadIdx.x == 0) atomicExch(err, 1u);
}

cudaError_t launch_stuck_wait(unsigned *err, unsigned long long wait_ns, cudaStream_t st) {
    stuck_wait_kernel<<<1, 32, 0, st>>>(err, wait_ns);
    return cudaGetLastError();
}

}  // namespace vc
