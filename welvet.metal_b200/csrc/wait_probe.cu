// Bounded-wait probe: one thread waits on an mbarrier that nothing arrives at,
// through the same mbar_wait_for primitive every pipeline kernel of this library
// uses, with a caller-chosen limit. The wait runs out, the thread records
// kErrWaitOther in the error word and the kernel returns normally: no trap, no
// copy in flight, no TMEM held, so the context stays usable. The host then reads
// the error word (status 4 with the reason), which is the path a real pipeline
// stall takes. Used by the failure-handling test; it reads and writes nothing
// else.
#include "common.cuh"
#include "kernels.h"

namespace wv {
namespace {

__global__ void wait_probe_kernel(uint32_t* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // phase 0 never completes: no thread arrives
    mbar_wait_for(&bar, 0, &abort_flag, err, kErrWaitOther, limit_ns);
  }
  __syncthreads();
}

}  // namespace

cudaError_t wait_probe(uint32_t* err, uint64_t limit_ns, cudaStream_t s) {
  wait_probe_kernel<<<1, 32, 0, s>>>(err, limit_ns);
  return cudaGetLastError();
}

}  // namespace wv
