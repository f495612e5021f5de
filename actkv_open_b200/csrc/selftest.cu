// Self-test of the failure path of the pipelined kernels: a bounded mbarrier wait that nothing
// satisfies.  The wait is the same helper every TMA / MMA / epilogue role uses (umma::mbar_wait):
// after ~2^31 cycles it gives up, raises the block's abort flag, sets ACTKV_DEV_TIMEOUT in the
// status word and returns false, so the kernel ends normally and the context stays usable.  No
// trap, no fault: it lets a test show that a stalled pipeline reports instead of hanging.
#include "common.cuh"
#include "kernels.cuh"
#include "umma_common.cuh"

namespace actkv {

namespace {

__global__ void bounded_wait_probe_kernel(int32_t* status, long long* waited) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    umma::mbar_init(umma::smem_u32(&bar), 1);          // one arrival completes phase 0: none comes
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const long long t0 = clock64();
  const bool done = umma::mbar_wait(umma::smem_u32(&bar), 0, &abort_flag, status);
  const long long dt = clock64() - t0;
  if (threadIdx.x == 0) *waited = done ? -1 : dt;
}

}  // namespace

cudaError_t launch_bounded_wait_probe(int32_t* status, long long* waited, cudaStream_t st) {
  bounded_wait_probe_kernel<<<1, 32, 0, st>>>(status, waited);
  return cudaGetLastError();
}

}  // namespace actkv
