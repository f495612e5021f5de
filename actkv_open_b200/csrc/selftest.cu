// Self-tests.  (1) The failure path of the pipelined kernels: a bounded mbarrier wait that nothing
// satisfies.  The wait is the same helper every TMA / MMA / epilogue role uses (umma::mbar_wait):
// after ~2^31 cycles it gives up, raises the block's abort flag, sets ACTKV_DEV_TIMEOUT in the
// status word and returns false, so the kernel ends normally and the context stays usable.  No
// trap, no fault: it lets a test show that a stalled pipeline reports instead of hanging.
// (2) The rate at which HBM serves the paged cache in the two read patterns (kv_gather_kernel).
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

// Read-only sweep of a paged cache in the two access patterns its kernels can use, to time what
// HBM serves each: mode 0 reads one head per CTA (CTA c takes head c % Hkv of blocks c / Hkv,
// c / Hkv + gridDim / Hkv, ...: per block BS pieces of head_bytes, row_bytes apart); mode 1 reads
// whole blocks (BS * row_bytes contiguous).  Both read every byte once.  The loads are folded into
// a checksum that is written only if it equals a value no cache of real data produces.
__global__ void __launch_bounds__(256) kv_gather_kernel(const uint4* __restrict__ kv, int64_t n_blocks, int BS,
                                                        int row_bytes, int head_bytes, int mode,
                                                        unsigned long long* sink) {
  const int64_t blk_u4 = int64_t(BS) * row_bytes / 16;       // uint4 per block
  uint32_t acc = 0;
  if (mode == 0) {
    const int hkv = row_bytes / head_bytes, per_tok = head_bytes / 16, n = BS * per_tok;
    const int h = int(blockIdx.x) % hkv;
    const int64_t b0 = blockIdx.x / hkv, bstep = gridDim.x / hkv;
    for (int64_t b = b0; b < n_blocks; b += 4 * bstep)
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t bb = b + k * bstep;
          v[k] = bb < n_blocks ? kv[bb * blk_u4 + int64_t(i / per_tok) * (row_bytes / 16) + h * per_tok + i % per_tok]
                               : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) acc ^= v[k].x ^ v[k].y ^ v[k].z ^ v[k].w;
      }
  } else {
    for (int64_t b = blockIdx.x; b < n_blocks; b += 4 * int64_t(gridDim.x))
      for (int64_t i = threadIdx.x; i < blk_u4; i += blockDim.x) {
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t bb = b + k * int64_t(gridDim.x);
          v[k] = bb < n_blocks ? kv[bb * blk_u4 + i] : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) acc ^= v[k].x ^ v[k].y ^ v[k].z ^ v[k].w;
      }
  }
  if (acc == 0x9e3779b9u && sink) atomicAdd(sink, 1ull);
}

}  // namespace

cudaError_t launch_bounded_wait_probe(int32_t* status, long long* waited, cudaStream_t st) {
  bounded_wait_probe_kernel<<<1, 32, 0, st>>>(status, waited);
  return cudaGetLastError();
}

cudaError_t launch_kv_gather(const void* kv, int64_t n_blocks, int BS, int row_bytes, int head_bytes, int mode,
                             unsigned long long* sink, cudaStream_t st) {
  // mode 0: a multiple of Hkv CTAs, so that every head of every block is read once
  const int hkv = row_bytes / head_bytes;
  int grid = device_sm_count() * 8;
  if (mode == 0) grid = (grid / hkv) * hkv;
  kv_gather_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(kv), n_blocks, BS, row_bytes, head_bytes, mode,
                                         sink);
  return cudaGetLastError();
}

}  // namespace actkv
