// actkv_keep_mask_static: the keep-mask selection of actkv_keep_mask for callers that cannot
// allocate device memory (an allocator-less host runtime, a memory pool that is already carved up,
// a plugin whose host forbids cudaMalloc while it serves).  Its scratch is this file's static
// device array instead of a caller workspace; inputs and outputs are still the caller's.
#include <stdio.h>

#include <mutex>

#include "kernels.cuh"

namespace actkv {

// Per-token reduced scores of every session of one call: R * max_seq floats at most.
constexpr size_t kStaticScratchFloats = size_t(1) << 20;   // 4 MiB, held by each GPU that loads the library
static __device__ __align__(256) float g_keep_scratch[kStaticScratchFloats];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_keep_scratch on the current device, looked up once per device.  In host
// code `g_keep_scratch` names a host-side stand-in, never the device array, so it is only ever
// passed to kernels through this address.
cudaError_t scratch_for_current_device(float** out, int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  *dev_out = dev;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_keep_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace actkv

using namespace actkv;

namespace actkv {
void set_last_error(const char* msg);   // capi.cu: the message actkv_last_error() returns
}

namespace {
int fail_static(int code, const char* fmt, size_t a = 0, size_t b = 0) {
  char buf[256];
  snprintf(buf, sizeof(buf), fmt, a, b);
  actkv::set_last_error(buf);
  return code;
}
}  // namespace

extern "C" {

int actkv_keep_mask_static(const float* scores, const int64_t* scores_off, int64_t scores_stride_r,
                           int64_t scores_stride_l, int64_t scores_stride_x, int n_lead, int n_red,
                           int head_reduce, const uint8_t* pinned, int64_t pinned_stride_r, int protected_prefix,
                           const int32_t* seq_used, const int32_t* budget, int evict_semantics, uint8_t* keep,
                           int64_t keep_stride_r, int32_t* kept, int R, int max_seq, int32_t* status,
                           void* stream) {
  if (head_reduce != ACTKV_REDUCE_MEAN && head_reduce != ACTKV_REDUCE_MAX)
    return fail_static(ACTKV_ERR_HEAD_REDUCE, "head_reduce must be mean or max");
  if (n_lead <= 0 || n_red <= 0 || R < 0 || max_seq < 0) return fail_static(ACTKV_ERR_INVALID, "bad sizes");
  if (size_t(R) * size_t(max_seq) > kStaticScratchFloats)
    return fail_static(ACTKV_ERR_WORKSPACE,
                       "R * max_seq = %zu exceeds the static scratch of %zu floats (4 MiB); split the batch "
                       "or use actkv_keep_mask with a workspace",
                       size_t(R) * size_t(max_seq), kStaticScratchFloats);
  actkv::set_last_error("");
  if (R == 0) return ACTKV_OK;
  float* scratch = nullptr;
  int dev = 0;
  cudaError_t e = scratch_for_current_device(&scratch, &dev);
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "static scratch set-up on device %d: %s", dev, cudaGetErrorString(e));
    actkv::set_last_error(buf);
    return ACTKV_ERR_CUDA;
  }
  // Every entry of the scratch that the kernel reads it has written first in the same launch, so
  // nothing needs clearing between calls.
  KeepMaskArgs a{scores, scores_off, scores_stride_r, scores_stride_l, scores_stride_x, n_lead, n_red,
                 head_reduce, pinned, pinned_stride_r, protected_prefix, seq_used, budget, evict_semantics,
                 keep, keep_stride_r, kept, scratch, max_seq, status};
  e = launch_keep_mask(a, R, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "keep_mask_static: %s", cudaGetErrorString(e));
    actkv::set_last_error(buf);
    return ACTKV_ERR_CUDA;
  }
  return ACTKV_OK;
}

}  // extern "C"
