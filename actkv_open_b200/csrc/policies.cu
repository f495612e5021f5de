// Baseline eviction policies of the reference on the device (actkv/eviction.py:89-149).
//
// snapkv_scores_kernel: SnapKV's per-layer token scores, the sum of the attention rows of the
//   last w observed query tokens (oldest first, each row over its own length) average-pooled with
//   kernel `pool` (stride 1, zero padding pool / 2, divisor pool; the same summation order as the
//   reference's torch ops), plus the pinned mask of the observation window [length - w, length).
//   The keep mask then comes from the keep-mask kernels (protected prefix and window pinned, the
//   top budget - w of the rest, ties to the lowest index), and keep_indices_kernel turns each
//   layer's mask into its sorted keep indices.
// streaming_keep_kernel: StreamingLLM's keep indices, the protected prefix and the last `budget`
//   tokens, the same in every layer.
// snapkv_gather_kernel: SnapKV.apply_keep, each stored row and layer gathered by the layer's keep
//   indices (entries past the row's length dropped) into the other half of a double buffer.
#include "common.cuh"
#include "kernels.cuh"

namespace actkv {

namespace {

constexpr int kScoreTile = 256;

__global__ void __launch_bounds__(kScoreTile) snapkv_scores_kernel(SnapScoreArgs a) {
  __shared__ float acc[kScoreTile + kSnapMaxPool];
  const int l = blockIdx.x, t0 = blockIdx.y * kScoreTile;
  const int pad = a.pool / 2;
  const int n = kScoreTile + a.pool - 1;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int t = t0 - pad + i;
    float v = 0.0f;
    if (t >= 0 && t < a.length)
      for (int k = 0; k < a.w; ++k) {
        const int s = a.slots[k];
        const int len = min(a.lens[int64_t(s) * a.lens_stride_slot + l], a.length);
        if (t < len) v += a.rows[int64_t(s) * a.stride_slot + int64_t(l) * a.stride_l + t];
      }
    acc[i] = v;
  }
  __syncthreads();
  const int t = t0 + threadIdx.x;
  if (t < a.length) {
    float p = acc[threadIdx.x + pad];
    if (a.pool > 1) {
      float sum = 0.0f;
      for (int j = 0; j < a.pool; ++j) sum += acc[threadIdx.x + j];
      p = sum / float(a.pool);
    }
    a.scores[int64_t(l) * a.stride_out + t] = p;
    a.pinned[int64_t(l) * a.stride_out + t] = t >= a.length - a.w ? 1 : 0;
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) {
    a.seq[l] = a.length;
    a.budget_rest[l] = a.rest;
  }
}

// Row l's kept positions in order; exactly K of them are expected.
__global__ void __launch_bounds__(1024) keep_indices_kernel(const uint8_t* keep, int64_t keep_stride, int length,
                                                            int64_t* out, int64_t out_stride, int K,
                                                            int32_t* status) {
  __shared__ int red[33];
  const int l = blockIdx.x;
  int base = 0;
  for (int t0 = 0; t0 < length; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    const bool k = t < length && keep[int64_t(l) * keep_stride + t] != 0;
    int total;
    const int pos = base + block_excl_count(k, red, &total);
    if (k && pos < K) out[int64_t(l) * out_stride + pos] = t;
    base += total;
  }
  if (threadIdx.x == 0 && base != K) flag(status, ACTKV_DEV_BAD_INDEX);
}

__global__ void streaming_keep_kernel(int64_t* out, int64_t out_stride, int length, int protected_tokens,
                                      int budget) {
  const int l = blockIdx.x;
  for (int i = threadIdx.x; i < protected_tokens + budget; i += blockDim.x)
    out[int64_t(l) * out_stride + i] = i < protected_tokens ? i : length - budget + (i - protected_tokens);
}

__global__ void __launch_bounds__(256) snapkv_gather_kernel(SnapGatherArgs a) {
  __shared__ int red[32];
  const int s = a.slots[blockIdx.x], l = blockIdx.y;
  const int len = a.lens[int64_t(s) * a.lens_stride_slot + l];
  const int64_t* kp = a.keep + int64_t(l) * a.keep_stride;
  const float* src = a.src + int64_t(s) * a.stride_slot + int64_t(l) * a.stride_l;
  float* dst = a.dst + int64_t(s) * a.stride_slot + int64_t(l) * a.stride_l;
  int cnt = 0;
  for (int j = threadIdx.x; j < a.K; j += blockDim.x) {
    const int64_t t = kp[j];
    if (t >= 0 && t < len) {          // keep is sorted: these j form the prefix [0, cnt)
      dst[j] = src[t];
      ++cnt;
    }
  }
  cnt = block_sum(cnt, red);
  if (threadIdx.x == 0) a.lens[int64_t(s) * a.lens_stride_slot + l] = cnt;
}

}  // namespace

cudaError_t launch_snapkv_scores(const SnapScoreArgs& a, int L, cudaStream_t st) {
  if (L <= 0 || a.length <= 0) return cudaSuccess;
  snapkv_scores_kernel<<<dim3(L, (a.length + kScoreTile - 1) / kScoreTile), kScoreTile, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_keep_indices(const uint8_t* keep, int64_t keep_stride, int length, int64_t* out,
                                int64_t out_stride, int K, int L, int32_t* status, cudaStream_t st) {
  if (L <= 0) return cudaSuccess;
  keep_indices_kernel<<<L, 1024, 0, st>>>(keep, keep_stride, length, out, out_stride, K, status);
  return cudaGetLastError();
}

cudaError_t launch_streaming_keep(int64_t* out, int64_t out_stride, int L, int length, int protected_tokens,
                                  int budget, cudaStream_t st) {
  if (L <= 0) return cudaSuccess;
  streaming_keep_kernel<<<L, 256, 0, st>>>(out, out_stride, length, protected_tokens, budget);
  return cudaGetLastError();
}

cudaError_t launch_snapkv_gather(const SnapGatherArgs& a, int n, int L, cudaStream_t st) {
  if (n <= 0 || L <= 0) return cudaSuccess;
  snapkv_gather_kernel<<<dim3(n, L), 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace actkv
