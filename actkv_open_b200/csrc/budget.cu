// Adaptive budget (ActKV Algorithm 2, actkv/budget.py:9-104) on the device.
//
// confidence_kernel (one CTA per logit row): T = -(1/k) sum of the k largest log-softmax values =
//   lse(x) - (sum of the k largest x) / k.  lse from a block max and a block sum of exp; the sum of
//   the k largest values from a radix select of the k-th largest (4 passes of 8-bit digits over
//   order-preserving keys) plus the values above it, so ties at the boundary count exactly as
//   torch.topk's values do.  T is appended to the row's session trace (trace_len advances), so
//   recording a decode step needs no host round trip.
// budget_kernel (one CTA per session): the reference's trace_confidence + fit_slope +
//   ConfidenceBudget.next_budget on the session's whole trace: sliding-window minima into shared
//   memory, the bottom_pct quantile by two radix selects (linear interpolation as torch.quantile /
//   torch.lerp), least-squares slope of the kept windows in double, then the budget step (grow by
//   scale_up when the slope is negative; with `bidirectional`, shrink by scale_down after
//   shrink_patience rising slopes).  With seq_used given it steps only sessions whose unprotected
//   length exceeds the budget (the reference's end_round, actkv/hf/session.py:186-193), and it can
//   write the new budget straight into the eviction step's budget array.
#include "common.cuh"
#include "kernels.cuh"

namespace actkv {

namespace {

constexpr int kBudgetThreads = 1024;

__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Key of rank `want` in descending order (0 = the largest) among the n keys key_of(0..n-1).
// All threads of the block call it; hist holds 256 counters, sh 2 ints.
template <typename KeyFn>
__device__ uint32_t block_select_desc(int n, int want, KeyFn key_of, uint32_t* hist, int* sh) {
  uint32_t prefix = 0, mask = 0;
  int rem = want;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t key = key_of(i);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0, bin = 255;
      for (; bin > 0; --bin) {
        if (acc + int(hist[bin]) > rem) break;
        acc += int(hist[bin]);
      }
      sh[0] = bin;
      sh[1] = rem - acc;
    }
    __syncthreads();
    prefix |= uint32_t(sh[0]) << shift;
    mask |= 255u << shift;
    rem = sh[1];
    __syncthreads();
  }
  return prefix;
}

template <typename T>
__global__ void __launch_bounds__(kBudgetThreads) confidence_kernel(ConfidenceArgs a) {
  __shared__ float redf[32];
  __shared__ double redd[32];
  __shared__ int redi[32];
  __shared__ uint32_t hist[256];
  __shared__ int sh[2];
  const int row = blockIdx.x;
  const T* x = static_cast<const T*>(a.logits) + int64_t(row) * a.row_stride;
  const int V = a.V;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, to_f32(x[i]));
  m = block_max(m, redf);
  float s = 0.0f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) s += expf(to_f32(x[i]) - m);
  s = block_sum(s, redf);
  const float lse = m + logf(s);
  const int k = min(a.k, V);
  const uint32_t tk = block_select_desc(V, k - 1, [&](int i) { return order_key(to_f32(x[i])); }, hist, sh);
  double above = 0.0;
  int n_above = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = to_f32(x[i]);
    if (order_key(v) > tk) {
      above += double(v);
      ++n_above;
    }
  }
  above = block_sum(above, redd);
  n_above = block_sum(n_above, redi);
  if (threadIdx.x == 0) {
    const double top = above + double(k - n_above) * double(key_to_float(tk));
    const float conf = float(double(lse) - top / double(k));
    const int r = a.sessions ? a.sessions[row] : row;
    const int pos = a.trace_len[r];
    if (pos < a.capacity) {
      a.trace[int64_t(r) * a.capacity + pos] = conf;
      a.trace_len[r] = pos + 1;
    } else {
      flag(a.status, ACTKV_DEV_BAD_INDEX);
    }
  }
}

__global__ void __launch_bounds__(kBudgetThreads) budget_kernel(BudgetArgs a) {
  extern __shared__ float pooled[];                   // [kBudgetMaxPooled]
  __shared__ double redd[32];
  __shared__ uint32_t hist[256];
  __shared__ int sh[2];
  const int r = blockIdx.x;
  const int b0 = a.budget[r];
  if (a.seq_used && !(a.seq_used[r] - a.protected_tokens > b0)) {
    // not over budget: the reference keeps the current budget and takes no slope
    if (threadIdx.x == 0) {
      if (a.slope) a.slope[r] = nan("");
      if (a.budget_out) a.budget_out[r] = b0;
    }
    return;
  }
  const int n = min(a.trace_len[r], int(a.capacity));
  const float* t = a.trace + int64_t(r) * a.capacity;
  const int w = n < a.window ? n : a.window;
  const int P = n == 0 ? 0 : (n - w) / a.stride + 1;
  if (P > kBudgetMaxPooled) {
    if (threadIdx.x == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
    return;
  }
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    float v = t[int64_t(i) * a.stride];
    for (int j = 1; j < w; ++j) v = fminf(v, t[int64_t(i) * a.stride + j]);
    pooled[i] = v;
  }
  __syncthreads();
  double slope = 0.0;
  if (P >= 2) {
    auto key_of = [&](int i) { return order_key(pooled[i]); };
    const double pos = (a.bottom_pct / 100.0) * double(P - 1);
    const int lo = int(floor(pos));
    const int hi = min(lo + 1, P - 1);
    const double wt = pos - double(lo);
    const double vlo = key_to_float(block_select_desc(P, P - 1 - lo, key_of, hist, sh));
    const double vhi = key_to_float(block_select_desc(P, P - 1 - hi, key_of, hist, sh));
    const double thr = wt < 0.5 ? vlo + wt * (vhi - vlo) : vhi - (vhi - vlo) * (1.0 - wt);
    double cnt = 0.0, sx = 0.0, sy = 0.0;
    for (int i = threadIdx.x; i < P; i += blockDim.x)
      if (double(pooled[i]) <= thr) {
        cnt += 1.0;
        sx += double(i);
        sy += double(pooled[i]);
      }
    cnt = block_sum(cnt, redd);
    sx = block_sum(sx, redd);
    sy = block_sum(sy, redd);
    if (cnt >= 2.0) {
      const double xm = sx / cnt, ym = sy / cnt;
      double var = 0.0, cov = 0.0;
      for (int i = threadIdx.x; i < P; i += blockDim.x)
        if (double(pooled[i]) <= thr) {
          const double dx = double(i) - xm;
          var += dx * dx;
          cov += dx * (double(pooled[i]) - ym);
        }
      var = block_sum(var, redd);
      cov = block_sum(cov, redd);
      if (var != 0.0) slope = cov / var;
    }
  }
  if (threadIdx.x == 0) {
    int b = b0, rising = a.rising[r];
    if (slope < 0.0) {
      b = min(int(double(b) * a.scale_up), a.upper);
      rising = 0;
    } else if (a.bidirectional && slope > a.shrink_slope) {
      if (++rising >= a.shrink_patience) {
        b = max(int(double(b) / a.scale_down), a.lower);
        rising = 0;
      }
    } else {
      rising = 0;
    }
    a.budget[r] = b;
    a.rising[r] = rising;
    if (a.slope) a.slope[r] = slope;
    if (a.budget_out) a.budget_out[r] = b;
  }
}

}  // namespace

cudaError_t launch_confidence(const ConfidenceArgs& a, int dtype, int B, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  if (dtype == ACTKV_F32)
    confidence_kernel<float><<<B, kBudgetThreads, 0, st>>>(a);
  else if (dtype == ACTKV_F16)
    confidence_kernel<__half><<<B, kBudgetThreads, 0, st>>>(a);
  else
    confidence_kernel<__nv_bfloat16><<<B, kBudgetThreads, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_budget(const BudgetArgs& a, int R, cudaStream_t st) {
  if (R <= 0) return cudaSuccess;
  const int smem = kBudgetMaxPooled * int(sizeof(float));
  cudaError_t e = cudaFuncSetAttribute(budget_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  budget_kernel<<<R, kBudgetThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace actkv
