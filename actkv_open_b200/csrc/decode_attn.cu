// Paged decode attention with its log-sum-exp (flash decoding), on CUDA cores: the GPU form of the
// reference's paged_decode_attention_ref (actkv/kernels/lse_attn.py:42-60), one query per session:
//   out[r, hq, :] = softmax_t(scale * q[r, hq] . k[t, h]) @ v[t, h],  lse[r, hq] = logsumexp_t(...)
// over t < seq_used[r], h = hq / G.
//
// One query token per session makes this HBM-bound (each K/V row is read once and used by the G
// query heads of its KV head), so it runs on CUDA cores: a CTA takes one (session, KV head, token
// split); each warp walks a contiguous run of its split's tokens with lane i holding dims
// [i*DPL, i*DPL + DPL) of q, k, v and of the G output accumulators: a token's G logits are warp
// sums, then the online softmax (running max m, sum l, rescaled accumulator) in log2 units.  The
// warps merge in shared memory, the splits in decode_combine_kernel.
//
// A lane's DPL elements of a K / V row are one vector load (the host requires the rows aligned to
// it), and kTok tokens' loads are issued before the first is used: the bytes in flight per SM,
// not the arithmetic, bound this kernel.  The G partial logits of a token are reduced together
// (each butterfly step halves the values a lane carries, then one shuffle per head broadcasts
// the sums), G + 4 + log2 G shuffles instead of 5 G.
#include "common.cuh"
#include "kernels.cuh"

namespace actkv {

namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kTok = 8;                           // tokens whose loads a warp keeps in flight

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// DPL consecutive elements as one load of DPL * sizeof(T) bytes, converted to fp32.
template <typename T, int DPL> struct RowVec;
template <> struct RowVec<float, 4> { using V = float4; };
template <> struct RowVec<float, 2> { using V = float2; };
template <> struct RowVec<__nv_bfloat16, 4> { using V = uint2; };
template <> struct RowVec<__nv_bfloat16, 2> { using V = uint32_t; };
template <> struct RowVec<__half, 4> { using V = uint2; };
template <> struct RowVec<__half, 2> { using V = uint32_t; };

template <typename T, int DPL>
__device__ __forceinline__ void load_row(const T* p, float (&x)[DPL]) {
  using V = typename RowVec<T, DPL>::V;
  static_assert(sizeof(V) == DPL * sizeof(T), "one vector per lane");
  const V v = __ldg(reinterpret_cast<const V*>(p));
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < DPL; ++i) x[i] = to_f32(e[i]);
}

// x[g] holds lane partials of G sums; on return x[g] is sum g on every lane.  Butterfly steps
// with offsets 16, 8, ... each hand half of the remaining values to the partner lane, so after
// log2 G steps a lane carries one value (that of head lane >> (5 - log2 G)); the remaining
// offsets finish its sum and a shuffle per head broadcasts the G results.
template <int G>
__device__ __forceinline__ void warp_sums(float (&x)[G]) {
  constexpr unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  int o = 16;
#pragma unroll
  for (int n = G; n > 1; n >>= 1, o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float keep = hi ? x[i + n / 2] : x[i];
      const float send = hi ? x[i] : x[i + n / 2];
      x[i] = keep + __shfl_xor_sync(full, send, o);
    }
  }
  float v = x[0];
  for (; o > 0; o >>= 1) v += __shfl_xor_sync(full, v, o);
  constexpr int shift = G == 1 ? 5 : G == 2 ? 4 : G == 4 ? 3 : 2;
#pragma unroll
  for (int g = 0; g < G; ++g) x[g] = __shfl_sync(full, v, G == 1 ? 0 : g << shift);
}

template <typename T, int G, int DPL>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(DecodeArgs a) {
  constexpr int D = 32 * DPL;
  __shared__ float s_m[kDecWarps][G], s_l[kDecWarps][G];
  __shared__ float s_acc[kDecWarps][G][D];
  const int sp = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.seq_used[r];
  const int per = (S + a.splits - 1) / a.splits;
  const int s0 = min(S, sp * per), s1 = min(S, s0 + per);
  // this warp's contiguous run of the split
  const int wper = (s1 - s0 + kDecWarps - 1) / kDecWarps;
  const int t0 = min(s1, s0 + warp * wper), t1 = min(s1, t0 + wper);
  const float c2 = a.scale * kLog2e;
  float q[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i)
      q[g][i] = to_f32(static_cast<const T*>(a.q)[r * a.q_stride_r + (h * G + g) * a.q_stride_h + lane * DPL + i]) *
                c2;
  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[g][i] = 0.0f;
  }
  const T* kv = static_cast<const T*>(a.kv);
  // kTok tokens at a time: their K / V loads are all in flight before the first is used
  for (int tb = t0; tb < t1; tb += kTok) {
    float k[kTok][DPL], v[kTok][DPL];
    bool use[kTok];
#pragma unroll
    for (int u = 0; u < kTok; ++u) {
      const int t = tb + u;
      const int lb = t / a.BS;
      const int blk = t < t1 && lb < a.MB ? a.block_table[r * a.bt_stride_r + lb] : -1;
      use[u] = t < t1 && blk >= 0 && blk < a.NB;
      if (t < t1 && !use[u] && lane == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      const int64_t row = use[u] ? int64_t(blk) * a.kv_stride_b + int64_t(t % a.BS) * a.kv_stride_s +
                                       int64_t(h) * a.kv_stride_h + lane * DPL
                                 : 0;
      if (use[u]) {
        load_row<T, DPL>(kv + row, k[u]);
        load_row<T, DPL>(kv + a.kv_stride_kv + row, v[u]);
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) k[u][i] = v[u][i] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < kTok; ++u) {
      if (!use[u]) continue;
      float x[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        x[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) x[g] = fmaf(q[g][i], k[u][i], x[g]);
      }
      warp_sums<G>(x);                                  // the G logits, in log2 units, on every lane
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float mn = fmaxf(m[g], x[g]);
        const float corr = ex2f(m[g] - mn);             // 0 while m is still -inf
        const float p = ex2f(x[g] - mn);
        l[g] = fmaf(l[g], corr, p);
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] = fmaf(acc[g][i], corr, p * v[u][i]);
        m[g] = mn;
      }
    }
  }
  // merge the warps
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) s_acc[warp][g][lane * DPL + i] = acc[g][i];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += kDecThreads) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, s_m[w][g]);
    float L = 0.0f, A = 0.0f;
    if (M != -INFINITY)
      for (int w = 0; w < kDecWarps; ++w) {
        if (s_m[w][g] == -INFINITY) continue;
        const float f = ex2f(s_m[w][g] - M);
        L = fmaf(s_l[w][g], f, L);
        A = fmaf(s_acc[w][g][d], f, A);
      }
    const int64_t pi = (int64_t(r) * a.Hq + h * G + g) * a.splits + sp;
    a.part_acc[pi * D + d] = A;
    if (d == 0) {
      a.part_m[pi] = M;
      a.part_l[pi] = L;
    }
  }
}

__global__ void decode_combine_kernel(DecodeArgs a) {
  const int r = blockIdx.y, hq = blockIdx.x;
  const int64_t base = (int64_t(r) * a.Hq + hq) * a.splits;
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.part_m[base + s]);
  float L = 0.0f;
  if (M != -INFINITY)
    for (int s = 0; s < a.splits; ++s)
      if (a.part_m[base + s] != -INFINITY) L = fmaf(a.part_l[base + s], exp2f(a.part_m[base + s] - M), L);
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float A = 0.0f;
    if (M != -INFINITY)
      for (int s = 0; s < a.splits; ++s)
        if (a.part_m[base + s] != -INFINITY)
          A = fmaf(a.part_acc[(base + s) * a.D + d], exp2f(a.part_m[base + s] - M), A);
    a.out[r * a.out_stride_r + hq * a.out_stride_h + d] = L > 0.0f ? A / L : 0.0f;
  }
  if (threadIdx.x == 0)
    a.lse[r * a.lse_stride_r + hq] = L > 0.0f ? (M + log2f(L)) * 0.69314718055994531f : -INFINITY;
}

template <typename T, int DPL>
cudaError_t launch_dec_g(const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  switch (a.G) {
    case 1: decode_attn_kernel<T, 1, DPL><<<grid, kDecThreads, 0, st>>>(a); break;
    case 2: decode_attn_kernel<T, 2, DPL><<<grid, kDecThreads, 0, st>>>(a); break;
    case 4: decode_attn_kernel<T, 4, DPL><<<grid, kDecThreads, 0, st>>>(a); break;
    default: decode_attn_kernel<T, 8, DPL><<<grid, kDecThreads, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_dec_t(const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  return a.D == 64 ? launch_dec_g<T, 2>(a, grid, st) : launch_dec_g<T, 4>(a, grid, st);
}

}  // namespace

bool decode_supported(int D, int G) { return (D == 64 || D == 128) && (G == 1 || G == 2 || G == 4 || G == 8); }

cudaError_t launch_decode_attention(const DecodeArgs& a, int dtype, cudaStream_t st) {
  const dim3 grid(a.splits, a.Hkv, a.R);
  cudaError_t e = dtype == ACTKV_F32   ? launch_dec_t<float>(a, grid, st)
                  : dtype == ACTKV_F16 ? launch_dec_t<__half>(a, grid, st)
                                       : launch_dec_t<__nv_bfloat16>(a, grid, st);
  if (e != cudaSuccess) return e;
  decode_combine_kernel<<<dim3(a.Hq, a.R), 128, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace actkv
