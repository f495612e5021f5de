// Paged decode attention with its log-sum-exp (flash decoding), on CUDA cores (fp32 caches, head_dim
// 64; bf16 / fp16 caches with head_dim 128 take the tensor-core kernel of decode_tc.cu): the GPU form of the
// reference's paged_decode_attention_ref (actkv/kernels/lse_attn.py:42-60), one query per session:
//   out[r, hq, :] = softmax_t(scale * q[r, hq] . k[t, h]) @ v[t, h],  lse[r, hq] = logsumexp_t(...)
// over t < seq_used[r], h = hq / G.
//
// One query token per session makes this HBM-bound (each K/V row is read once and used by the G
// query heads of its KV head), so it runs on CUDA cores: a CTA takes one (session, KV head, token
// split); each warp walks a contiguous run of its split's tokens with lane i holding dims
// [i*DPL, i*DPL + DPL) of q and of the G output accumulators.  The warps merge in shared memory,
// the splits in decode_combine_kernel.
//
// What bounds it is the bytes each SM keeps in flight (Little's law), so the K / V rows do not go
// through registers: every warp owns a ring of kStages stages in shared memory (kU tokens' K and V
// rows each, kWarpRing bytes in all) filled by 16-byte cp.async copies, one commit group per
// stage; it waits for the oldest stage, folds its tokens, and refills the slot with the stage
// kStages ahead.  A stage's kU * G partial logits are reduced together (each butterfly step halves
// the values a lane carries, then one shuffle per value broadcasts the sums); then the online
// softmax (running max m, sum l, rescaled accumulator) in log2 units.
#include "common.cuh"
#include "kernels.cuh"

namespace actkv {

namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kWarpRing = 8192;                   // bytes of K / V ring per warp
constexpr int kMaxStages = 16, kMaxU = 4;
constexpr int kMetaBytes = kDecWarps * kMaxStages * kMaxU * 4;   // each ring slot's paged block ids
constexpr int kDecSmem = kDecWarps * kWarpRing + kMetaBytes;
// tokens per ring stage: their kU * G logits are reduced together
constexpr int dec_tokens_per_stage(int G) { return G >= 4 ? 2 : 4; }

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// DPL consecutive elements of shared memory as one load, converted to fp32.
template <typename T, int DPL> struct RowVec;
template <> struct RowVec<float, 4> { using V = float4; };
template <> struct RowVec<float, 2> { using V = float2; };
template <> struct RowVec<__nv_bfloat16, 4> { using V = uint2; };
template <> struct RowVec<__nv_bfloat16, 2> { using V = uint32_t; };
template <> struct RowVec<__half, 4> { using V = uint2; };
template <> struct RowVec<__half, 2> { using V = uint32_t; };

template <typename T, int DPL>
__device__ __forceinline__ void load_row(const uint8_t* p, float (&x)[DPL]) {
  using V = typename RowVec<T, DPL>::V;
  static_assert(sizeof(V) == DPL * sizeof(T), "one vector per lane");
  const V v = *reinterpret_cast<const V*>(p);
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < DPL; ++i) x[i] = to_f32(e[i]);
}

// d = a * b + c on two fp32 lanes at once (Blackwell's paired FMA: half the issue slots of two
// fmaf, each lane rounded as fmaf rounds it).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

constexpr int ilog2(int n) { return n <= 1 ? 0 : 1 + ilog2(n / 2); }

// x[i] holds lane partials of N sums; on return x[i] is sum i on every lane.  Butterfly steps
// with offsets 16, 8, ... each hand half of the remaining values to the partner lane, so after
// log2 N steps a lane carries one value (that of sum lane >> (5 - log2 N)); the remaining
// offsets finish its sum and a shuffle per value broadcasts the N results.
template <int N>
__device__ __forceinline__ void warp_sums(float (&x)[N]) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "a power of two up to 32");
  constexpr unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  int o = 16;
#pragma unroll
  for (int n = N; n > 1; n >>= 1, o >>= 1) {
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
  constexpr int shift = 5 - ilog2(N);
#pragma unroll
  for (int i = 0; i < N; ++i) x[i] = __shfl_sync(full, v, (i << shift) & 31);
}

template <typename T, int G, int DPL>
__global__ void __launch_bounds__(kDecThreads, decode_ctas_per_sm(G)) decode_attn_kernel(DecodeArgs a) {
  constexpr int kU = dec_tokens_per_stage(G);
  constexpr int D = 32 * DPL;
  constexpr int RB = D * int(sizeof(T));           // bytes of one K or V row
  constexpr int kStageBytes = 2 * RB * kU;         // [u][K, V][RB]
  constexpr int kStages = kWarpRing / kStageBytes;
  constexpr int kChunks = kStageBytes / 16;        // 16-byte copies per stage
  constexpr int kRowChunks = RB / 16;
  static_assert(kStages >= 2 && kStages <= kMaxStages && kWarpRing % kStageBytes == 0, "ring of whole stages");
  static_assert(kChunks % 32 == 0 && kU <= kMaxU && kU % 2 == 0 && DPL % 2 == 0, "whole warps of copies, pairs");
  static_assert(kDecWarps * (2 * G + G * D) * 4 <= kDecWarps * kWarpRing, "the warp merge reuses the ring");
  extern __shared__ __align__(128) uint8_t dsmem[];
  const int sp = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
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
  float m[G], l[G];
  float2 acc[G][DPL / 2];                          // dims (2i, 2i + 1) of the lane's slice
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) acc[g][i] = make_float2(0.0f, 0.0f);
  }
  const uint8_t* kv = static_cast<const uint8_t*>(a.kv);
  uint8_t* ring = dsmem + warp * kWarpRing;
  int* meta = reinterpret_cast<int*>(dsmem + kDecWarps * kWarpRing) + warp * kMaxStages * kMaxU;
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
  // Copies of the kU tokens from tb into ring slot `slot`.  Lane u < kU resolves token tb + u
  // (its paged block: -1 past the run or for an id outside the pool; its row in the block) for
  // the other lanes and records the block id for the fold.
  auto issue = [&](int slot, int tb) {
    int blk = -1, row = 0;
    if (lane < kU) {
      const int t = tb + lane;
      if (t < t1) {
        const int lb = t / a.BS;
        row = t - lb * a.BS;
        blk = lb < a.MB ? a.block_table[r * a.bt_stride_r + lb] : -1;
        if (blk < 0 || blk >= a.NB) {
          blk = -1;
          flag(a.status, ACTKV_DEV_BAD_INDEX);
        }
      }
      meta[slot * kU + lane] = blk;
    }
#pragma unroll
    for (int j = 0; j < kChunks / 32; ++j) {
      const int c = lane + 32 * j;
      const int u = c / (2 * kRowChunks), rem = c % (2 * kRowChunks);
      const int half = rem / kRowChunks, off = (rem % kRowChunks) * 16;
      const int bu = __shfl_sync(full, blk, u), ru = __shfl_sync(full, row, u);
      if (bu >= 0) {
        const int64_t e = (half ? a.kv_stride_kv : 0) + int64_t(bu) * a.kv_stride_b + int64_t(ru) * a.kv_stride_s +
                          int64_t(h) * a.kv_stride_h;
        cp_async16(ring_s + slot * kStageBytes + (u * 2 + half) * RB + off, kv + e * int64_t(sizeof(T)) + off);
      }
    }
  };
  const int nst = (t1 - t0 + kU - 1) / kU;         // stages this warp folds
#pragma unroll
  for (int st = 0; st < kStages; ++st) {
    if (st < nst) issue(st, t0 + st * kU);
    cp_async_commit();
  }
  for (int st = 0; st < nst; ++st) {
    const int slot = st % kStages;
    cp_async_wait<kStages - 1>();                  // this lane's copies of stage st have landed
    __syncwarp();                                  // ... and every other lane's, and the block ids
    const uint8_t* sb = ring + slot * kStageBytes;
    bool use[kU];
    float x[kU * G], k[kU][DPL], v[kU][DPL];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      use[u] = meta[slot * kU + u] >= 0;
      if (use[u]) {
        load_row<T, DPL>(sb + (u * 2) * RB + lane * DPL * int(sizeof(T)), k[u]);
        load_row<T, DPL>(sb + (u * 2 + 1) * RB + lane * DPL * int(sizeof(T)), v[u]);
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) k[u][i] = v[u][i] = 0.0f;
      }
    }
    // partial logits of tokens u and u + 1 together, each summed over i in order
#pragma unroll
    for (int u = 0; u < kU; u += 2)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float2 d = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < DPL; ++i) d = ffma2(make_float2(q[g][i], q[g][i]), make_float2(k[u][i], k[u + 1][i]), d);
        x[u * G + g] = d.x;
        x[(u + 1) * G + g] = d.y;
      }
    __syncwarp();                                  // the slot is read: refill it
    if (st + kStages < nst) issue(slot, t0 + (st + kStages) * kU);
    cp_async_commit();
    warp_sums<kU * G>(x);                          // the logits, in log2 units, on every lane
    // online softmax over the stage's tokens at once: one rescale of the running sums per stage
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mn = m[g];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (use[u]) mn = fmaxf(mn, x[u * G + g]);
      if (mn == -INFINITY) continue;               // no token of the stage is in the pool
      const float corr = ex2f(m[g] - mn);          // 0 while m is still -inf
      float p[kU], ls = 0.0f;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        p[u] = use[u] ? ex2f(x[u * G + g] - mn) : 0.0f;
        ls += p[u];
      }
      l[g] = fmaf(l[g], corr, ls);
#pragma unroll
      for (int i = 0; i < DPL / 2; ++i) {
        float2 y = ffma2(acc[g][i], make_float2(corr, corr), make_float2(0.0f, 0.0f));
#pragma unroll
        for (int u = 0; u < kU; ++u) y = ffma2(make_float2(p[u], p[u]), make_float2(v[u][2 * i], v[u][2 * i + 1]), y);
        acc[g][i] = y;
      }
      m[g] = mn;
    }
  }
  cp_async_wait_all();
  __syncthreads();                                 // every ring is drained: reuse it for the merge
  float* s_m = reinterpret_cast<float*>(dsmem);                 // [kDecWarps][G]
  float* s_l = s_m + kDecWarps * G;                             // [kDecWarps][G]
  float* s_acc = s_l + kDecWarps * G;                           // [kDecWarps][G][D]
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      s_m[warp * G + g] = m[g];
      s_l[warp * G + g] = l[g];
    }
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) {
      s_acc[(warp * G + g) * D + lane * DPL + 2 * i] = acc[g][i].x;
      s_acc[(warp * G + g) * D + lane * DPL + 2 * i + 1] = acc[g][i].y;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += kDecThreads) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, s_m[w * G + g]);
    float L = 0.0f, A = 0.0f;
    if (M != -INFINITY)
      for (int w = 0; w < kDecWarps; ++w) {
        if (s_m[w * G + g] == -INFINITY) continue;
        const float f = ex2f(s_m[w * G + g] - M);
        L = fmaf(s_l[w * G + g], f, L);
        A = fmaf(s_acc[(w * G + g) * D + d], f, A);
      }
    const int64_t pi = (int64_t(r) * a.Hq + h * G + g) * a.splits + sp;
    a.part_acc[pi * D + d] = A;
    if (d == 0) {
      a.part_m[pi] = M;
      a.part_l[pi] = L;
    }
  }
}

// One CTA per (session, query head): the splits' weights 2^(m_s - M) once into shared memory,
// then thread d sums its dimension over the splits with independent loads.
constexpr int kCombineThreads = 128;
static_assert(kCombineThreads >= kDecodeMaxSplits, "a thread per split");

__global__ void __launch_bounds__(kCombineThreads) decode_combine_kernel(DecodeArgs a) {
  __shared__ float w[kCombineThreads], red[32];
  const int r = blockIdx.y, hq = blockIdx.x;
  const int64_t base = (int64_t(r) * a.Hq + hq) * a.splits;
  const int ns = a.splits;                          // <= kCombineThreads (decode_splits)
  const float ms = threadIdx.x < ns ? a.part_m[base + threadIdx.x] : -INFINITY;
  const float ls = threadIdx.x < ns ? a.part_l[base + threadIdx.x] : 0.0f;
  const float M = block_max(ms, red);
  const float ws = M != -INFINITY && ms != -INFINITY ? ex2f(ms - M) : 0.0f;
  w[threadIdx.x] = ws;
  const float L = block_sum(ws * ls, red);          // block_sum's barriers also publish w
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
  for (int d = threadIdx.x; d < a.D; d += kCombineThreads) {
    const float* pa = a.part_acc + base * a.D + d;
    float A0 = 0.0f, A1 = 0.0f, A2 = 0.0f, A3 = 0.0f;
    int s = 0;
    for (; s + 4 <= ns; s += 4) {
      A0 = fmaf(pa[int64_t(s) * a.D], w[s], A0);
      A1 = fmaf(pa[int64_t(s + 1) * a.D], w[s + 1], A1);
      A2 = fmaf(pa[int64_t(s + 2) * a.D], w[s + 2], A2);
      A3 = fmaf(pa[int64_t(s + 3) * a.D], w[s + 3], A3);
    }
    for (; s < ns; ++s) A0 = fmaf(pa[int64_t(s) * a.D], w[s], A0);
    a.out[r * a.out_stride_r + hq * a.out_stride_h + d] = ((A0 + A1) + (A2 + A3)) * inv;
  }
  if (threadIdx.x == 0)
    a.lse[r * a.lse_stride_r + hq] = L > 0.0f ? (M + log2f(L)) * 0.69314718055994531f : -INFINITY;
}

template <typename T, int G, int DPL>
cudaError_t launch_dec(const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  auto k = decode_attn_kernel<T, G, DPL>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmem);
  if (e != cudaSuccess) return e;
  k<<<grid, kDecThreads, kDecSmem, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int DPL>
cudaError_t launch_dec_g(const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  switch (a.G) {
    case 1: return launch_dec<T, 1, DPL>(a, grid, st);
    case 2: return launch_dec<T, 2, DPL>(a, grid, st);
    case 4: return launch_dec<T, 4, DPL>(a, grid, st);
    default: return launch_dec<T, 8, DPL>(a, grid, st);
  }
}

template <typename T>
cudaError_t launch_dec_t(const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  return a.D == 64 ? launch_dec_g<T, 2>(a, grid, st) : launch_dec_g<T, 4>(a, grid, st);
}

}  // namespace

bool decode_supported(int D, int G) { return (D == 64 || D == 128) && (G == 1 || G == 2 || G == 4 || G == 8); }

cudaError_t launch_decode_attention(const DecodeArgs& a, int dtype, cudaStream_t st) {
  const dim3 grid(a.splits, a.Hkv, a.R);
  cudaError_t e;
  if (decode_tc_supported(a, dtype)) {
    e = launch_decode_tc(a, dtype, st, nullptr);
  } else {
    e = dtype == ACTKV_F32   ? launch_dec_t<float>(a, grid, st)
        : dtype == ACTKV_F16 ? launch_dec_t<__half>(a, grid, st)
                             : launch_dec_t<__nv_bfloat16>(a, grid, st);
  }
  if (e != cudaSuccess) return e;
  decode_combine_kernel<<<dim3(a.Hq, a.R), kCombineThreads, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace actkv
