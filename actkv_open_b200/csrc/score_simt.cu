// LSE-recovery scoring on CUDA cores (any cache/query dtype, head_dim <= 256, any GQA group).
//
// Computes, for session r, layer l, KV head h and token t < seq_used[r] (Algorithm 3,
// actkv/kernels/lse_attn.py:63-78 / :85-130):
//   p_j(t) = max_{g<G} exp(scale * <q_j[h*G+g], k_t[h]> - lse_j[h*G+g])
// summed over the action tokens j that see t (causal region: t <= seq_used - A + j), then folded
// into `out` as a fresh mean, a running-mean continuation, or (A = 1) the reference's exact
// running-mean update out += (p - out) / (n + 1).
//
// One CTA per (token chunk, KV head, session*layer).  The K chunk of the head is gathered through
// the block table into shared memory as fp32 once; query rows stream through shared memory in
// chunks; each thread owns one token and a residue class of the queries (QL lanes per token),
// and the QL partial sums are combined with shuffles.  This path also serves as the check for the
// tcgen05 path on shapes where both run.
#include "common.cuh"
#include "score_common.cuh"

namespace actkv {

template <typename KT, typename QT, int QL>
__global__ void __launch_bounds__(QL == 1 ? 128 : 256) score_simt_kernel(ScoreArgs a) {
  constexpr int NT = QL == 1 ? 128 : 256;
  constexpr int TOK = NT / QL;
  extern __shared__ float smem[];
  const int D = a.D, G = a.G, DP = a.D + 1;
  float* ks = smem;                         // [TOK][DP]
  float* qs = ks + TOK * DP;                // [QROWS][DP]
  float* ls = qs + a.qrows * DP;            // [QROWS]
  const int h = blockIdx.y;
  const int r = blockIdx.z / a.L, l = blockIdx.z % a.L;
  const int S = a.seq_used[r];
  const int t0 = blockIdx.x * TOK;
  if (t0 >= S) return;
  const int a0 = a.act_off ? a.act_off[r] : r;
  const int A = a.act_off ? a.act_off[r + 1] - a0 : 1;

  // gather the K chunk [TOK][D] of head h through the block table
  const KT* kvl = static_cast<const KT*>(a.kv) + l * a.kv_stride_l;
  const int32_t* bt = a.block_table + r * a.bt_stride_r;
  for (int idx = threadIdx.x; idx < TOK * D; idx += NT) {
    const int tl = idx / D, d = idx - tl * D;
    const int t = t0 + tl;
    float v = 0.0f;
    if (t < S) {
      const int blk = t / a.BS;
      int phys = blk < a.MB ? bt[blk] : -1;
      if (phys < 0 || phys >= a.NB) {
        flag(a.status, ACTKV_DEV_BAD_INDEX);
      } else {
        v = to_f32(kvl[phys * a.kv_stride_b + (t - blk * a.BS) * a.kv_stride_s + h * a.kv_stride_h + d]);
      }
    }
    ks[tl * DP + d] = v;
  }

  const int tl = threadIdx.x / QL, ql = threadIdx.x % QL;
  const int t = t0 + tl;
  const int first_q = t - (S - A);          // first action token that sees t (<= 0: all)
  const QT* qb = static_cast<const QT*>(a.q) + l * a.q_stride_l;
  const float* lb = a.lse + l * a.lse_stride_l;
  const int qc = a.qrows / G;               // queries per chunk
  float sum = 0.0f;
  for (int c0 = 0; c0 < A; c0 += qc) {
    __syncthreads();
    const int nq = min(qc, A - c0);
    for (int idx = threadIdx.x; idx < nq * G * D; idx += NT) {
      const int row = idx / D, d = idx - row * D;
      const int j = row / G, g = row - j * G;
      qs[row * DP + d] = to_f32(qb[(a0 + c0 + j) * a.q_stride_a + (h * G + g) * a.q_stride_h + d]);
    }
    for (int row = threadIdx.x; row < nq * G; row += NT) {
      const int j = row / G, g = row - j * G;
      ls[row] = lb[(a0 + c0 + j) * a.lse_stride_a + h * G + g];
    }
    __syncthreads();
    if (t < S) {
      const float* kr = ks + tl * DP;
      for (int j = ql; j < nq; j += QL) {
        if (c0 + j < first_q) continue;     // causal: token j does not see t yet
        float best = -INFINITY;
        for (int g = 0; g < G; ++g) {
          const float* qr = qs + (j * G + g) * DP;
          float dot = 0.0f;
          for (int d = 0; d < D; ++d) dot = fmaf(kr[d], qr[d], dot);
          const float p = expf(__fsub_rn(__fmul_rn(dot, a.scale), ls[j * G + g]));
          best = fmaxf(best, p);
        }
        sum += best;
      }
    }
  }
#pragma unroll
  for (int o = 1; o < QL; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (ql == 0 && t < S) {
    float* o = a.out + (a.out_off ? a.out_off[r] : r * a.out_stride_r) + l * a.out_stride_l +
               h * a.out_stride_h + t;
    *o = finalize_score(sum, A, first_q, o, a.n_seen ? a.n_seen[r] : -1);
  }
}

template <typename KT, typename QT>
cudaError_t launch_simt_typed(const ScoreArgs& a, int max_W, int max_A, cudaStream_t st) {
  const bool narrow = max_A <= 2;
  const int tok = narrow ? 128 : 64;
  dim3 grid((max_W + tok - 1) / tok, a.Hkv, a.R * a.L);
  const size_t sm = size_t(tok * (a.D + 1) + a.qrows * (a.D + 1) + a.qrows) * sizeof(float);
  if (narrow) {
    auto k = score_simt_kernel<KT, QT, 1>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    if (e != cudaSuccess) return e;
    k<<<grid, 128, sm, st>>>(a);
  } else {
    auto k = score_simt_kernel<KT, QT, 4>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    if (e != cudaSuccess) return e;
    k<<<grid, 256, sm, st>>>(a);
  }
  return cudaGetLastError();
}

template <typename KT>
cudaError_t launch_simt_q(const ScoreArgs& a, int q_dtype, int max_W, int max_A, cudaStream_t st) {
  switch (q_dtype) {
    case ACTKV_F32: return launch_simt_typed<KT, float>(a, max_W, max_A, st);
    case ACTKV_F16: return launch_simt_typed<KT, __half>(a, max_W, max_A, st);
    default: return launch_simt_typed<KT, __nv_bfloat16>(a, max_W, max_A, st);
  }
}

cudaError_t launch_score_simt(const ScoreArgs& a, int kv_dtype, int q_dtype, int max_W, int max_A,
                              cudaStream_t st) {
  switch (kv_dtype) {
    case ACTKV_F32: return launch_simt_q<float>(a, q_dtype, max_W, max_A, st);
    case ACTKV_F16: return launch_simt_q<__half>(a, q_dtype, max_W, max_A, st);
    default: return launch_simt_q<__nv_bfloat16>(a, q_dtype, max_W, max_A, st);
  }
}

}  // namespace actkv
