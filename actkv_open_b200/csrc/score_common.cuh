// Arguments and the final fold shared by the two scoring kernels.
#pragma once
#include "common.cuh"

namespace actkv {

constexpr int kMaxLayerGroups = 16;

struct ScoreArgs {
  const void* q;
  int64_t q_stride_l, q_stride_a, q_stride_h;
  const float* lse;
  int64_t lse_stride_l, lse_stride_a;
  const int32_t* act_off;        // [R+1] or nullptr: session r has one query, row r
  const void* kv;
  int64_t kv_stride_l, kv_stride_kv, kv_stride_b, kv_stride_s, kv_stride_h;
  const int32_t* block_table;
  int64_t bt_stride_r;
  const int32_t* seq_used;
  float* out;
  const int64_t* out_off;
  int64_t out_stride_r, out_stride_l, out_stride_h;
  const int32_t* n_seen;         // nullptr: fresh mean
  int R, L, MB, NB, BS, Hq, Hkv, G, D;
  int qrows;                     // SIMT: query rows per shared-memory chunk
  float scale;
  int32_t* status;
  // tensor-core walkers: with `filter`, only sessions with cols_lo <= A*G <= cols_hi are scored by
  // this launch (the host launches each width class on its own shared-memory layout)
  int filter, cols_lo, cols_hi;
  // queries streamed in by layer groups (CTA-pair kernel only): group g is layers
  // [lgrp[g], lgrp[g + 1]), and its queries may be read once *ready - ready_base >= g + 1 (modulo
  // 2^32).  Every work group takes its share of group 0, then of group 1, ...  n_lgroups == 0:
  // one group of all layers, nothing to wait for.
  const uint32_t* ready;
  uint32_t ready_base;
  int n_lgroups;
  int lgrp[kMaxLayerGroups + 1];
};

// Fold the sum over the action tokens that saw this token into the stored score.
//   fresh (n0 < 0):  sum / A                       (A sequential reference calls from zero)
//   A == 1:          out + (p - out) / (n0 + 1)    (lse_attn.py:78, same operation order)
//   otherwise:       ((n0 + m) * out + sum) / (n0 + A), m = first action token that sees t
__device__ __forceinline__ float finalize_score(float sum, int A, int first_q, const float* o, int n0) {
  if (n0 < 0) return A > 0 ? __fdiv_rn(sum, float(A)) : 0.0f;
  const float out0 = *o;
  if (A == 0) return out0;
  if (A == 1) return __fadd_rn(out0, __fdiv_rn(__fsub_rn(sum, out0), __fadd_rn(float(n0), 1.0f)));
  const int m = first_q > 0 ? first_q : 0;
  return __fdiv_rn(__fadd_rn(__fmul_rn(float(n0 + m), out0), sum), float(n0 + A));
}

cudaError_t launch_score_simt(const ScoreArgs& a, int kv_dtype, int q_dtype, int max_W, int max_A,
                              cudaStream_t st);

}  // namespace actkv
