// Epilogue and operand helpers shared by the tcgen05 scoring kernels (score_umma.cu, one CTA per
// tile; score_pair.cu, a CTA pair per tile).
#pragma once

#include "score_common.cuh"
#include "umma_common.cuh"

namespace actkv {
namespace umma {

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return uint32_t(__bfloat16_as_ushort(lo)) | (uint32_t(__bfloat16_as_ushort(hi)) << 16);
}

// Row of the query-side lse tile for a column whose term is c (= -lse/scale, 0 for padding):
// c1 + c2 + c3 reproduces c to fp32 precision.
__device__ __forceinline__ uint4 lse_split_row(float c) {
  const __nv_bfloat16 c1 = __float2bfloat16_rn(c);
  const float r1 = c - __bfloat162float(c1);
  const __nv_bfloat16 c2 = __float2bfloat16_rn(r1);
  const __nv_bfloat16 c3 = __float2bfloat16_rn(r1 - __bfloat162float(c2));
  return make_uint4(pack_bf16x2(c1, c2), pack_bf16x2(c3, __float2bfloat16_rn(0.0f)), 0u, 0u);
}

// Fold one 32-column batch of a token row.  Column g of action token j holds x_g - lse_g/scale
// (the lse step already added); for each j: sum += 2^(s2 * max_g column), s2 = scale*log2(e),
// i.e. max_g exp(x_g*scale - lse_g).  CHECK: partial batch (j >= A) or causal rows.
template <int G, bool CHECK>
__device__ __forceinline__ void fold_batch(const float (&v)[32], float s2, int jb, int A, int first_q,
                                           float& sum) {
#pragma unroll
  for (int qq = 0; qq < 32 / G; ++qq) {
    const float* c = v + qq * G;
    float m;
    if constexpr (G == 1) {
      m = c[0];
    } else if constexpr (G == 2) {
      m = fmaxf(c[0], c[1]);
    } else {
      m = fmaxf(fmax3(c[0], c[1], c[2]), c[3]);
#pragma unroll
      for (int g = 4; g < G; g += 4) m = fmax3(m, fmax3(c[g], c[g + 1], c[g + 2]), c[g + 3]);
    }
    const float p = ex2(s2 * m);
    if (CHECK) {
      const int j = jb + qq;
      if (j < A && j >= first_q) sum += p;
    } else {
      sum += p;
    }
  }
}

// ------------------------------------------------------------------------------------ schedule
struct Unit {
  int r, l, h, tile;
  int S, A, a0, T, nch;
  bool seg_first;   // first unit of its (r, l, h) segment in this CTA's range
  bool seg_last;    // last unit of its segment in this CTA's range
};

// Walks one work group's contiguous share of the flattened (r, l, h, tile) space (tile fastest),
// tiles of TILE tokens; a work group is a CTA (one-CTA kernel) or a CTA pair.  WINDOWED: of the
// layers [lw0, lw1) only (one layer group of a streamed call), else of all layers.  Every thread of
// the group builds the same one; after the initial seek it only increments counters.
template <int TILE, bool WINDOWED = false>
struct Walker {
  const ScoreArgs* a;
  int qpc;
  int lw0_, lw1_;                   // WINDOWED only
  int64_t u, u_begin, u_end;
  int r, l, h, tile;
  int S, A, a0, T, nch;

  __device__ void load_session(int rr) {
    S = a->seq_used[rr];
    a0 = a->act_off[rr];
    A = a->act_off[rr + 1] - a0;
    T = (S + TILE - 1) / TILE;
    nch = (A + qpc - 1) / qpc;
    if (a->filter && (A * a->G < a->cols_lo || A * a->G > a->cols_hi)) T = 0;   // another launch's
  }
  __device__ int64_t weight() const { return 1 + nch; }
  __device__ int lw0() const {
    if constexpr (WINDOWED) return lw0_;
    else return 0;
  }
  __device__ int lw1() const {
    if constexpr (WINDOWED) return lw1_;
    else return a->L;
  }
  __device__ int64_t units() const { return int64_t(lw1() - lw0()) * a->Hkv * T; }

  __device__ int64_t first_unit(int64_t x) {
    int64_t U = 0, C = 0;
    for (int rr = 0; rr < a->R; ++rr) {
      load_session(rr);
      const int64_t n = units(), c = n * weight();
      if (x < C + c) return U + (x - C + weight() - 1) / weight();
      U += n;
      C += c;
    }
    return U;
  }

  __device__ void init(const ScoreArgs* args, int qpc_, int group, int n_groups) {
    init(args, qpc_, group, n_groups, 0, args->L);
  }
  __device__ void init(const ScoreArgs* args, int qpc_, int group, int n_groups, int l_begin, int l_end) {
    a = args;
    qpc = qpc_;
    lw0_ = l_begin;
    lw1_ = l_end;
    int64_t W = 0;
    for (int rr = 0; rr < a->R; ++rr) {
      load_session(rr);
      W += units() * weight();
    }
    const int64_t lo = W * group / n_groups, hi = W * (group + 1) / n_groups;
    u = u_begin = first_unit(lo);
    u_end = first_unit(hi);
    // seek (r, l, h, tile) of unit u: the only divisions of the walk
    int64_t U = 0;
    r = 0;
    load_session(0);
    while (r + 1 < a->R && u >= U + units()) {
      U += units();
      ++r;
      load_session(r);
    }
    const int64_t local = u - U;
    tile = T ? int(local % T) : 0;
    const int64_t lh = T ? local / T : 0;
    h = int(lh % a->Hkv);
    l = lw0() + int(lh / a->Hkv);
  }

  __device__ bool next(Unit& x) {
    if (u >= u_end) return false;
    while (T == 0) {                  // sessions without tokens have no units
      ++r;
      load_session(r);
      tile = h = 0;
      l = lw0();
    }
    x.r = r;
    x.l = l;
    x.h = h;
    x.tile = tile;
    x.S = S;
    x.A = A;
    x.a0 = a0;
    x.T = T;
    x.nch = nch;
    x.seg_first = tile == 0 || u == u_begin;
    x.seg_last = tile == T - 1 || u + 1 == u_end;
    ++u;
    if (++tile == T) {
      tile = 0;
      if (++h == a->Hkv) {
        h = 0;
        if (++l == lw1()) {
          l = lw0();
          if (u < u_end) {
            ++r;
            load_session(r);
          }
        }
      }
    }
    return true;
  }
};

}  // namespace umma
}  // namespace actkv
