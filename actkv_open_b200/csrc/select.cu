// Keep-score update (ActionLRFU, actkv/eviction.py:198-210 with top_p_mask :36-50) and keep-mask
// selection (actkv/paged.py:23-46), one CTA per (session, layer) / per session.
//
// Both selections are radix selects over the 32-bit key of each float, 8 bits per pass, with
// per-warp shared-memory histograms (no global atomics, no sort):
//   keep mask : count-weighted  -> the budget-th largest candidate score (top-k threshold)
//   nucleus   : mass-weighted   -> the entry at which the descending cumulative mass first
//                                  reaches top_p * total (the crossing entry)
// Masses are accumulated as 64-bit fixed point, so histogram sums do not depend on the order in
// which threads add them: the result is the same on every run.  Ties at a threshold go to the
// lowest token index (a block-wide ballot scan counts the equal entries in index order).
#include "kernels.cuh"

namespace actkv {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kBins = 256;

// Finds, from the highest bin down, the bin where the running sum of `w` first reaches `need`.
// Executed by warp 0; lane i owns bins [8i, 8i + 8).  Returns via shared out[0] = bin (or -1 when
// the total never reaches need), out_above = sum of w over bins above it.
template <typename W>
__device__ void find_crossing_bin(const W* w, W need, int* out_bin, W* out_above) {
  const int lane = threadIdx.x & 31;
  W mine = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) mine += w[lane * 8 + k];
  // suffix sum over lanes above this one
  W incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    W y = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += y;
  }
  W above = incl - mine;           // bins owned by higher lanes
  if (lane == 0) *out_bin = -1;
  __syncwarp();
  if (above < need && need <= incl) {
    W acc = above;
    for (int k = 7; k >= 0; --k) {
      const W v = w[lane * 8 + k];
      if (acc + v >= need && v > 0) {
        *out_bin = lane * 8 + k;
        *out_above = acc;
        break;
      }
      acc += v;
    }
  }
  __syncwarp();
}

// ----------------------------------------------------------------------------------- keep mask
__global__ void __launch_bounds__(kSelThreads) keep_mask_kernel(KeepMaskArgs a) {
  __shared__ uint32_t hist[kSelWarps][kBins];
  __shared__ uint32_t tot[kBins];
  __shared__ int red[33];
  __shared__ int sel_bin;
  __shared__ uint32_t sel_above;
  const int r = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int n = a.seq_used[r];
  const float* sc = a.scores + (a.scores_off ? a.scores_off[r] : r * a.stride_r);
  const uint8_t* pin = a.pinned ? a.pinned + r * a.pinned_stride_r : nullptr;
  uint8_t* keep = a.keep + r * a.keep_stride_r;
  float* s = a.s_ws + r * a.max_seq;
  if (n > a.max_seq) {
    if (threadIdx.x == 0) {
      flag(a.status, ACTKV_DEV_BAD_INDEX);
      if (a.kept) a.kept[r] = 0;
    }
    return;
  }
  auto is_prot = [&](int t) { return t < a.protected_prefix || (pin && pin[t]); };

  // pass 1: reduce heads (dim -2) then average the leading rows; count protected tokens
  int n_prot = 0;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    float acc = 0.0f;
    for (int l = 0; l < a.n_lead; ++l) {
      const float* row = sc + l * a.stride_l + t;
      float v;
      if (a.reduce == ACTKV_REDUCE_MAX) {
        v = row[0];
        for (int x = 1; x < a.n_red; ++x) v = fmaxf(v, row[x * a.stride_x]);
      } else {
        v = row[0];
        for (int x = 1; x < a.n_red; ++x) v += row[x * a.stride_x];
        v = __fdiv_rn(v, float(a.n_red));
      }
      acc += v;
    }
    s[t] = __fdiv_rn(acc, float(a.n_lead));
    n_prot += is_prot(t);
  }
  n_prot = block_sum(n_prot, red);
  const int n_cand = n - n_prot;
  const int budget = a.budget[r];
  const bool keep_all = (a.evict_semantics && n_cand <= budget) || budget >= n_cand;
  const int k = budget < n_cand ? (budget > 0 ? budget : 0) : n_cand;
  if (keep_all || k == 0) {
    for (int t = threadIdx.x; t < n; t += blockDim.x) keep[t] = keep_all ? 1 : is_prot(t);
    if (threadIdx.x == 0 && a.kept) a.kept[r] = keep_all ? n : n_prot;
    return;
  }
  // radix select of the k-th largest candidate key
  uint32_t prefix = 0, pmask = 0;
  uint32_t need = uint32_t(k);
  uint32_t eq_count = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < kSelWarps * kBins; i += blockDim.x) (&hist[0][0])[i] = 0;
    __syncthreads();
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
      if (is_prot(t)) continue;
      const uint32_t u = order_key(s[t]);
      if ((u & pmask) == prefix) atomicAdd(&hist[warp][(u >> shift) & 0xff], 1u);
    }
    __syncthreads();
    if (threadIdx.x < kBins) {
      uint32_t c = 0;
      for (int w = 0; w < kSelWarps; ++w) c += hist[w][threadIdx.x];
      tot[threadIdx.x] = c;
    }
    __syncthreads();
    if (warp == 0) find_crossing_bin<uint32_t>(tot, need, &sel_bin, &sel_above);
    __syncthreads();
    const int b = sel_bin;
    if (b < 0) {                                      // cannot happen: k <= #candidates
      if (threadIdx.x == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      return;
    }
    need -= sel_above;
    eq_count = tot[b];
    prefix |= uint32_t(b) << shift;
    pmask |= 0xffu << shift;
    __syncthreads();
  }
  // final pass: protected, above the threshold, or among the first `need` equal ones by index
  const bool ties = eq_count > need;
  int eq_seen = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int t = base + threadIdx.x;
    const bool in = t < n;
    const bool prot = in && is_prot(t);
    const uint32_t u = in && !prot ? order_key(s[t]) : 0u;
    const bool cand = in && !prot;
    const bool eq = cand && u == prefix;
    bool take = prot || (cand && u > prefix);
    if (ties) {
      int tot_eq;
      const int rank = block_excl_count(eq, red, &tot_eq) + eq_seen;
      take = take || (eq && uint32_t(rank) < need);
      eq_seen += tot_eq;
    } else {
      take = take || eq;
    }
    if (in) keep[t] = take;
  }
  if (threadIdx.x == 0 && a.kept) a.kept[r] = n_prot + k;
}

// ----------------------------------------------------------------------------------- ActionLRFU
struct LrfuSmem {
  uint32_t hc[kSelWarps][kBins];
  unsigned long long hm[kSelWarps][kBins];
  unsigned long long tm[kBins];
  uint32_t tc[kBins];
  double dred[32];
  float fred[32];
  int ired[33];
  int sel_bin;
  unsigned long long sel_above;
};

// grid (L, R)
__global__ void __launch_bounds__(kSelThreads) lrfu_kernel(LrfuArgs a) {
  extern __shared__ __align__(16) unsigned char lrfu_smem_raw[];
  LrfuSmem& sm = *reinterpret_cast<LrfuSmem*>(lrfu_smem_raw);
  const int l = blockIdx.x, r = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int n = a.seq_used[r];
  const float* src = a.src + (a.src_off ? a.src_off[r] : r * a.src_stride_r) + l * a.src_stride_l;
  float* ks = a.ks + r * a.ks_stride_r + l * a.ks_stride_l;
  float* act = a.act + r * a.act_stride_r + l * a.act_stride_l;
  const uint8_t* pin = a.pinned ? a.pinned + r * a.pinned_stride_r : nullptr;
  auto excluded = [&](int t) { return t < a.protected_prefix || (pin && pin[t]); };

  // pass 1: head reduction -> act, total mass, largest entry, number of positive entries
  double total = 0.0;
  float vmax = 0.0f;
  int n_pos = 0;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    float v = src[t];
    if (a.reduce == ACTKV_REDUCE_MAX) {
      for (int h = 1; h < a.H; ++h) v = fmaxf(v, src[h * a.src_stride_h + t]);
    } else {
      for (int h = 1; h < a.H; ++h) v += src[h * a.src_stride_h + t];
      v = __fdiv_rn(v, float(a.H));
    }
    act[t] = v;
    if (!excluded(t)) {
      total += v;
      if (v > 0.0f) {
        vmax = fmaxf(vmax, v);
        ++n_pos;
      }
    }
  }
  __syncthreads();
  total = block_sum(total, sm.dred);
  vmax = block_max(vmax, sm.fred);
  n_pos = block_sum(n_pos, sm.ired);
  const float total_f = float(total);
  const bool any_hit = (a.n_act == nullptr || a.n_act[r] > 0) && total_f > 0.0f && n_pos > 0;

  bool hit_all = false;
  uint32_t tau = 0;                 // bit pattern of the crossing value
  unsigned long long take_eq = 0;   // how many entries equal to tau are hits
  unsigned long long eq_count = 0;
  double fx = 0.0;
  if (any_hit) {
    // fixed point: n_pos * vmax * 2^e < 2^62
    int e2;
    frexp(double(vmax) * double(n_pos), &e2);
    fx = ldexp(1.0, 62 - e2);
    const float target_f = __fmul_rn(a.top_p, total_f);
    unsigned long long need = (unsigned long long)ceil(double(target_f) * fx);
    if (need == 0) need = 1;
    uint32_t prefix = 0, pmask = 0;
    for (int pass = 0; pass < 4 && !hit_all; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = threadIdx.x; i < kSelWarps * kBins; i += blockDim.x) {
        (&sm.hc[0][0])[i] = 0;
        (&sm.hm[0][0])[i] = 0;
      }
      __syncthreads();
      for (int t = threadIdx.x; t < n; t += blockDim.x) {
        if (excluded(t)) continue;
        const float v = act[t];
        if (!(v > 0.0f)) continue;
        const uint32_t u = __float_as_uint(v);
        if ((u & pmask) != prefix) continue;
        const int b = (u >> shift) & 0xff;
        atomicAdd(&sm.hc[warp][b], 1u);
        atomicAdd(&sm.hm[warp][b], (unsigned long long)(double(v) * fx));
      }
      __syncthreads();
      if (threadIdx.x < kBins) {
        uint32_t c = 0;
        unsigned long long m = 0;
        for (int w = 0; w < kSelWarps; ++w) {
          c += sm.hc[w][threadIdx.x];
          m += sm.hm[w][threadIdx.x];
        }
        sm.tc[threadIdx.x] = c;
        sm.tm[threadIdx.x] = m;
      }
      __syncthreads();
      if (warp == 0) find_crossing_bin<unsigned long long>(sm.tm, need, &sm.sel_bin, &sm.sel_above);
      __syncthreads();
      const int b = sm.sel_bin;
      if (b < 0) {
        hit_all = pass == 0;        // the mass never reaches the target: every positive entry
        if (pass > 0 && threadIdx.x == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      } else {
        need -= sm.sel_above;
        eq_count = sm.tc[b];
        prefix |= uint32_t(b) << shift;
        pmask |= 0xffu << shift;
      }
      __syncthreads();
    }
    tau = prefix;
    if (!hit_all) {
      const unsigned long long unit = (unsigned long long)(double(__uint_as_float(tau)) * fx);
      take_eq = unit ? (need + unit - 1) / unit : eq_count;
      if (take_eq < 1) take_eq = 1;
      if (take_eq > eq_count) take_eq = eq_count;
    }
  }
  // final pass: ks = fl(decay*ks) (+ a for hits); protected tokens untouched
  const bool ties = any_hit && !hit_all && eq_count > take_eq;
  int eq_seen = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int t = base + threadIdx.x;
    const bool in = t < n;
    const bool ex = in && excluded(t);
    const float v = in ? act[t] : 0.0f;
    const bool pos = in && !ex && v > 0.0f;
    const uint32_t u = __float_as_uint(v);
    bool hit = false;
    if (any_hit && pos) hit = hit_all || u > tau;
    const bool eq = any_hit && !hit_all && pos && u == tau;
    if (ties) {
      int tot_eq;
      const int rank = block_excl_count(eq, sm.ired, &tot_eq) + eq_seen;
      hit = hit || (eq && (unsigned long long)rank < take_eq);
      eq_seen += tot_eq;
    } else {
      hit = hit || eq;
    }
    if (in && !ex) {
      float k = __fmul_rn(ks[t], a.decay);
      if (hit) k = __fadd_rn(k, v);
      ks[t] = k;
    }
  }
}

size_t lrfu_smem_bytes() { return sizeof(LrfuSmem); }

}  // namespace actkv
