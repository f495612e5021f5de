// Keep-score update (ActionLRFU, actkv/eviction.py:198-210 with top_p_mask :36-50 and the head
// reduction of reduce_heads :20-33) and keep-mask selection (actkv/paged.py:23-46).
//
// Rows that fit (the usual case) are selected by a cluster of kCl CTAs per row (see "cluster-parallel
// selection" below): the row's keys are split over the CTAs' shared memories and the histograms
// are merged through distributed shared memory; the ActionLRFU cluster kernel also does the head
// reduction, so it is one launch; the keep mask is reduce + select.  Longer rows take the
// one-CTA-per-row kernels:
//   reduce  grid-wide (many CTAs per row, strided): the head mean (LRFU) or the head-then-layer
//           mean (keep mask) of every token, written to the act output / the scratch row;
//   select  one CTA (1024 threads) per row: the row becomes 32-bit order keys held in shared
//           memory (rows of more than kSmemKeyCap tokens stay in global memory), then a 3-pass
//           radix select (11, 11, 10 bits; one block-wide histogram per pass) finds the threshold:
//             keep mask : count-weighted -> the budget-th largest candidate score (top-k)
//             nucleus   : mass-weighted  -> the entry at which the descending cumulative mass
//                                           first reaches top_p * total (the crossing entry)
//           and a last pass writes the mask / updates the keep scores.
// Masses are 64-bit fixed point, so histogram sums do not depend on the order in which threads add
// them: the result is the same on every run.  The nucleus histogram updates are aggregated per
// warp (mass_add_warp), because probabilities cluster in a few exponents and per-token atomics on
// those bins serialise.  Ties at a threshold go to the lowest token index
// (a block-wide ballot scan counts the equal entries in index order).  Key 0 marks a token that
// takes no part in the selection (protected, or not positive for the nucleus).
#include <cooperative_groups.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace actkv {

constexpr int kSelThreads = 1024;
constexpr int kBins = 2048;
// radix digits of the 32-bit key, most significant first: bits 31..21, 20..10, 9..0
__device__ __forceinline__ int pass_shift(int p) { return p == 0 ? 21 : (p == 1 ? 10 : 0); }
__device__ __forceinline__ uint32_t pass_mask(int p) { return p < 2 ? 0x7FFu : 0x3FFu; }
// nucleus keys are positive floats (bit 31 clear): bits 30..20, 19..9, 8..0, so that the first
// digit splits every exponent into 8 bins and the few exponents most probabilities share spread
__device__ __forceinline__ int npass_shift(int p) { return p == 0 ? 20 : (p == 1 ? 9 : 0); }
__device__ __forceinline__ uint32_t npass_mask(int p) { return p < 2 ? 0x7FFu : 0x1FFu; }
constexpr int kSmemKeyCap = 49152;          // keep mask: tokens per row whose keys fit in shared memory
constexpr int kLrfuKeyCap = 36864;          // ActionLRFU: the same, beside its larger histograms
constexpr int kReduceThreads = 256;

// Highest bin b whose suffix sum (bins > b) is < need <= suffix sum including b; warp 0 only.
// Lane i owns nb/32 consecutive bins.  out_bin = -1 when the total never reaches need.
template <typename W>
__device__ void find_crossing_bin(const W* w, int nb, W need, int* out_bin, W* out_above) {
  const int lane = threadIdx.x & 31;
  const int per = nb / 32;
  W mine = 0;
  for (int k = 0; k < per; ++k) mine += w[lane * per + k];
  W incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const W y = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += y;
  }
  const W above = incl - mine;
  if (lane == 0) *out_bin = -1;
  __syncwarp();
  if (above < need && need <= incl) {
    W acc = above;
    for (int k = per - 1; k >= 0; --k) {
      const W v = w[lane * per + k];
      if (v > 0 && acc + v >= need) {
        *out_bin = lane * per + k;
        *out_above = acc;
        break;
      }
      acc += v;
    }
  }
  __syncwarp();
}

// Fixed-point mass of a positive float given by its bits: floor(v * 2^F), computed exactly from
// the mantissa and exponent with shifts (the same value as the floating-point product, floored).
__device__ __forceinline__ unsigned long long fixed_mass(uint32_t bits, int F) {
  int e = int((bits >> 23) & 0xFF);
  uint32_t m = bits & 0x7FFFFFu;
  if (e) m |= 0x800000u;
  else e = 1;
  const int sh = e - 150 + F;               // v = m * 2^(e - 150)
  if (sh >= 0) return (unsigned long long)m << sh;
  return sh > -32 ? (unsigned long long)(m >> -sh) : 0ull;
}

// Adds (count 1, mass m) to bin `bin` for every active lane, aggregated per warp: lanes with the
// same bin are grouped with __match_any_sync, the group's mass is summed exactly in four 16-bit
// pieces with __reduce_add_sync, and one lane per group adds it to the bin with native 32-bit
// atomics (low word, its carry, high word), so hot bins see one update per warp and no
// compare-and-swap loop.  All 32 lanes must call it.
__device__ __forceinline__ void mass_add_warp(uint32_t* hc, uint32_t* hlo, uint32_t* hhi, int bin,
                                              unsigned long long m, bool active) {
  const unsigned peers = __match_any_sync(0xffffffffu, active ? bin : -1);
  unsigned long long sum = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    sum += (unsigned long long)__reduce_add_sync(peers, unsigned(m >> (16 * c)) & 0xFFFFu) << (16 * c);
  if (active && int(threadIdx.x & 31) == __ffs(peers) - 1) {
    atomicAdd(&hc[bin], unsigned(__popc(peers)));
    const uint32_t lo = uint32_t(sum), hi = uint32_t(sum >> 32);
    const uint32_t old = atomicAdd(&hlo[bin], lo);
    const uint32_t carry = (old + lo) < old ? 1u : 0u;
    if (hi | carry) atomicAdd(&hhi[bin], hi + carry);
  }
}

// grid-stride helper: CTAs per row for the reduce launches
inline int reduce_ctas_per_row(int rows) {
  const int want = (2 * device_sm_count() + rows - 1) / (rows > 0 ? rows : 1);
  return want < 1 ? 1 : (want > 128 ? 128 : want);
}

// ======================================================================================= keep mask
// s[r][t] = mean over the leading rows of (reduce over x of scores(r, l, x, t)); grid (X, R)
__global__ void __launch_bounds__(kReduceThreads) keep_reduce_kernel(KeepMaskArgs a) {
  const int r = blockIdx.y;
  const int n = a.seq_used[r];
  if (n > a.max_seq) return;                          // the select kernel reports it
  const float* sc = a.scores + (a.scores_off ? a.scores_off[r] : r * a.stride_r);
  float* s = a.s_ws + r * a.max_seq;
  if (a.n_red == 1) {
    // one value per leading row (the pipeline's [L, S] keep scores): the rows' loads are issued 8
    // at a time, then added in row order (the same sum as the general loop below)
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x) {
      float acc = 0.0f;
      int l = 0;
      for (; l + 8 <= a.n_lead; l += 8) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __ldg(sc + (l + k) * a.stride_l + t);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc += v[k];
      }
      for (; l < a.n_lead; ++l) acc += __ldg(sc + l * a.stride_l + t);
      s[t] = __fdiv_rn(acc, float(a.n_lead));
    }
    return;
  }
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (int l = 0; l < a.n_lead; ++l) {
      const float* row = sc + l * a.stride_l + t;
      float v = row[0];
      if (a.reduce == ACTKV_REDUCE_MAX) {
        for (int x = 1; x < a.n_red; ++x) v = fmaxf(v, row[x * a.stride_x]);
      } else {
        for (int x = 1; x < a.n_red; ++x) v += row[x * a.stride_x];
        v = __fdiv_rn(v, float(a.n_red));
      }
      acc += v;
    }
    s[t] = __fdiv_rn(acc, float(a.n_lead));
  }
}

__global__ void __launch_bounds__(kSelThreads) keep_select_kernel(KeepMaskArgs a) {
  extern __shared__ uint32_t skeys[];                 // [kSmemKeyCap] when the row fits
  __shared__ uint32_t hist[kBins];
  __shared__ int red[33];
  __shared__ int sel_bin;
  __shared__ uint32_t sel_above;
  const int r = blockIdx.x;
  const int n = a.seq_used[r];
  const uint8_t* pin = a.pinned ? a.pinned + r * a.pinned_stride_r : nullptr;
  uint8_t* keep = a.keep + r * a.keep_stride_r;
  if (n > a.max_seq) {
    if (threadIdx.x == 0) {
      flag(a.status, ACTKV_DEV_BAD_INDEX);
      if (a.kept) a.kept[r] = 0;
    }
    return;
  }
  float* s = a.s_ws + r * a.max_seq;
  const bool in_smem = n <= kSmemKeyCap;
  uint32_t* keys = in_smem ? skeys : reinterpret_cast<uint32_t*>(s);   // converted in place otherwise
  // keys: order_key(score), 0 for protected tokens
  int n_prot = 0;
  for (int t0 = threadIdx.x; t0 < n; t0 += 4 * blockDim.x) {
    float v[4];
    bool pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {                      // four independent loads in flight
      const int t = t0 + i * blockDim.x;
      v[i] = t < n ? s[t] : 0.0f;
      pr[i] = t < n && (t < a.protected_prefix || (pin && pin[t]));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + i * blockDim.x;
      if (t >= n) break;
      uint32_t k = 0;
      if (!pr[i]) {
        k = order_key(v[i]);
        if (k == 0) k = 1;                             // never collide with the protected mark
      }
      keys[t] = k;
      n_prot += pr[i];
    }
  }
  n_prot = block_sum(n_prot, red);                    // includes __syncthreads
  const int n_cand = n - n_prot;
  const int budget = a.budget[r];
  const bool keep_all = budget >= n_cand;
  const int k = keep_all ? n_cand : (budget > 0 ? budget : 0);
  if (keep_all || k == 0) {
    for (int t = threadIdx.x; t < n; t += blockDim.x) keep[t] = keep_all ? 1 : (keys[t] == 0);
    if (threadIdx.x == 0 && a.kept) a.kept[r] = keep_all ? n : n_prot;
    return;
  }
  uint32_t prefix = 0, pmask = 0, need = uint32_t(k), eq_count = 0;
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass_shift(pass);
    const uint32_t dmask = pass_mask(pass);
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
      const uint32_t u = keys[t];
      if (u != 0 && (u & pmask) == prefix) atomicAdd(&hist[(u >> shift) & dmask], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) find_crossing_bin<uint32_t>(hist, int(dmask) + 1, need, &sel_bin, &sel_above);
    __syncthreads();
    const int b = sel_bin;
    if (b < 0) {                                      // cannot happen: k <= #candidates
      if (threadIdx.x == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      return;
    }
    need -= sel_above;
    eq_count = hist[b];
    prefix |= uint32_t(b) << shift;
    pmask |= dmask << shift;
    __syncthreads();
  }
  // final pass: protected, above the threshold, or among the first `need` equal ones by index
  const bool ties = eq_count > need;
  int eq_seen = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int t = base + threadIdx.x;
    const bool in = t < n;
    const uint32_t u = in ? keys[t] : 0u;
    const bool prot = in && u == 0;
    const bool eq = in && !prot && u == prefix;
    bool take = prot || (in && u > prefix);
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

// ------------------------------------------------------------------ cluster-parallel selection
// One row (session) is shared by the kCl CTAs of a thread-block cluster: CTA c holds the keys of
// a contiguous slice of the tokens in its shared memory.  Each radix pass builds a local histogram
// per CTA; CTA c then sums bins [c*kBins/kCl, (c+1)*kBins/kCl) over the cluster through distributed
// shared memory, CTA 0's first warp finds the crossing bin over those merged slices and writes the
// result into every CTA.  Counts (protected tokens, equal keys before a CTA's slice) are exchanged
// by every CTA writing its own into a slot of every CTA, then summed in rank order, so the result
// does not depend on timing.  cluster.sync() separates every phase: no CTA reads or writes another's
// shared memory after that one could have moved past the phase or exited.
constexpr int kCl = 4;
constexpr int kSlice = kBins / kCl;

// Broadcast this CTA's v into slot [rank] of `slots` in every CTA of the cluster (thread 0 only).
__device__ __forceinline__ void cluster_put(cg::cluster_group& cl, uint32_t* slots, uint32_t v) {
  const unsigned me = cl.block_rank();
  for (unsigned q = 0; q < kCl; ++q) cl.map_shared_rank(slots, q)[me] = v;
}

// Merge the cluster's local histograms into this CTA's slice (mslice) and broadcast the slice's
// total; the one CTA whose slice holds the crossing bin (the highest bin whose suffix sum reaches
// need) finds it in its own shared memory and writes (bin, count above it, count in it) into every
// CTA's sel[3] (0xFFFFFFFF in sel[0] when the total never reaches need).  Three cluster barriers;
// all threads of all CTAs call it.  `stot` holds kCl slice totals, `red` 33 ints of scratch.
__device__ void cluster_crossing_u32(cg::cluster_group& cl, uint32_t* hist, uint32_t* mslice, uint32_t* stot,
                                     uint32_t need, int nbins, uint32_t* sel, int* red) {
  const unsigned me = cl.block_rank();
  cl.sync();                                         // every local histogram is complete
  uint32_t part = 0;
  for (int i = threadIdx.x; i < kSlice; i += blockDim.x) {
    uint32_t v = 0;
    const int b = int(me) * kSlice + i;
    if (b < nbins)
      for (unsigned q = 0; q < kCl; ++q) v += cl.map_shared_rank(hist, q)[b];
    mslice[i] = v;
    part += v;
  }
  const uint32_t tot = uint32_t(block_sum(int(part), red));   // counts fit in int (< 2^31 tokens)
  if (threadIdx.x == 0) cluster_put(cl, stot, tot);
  cl.sync();                                         // every slice is merged, its total everywhere
  uint32_t above = 0, total = 0;
  for (unsigned q = 0; q < kCl; ++q) {
    total += stot[q];
    if (q > me) above += stot[q];
  }
  if (threadIdx.x < 32) {
    if (above < need && need <= above + stot[me]) {  // the crossing is in this slice
      __shared__ int b_local;
      __shared__ uint32_t b_above;
      find_crossing_bin<uint32_t>(mslice, kSlice, need - above, &b_local, &b_above);
      if (threadIdx.x == 0) {
        for (unsigned q = 0; q < kCl; ++q) {
          uint32_t* d = cl.map_shared_rank(sel, q);
          d[0] = me * kSlice + uint32_t(b_local);
          d[1] = above + b_above;
          d[2] = mslice[b_local];
        }
      }
    } else if (me == 0 && total < need && threadIdx.x == 0) {
      for (unsigned q = 0; q < kCl; ++q) cl.map_shared_rank(sel, q)[0] = 0xFFFFFFFFu;
    }
  }
  cl.sync();                                         // sel is in every CTA
}

// keep mask, one cluster per row: the same selection as keep_select_kernel (top `budget` keys,
// ties to the lowest index, protected tokens always kept).  Rows up to kCl * kSmemKeyCap tokens.
__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kSelThreads)
    keep_select_cluster_kernel(KeepMaskArgs a) {
  extern __shared__ uint32_t skeys[];                 // this CTA's slice of the row
  __shared__ uint32_t hist[kBins];
  __shared__ uint32_t mslice[kSlice];
  __shared__ uint32_t slots[kCl];
  __shared__ uint32_t stot[kCl];
  __shared__ uint32_t sel[3];
  __shared__ int red[33];
  cg::cluster_group cl = cg::this_cluster();
  const int me = int(cl.block_rank());
  const int r = blockIdx.y;
  const int n = a.seq_used[r];
  uint8_t* keep = a.keep + r * a.keep_stride_r;
  if (n > a.max_seq || (n + kCl - 1) / kCl > kSmemKeyCap) {   // uniform over the cluster: no one waits
    if (threadIdx.x == 0 && me == 0) {
      flag(a.status, ACTKV_DEV_BAD_INDEX);
      if (a.kept) a.kept[r] = 0;
    }
    return;
  }
  const uint8_t* pin = a.pinned ? a.pinned + r * a.pinned_stride_r : nullptr;
  const float* s = a.s_ws + r * a.max_seq;
  const int per = (n + kCl - 1) / kCl;
  const int t0 = min(n, me * per), m = min(n, t0 + per) - t0;    // tokens [t0, t0 + m)
  uint32_t n_prot = 0;
  // four tokens per thread and step, their loads issued before the keys are formed
  for (int i0 = threadIdx.x; i0 < m; i0 += 4 * int(blockDim.x)) {
    float v[4];
    uint8_t pb[4];
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
      const int i = i0 + k4 * int(blockDim.x);
      v[k4] = i < m ? __ldg(s + t0 + i) : 0.0f;
      pb[k4] = i < m && pin ? __ldg(pin + t0 + i) : uint8_t(0);
    }
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
      const int i = i0 + k4 * int(blockDim.x);
      if (i >= m) break;
      const int t = t0 + i;
      const bool pr = t < a.protected_prefix || pb[k4];
      uint32_t k = 0;
      if (!pr) {
        k = order_key(v[k4]);
        if (k == 0) k = 1;                             // never collide with the protected mark
      }
      skeys[i] = k;
      n_prot += pr;
    }
  }
  n_prot = uint32_t(block_sum(int(n_prot), red));
  cl.sync();                                           // every CTA of the cluster has started
  if (threadIdx.x == 0) cluster_put(cl, slots, n_prot);
  cl.sync();
  uint32_t prot_total = 0;
  for (int q = 0; q < kCl; ++q) prot_total += slots[q];
  const int n_cand = n - int(prot_total);
  const int budget = a.budget[r];
  const bool keep_all = budget >= n_cand;
  const int k = keep_all ? n_cand : (budget > 0 ? budget : 0);
  if (keep_all || k == 0) {                            // uniform; no further cluster traffic
    for (int i = threadIdx.x; i < m; i += blockDim.x) keep[t0 + i] = keep_all ? 1 : (skeys[i] == 0);
    if (threadIdx.x == 0 && me == 0 && a.kept) a.kept[r] = keep_all ? n : int(prot_total);
    return;
  }
  uint32_t prefix = 0, pmask = 0, need = uint32_t(k), eq_count = 0;
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass_shift(pass);
    const uint32_t dmask = pass_mask(pass);
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      const uint32_t u = skeys[i];
      if (u != 0 && (u & pmask) == prefix) atomicAdd(&hist[(u >> shift) & dmask], 1u);
    }
    __syncthreads();
    cluster_crossing_u32(cl, hist, mslice, stot, need, int(dmask) + 1, sel, red);
    if (sel[0] == 0xFFFFFFFFu) {                       // cannot happen: k <= #candidates (uniform)
      if (threadIdx.x == 0 && me == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      return;
    }
    need -= sel[1];
    eq_count = sel[2];
    prefix |= sel[0] << shift;
    pmask |= dmask << shift;
  }
  // equal keys before this CTA's slice, for ranking ties by index
  const bool ties = eq_count > need;
  uint32_t eq_seen = 0;
  if (ties) {
    int mine = 0;
    for (int i = threadIdx.x; i < m; i += blockDim.x) mine += skeys[i] == prefix;
    mine = block_sum(mine, red);
    cl.sync();                                         // the last pass's reads of sel are done
    if (threadIdx.x == 0) cluster_put(cl, slots, uint32_t(mine));
    cl.sync();
    for (int q = 0; q < me; ++q) eq_seen += slots[q];
  }
  for (int base = 0; base < m; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool in = i < m;
    const uint32_t u = in ? skeys[i] : 0u;
    const bool prot = in && u == 0;
    const bool eq = in && !prot && u == prefix;
    bool take = prot || (in && u > prefix);
    if (ties) {
      int tot_eq;
      const int rank = block_excl_count(eq, red, &tot_eq) + int(eq_seen);
      take = take || (eq && uint32_t(rank) < need);
      eq_seen += uint32_t(tot_eq);
    } else {
      take = take || eq;
    }
    if (in) keep[t0 + i] = take;
  }
  if (threadIdx.x == 0 && me == 0 && a.kept) a.kept[r] = int(prot_total) + k;
}

cudaError_t launch_keep_mask(const KeepMaskArgs& a, int R, cudaStream_t st) {
  if (R <= 0) return cudaSuccess;
  keep_reduce_kernel<<<dim3(reduce_ctas_per_row(R), R), kReduceThreads, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (a.max_seq <= int64_t(kCl) * kSmemKeyCap) {
    // a cluster of kCl CTAs per row, each with its slice of the keys in shared memory
    const int per = int((a.max_seq + kCl - 1) / kCl);
    const size_t sm = size_t(per > 0 ? per : 1) * sizeof(uint32_t);
    e = cudaFuncSetAttribute(keep_select_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    if (e != cudaSuccess) return e;
    keep_select_cluster_kernel<<<dim3(kCl, R), kSelThreads, sm, st>>>(a);
    return cudaGetLastError();
  }
  const int cap = a.max_seq < kSmemKeyCap ? int(a.max_seq) : kSmemKeyCap;
  const size_t sm = size_t(cap > 0 ? cap : 1) * sizeof(uint32_t);
  e = cudaFuncSetAttribute(keep_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  if (e != cudaSuccess) return e;
  keep_select_kernel<<<R, kSelThreads, sm, st>>>(a);
  return cudaGetLastError();
}

// ======================================================================================= ActionLRFU
// act(r, l, t) = reduce over h of src(r, l, h, t); grid (X, L, R)
__global__ void __launch_bounds__(kReduceThreads) headmean_kernel(LrfuArgs a) {
  const int l = blockIdx.y, r = blockIdx.z;
  const int n = a.seq_used[r];
  const float* src = a.src + (a.src_off ? a.src_off[r] : r * a.src_stride_r) + l * a.src_stride_l;
  float* act = a.act + r * a.act_stride_r + l * a.act_stride_l;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x) {
    float v = src[t];
    if (a.reduce == ACTKV_REDUCE_MAX) {
      for (int h = 1; h < a.H; ++h) v = fmaxf(v, src[h * a.src_stride_h + t]);
    } else {
      for (int h = 1; h < a.H; ++h) v += src[h * a.src_stride_h + t];
      v = __fdiv_rn(v, float(a.H));
    }
    act[t] = v;
  }
}

struct LrfuSelSmem {                        // 57.5 KB; with kLrfuKeyCap keys 217.5 KB
  unsigned long long hm[kBins];             // combined masses for the crossing search
  uint32_t h16[4][kBins];                   // rows <= 65535 tokens: 16-bit chunk sums of the mass
  uint32_t hc[kBins];
  __device__ uint32_t* hlo() { return h16[0]; }        // longer rows: low / high 32-bit words (with carry)
  __device__ uint32_t* hhi() { return h16[1]; }
  double dred[32];
  float fred[32];
  int ired[33];
  int sel_bin;
  unsigned long long sel_above;
};

static_assert(sizeof(LrfuSelSmem) + size_t(kLrfuKeyCap) * 4 <= 232448, "LRFU select exceeds 227 KB of smem");
static_assert(size_t(kSmemKeyCap) * 4 + 8192 + 512 <= 232448, "keep select exceeds 227 KB of smem");

// grid (L, R): nucleus of act over the non-excluded tokens, then the keep-score update
__global__ void __launch_bounds__(kSelThreads) lrfu_select_kernel(LrfuArgs a) {
  extern __shared__ __align__(16) unsigned char lrfu_smem_raw[];
  LrfuSelSmem& sm = *reinterpret_cast<LrfuSelSmem*>(lrfu_smem_raw);
  uint32_t* skeys = reinterpret_cast<uint32_t*>(lrfu_smem_raw + sizeof(LrfuSelSmem));
  const int l = blockIdx.x, r = blockIdx.y;
  const int n = a.seq_used[r];
  float* ks = a.ks + r * a.ks_stride_r + l * a.ks_stride_l;
  const float* act = a.act + r * a.act_stride_r + l * a.act_stride_l;
  const uint8_t* pin = a.pinned ? a.pinned + r * a.pinned_stride_r : nullptr;
  auto excluded = [&](int t) { return t < a.protected_prefix || (pin && pin[t]); };
  const bool in_smem = n <= kLrfuKeyCap;
  // key of a token taking part in the nucleus: its (positive) value's bits; 0 otherwise
  auto key_at = [&](int t) -> uint32_t {
    const float v = act[t];
    return (!excluded(t) && v > 0.0f) ? __float_as_uint(v) : 0u;
  };

  double total = 0.0;
  float vmax = 0.0f;
  int n_pos = 0;
  for (int t0 = threadIdx.x; t0 < n; t0 += 4 * blockDim.x) {
    float va[4];
    bool exa[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {                      // four independent loads in flight
      const int t = t0 + i * blockDim.x;
      va[i] = t < n ? act[t] : 0.0f;
      exa[i] = t < n && excluded(t);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + i * blockDim.x;
      if (t >= n) break;
      const float v = va[i];
      uint32_t key = 0;
      if (!exa[i]) {
        total += v;
        if (v > 0.0f) {
          vmax = fmaxf(vmax, v);
          ++n_pos;
          key = __float_as_uint(v);
        }
      }
      if (in_smem) skeys[t] = key;
    }
  }
  __syncthreads();
  total = block_sum(total, sm.dred);
  vmax = block_max(vmax, sm.fred);
  n_pos = block_sum(n_pos, sm.ired);
  const float total_f = float(total);
  const bool any_hit = (a.n_act == nullptr || a.n_act[r] > 0) && total_f > 0.0f && n_pos > 0;

  bool hit_all = false;
  uint32_t tau = 0;
  unsigned long long take_eq = 0, eq_count = 0;
  if (any_hit) {
    int e2;
    frexp(double(vmax) * double(n_pos), &e2);
    const int F = 62 - e2;                            // n_pos * vmax * 2^F < 2^62
    const double fx = ldexp(1.0, F);
    const float target_f = __fmul_rn(a.top_p, total_f);
    unsigned long long need = (unsigned long long)ceil(double(target_f) * fx);
    if (need == 0) need = 1;
    uint32_t prefix = 0, pmask = 0;
    for (int pass = 0; pass < 3 && !hit_all; ++pass) {
      const int shift = npass_shift(pass);
      const uint32_t dmask = npass_mask(pass);
      for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        sm.hc[i] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) sm.h16[c][i] = 0;
      }
      __syncthreads();
      const bool chunked = n <= 65535;
      if (chunked) {
        // per token: count + four 16-bit mass pieces, fire-and-forget 32-bit atomics
        for (int t = threadIdx.x; t < n; t += blockDim.x) {
          const uint32_t u = in_smem ? skeys[t] : key_at(t);
          if (u == 0 || (u & pmask) != prefix) continue;
          const int bin = int((u >> shift) & dmask);
          const unsigned long long m = fixed_mass(u, F);
          atomicAdd(&sm.hc[bin], 1u);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t part = unsigned(m >> (16 * c)) & 0xFFFFu;
            if (part) atomicAdd(&sm.h16[c][bin], part);
          }
        }
      } else {
        for (int base = 0; base < n; base += blockDim.x) {
          const int t = base + threadIdx.x;
          const uint32_t u = t < n ? key_at(t) : 0u;
          const bool active = u != 0 && (u & pmask) == prefix;
          const unsigned long long m = active ? fixed_mass(u, F) : 0ull;
          mass_add_warp(sm.hc, sm.hlo(), sm.hhi(), int((u >> shift) & dmask), m, active);
        }
      }
      __syncthreads();
      for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        if (chunked) {
          unsigned long long v = 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) v += (unsigned long long)sm.h16[c][i] << (16 * c);
          sm.hm[i] = v;
        } else {
          sm.hm[i] = (unsigned long long)sm.hhi()[i] << 32 | sm.hlo()[i];
        }
      }
      __syncthreads();
      if (threadIdx.x < 32)
        find_crossing_bin<unsigned long long>(sm.hm, int(dmask) + 1, need, &sm.sel_bin, &sm.sel_above);
      __syncthreads();
      const int b = sm.sel_bin;
      if (b < 0) {
        hit_all = pass == 0;                          // the target exceeds the whole mass: every positive
        if (pass > 0 && threadIdx.x == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      } else {
        need -= sm.sel_above;
        eq_count = sm.hc[b];
        prefix |= uint32_t(b) << shift;
        pmask |= dmask << shift;
      }
      __syncthreads();
    }
    tau = prefix;
    if (!hit_all) {
      const unsigned long long unit = fixed_mass(tau, F);
      take_eq = unit ? (need + unit - 1) / unit : eq_count;
      if (take_eq < 1) take_eq = 1;
      if (take_eq > eq_count) take_eq = eq_count;
    }
  }
  // final pass: ks = fl(decay*ks) (+ a for hits); excluded tokens untouched
  const bool ties = any_hit && !hit_all && eq_count > take_eq;
  int eq_seen = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int t = base + threadIdx.x;
    const bool in = t < n;
    const bool ex = in && excluded(t);
    const float v = in ? act[t] : 0.0f;
    const bool pos = in && !ex && v > 0.0f;
    const uint32_t u = __float_as_uint(v);
    bool hit = any_hit && pos && (hit_all || u > tau);
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

// ActionLRFU nucleus + keep-score update on a cluster of kCl CTAs per (layer, session) row: the
// same result as lrfu_select_kernel (sums combined in rank order), with each CTA's slice of the
// keys (and its exclusion flags) in shared memory.  Rows up to kCl * kLrfuClCap tokens (134,656;
// the 16-bit mass pieces of one CTA cannot overflow).
struct LrfuClSmem {
  unsigned long long hm[kBins];             // local masses (from the 16-bit pieces)
  uint32_t h16[4][kBins];
  uint32_t hc[kBins];
  unsigned long long mhm[kSlice];           // this CTA's merged slice
  uint32_t mhc[kSlice];
  uint32_t slots[4][kCl];                   // exchanged per-CTA values
  uint32_t sel[5];                          // bin, above (lo, hi), eq count, found
  double dred[32];
  float fred[32];
  int ired[33];
  int b_local;
  unsigned long long b_above;
};
// keys (4 B) and exclusion flags (1 B) per token of a CTA's slice beside LrfuClSmem in 227 KB
constexpr int kLrfuClCap = 33664;
// Tokens of a row per CTA of the ActionLRFU cluster: a multiple of 4, so that every slice starts
// on a 16-byte boundary of the row (the head reduction reads 4 tokens per load).
__host__ __device__ inline int lrfu_slice(int64_t n) { return int(((n + kCl - 1) / kCl + 3) & ~int64_t(3)); }
static_assert(sizeof(LrfuClSmem) + size_t(kLrfuClCap) * 5 <= 232448, "LRFU cluster select exceeds 227 KB");
static_assert(kLrfuClCap <= 65535 && kLrfuClCap % 4 == 0, "16-bit mass pieces per CTA; slices of whole 4-token groups");

constexpr int kClThreads = 512;                      // 2 CTAs per SM: a config-2 step's rows in one wave

__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kClThreads, 2)
    lrfu_select_cluster_kernel(LrfuArgs a) {
  extern __shared__ __align__(16) unsigned char lrfu_cl_raw[];
  LrfuClSmem& sm = *reinterpret_cast<LrfuClSmem*>(lrfu_cl_raw);
  uint32_t* skeys = reinterpret_cast<uint32_t*>(lrfu_cl_raw + sizeof(LrfuClSmem));
  // 1 where the token takes no part (protected or pinned): the final pass skips it
  uint8_t* sexcl = reinterpret_cast<uint8_t*>(skeys + lrfu_slice(a.max_seq));
  cg::cluster_group cl = cg::this_cluster();
  const unsigned me = cl.block_rank();
  const int l = blockIdx.y, r = blockIdx.z;
  const int n = a.seq_used[r];
  if (n > a.max_seq || lrfu_slice(n) > kLrfuClCap) {   // uniform over the cluster
    if (threadIdx.x == 0 && me == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
    return;
  }
  float* ks = a.ks + r * a.ks_stride_r + l * a.ks_stride_l;
  float* act = a.act + r * a.act_stride_r + l * a.act_stride_l;
  const float* src = a.src + (a.src_off ? a.src_off[r] : r * a.src_stride_r) + l * a.src_stride_l;
  const uint8_t* pin = a.pinned ? a.pinned + r * a.pinned_stride_r : nullptr;
  auto excluded = [&](int t) { return t < a.protected_prefix || (pin && pin[t]); };
  const int per = lrfu_slice(n);
  const int t0 = min(n, int(me) * per), m = min(n, t0 + per) - t0;

  // the head reduction of this slice (as headmean_kernel: heads in order, one division), written
  // to act, then the nucleus keys
  double total = 0.0;
  float vmax = 0.0f;
  int n_pos = 0;
  auto take = [&](int i, float v) {
    const int t = t0 + i;
    uint32_t key = 0;
    const bool ex = excluded(t);
    sexcl[i] = ex;
    if (!ex) {
      total += v;
      if (v > 0.0f) {
        vmax = fmaxf(vmax, v);
        ++n_pos;
        key = __float_as_uint(v);
      }
    }
    skeys[i] = key;
  };
  auto fold = [&](float v, float w) { return a.reduce == ACTKV_REDUCE_MAX ? fmaxf(v, w) : v + w; };
  const bool vec = ((reinterpret_cast<uintptr_t>(src + t0) | reinterpret_cast<uintptr_t>(act + t0)) & 15) == 0 &&
                   (a.src_stride_h & 3) == 0;
  // 4 tokens per thread and step with 16-byte loads, the loads of up to 8 heads issued before they
  // are folded (in head order); the scalar loop below takes the rest
  const int m4 = vec ? (m & ~3) : 0;
  for (int i = threadIdx.x * 4; i < m4; i += blockDim.x * 4) {
    const float* p = src + t0 + i;
    float4 v = __ldg(reinterpret_cast<const float4*>(p));
    for (int h0 = 1; h0 < a.H; h0 += 8) {
      float4 w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (h0 + k < a.H) w[k] = __ldg(reinterpret_cast<const float4*>(p + (h0 + k) * a.src_stride_h));
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (h0 + k < a.H) {
          v.x = fold(v.x, w[k].x);
          v.y = fold(v.y, w[k].y);
          v.z = fold(v.z, w[k].z);
          v.w = fold(v.w, w[k].w);
        }
    }
    if (a.reduce != ACTKV_REDUCE_MAX) {
      const float hf = float(a.H);
      v = make_float4(__fdiv_rn(v.x, hf), __fdiv_rn(v.y, hf), __fdiv_rn(v.z, hf), __fdiv_rn(v.w, hf));
    }
    *reinterpret_cast<float4*>(act + t0 + i) = v;
    take(i, v.x);
    take(i + 1, v.y);
    take(i + 2, v.z);
    take(i + 3, v.w);
  }
  for (int i = m4 + threadIdx.x; i < m; i += blockDim.x) {
    const int t = t0 + i;
    float v = src[t];
    for (int h = 1; h < a.H; ++h) v = fold(v, src[h * a.src_stride_h + t]);
    if (a.reduce != ACTKV_REDUCE_MAX) v = __fdiv_rn(v, float(a.H));
    act[t] = v;
    take(i, v);
  }
  total = block_sum(total, sm.dred);
  vmax = block_max(vmax, sm.fred);
  n_pos = block_sum(n_pos, sm.ired);
  cl.sync();                                           // every CTA of the cluster has started
  if (threadIdx.x == 0) {
    const unsigned long long tb = __double_as_longlong(total);
    for (unsigned q = 0; q < kCl; ++q) {
      uint32_t (*d)[kCl] = cl.map_shared_rank(sm.slots, q);
      d[0][me] = uint32_t(tb);
      d[1][me] = uint32_t(tb >> 32);
      d[2][me] = __float_as_uint(vmax);
      d[3][me] = uint32_t(n_pos);
    }
  }
  cl.sync();
  total = 0.0;
  vmax = 0.0f;
  n_pos = 0;
  for (unsigned q = 0; q < kCl; ++q) {                 // rank order: the same sum in every CTA
    total += __longlong_as_double((long long)((unsigned long long)sm.slots[1][q] << 32 | sm.slots[0][q]));
    vmax = fmaxf(vmax, __uint_as_float(sm.slots[2][q]));
    n_pos += int(sm.slots[3][q]);
  }
  const float total_f = float(total);
  const bool any_hit = (a.n_act == nullptr || a.n_act[r] > 0) && total_f > 0.0f && n_pos > 0;

  bool hit_all = false;
  uint32_t tau = 0;
  unsigned long long take_eq = 0, eq_count = 0;
  if (any_hit) {                                       // uniform
    int e2;
    frexp(double(vmax) * double(n_pos), &e2);
    const int F = 62 - e2;                             // n_pos * vmax * 2^F < 2^62
    const double fx = ldexp(1.0, F);
    const float target_f = __fmul_rn(a.top_p, total_f);
    unsigned long long need = (unsigned long long)ceil(double(target_f) * fx);
    if (need == 0) need = 1;
    uint32_t prefix = 0, pmask = 0;
    for (int pass = 0; pass < 3 && !hit_all; ++pass) {
      const int shift = npass_shift(pass);
      const uint32_t dmask = npass_mask(pass);
      const int nbins = int(dmask) + 1;
      for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        sm.hc[i] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) sm.h16[c][i] = 0;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < m; i += blockDim.x) {
        const uint32_t u = skeys[i];
        if (u == 0 || (u & pmask) != prefix) continue;
        const int bin = int((u >> shift) & dmask);
        const unsigned long long mass = fixed_mass(u, F);
        atomicAdd(&sm.hc[bin], 1u);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t part = unsigned(mass >> (16 * c)) & 0xFFFFu;
          if (part) atomicAdd(&sm.h16[c][bin], part);
        }
      }
      __syncthreads();
      for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        unsigned long long v = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) v += (unsigned long long)sm.h16[c][i] << (16 * c);
        sm.hm[i] = v;
      }
      cl.sync();                                       // every local histogram is complete
      unsigned long long part_m = 0;
      for (int i = threadIdx.x; i < kSlice; i += blockDim.x) {
        unsigned long long v = 0;
        uint32_t c = 0;
        const int b = int(me) * kSlice + i;
        if (b < nbins)
          for (unsigned q = 0; q < kCl; ++q) {
            v += cl.map_shared_rank(sm.hm, q)[b];
            c += cl.map_shared_rank(sm.hc, q)[b];
          }
        sm.mhm[i] = v;
        sm.mhc[i] = c;
        part_m += v;
      }
      part_m = block_sum(part_m, reinterpret_cast<unsigned long long*>(sm.dred));
      if (threadIdx.x == 0)
        for (unsigned q = 0; q < kCl; ++q) {
          uint32_t (*d)[kCl] = cl.map_shared_rank(sm.slots, q);
          d[0][me] = uint32_t(part_m);
          d[1][me] = uint32_t(part_m >> 32);
        }
      cl.sync();                                       // merged slices and their masses everywhere
      unsigned long long above = 0, all = 0;
      for (unsigned q = 0; q < kCl; ++q) {
        const unsigned long long t = (unsigned long long)sm.slots[1][q] << 32 | sm.slots[0][q];
        all += t;
        if (q > me) above += t;
      }
      const unsigned long long mine = (unsigned long long)sm.slots[1][me] << 32 | sm.slots[0][me];
      if (threadIdx.x < 32 && above < need && need <= above + mine) {
        find_crossing_bin<unsigned long long>(sm.mhm, kSlice, need - above, &sm.b_local, &sm.b_above);
        if (threadIdx.x == 0) {
          const unsigned long long ab = above + sm.b_above;
          for (unsigned q = 0; q < kCl; ++q) {
            uint32_t* d = cl.map_shared_rank(sm.sel, q);
            d[0] = me * kSlice + uint32_t(sm.b_local);
            d[1] = uint32_t(ab);
            d[2] = uint32_t(ab >> 32);
            d[3] = sm.mhc[sm.b_local];
            d[4] = 1u;
          }
        }
      } else if (threadIdx.x == 0 && me == 0 && all < need) {
        for (unsigned q = 0; q < kCl; ++q) cl.map_shared_rank(sm.sel, q)[4] = 0u;
      }
      cl.sync();                                       // sel is in every CTA
      if (!sm.sel[4]) {
        hit_all = pass == 0;                           // the target exceeds the whole mass: every positive
        if (pass > 0 && threadIdx.x == 0 && me == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      } else {
        need -= (unsigned long long)sm.sel[2] << 32 | sm.sel[1];
        eq_count = sm.sel[3];
        prefix |= sm.sel[0] << shift;
        pmask |= dmask << shift;
      }
      // no barrier here: the next pass rewrites sel and slots only after two more cluster
      // barriers, which every CTA reaches after these reads, and nothing reads another CTA's
      // memory between here and the kernel's end except through the ties exchange (behind its own
      // barrier)
    }
    tau = prefix;
    if (!hit_all) {
      const unsigned long long unit = fixed_mass(tau, F);
      take_eq = unit ? (need + unit - 1) / unit : eq_count;
      if (take_eq < 1) take_eq = 1;
      if (take_eq > eq_count) take_eq = eq_count;
    }
  }
  const bool ties = any_hit && !hit_all && eq_count > take_eq;     // uniform
  unsigned long long eq_seen = 0;
  if (ties) {
    int mine = 0;
    for (int i = threadIdx.x; i < m; i += blockDim.x) mine += skeys[i] == tau;
    mine = block_sum(mine, sm.ired);
    if (threadIdx.x == 0)
      for (unsigned q = 0; q < kCl; ++q) cl.map_shared_rank(sm.slots, q)[0][me] = uint32_t(mine);
    cl.sync();
    for (unsigned q = 0; q < me; ++q) eq_seen += sm.slots[0][q];
  }
  // final pass over this CTA's slice: ks = fl(decay*ks) (+ a for hits); excluded tokens untouched.
  // The keep scores of four steps are loaded together; the exclusions come from shared memory.
  for (int base0 = 0; base0 < m; base0 += 4 * int(blockDim.x)) {
    float kv[4];
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const int i = base0 + s4 * int(blockDim.x) + int(threadIdx.x);
      kv[s4] = i < m && !sexcl[i] ? __ldcg(ks + t0 + i) : 0.0f;
    }
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const int base = base0 + s4 * int(blockDim.x);
      if (base >= m) break;                           // uniform
      const int i = base + threadIdx.x;
      const bool in = i < m;
      const uint32_t u = in ? skeys[i] : 0u;          // key != 0: taking part and positive
      const bool pos = u != 0;
      bool hit = any_hit && pos && (hit_all || u > tau);
      const bool eq = any_hit && !hit_all && pos && u == tau;
      if (ties) {
        int tot_eq;
        const int rank = block_excl_count(eq, sm.ired, &tot_eq);
        hit = hit || (eq && eq_seen + (unsigned long long)rank < take_eq);
        eq_seen += (unsigned long long)tot_eq;
      } else {
        hit = hit || eq;
      }
      if (in && !sexcl[i]) {
        float k = __fmul_rn(kv[s4], a.decay);
        if (hit) k = __fadd_rn(k, __uint_as_float(u));
        ks[t0 + i] = k;
      }
    }
  }
}

cudaError_t launch_lrfu(const LrfuArgs& a, int R, int L, cudaStream_t st) {
  if (R <= 0 || L <= 0) return cudaSuccess;
  cudaError_t e;
  if (a.max_seq > 0 && lrfu_slice(a.max_seq) <= kLrfuClCap) {
    // one cluster per row; the head reduction happens inside
    const int per = lrfu_slice(a.max_seq);
    const size_t sm = sizeof(LrfuClSmem) + size_t(per) * (sizeof(uint32_t) + 1);
    e = cudaFuncSetAttribute(lrfu_select_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    if (e != cudaSuccess) return e;
    lrfu_select_cluster_kernel<<<dim3(kCl, L, R), kClThreads, sm, st>>>(a);
    return cudaGetLastError();
  }
  headmean_kernel<<<dim3(reduce_ctas_per_row(R * L), L, R), kReduceThreads, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // the row lengths are on the device: room for kLrfuKeyCap keys, rows beyond it use global memory
  const size_t sm = sizeof(LrfuSelSmem) + size_t(kLrfuKeyCap) * sizeof(uint32_t);
  e = cudaFuncSetAttribute(lrfu_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  if (e != cudaSuccess) return e;
  lrfu_select_kernel<<<dim3(L, R), kSelThreads, sm, st>>>(a);
  return cudaGetLastError();
}

}  // namespace actkv
