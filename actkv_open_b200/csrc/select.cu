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

#include <cstddef>

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
  pdl_wait();                                   // launched by launch_pdl: see common.cuh
  pdl_trigger();
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
// per CTA and publishes it (with its sums per group of 32 bins) in the CTA's own shared memory;
// after one cluster barrier every CTA reads the group sums of all CTAs, then the 32 bins of the
// crossing group, through distributed shared memory and finds the crossing bin itself.  Every sum
// over the CTAs is taken in rank order, so all CTAs reach the same result and it does not depend on
// timing.  Barriers: a CTA publishes only after every CTA has finished reading its previous publish
// (the arrive after the reads, the wait before the next publish), and waits once more before it
// exits, so no CTA reads the shared memory of a CTA that has moved on or exited.
constexpr int kCl = 4;
constexpr int kGroups = kBins / 32;

// The two halves of a cluster barrier, for every thread of every CTA of the cluster (in order:
// arrive, wait, arrive, wait, ...).  arrive releases this thread's earlier shared-memory accesses
// (reads of other CTAs included); wait acquires every other thread's.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory"); }

// Distributed shared memory through shared::cluster addresses: dsmem(p, q) is the address of the
// variable at p in the shared memory of cluster rank q; the loads read it there.
__device__ __forceinline__ uint32_t dsmem(const void* p, unsigned q) {
  uint32_t a;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(uint32_t(__cvta_generic_to_shared(p))), "r"(q));
  return a;
}
__device__ __forceinline__ uint32_t ld_dsmem(uint32_t a, uint32_t) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ unsigned long long ld_dsmem(uint32_t a, unsigned long long) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(a));
  return v;
}
// Two consecutive values in one request (the address aligned to their combined size).
__device__ __forceinline__ void ld_dsmem2(uint32_t a, uint32_t& x, uint32_t& y) {
  asm volatile("ld.shared::cluster.v2.u32 {%0, %1}, [%2];" : "=r"(x), "=r"(y) : "r"(a));
}
__device__ __forceinline__ void ld_dsmem2(uint32_t a, unsigned long long& x, unsigned long long& y) {
  asm volatile("ld.shared::cluster.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "r"(a));
}

// Suffix sum over the lanes of a warp: lane i gets the sum over lanes >= i.
template <typename W>
__device__ __forceinline__ W warp_suffix_sum(W v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const W y = __shfl_down_sync(0xffffffffu, v, o);
    if (lane + o < 32) v += y;
  }
  return v;
}

// One CTA's copy of a radix pass's result over the cluster (warp 0 writes it).
template <typename W>
struct Crossing {
  W above;                  // weight of the bins above the crossing bin
  uint32_t bin;             // the crossing bin
  uint32_t count;           // keys in it, over the cluster
  uint32_t eq_before;       // keys in it in the CTAs of lower rank
  uint32_t found;           // 0: the cluster's total weight is below need
};

// The crossing bin of a radix pass over the cluster: the highest bin whose weight above it is
// < need <= its weight plus the weight above it.  Every CTA publishes, at the same offsets of its
// own shared memory, its bins' weights (bins[kBins]), their sums per group of 32 bins
// (groups[kGroups]) and its bins' key counts (counts; nullptr when the weights are the counts).
// Warp 0 of every CTA, after the barrier that follows the publish: the group sums of all CTAs, then
// the 32 bins of the crossing group, each summed in rank order, so every CTA finds the same bin.
// Remote reads cost per request, so each lane takes its two groups in one request and only the
// lane of the crossing bin reads the counts.  groups: aligned to 2 * sizeof(W).
template <typename W>
__device__ void cluster_crossing(cg::cluster_group& cl, const W* bins, const W* groups, const uint32_t* counts,
                                 W need, Crossing<W>* out) {
  const int lane = threadIdx.x & 31;
  const unsigned me = cl.block_rank();
  W g_lo = 0, g_hi = 0;                                // groups 2 * lane and 2 * lane + 1
  {
    W lo[kCl], hi[kCl];                                // every load issued before the sums
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q) ld_dsmem2(dsmem(groups + 2 * lane, q), lo[q], hi[q]);
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q) {
      g_lo += lo[q];
      g_hi += hi[q];
    }
  }
  const W pair = g_lo + g_hi;
  const W incl = warp_suffix_sum(pair);
  const W above_pair = incl - pair;
  const unsigned hit = __ballot_sync(0xffffffffu, above_pair < need && need <= incl);
  if (hit == 0) {                                      // uniform over the warp
    if (lane == 0) out->found = 0;
    return;
  }
  const int src = __ffs(hit) - 1;
  W above = __shfl_sync(0xffffffffu, above_pair, src);
  const W hi_w = __shfl_sync(0xffffffffu, g_hi, src);
  int group = 2 * src + 1;
  if (need > above + hi_w) {
    group = 2 * src;
    above += hi_w;
  }
  const int b = group * 32 + lane;
  W w = 0, wq[kCl];
#pragma unroll
  for (unsigned q = 0; q < kCl; ++q) wq[q] = ld_dsmem(dsmem(bins + b, q), W());
#pragma unroll
  for (unsigned q = 0; q < kCl; ++q) w += wq[q];
  const W above_b = above + (warp_suffix_sum(w) - w);
  const unsigned hb = __ballot_sync(0xffffffffu, w > 0 && above_b < need && need <= above_b + w);
  if (hb == 0) {                                       // cannot happen: the group holds the crossing
    if (lane == 0) out->found = 0;
    return;
  }
  if (lane == __ffs(hb) - 1) {
    uint32_t c = 0, c_before = 0;
    uint32_t cq[kCl];
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q)
      cq[q] = counts ? ld_dsmem(dsmem(counts + b, q), uint32_t()) : uint32_t(wq[q]);
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q) {
      c += cq[q];
      if (q < me) c_before += cq[q];
    }
    out->above = above_b;
    out->bin = uint32_t(b);
    out->count = c;
    out->eq_before = c_before;
    out->found = 1;
  }
}

// keep mask, one cluster per row: the same selection as keep_select_kernel (top `budget` keys,
// ties to the lowest index, protected tokens always kept).  Rows up to kCl * kSmemKeyCap tokens.
// One cluster barrier per radix pass (see cluster_crossing); the barrier that guards a CTA's
// published histogram against its next publish is split around the next pass's scan.
__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kSelThreads)
    keep_select_cluster_kernel(KeepMaskArgs a) {
  pdl_wait();                                   // launched by launch_pdl: see common.cuh
  pdl_trigger();
  extern __shared__ uint32_t skeys[];                 // this CTA's slice of the row
  __shared__ uint32_t hist[kBins];                    // this pass's counts (local)
  __shared__ uint32_t pub[kBins];                     // published: counts per bin
  __shared__ __align__(16) uint32_t gpub[kGroups];    // published: counts per group of 32 bins
  __shared__ uint32_t p_prot;                         // published: protected tokens in this slice
  __shared__ uint32_t c_prot;                         // the cluster's, summed in rank order
  __shared__ Crossing<uint32_t> sel;
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
  if (threadIdx.x == 0) p_prot = n_prot;
  cluster_arrive();
  cluster_wait();                                      // every CTA has started and published
  if (threadIdx.x == 0) {
    uint32_t tot = 0;
    uint32_t pq[kCl];
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q) pq[q] = ld_dsmem(dsmem(&p_prot, q), 0u);
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q) tot += pq[q];
    c_prot = tot;
  }
  __syncthreads();
  cluster_arrive();                                    // this CTA's reads of the others are done
  const uint32_t prot_total = c_prot;
  const int n_cand = n - int(prot_total);
  const int budget = a.budget[r];
  const bool keep_all = budget >= n_cand;
  const int k = keep_all ? n_cand : (budget > 0 ? budget : 0);
  if (keep_all || k == 0) {                            // uniform; no further cluster traffic
    for (int i = threadIdx.x; i < m; i += blockDim.x) keep[t0 + i] = keep_all ? 1 : (skeys[i] == 0);
    if (threadIdx.x == 0 && me == 0 && a.kept) a.kept[r] = keep_all ? n : int(prot_total);
    cluster_wait();                                    // no CTA still reads this one's shared memory
    return;
  }
  uint32_t prefix = 0, pmask = 0, need = uint32_t(k), eq_count = 0, eq_before = 0;
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
    cluster_wait();                                    // no CTA still reads what this one published
    for (int g = int(threadIdx.x >> 5); g < kGroups; g += int(blockDim.x >> 5)) {
      const int b = g * 32 + int(threadIdx.x & 31);
      const uint32_t v = hist[b];
      pub[b] = v;
      const uint32_t gs = warp_sum(v);
      if ((threadIdx.x & 31) == 0) gpub[g] = gs;
    }
    cluster_arrive();
    cluster_wait();                                    // every CTA's histogram is published
    if (threadIdx.x < 32) cluster_crossing<uint32_t>(cl, pub, gpub, nullptr, need, &sel);
    __syncthreads();
    cluster_arrive();                                  // this CTA's reads of the others are done
    if (!sel.found) {                                  // cannot happen: k <= #candidates (uniform)
      if (threadIdx.x == 0 && me == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      cluster_wait();
      return;
    }
    need -= sel.above;
    eq_count = sel.count;
    eq_before = sel.eq_before;
    prefix |= sel.bin << shift;
    pmask |= dmask << shift;
  }
  // ties at the threshold go to the lowest index: the last pass resolved every bit of the keys,
  // so its crossing bin counted exactly the keys equal to it, eq_before of them before this slice
  const bool ties = eq_count > need;
  uint32_t eq_seen = ties ? eq_before : 0u;
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
  cluster_wait();                                      // no CTA still reads this one's shared memory
}

cudaError_t launch_keep_mask(const KeepMaskArgs& a, int R, cudaStream_t st) {
  if (R <= 0) return cudaSuccess;
  cudaError_t e = launch_pdl(keep_reduce_kernel, dim3(reduce_ctas_per_row(R), R), dim3(kReduceThreads), 0, st, a);
  if (e != cudaSuccess) return e;
  if (a.max_seq <= int64_t(kCl) * kSmemKeyCap) {
    // a cluster of kCl CTAs per row, each with its slice of the keys in shared memory
    const int per = int((a.max_seq + kCl - 1) / kCl);
    const size_t sm = size_t(per > 0 ? per : 1) * sizeof(uint32_t);
    e = cudaFuncSetAttribute(keep_select_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    if (e != cudaSuccess) return e;
    return launch_pdl(keep_select_cluster_kernel, dim3(kCl, R), dim3(kSelThreads), sm, st, a);
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
// keys (and its exclusion flags) in shared memory.  Rows up to kCl * kLrfuClCap tokens (132,656;
// the 16-bit mass pieces of one CTA cannot overflow).
//
// One cluster barrier per radix pass: each CTA publishes its bin masses and counts, and the masses
// of each group of 32 bins, in its own shared memory; after the barrier every CTA finds the
// crossing bin itself (the group masses of all CTAs, then the 32 bins of the crossing group, each
// summed in rank order, so every CTA reaches the same bin).  The barrier that keeps a CTA from
// republishing while another still reads it is split in two: the arrive follows this CTA's
// reads, the wait precedes its next publish, so the next pass's scan of the keys runs in between.
// After the last pass every key is resolved, so a CTA's count in the crossing bin is its number
// of keys equal to the threshold: the tie ranks come from the same reads.

struct LrfuClSmem {
  uint32_t h16[4][kBins];                   // this pass's 16-bit mass pieces (local)
  uint32_t hcl[kBins];                      // this pass's counts (local)
  unsigned long long hm[kBins];             // published: mass per bin
  unsigned long long gm[kGroups];           // published: mass per group of 32 bins
  uint32_t hc[kBins];                       // published: count per bin
  double p_total;                           // published: this slice's sum, max and positives
  float p_vmax;
  int p_npos;
  double c_total;                           // the cluster's, combined in rank order
  float c_vmax;
  int c_npos;
  Crossing<unsigned long long> sel;         // this pass's result (warp 0 writes)
  double dred[32];
  float fred[32];
  int ired[33];
};
// keys (4 B) and exclusion flags (1 B) per token of a CTA's slice beside LrfuClSmem in 227 KB
constexpr int kLrfuClCap = 33164;
// Tokens of a row per CTA of the ActionLRFU cluster: a multiple of 4, so that every slice starts
// on a 16-byte boundary of the row (the head reduction reads 4 tokens per load).
__host__ __device__ inline int lrfu_slice(int64_t n) { return int(((n + kCl - 1) / kCl + 3) & ~int64_t(3)); }
static_assert(sizeof(LrfuClSmem) + size_t(kLrfuClCap) * 5 <= 232448, "LRFU cluster select exceeds 227 KB");
static_assert(offsetof(LrfuClSmem, gm) % 16 == 0, "group masses are read two per 16-byte request");
static_assert(kLrfuClCap <= 65535 && kLrfuClCap % 4 == 0, "16-bit mass pieces per CTA; slices of whole 4-token groups");
static_assert(int64_t(kCl) * kLrfuClCap >= 131072, "a 131072-token row takes the cluster path");

constexpr int kClThreads = 512;                      // 2 CTAs per SM: a config-2 step's rows in one wave

__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kClThreads, 2)
    lrfu_select_cluster_kernel(LrfuArgs a) {
  pdl_wait();                                   // launched by launch_pdl: see common.cuh
  pdl_trigger();
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
  // every 128-byte line of the slice's per-head scores and keep scores asked of L2 up front: the
  // head reduction's loads, limited by the registers a thread can keep in flight, and the final
  // pass's then wait on L2 rather than on HBM
  {
    const int lines = (m * 4 + 127) / 128;            // (lines - 1) * 128 < m * 4: inside the row
    for (int j = threadIdx.x; j < lines * (a.H + 1); j += blockDim.x) {
      const int h = j / lines, k = j - h * lines;
      const char* row = h < a.H ? reinterpret_cast<const char*>(src + int64_t(h) * a.src_stride_h + t0)
                                : reinterpret_cast<const char*>(ks + t0);
      asm volatile("prefetch.L2 [%0];" ::"l"(row + k * 128));
    }
  }

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

  // the row's sum, maximum and positive count: published here, read from every CTA after one
  // barrier and combined in rank order (the same values in every CTA)
  if (threadIdx.x == 0) {
    sm.p_total = total;
    sm.p_vmax = vmax;
    sm.p_npos = n_pos;
  }
  cluster_arrive();
  cluster_wait();                                      // every CTA has started and published
  if (threadIdx.x == 0) {
    double tt = 0.0;
    float vm = 0.0f;
    int np = 0;
    unsigned long long tq[kCl];
    uint32_t vq[kCl], nq[kCl];
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q) {
      tq[q] = ld_dsmem(dsmem(&sm.p_total, q), 0ull);
      vq[q] = ld_dsmem(dsmem(&sm.p_vmax, q), 0u);
      nq[q] = ld_dsmem(dsmem(&sm.p_npos, q), 0u);
    }
#pragma unroll
    for (unsigned q = 0; q < kCl; ++q) {             // rank order
      tt += __longlong_as_double((long long)tq[q]);
      vm = fmaxf(vm, __uint_as_float(vq[q]));
      np += int(nq[q]);
    }
    sm.c_total = tt;
    sm.c_vmax = vm;
    sm.c_npos = np;
  }
  __syncthreads();
  cluster_arrive();                                    // this CTA's reads of the others are done
  total = sm.c_total;
  vmax = sm.c_vmax;
  n_pos = sm.c_npos;
  const float total_f = float(total);
  const bool any_hit = (a.n_act == nullptr || a.n_act[r] > 0) && total_f > 0.0f && n_pos > 0;

  bool hit_all = false;
  uint32_t tau = 0;
  unsigned long long take_eq = 0, eq_count = 0, eq_before = 0;
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
      for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        sm.hcl[i] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) sm.h16[c][i] = 0;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < m; i += blockDim.x) {
        const uint32_t u = skeys[i];
        if (u == 0 || (u & pmask) != prefix) continue;
        const int bin = int((u >> shift) & dmask);
        const unsigned long long mass = fixed_mass(u, F);
        atomicAdd(&sm.hcl[bin], 1u);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t part = unsigned(mass >> (16 * c)) & 0xFFFFu;
          if (part) atomicAdd(&sm.h16[c][bin], part);
        }
      }
      __syncthreads();
      cluster_wait();                                  // no CTA still reads what this one published
      // publish the bins' masses and counts and the mass of each group of 32 bins (warp w takes
      // groups w, w + 16, ...; lane i bin 32 g + i)
      for (int g = int(threadIdx.x >> 5); g < kGroups; g += int(blockDim.x >> 5)) {
        const int b = g * 32 + int(threadIdx.x & 31);
        unsigned long long v = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) v += (unsigned long long)sm.h16[c][b] << (16 * c);
        sm.hm[b] = v;
        sm.hc[b] = sm.hcl[b];
        v = warp_sum(v);
        if ((threadIdx.x & 31) == 0) sm.gm[g] = v;
      }
      cluster_arrive();
      cluster_wait();                                  // every CTA's histogram is published
      if (threadIdx.x < 32) cluster_crossing<unsigned long long>(cl, sm.hm, sm.gm, sm.hc, need, &sm.sel);
      __syncthreads();
      cluster_arrive();                                // this CTA's reads of the others are done
      if (!sm.sel.found) {                             // uniform over the cluster
        hit_all = pass == 0;                           // the target exceeds the whole mass: every positive
        if (pass > 0 && threadIdx.x == 0 && me == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
      } else {
        need -= sm.sel.above;
        eq_count = sm.sel.count;
        eq_before = sm.sel.eq_before;
        prefix |= sm.sel.bin << shift;
        pmask |= dmask << shift;
      }
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
  // keys equal to tau in the CTAs of lower rank: the last pass resolved every bit of the keys, so
  // its crossing bin counted exactly those
  unsigned long long eq_seen = ties ? eq_before : 0ull;
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
  cluster_wait();                                     // no CTA still reads this one's shared memory
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
    return launch_pdl(lrfu_select_cluster_kernel, dim3(kCl, L, R), dim3(kClThreads), sm, st, a);
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
