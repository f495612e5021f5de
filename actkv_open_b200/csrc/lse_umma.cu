// Causal log-sum-exp of the action region on the sm_100a tensor cores (tcgen05 + TMA + TMEM).
//
// The eviction step consumes lse[l, j, hq] = log sum_{t <= S-A+j} exp(scale * q[j, hq] . k[t, h])
// for every action token j of every session: the LSE by-product of the attention backend, which
// the reference takes from paged_decode_attention_ref called with seq_used = S - A + j + 1
// (actkv/kernels/lse_attn.py:42-60; causal region as in the eviction glue).  Here it is computed
// directly from the paged cache, for all layers and sessions in one launch:
//
//   unit = (session r, layer l, KV head h, token split sp, row group rg): up to kGroupBlocks row
//   blocks of 128 query rows (row = j*G + g of action token j) resident in shared memory, against
//   the split's key tiles of 128 tokens.  Each key tile is read once and used by every row block
//   of the group (streaming it once per row block measured TMA-bound at ~4 TB/s of 2 KB boxes).
//   MMA:      X_b[128 rows, 128 tokens] = Q_b[128, D] * K_tile[128, D]^T per row block b
//             (M=128, N=128, 8 K=16 steps), into TMEM slot b (4 slots x 128 columns)
//   epilogue: one thread per row and warpgroup (four warpgroups, warpgroup w owns the token
//             columns [32w, 32w+32) of every slot): online max m and sum s of
//             2^(x * scale * log2 e) over the visible tokens (t <= S - A + j), one partial (m, s)
//             per (row, split, warpgroup)
//   lse_combine_kernel merges a row's partials: lse = ln 2 * (M + log2 sum_i s_i 2^(m_i - M)).
//
// Warp roles as in the scoring kernel: warp 0 TMA producer (the group's Q rows once per unit;
// K tiles of 128 tokens = 128/BS paged blocks through a 2-stage ring, one TMA box per block and
// D-half; the next tile's block ids read before waiting for a stage), warp 1 TMEM allocator +
// single-thread MMA issuer, warps 2-17 the four epilogue warpgroups (the exponentials bound the
// kernel; four warps per scheduler keep the MUFU unit fed across the load and max phases).  Each
// TMEM slot has its own full / empty barriers, and the epilogue hands a slot back as soon as it
// holds the values in registers, so the MMAs of the next tile's row block b overlap the math.
// Units are dealt round-robin over the persistent CTAs; a split is at most kLseSplitTiles tiles,
// which bounds the cost of one unit (load balance over mixed lengths).
//
// Every wait is bounded (sets ACTKV_DEV_TIMEOUT, raises a shared abort flag, unwinds and frees
// TMEM); no trap, no unbounded spin.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"
#include "umma_common.cuh"

namespace actkv {
namespace lse_umma {

using namespace umma;

constexpr int kEpiGroups = kLseParts;                     // epilogue warpgroups, 32 token columns each
constexpr int kThreads = 64 + 128 * kEpiGroups;
constexpr int kRows = 128;                                // query rows per row block (MMA M)
constexpr int kTileN = kLseTileTokens;                    // tokens per key tile (MMA N)
constexpr int kGroupBlocks = 4;                           // row blocks resident per unit (TMEM slots)
constexpr int kKStages = 2;
constexpr uint32_t kQBlockBytes = 2 * kRows * 128;        // two D-halves of 128 rows x 128 B
constexpr uint32_t kKStageBytes = 2 * kTileN * 128;       // two D-halves of 128 rows x 128 B
constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = kGroupBlocks * kQBlockBytes;
constexpr uint32_t kBarOff = kKOff + kKStages * kKStageBytes;
// barriers: k_full[2] k_empty[2] q_full q_empty acc_full[4] acc_empty[4], then the TMEM address
// and the abort flag
constexpr uint32_t kNumBars = 2 * kKStages + 2 + 2 * kGroupBlocks;
constexpr uint32_t kSmemBytes = kBarOff + kNumBars * 8 + 16;
static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA can have");
static_assert(kTileN == 128 && kGroupBlocks * kTileN == 512, "one TMEM slot of 128 columns per row block");
static_assert(kEpiGroups * 32 == kTileN, "each epilogue warpgroup owns 32 columns of a slot");

struct LUnit {
  int r, l, h, sp, rg;
  int S, A, a0;
  int j0, nb;                   // first action token of the group, row blocks in it
  int t0, t1;                   // key tiles [t0, t1) of this split that some row of the group sees
};

// Units of session r: L * Hkv * nsp * ngroups, ordered (l, h, sp, rg).  CTA c takes units c,
// c + grid, c + 2 grid, ...; every thread walks the same sequence.
struct LWalker {
  const LseArgs* a;
  int G;
  int64_t u, step, base, n_r;
  int r, S, A, a0, nrb, ngr, nsp;

  __device__ void load(int rr) {
    S = a->seq_used[rr];
    a0 = a->act_off[rr];
    A = a->act_off[rr + 1] - a0;
    nrb = A > 0 ? (A * G + kRows - 1) / kRows : 0;
    ngr = (nrb + kGroupBlocks - 1) / kGroupBlocks;
    const int T = (S + kTileN - 1) / kTileN;
    nsp = (T + kLseSplitTiles - 1) / kLseSplitTiles;
    if (nsp > a->nsplit) nsp = a->nsplit;     // the host checks max_seq; flagged by the combine
    n_r = int64_t(a->L) * a->Hkv * nsp * ngr;
  }
  __device__ void init(const LseArgs* args) {
    a = args;
    G = a->G;
    u = blockIdx.x;
    step = gridDim.x;
    base = 0;
    r = 0;
    if (a->R > 0) load(0);
  }
  __device__ bool next(LUnit& x) {
    while (r < a->R && u >= base + n_r) {
      base += n_r;
      ++r;
      if (r < a->R) load(r);
    }
    if (r >= a->R) return false;
    int64_t v = u - base;
    x.rg = int(v % ngr);
    v /= ngr;
    x.sp = int(v % nsp);
    v /= nsp;
    x.h = int(v % a->Hkv);
    x.l = int(v / a->Hkv);
    x.r = r;
    x.S = S;
    x.A = A;
    x.a0 = a0;
    x.j0 = x.rg * kGroupBlocks * (kRows / G);
    x.nb = min(kGroupBlocks, nrb - x.rg * kGroupBlocks);
    const int j_last = min(A, x.j0 + x.nb * (kRows / G)) - 1;
    const int last_tok = S - A + j_last;                     // the group's last visible token
    const int T_u = last_tok >= 0 ? last_tok / kTileN + 1 : 0;
    x.t0 = x.sp * kLseSplitTiles;
    x.t1 = min(T_u, x.t0 + kLseSplitTiles);
    u += step;
    return true;
  }
};

template <int G, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    lse_umma_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_q,
                    LseArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kBarOff + kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kBarOff + kNumBars * 8 + 4);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int B_KFULL = 0, B_KEMPTY = kKStages, B_QFULL = 2 * kKStages, B_QEMPTY = 2 * kKStages + 1,
            B_AFULL = 2 * kKStages + 2, B_AEMPTY = 2 * kKStages + 2 + kGroupBlocks;
  const unsigned full = 0xffffffffu;

  if ((base & 1023u) != 0) {                    // swizzled operands need 1024-byte alignment
    if (threadIdx.x == 0) flag(a.status, ACTKV_DEV_MISALIGNED);
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(bar(B_KFULL + i), 1);
      mbar_init(bar(B_KEMPTY + i), 1);
    }
    mbar_init(bar(B_QFULL), 1);
    mbar_init(bar(B_QEMPTY), 1);
    for (int i = 0; i < kGroupBlocks; ++i) {
      mbar_init(bar(B_AFULL + i), 1);
      mbar_init(bar(B_AEMPTY + i), 4 * kEpiGroups);   // one arrive per epilogue warp
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  LWalker wk;
  wk.init(&a);
  LUnit x;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_k)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_q)) : "memory");
    }
    const int bpt = kTileN / a.BS;               // paged blocks per key tile (<= 16: one per lane)
    // lane b's block id of key tile t (block b of the tile); -2 past the session's blocks
    auto read_id = [&](const LUnit& u, int t) -> int {
      const int first = t * bpt;
      if (lane >= min(bpt, (u.S + a.BS - 1) / a.BS - first)) return -2;
      const int lb = first + lane;
      return lb < a.MB ? a.block_table[u.r * a.bt_stride_r + lb] : -1;
    };
    uint32_t kiter = 0, qiter = 0;
    bool ok = true;
    while (ok && wk.next(x)) {
      if (x.t0 >= x.t1) continue;
      int id = read_id(x, x.t0);                  // in flight while waiting for the query buffer
      bool w = mbar_wait(bar(B_QEMPTY), (qiter & 1u) ^ 1u, abort_flag, a.status);
      if (!__all_sync(full, w)) break;
      if (lane == 0) {
        mbar_expect_tx(bar(B_QFULL), uint32_t(x.nb) * kQBlockBytes);
        for (int b = 0; b < x.nb; ++b)
          for (int hf = 0; hf < 2; ++hf)
            tma_load_4d(base + kQOff + b * kQBlockBytes + hf * (kQBlockBytes / 2), &tmap_q, bar(B_QFULL), hf * 64,
                        x.h * G, x.a0 + x.j0 + b * (kRows / G), x.l);
      }
      ++qiter;
      for (int t = x.t0; t < x.t1; ++t) {
        const int cur = id;
        if (t + 1 < x.t1) id = read_id(x, t + 1);   // in flight while this tile waits for a stage
        const int stage = kiter % kKStages;
        w = mbar_wait(bar(B_KEMPTY + stage), ((kiter / kKStages) & 1u) ^ 1u, abort_flag, a.status);
        if (!__all_sync(full, w)) {
          ok = false;
          break;
        }
        const int nblk = min(bpt, (x.S + a.BS - 1) / a.BS - t * bpt);
        int phys = 0;
        if (lane < nblk) {
          phys = cur;
          if (phys < 0 || phys >= a.NB) {
            flag(a.status, ACTKV_DEV_BAD_INDEX);
            phys = 0;
          }
        }
        if (lane == 0) mbar_expect_tx(bar(B_KFULL + stage), uint32_t(nblk) * a.BS * 128u * 2u);
        __syncwarp();
        // lane b copies paged block b (both D-halves): the boxes go out in parallel
        const uint32_t kdst = base + kKOff + stage * kKStageBytes;
        if (lane < nblk)
          for (int hf = 0; hf < 2; ++hf)
            tma_load_4d(kdst + hf * (kKStageBytes / 2) + lane * a.BS * 128, &tmap_k, bar(B_KFULL + stage), hf * 64,
                        x.h, phys * a.BS, x.l);
        ++kiter;
      }
    }
    if (*abort_flag && lane == 0) {
      // let copies already issued land before the CTA can exit (bounded)
      for (int s = 0; s < kKStages; ++s) {
        const uint32_t uses = kiter / kKStages + (uint32_t(s) < kiter % kKStages ? 1u : 0u);
        if (uses) mbar_drain(bar(B_KFULL + s), (uses - 1) & 1u);
      }
      if (qiter) mbar_drain(bar(B_QFULL), (qiter - 1) & 1u);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t idesc = instr_desc_mn(kRows, kTileN, BF16);
    uint32_t kiter = 0, qiter = 0;
    uint32_t slot_uses[kGroupBlocks] = {0, 0, 0, 0};
    int last_commit_bar = -1;
    uint32_t last_commit_parity = 0;
    bool ok = true;
    while (ok && wk.next(x)) {
      if (x.t0 >= x.t1) continue;
      if (!mbar_wait(bar(B_QFULL), qiter & 1u, abort_flag, a.status)) break;
      ++qiter;
      for (int t = x.t0; t < x.t1 && ok; ++t) {
        const int stage = kiter % kKStages;
        if (!mbar_wait(bar(B_KFULL + stage), (kiter / kKStages) & 1u, abort_flag, a.status)) {
          ok = false;
          break;
        }
        const uint32_t kaddr = base + kKOff + stage * kKStageBytes;
        for (int b = 0; b < x.nb; ++b) {
          if (!mbar_wait(bar(B_AEMPTY + b), (slot_uses[b] & 1u) ^ 1u, abort_flag, a.status)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t qaddr = base + kQOff + b * kQBlockBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t qoff = (k >> 2) * (kQBlockBytes / 2) + (k & 3) * 32;
            const uint32_t koff = (k >> 2) * (kKStageBytes / 2) + (k & 3) * 32;
            mma_f16(tmem + b * kTileN, sw128_desc(qaddr + qoff), sw128_desc(kaddr + koff), idesc, k > 0);
          }
          mma_commit(bar(B_AFULL + b));
          last_commit_bar = B_AFULL + b;
          last_commit_parity = slot_uses[b] & 1u;
          ++slot_uses[b];
        }
        if (!ok) break;
        mma_commit(bar(B_KEMPTY + stage));
        ++kiter;
      }
      if (!ok) break;
      mma_commit(bar(B_QEMPTY));                  // the unit's queries are no longer read
    }
    if (*abort_flag && last_commit_bar >= 0) mbar_drain(bar(last_commit_bar), last_commit_parity);
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ epilogue (4 x 4 warps)
    // Warp w reads TMEM lanes 32 (w % 4) .. + 31 = rows of every slot; warpgroup wg owns the
    // token columns [32 wg, 32 wg + 32) of every slot.
    const int wg = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(wg * 32);
    const float c2 = a.scale * kLog2e;
    const float ninf = -__int_as_float(0x7f800000);
    uint32_t slot_uses[kGroupBlocks] = {0, 0, 0, 0};
    bool ok = true;
    while (ok && wk.next(x)) {
      float m[kGroupBlocks], s[kGroupBlocks];
      int lim[kGroupBlocks];
#pragma unroll
      for (int b = 0; b < kGroupBlocks; ++b) {
        m[b] = ninf;
        s[b] = 0.0f;
        lim[b] = x.S - x.A + x.j0 + (b * kRows + row) / G;   // last token row b sees
      }
      for (int t = x.t0; t < x.t1 && ok; ++t) {
#pragma unroll
        for (int b = 0; b < kGroupBlocks; ++b) {
          if (b >= x.nb) break;
          const bool w = mbar_wait(bar(B_AFULL + b), slot_uses[b] & 1u, abort_flag, a.status);
          if (!__all_sync(full, w)) {
            ok = false;
            break;
          }
          fence_after();
          const int tok0 = t * kTileN + wg * 32;   // token of this warpgroup's first column
          float v[32];
          tmem_ld32(lane_addr + b * kTileN, v);
          tmem_wait(v);
          // loaded: the slot goes back to the tensor core before the math
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_AEMPTY + b));
          ++slot_uses[b];
          const int lb = lim[b];
          float mx = ninf;
          if (tok0 + 31 <= lb) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) mx = fmax3(mx, v[i], v[i + 1]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v[i] = tok0 + i <= lb ? v[i] : ninf;
              mx = fmaxf(mx, v[i]);
            }
          }
          if (mx != ninf) {                         // scale > 0: the max commutes with it
            const float mn = fmaxf(m[b], mx * c2);
            float acc0 = s[b] * ex2(m[b] - mn), acc1 = 0.0f;   // 0 while m is still -inf
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              acc0 += ex2(fmaf(v[i], c2, -mn));
              acc1 += ex2(fmaf(v[i + 1], c2, -mn));
            }
            m[b] = mn;
            s[b] = acc0 + acc1;
          }
        }
      }
      if (!ok) break;
#pragma unroll
      for (int b = 0; b < kGroupBlocks; ++b) {
        const int rr = b * kRows + row;
        const int j = x.j0 + rr / G, g = rr % G;
        if (b < x.nb && j < x.A) {
          float2* p = a.part +
                      (((int64_t(x.l) * a.sum_A + x.a0 + j) * a.Hq + x.h * G + g) * a.nsplit + x.sp) * kLseParts + wg;
          *p = make_float2(m[b], s[b]);
        }
      }
    }
    fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace lse_umma

// Merges each row's partials into its natural-log lse: one warp per row, its lanes reading the
// row's contiguous partials (coalesced), warp max and sum.  Grid (layer, session, row chunk); the
// row chunks stride over the session's A * Hq rows.  Rows that see no token (more action tokens
// than tokens) get -inf and flag ACTKV_DEV_BAD_INDEX, as does a session longer than the
// workspace's split count allows.
constexpr int kCombineThreads = 256;
constexpr int kCombineChunks = 16;

__global__ void __launch_bounds__(kCombineThreads) lse_combine_kernel(LseArgs a) {
  const int l = blockIdx.x, r = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.seq_used[r], a0 = a.act_off[r], A = a.act_off[r + 1] - a0;
  const int T = (S + kLseTileTokens - 1) / kLseTileTokens;
  int nsp = (T + kLseSplitTiles - 1) / kLseSplitTiles;
  if (nsp > a.nsplit) {
    if (threadIdx.x == 0 && blockIdx.z == 0) flag(a.status, ACTKV_DEV_BAD_INDEX);
    nsp = a.nsplit;
  }
  const int np = kLseParts * nsp;
  const float ninf = -__int_as_float(0x7f800000);
  const int wpb = kCombineThreads / 32;
  for (int idx = blockIdx.z * wpb + warp; idx < A * a.Hq; idx += gridDim.z * wpb) {
    const int j = idx / a.Hq, hq = idx % a.Hq;
    const float2* p = a.part + ((int64_t(l) * a.sum_A + a0 + j) * a.Hq + hq) * a.nsplit * kLseParts;
    float M = ninf;
    for (int i = lane; i < np; i += 32) M = fmaxf(M, p[i].x);
    M = warp_max(M);
    float lse = ninf;
    if (M != ninf) {
      float sum = 0.0f;
      for (int i = lane; i < np; i += 32) {
        const float2 v = p[i];
        if (v.x != ninf) sum += v.y * exp2f(v.x - M);
      }
      sum = warp_sum(sum);
      lse = (M + log2f(sum)) * 0.69314718055994531f;
    } else if (lane == 0) {
      flag(a.status, ACTKV_DEV_BAD_INDEX);
    }
    if (lane == 0) a.lse[int64_t(l) * a.lse_stride_l + int64_t(a0 + j) * a.lse_stride_a + hq] = lse;
  }
}

bool lse_umma_supported(const LseArgs& a, int kv_dtype, int q_dtype, const char** why) {
  auto no = [&](const char* w) {
    if (why) *why = w;
    return false;
  };
  if (kv_dtype != q_dtype || (kv_dtype != ACTKV_BF16 && kv_dtype != ACTKV_F16))
    return no("needs bf16 or fp16 q and cache of the same dtype");
  if (a.D != 128) return no("needs head_dim 128");
  if (!(a.G == 1 || a.G == 2 || a.G == 4 || a.G == 8 || a.G == 16)) return no("GQA group must be 1,2,4,8 or 16");
  if (a.BS % 8 != 0 || kLseTileTokens % a.BS != 0) return no("block_size must divide 128 and be a multiple of 8");
  if (a.kv_stride_b != int64_t(a.BS) * a.kv_stride_s) return no("kv blocks must be contiguous slots");
  const int64_t es = 2;
  if ((reinterpret_cast<uintptr_t>(a.kv) | reinterpret_cast<uintptr_t>(a.q)) % 16)
    return no("q and kv must be 16-byte aligned");
  if ((a.kv_stride_h * es) % 16 || (a.kv_stride_s * es) % 16 || (a.kv_stride_l * es) % 16)
    return no("kv strides must be multiples of 16 bytes");
  if ((a.q_stride_h * es) % 16 || (a.q_stride_a * es) % 16 || (a.q_stride_l * es) % 16)
    return no("q strides must be multiples of 16 bytes");
  return true;
}

template <int G, bool BF16>
static cudaError_t launch_lse_g(const CUtensorMap& mk, const CUtensorMap& mq, const LseArgs& a, int grid,
                                cudaStream_t st) {
  auto k = lse_umma::lse_umma_kernel<G, BF16>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(lse_umma::kSmemBytes));
  if (e != cudaSuccess) return e;
  k<<<grid, lse_umma::kThreads, lse_umma::kSmemBytes, st>>>(mk, mq, a);
  return cudaGetLastError();
}

template <bool BF16>
static cudaError_t launch_lse_t(const CUtensorMap& mk, const CUtensorMap& mq, const LseArgs& a, int grid,
                                cudaStream_t st) {
  switch (a.G) {
    case 1: return launch_lse_g<1, BF16>(mk, mq, a, grid, st);
    case 2: return launch_lse_g<2, BF16>(mk, mq, a, grid, st);
    case 4: return launch_lse_g<4, BF16>(mk, mq, a, grid, st);
    case 8: return launch_lse_g<8, BF16>(mk, mq, a, grid, st);
    default: return launch_lse_g<16, BF16>(mk, mq, a, grid, st);
  }
}

cudaError_t launch_region_lse(const LseArgs& a, int dtype, int grid, cudaStream_t st, const char** why) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    if (why) *why = "cuTensorMapEncodeTiled unavailable";
    return cudaErrorNotSupported;
  }
  const CUtensorMapDataType dt = dtype == ACTKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mk, mq;
  {
    const cuuint64_t dims[4] = {cuuint64_t(a.D), cuuint64_t(a.Hkv), cuuint64_t(a.NB) * a.BS, cuuint64_t(a.L)};
    const cuuint64_t strides[3] = {cuuint64_t(a.kv_stride_h) * 2, cuuint64_t(a.kv_stride_s) * 2,
                                   cuuint64_t(a.kv_stride_l) * 2};
    const cuuint32_t box[4] = {64, 1, cuuint32_t(a.BS), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&mk, dt, 4, const_cast<void*>(a.kv), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      if (why) *why = "cuTensorMapEncodeTiled rejected the K cache layout";
      return cudaErrorInvalidValue;
    }
  }
  {
    const cuuint64_t dims[4] = {cuuint64_t(a.D), cuuint64_t(a.Hq), cuuint64_t(a.sum_A), cuuint64_t(a.L)};
    const cuuint64_t strides[3] = {cuuint64_t(a.q_stride_h) * 2, cuuint64_t(a.q_stride_a) * 2,
                                   cuuint64_t(a.q_stride_l) * 2};
    const cuuint32_t box[4] = {64, cuuint32_t(a.G), cuuint32_t(lse_umma::kRows / a.G), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&mq, dt, 4, const_cast<void*>(a.q), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      if (why) *why = "cuTensorMapEncodeTiled rejected the query layout";
      return cudaErrorInvalidValue;
    }
  }
  cudaError_t e = dtype == ACTKV_BF16 ? launch_lse_t<true>(mk, mq, a, grid, st) : launch_lse_t<false>(mk, mq, a, grid, st);
  if (e != cudaSuccess) {
    if (why) *why = "lse_umma_kernel launch";
    return e;
  }
  lse_combine_kernel<<<dim3(a.L, a.R, kCombineChunks), kCombineThreads, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess && why) *why = "lse_combine_kernel launch";
  return e;
}

}  // namespace actkv
