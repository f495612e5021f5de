// LSE-recovery scoring on a CTA pair of sm_100a tensor cores (tcgen05.mma.cta_group::2).
//
// Same computation as score_umma.cu (scores of every (session, layer, KV head) over the causal
// action region: X = K_h * Q_h^T, then per token max over the GQA group of exp(x*scale - lse),
// causal mask, sum over the action tokens; actkv/kernels/lse_attn.py:63-78 / :85-130), with the
// tile shared by the two CTAs of a cluster:
//
//   M = 256 tokens per unit: CTA k of the pair holds tokens [128k, 128k + 128) of the tile in its
//       shared memory (8 paged blocks of 16 gathered by TMA through the block table) and
//       receives their 128 accumulator rows in its TMEM
//   N = up to 256 query columns per MMA chunk: CTA k holds columns [k N/2, (k+1) N/2) in its
//       shared memory, so each SM stores and streams half of every query chunk
//
// One thread of the even CTA issues the MMAs for both SMs.  Per SM and per 128 cycles of tensor
// work the operands read from shared memory are 4 KB of K plus 4 KB of Q (8 KB of Q in the
// one-CTA kernel), and a CTA holds up to four resident query chunks (A*G <= 1024; config 3's
// widest regions) in 128 KB.  Wider regions (config 4: A*G = 2048) go through the block path: a
// block of up to 8 consecutive tiles takes the query chunks four at a time and re-reads its K tiles
// (from L2) once per group of four.
//
// Every operand arrives by TMA, so no thread writes operand shared memory inside the loop: the lse
// term rides on the tensor core as in score_umma.cu (a ninth K = 16 step, ones x the three-term
// bf16 split of -lse/scale), and the split rows come from a pre-pass (lse_split_kernel) into a
// [L][sumA][Hq][8] bf16 workspace, loaded like the queries.  Both CTAs' copies complete on the even
// CTA's barriers (cp.async.bulk.tensor .cta_group::2, no multicast); the MMA commits arrive on both
// CTAs' barriers (tcgen05.commit .multicast::cluster); the odd CTA's epilogue warps release an
// accumulator on the even CTA's barrier.
//
// Warp roles (320 threads per CTA, one CTA per SM, persistent clusters of two):
//   warp 0    TMA producer of this CTA's halves (lane b: paged block b of the CTA's 128 tokens)
//   warp 1    TMEM allocator (both CTAs); the even CTA's lane 0 issues the MMAs
//   warps 2-9 epilogue, two warpgroups folding 128 columns each of this CTA's 128 token rows
// Every wait is bounded (see score_umma.cu); a timeout sets ACTKV_DEV_TIMEOUT and unwinds.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "score_common.cuh"
#include "score_tc.cuh"
#include "umma_common.cuh"

namespace actkv {
namespace pair {

using namespace umma;

constexpr int kThreads = 320;
constexpr int kHalfM = 128;                                 // token rows per CTA
constexpr int kTile = 2 * kHalfM;                           // tokens per unit
constexpr int kIdsAhead = 4;
constexpr uint32_t kQSlotBytes = 2 * 128 * 128;             // 128 query rows x two 128-byte D-halves
constexpr uint32_t kKStageBytes = 2 * kHalfM * 128;         // 128 token rows x two D-halves
constexpr uint32_t kExtHalfBytes = 128 * 16;                // one K half (8 elements) of 128 rows
constexpr uint32_t kLseSlotBytes = 2 * kExtHalfBytes;       // TMA'd first half, zero second half
constexpr uint32_t kOnesBytes = 2 * kExtHalfBytes;
constexpr int kBlockTiles = 8;                              // tiles sharing one pass of a wide region's queries
constexpr int kPartSlots = 8;                               // >= kBlockTiles units between the warpgroups
constexpr uint16_t kPairMask = 0x3;

template <int QS>
struct Layout {
  static constexpr int kQSlots = QS;                        // resident query chunks
  static constexpr int kKStages = QS == 2 ? 4 : 2;
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kKOff = kQOff + QS * kQSlotBytes;
  static constexpr uint32_t kLseOff = kKOff + kKStages * kKStageBytes;
  static constexpr uint32_t kOnesOff = kLseOff + QS * kLseSlotBytes;
  static constexpr uint32_t kPartOff = kOnesOff + kOnesBytes;
  static constexpr uint32_t kPartCntOff = kPartOff + kPartSlots * 2 * 128 * 4;
  static constexpr uint32_t kBlkIdsOff = kPartCntOff + kPartSlots * 128 * 4;   // [kBlockTiles][16] block ids
  static constexpr uint32_t kBarOff = kBlkIdsOff + kBlockTiles * 16 * 4;
  // kfull[S] kempty[S] qfull[QS] qempty[QS] afull[2] aempty[2], then the TMEM address, abort flag
  static constexpr int kNumBars = 2 * kKStages + 2 * QS + 4;
  static constexpr uint32_t kSmemBytes = kBarOff + kNumBars * 8 + 16;
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA can have");
};

// K-major, no swizzle: core matrices of 8 rows x 16 bytes, 8-row groups 128 B apart (stride), the
// second K half (elements 8-15) of every row kExtHalfBytes after the first (leading offset).
__device__ __forceinline__ uint64_t ext_desc(uint32_t addr) {
  uint64_t d = uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(kExtHalfBytes >> 4) << 16;
  d |= uint64_t(128 >> 4) << 32;
  d |= uint64_t(1) << 46;
  return d;
}

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Tiled TMA load into this CTA's shared memory whose completion counts on a barrier of either CTA
// of the pair (bar: a shared::cluster address).  No multicast.
__device__ __forceinline__ void tma2_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma2_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once the MMAs issued so far complete) on the barrier at this offset in both CTAs.
__device__ __forceinline__ void commit2(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(kPairMask)
      : "memory");
}

// Columns of chunk c (N of the MMA: a multiple of 32 so that each CTA's half holds whole query
// tokens for G <= 16).
__device__ __forceinline__ int chunk_cols(int A, int c, int qpc, int G) { return min(256, (A - c * qpc) * G); }
__device__ __forceinline__ int chunk_n(int ncols) { return (ncols + 31) & ~31; }

// u is the tile `nb` tiles after `first` in the same (session, layer, head) segment of a region
// wider than the query slots: it joins first's block.
template <int QS>
__device__ __forceinline__ bool same_block(const Unit& u, const Unit& first, int nb) {
  return u.nch > QS && u.r == first.r && u.l == first.l && u.h == first.h && u.tile == first.tile + nb;
}

// WIDE: some region has more query chunks than slots (A*G > 256*QS); every unit then goes through
// the block path (a unit of a narrower region is a block of one tile), in which a wide region's
// block of up to kBlockTiles consecutive tiles takes its query chunks QS at a time through the
// slots and re-reads the block's K tiles (from L2) once per group; each tile's chunks are still
// folded in chunk order.
template <int G, bool BF16, int QS, bool WIDE, bool STREAMED>
__global__ void __launch_bounds__(kThreads, 1)
    score_pair_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_l, ScoreArgs a) {
  using Lay = Layout<QS>;
  constexpr int NK = Lay::kKStages;
  constexpr int QPC = 256 / G;                  // query tokens per chunk (both CTAs)
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  const uint32_t rank = cta_rank();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::kBarOff + Lay::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lay::kBarOff + Lay::kNumBars * 8 + 4);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int B_KFULL = 0, B_KEMPTY = NK, B_QFULL = 2 * NK, B_QEMPTY = 2 * NK + QS, B_AFULL = 2 * NK + 2 * QS,
            B_AEMPTY = 2 * NK + 2 * QS + 2;
  const unsigned full = 0xffffffffu;

  if ((base & 1023u) != 0) {                    // the same in both CTAs: both return here
    if (threadIdx.x == 0) flag(a.status, ACTKV_DEV_MISALIGNED);
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NK; ++i) {
      mbar_init(bar(B_KFULL + i), 1);          // the even CTA's arrive.expect_tx
      mbar_init(bar(B_KEMPTY + i), 1);         // the MMA commit
    }
    for (int i = 0; i < QS; ++i) {
      mbar_init(bar(B_QFULL + i), 1);
      mbar_init(bar(B_QEMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_AFULL + i), 1);
      mbar_init(bar(B_AEMPTY + i), 16);        // one arrive per epilogue warp of both CTAs
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // constant operand halves: the key-side lse tile (every row [1, 1, 1, 0, ...], second K half
  // zero) and the zero second K half of every lse slot
  {
    const __nv_bfloat16 one = __float2bfloat16_rn(1.0f), zero = __float2bfloat16_rn(0.0f);
    const uint4 ones = make_uint4(pack_bf16x2(one, one), pack_bf16x2(one, zero), 0u, 0u);
    for (int i = threadIdx.x; i < 128 * (2 + QS); i += kThreads) {
      const int row = i & 127, part = i >> 7;  // part 0, 1: the ones tile's halves; 2..: lse slots
      uint4* p;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (part < 2) {
        p = reinterpret_cast<uint4*>(smem + Lay::kOnesOff + part * kExtHalfBytes + row * 16);
        if (part == 0) v = ones;
      } else {
        p = reinterpret_cast<uint4*>(smem + Lay::kLseOff + (part - 2) * kLseSlotBytes + kExtHalfBytes + row * 16);
      }
      *p = v;
    }
  }
  for (int i = threadIdx.x; i < kPartSlots * 128; i += kThreads)
    reinterpret_cast<uint32_t*>(smem + Lay::kPartCntOff)[i] = 0u;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  cluster_sync();                               // barriers and constant tiles ready in both CTAs
  fence_after();
  const uint32_t tmem = *tmem_slot;

  Walker<kTile, STREAMED> wk;
  // every role walks the layer groups in order, this pair's share of each (one group of all
  // layers when nothing is streamed)
  // (STREAMED: the host streams the queries in by layer groups; which share a pair takes rotates
  // with the group, so that no pair takes the larger share of every group.  Otherwise one group,
  // and the loops below compile to a single walk.)
  const int n_lg = STREAMED ? a.n_lgroups : 1;
  auto start_group = [&](int g) {
    const int np = int(gridDim.x >> 1);
    if constexpr (STREAMED)
      wk.init(&a, QPC, (int(blockIdx.x >> 1) + g) % np, np, a.lgrp[g], a.lgrp[g + 1]);
    else
      wk.init(&a, QPC, blockIdx.x >> 1, np);
  };
  Unit x;
  const int bpc = kHalfM / a.BS;                // paged blocks per CTA per unit

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_k)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_q)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_l)) : "memory");
    }
    // valid paged blocks of unit y in CTA k's half
    auto half_blocks = [&](const Unit& y, int k) -> int {
      const int first = y.tile * 2 * bpc + k * bpc;
      return max(0, min(bpc, (y.S + a.BS - 1) / a.BS - first));
    };
    auto read_id = [&](const Unit& y) -> int {
      if (y.nch == 0 || (!WIDE && y.nch > QS)) return -2;     // units the loop below skips
      if (lane >= half_blocks(y, rank)) return -2;
      const int lb = y.tile * 2 * bpc + rank * bpc + lane;
      return lb < a.MB ? a.block_table[y.r * a.bt_stride_r + lb] : -1;
    };
    Walker<kTile, STREAMED> ahead;
    Unit y;
    int ids[kIdsAhead] = {};
    auto pop_id = [&]() -> int {
      const int cur = ids[0];
#pragma unroll
      for (int i = 0; i + 1 < kIdsAhead; ++i) ids[i] = ids[i + 1];
      ids[kIdsAhead - 1] = ahead.next(y) ? read_id(y) : -2;
      return cur;
    };
    uint32_t kiter = 0;
    uint32_t quses[QS];
#pragma unroll
    for (int i = 0; i < QS; ++i) quses[i] = 0;
    bool ok = true;
    // query chunk c of unit u's segment (this CTA's half) and its lse rows into slot `slot`
    auto load_q = [&](const Unit& u, int slot, int c) -> bool {
      const bool w = mbar_wait(bar(B_QEMPTY + slot), (quses[slot] & 1u) ^ 1u, abort_flag, a.status);
      if (!__all_sync(full, w)) return false;
      if (lane == 0) {
        const uint32_t qf = peer_addr(bar(B_QFULL + slot), 0);
        if (rank == 0) mbar_expect_tx(bar(B_QFULL + slot), 2 * (kQSlotBytes + kExtHalfBytes));
        const int n = chunk_n(chunk_cols(u.A, c, QPC, G));
        const int row0 = u.a0 + c * QPC + int(rank) * (n / (2 * G));
        const uint32_t dst = base + Lay::kQOff + slot * kQSlotBytes;
        for (int hf = 0; hf < 2; ++hf)
          tma2_load_4d(dst + hf * (kQSlotBytes / 2), &tmap_q, qf, hf * 64, u.h * G, row0, u.l);
        tma2_load_4d(base + Lay::kLseOff + slot * kLseSlotBytes, &tmap_l, qf, 0, u.h * G, row0, u.l);
      }
      __syncwarp();
      ++quses[slot];
      return true;
    };
    auto load_k = [&](const Unit& u, int id) -> bool {
      const int stage = kiter % NK;
      const bool w = mbar_wait(bar(B_KEMPTY + stage), ((kiter / NK) & 1u) ^ 1u, abort_flag, a.status);
      if (!__all_sync(full, w)) return false;
      const int nmine = half_blocks(u, rank);
      int phys = 0;
      if (lane < nmine) {
        phys = id;
        if (phys < 0 || phys >= a.NB) {
          flag(a.status, ACTKV_DEV_BAD_INDEX);
          phys = 0;
        }
      }
      const uint32_t kf = peer_addr(bar(B_KFULL + stage), 0);
      if (rank == 0 && lane == 0)
        mbar_expect_tx(bar(B_KFULL + stage), uint32_t(half_blocks(u, 0) + half_blocks(u, 1)) * a.BS * 256u);
      __syncwarp();
      const uint32_t kdst = base + Lay::kKOff + stage * kKStageBytes;
      if (lane < nmine)
        for (int hf = 0; hf < 2; ++hf)
          tma2_load_4d(kdst + hf * (kKStageBytes / 2) + lane * a.BS * 128, &tmap_k, kf, hf * 64, u.h, phys * a.BS,
                       u.l);
      ++kiter;
      return true;
    };
    for (int g = 0; g < n_lg && ok; ++g) {
      start_group(g);
      if constexpr (STREAMED) {                 // this group's queries have landed
        const bool w = counter_wait(a.ready, a.ready_base + uint32_t(g) + 1u, abort_flag, a.status);
        if (!__all_sync(full, w)) {
          ok = false;
          break;
        }
      }
      ahead = wk;
#pragma unroll
      for (int i = 0; i < kIdsAhead; ++i) ids[i] = ahead.next(y) ? read_id(y) : -2;
      if constexpr (!WIDE) {
        // resident queries (A*G <= 256*QS): loaded once per segment, one K tile per unit
        while (ok && wk.next(x)) {
          const int id = pop_id();
          if (x.nch == 0 || x.nch > QS) continue;
          if (x.seg_first)
            for (int c = 0; c < x.nch && ok; ++c) ok = load_q(x, c, c);
          ok = ok && load_k(x, id);
        }
      } else {
        int* blk_ids = reinterpret_cast<int*>(smem + Lay::kBlkIdsOff);
        Unit nx;
        bool have = wk.next(x);
        int x_id = have ? pop_id() : -2;
        while (ok && have) {
          const Unit first = x;
          const bool wide = first.nch > QS;
          int nb = 0;
          bool nhave;
          int nx_id;
          while (true) {
            if (lane < bpc) blk_ids[nb * 16 + lane] = x_id;
            ++nb;
            nhave = wk.next(nx);
            nx_id = nhave ? pop_id() : -2;
            if (!wide || !(nhave && nb < kBlockTiles && same_block<QS>(nx, first, nb))) break;
            x = nx;
            x_id = nx_id;
          }
          for (int p = 0; p * QS < first.nch && ok; ++p) {
            if (wide || first.seg_first)
              for (int sl = 0; sl < QS && p * QS + sl < first.nch && ok; ++sl) ok = load_q(first, sl, p * QS + sl);
            for (int b = 0; b < nb && ok; ++b) {
              Unit u = first;
              u.tile = first.tile + b;
              ok = load_k(u, lane < bpc ? blk_ids[b * 16 + lane] : -2);
            }
          }
          x = nx;
          x_id = nx_id;
          have = nhave;
        }
      }
    }
    if (*abort_flag && rank == 0 && lane == 0) {
      // let copies already issued (by either CTA) land before the pair can exit (bounded)
      for (int s = 0; s < NK; ++s) {
        const uint32_t uses = kiter / NK + (uint32_t(s) < kiter % NK ? 1u : 0u);
        if (uses) mbar_drain(bar(B_KFULL + s), (uses - 1) & 1u);
      }
      for (int s = 0; s < QS; ++s)
        if (quses[s]) mbar_drain(bar(B_QFULL + s), (quses[s] - 1) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (rank == 0 && lane == 0) {
      uint32_t kiter = 0, acc_iter = 0;
      uint32_t quses[QS];
#pragma unroll
      for (int i = 0; i < QS; ++i) quses[i] = 0;
      uint32_t idesc[QS], idesc_l[QS];
      int last_commit_bar = -1;
      uint32_t last_commit_parity = 0;
      bool ok = true;
      const uint64_t d_ones = ext_desc(base + Lay::kOnesOff);
      // the query chunks c0 .. c0 + n - 1 of unit u into slots 0 .. n - 1: wait for them
      auto wait_q = [&](const Unit& u, int c0, int n) -> bool {
        for (int sl = 0; sl < n; ++sl) {
          if (!mbar_wait(bar(B_QFULL + sl), quses[sl] & 1u, abort_flag, a.status)) return false;
          ++quses[sl];
          const int nc = chunk_n(chunk_cols(u.A, c0 + sl, QPC, G));
          idesc[sl] = instr_desc_mn(kTile, nc, BF16);
          idesc_l[sl] = instr_desc_mn(kTile, nc, true);
        }
        return true;
      };
      // the MMAs of the query chunks in slots 0 .. n - 1 against the next K stage, one accumulator
      // each; release_q: the slots' last use
      auto mma_tile = [&](int n, bool release_q) -> bool {
        const int stage = kiter % NK;
        if (!mbar_wait(bar(B_KFULL + stage), (kiter / NK) & 1u, abort_flag, a.status)) return false;
        const uint64_t dk = sw128_desc(base + Lay::kKOff + stage * kKStageBytes);
        for (int sl = 0; sl < n; ++sl) {
          const int buf = acc_iter & 1;
          if (!mbar_wait(bar(B_AEMPTY + buf), ((acc_iter >> 1) & 1u) ^ 1u, abort_flag, a.status)) return false;
          fence_after();
          const uint64_t dq = sw128_desc(base + Lay::kQOff + sl * kQSlotBytes);
          const uint32_t d = tmem + buf * 256;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // start-address field is addr >> 4: a K step's byte offset adds without a carry out
            const uint32_t off = (k >> 2) * (kKStageBytes / 2) + (k & 3) * 32;
            mma2_f16(d, dk + (off >> 4), dq + (off >> 4), idesc[sl], k > 0);
          }
          // lse step: ones x (c1, c2, c3) adds -lse/scale to every column (bf16 operands)
          mma2_f16(d, d_ones, ext_desc(base + Lay::kLseOff + sl * kLseSlotBytes), idesc_l[sl], 1);
          commit2(bar(B_AFULL + buf));
          last_commit_bar = B_AFULL + buf;
          last_commit_parity = (acc_iter >> 1) & 1u;
          ++acc_iter;
          if (release_q) commit2(bar(B_QEMPTY + sl));
        }
        commit2(bar(B_KEMPTY + stage));
        ++kiter;
        return true;
      };
      for (int g = 0; g < n_lg && ok; ++g) {
        start_group(g);
        if constexpr (!WIDE) {
          while (ok && wk.next(x)) {
            if (x.nch == 0 || x.nch > QS) continue;
            if (x.seg_first) ok = wait_q(x, 0, x.nch);
            ok = ok && mma_tile(x.nch, x.seg_last);
          }
        } else {
          Unit nx;
          bool have = wk.next(x);
          while (ok && have) {
            const Unit first = x;
            const bool wide = first.nch > QS;
            int nb = 0;
            bool nhave;
            while (true) {
              ++nb;
              nhave = wk.next(nx);
              if (!wide || !(nhave && nb < kBlockTiles && same_block<QS>(nx, first, nb))) break;
              x = nx;
            }
            for (int p = 0; p * QS < first.nch && ok; ++p) {
              const int n = min(QS, first.nch - p * QS);
              if (wide || first.seg_first) ok = wait_q(first, p * QS, n);
              for (int b = 0; b < nb && ok; ++b) ok = mma_tile(n, wide ? b == nb - 1 : first.seg_last);
            }
            x = nx;
            have = nhave;
          }
        }
      }
      if (*abort_flag && last_commit_bar >= 0) mbar_drain(bar(last_commit_bar), last_commit_parity);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (2 x 4 warps)
    const int wg = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;           // this CTA's token row of the unit
    const int row_off = int(rank) * kHalfM + row;
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const float s2 = a.scale * kLog2e;
    float* part = reinterpret_cast<float*>(smem + Lay::kPartOff);
    uint32_t* part_cnt = reinterpret_cast<uint32_t*>(smem + Lay::kPartCntOff);
    const uint32_t aempty0 = peer_addr(bar(B_AEMPTY), 0);
    uint32_t acc_iter = 0, exch_iter = 0;
    bool ok = true;
    auto fold_chunk = [&](const Unit& u, int c, float& sum) -> bool {
      const int t = u.tile * kTile + row_off;
      const int first_q = t - (u.S - u.A);
      const bool causal_tile = u.tile * kTile + int(rank) * kHalfM + kHalfM - 1 > u.S - u.A;
      const int buf = acc_iter & 1;
      const bool w = mbar_wait(bar(B_AFULL + buf), (acc_iter >> 1) & 1u, abort_flag, a.status);
      if (!__all_sync(full, w)) return false;
      fence_after();
      const int ncols = chunk_cols(u.A, c, QPC, G);
      const int cb0 = wg * 4, cb1 = min((ncols + 31) / 32, cb0 + 4);
      const int jc = c * QPC;
      const uint32_t taddr = lane_addr + buf * 256;
      if (!(causal_tile || ncols < 256)) {
        // two 64-column loads (fewer wait::ld round trips: at G = 8 the fold is short and the
        // round trips bound the epilogue; measured 5% on the block path, neutral at G = 4)
        float v[64];
        const uint32_t t0 = taddr + cb0 * 32;
        const float(&lo)[32] = *reinterpret_cast<const float(*)[32]>(v);
        const float(&hi)[32] = *reinterpret_cast<const float(*)[32]>(v + 32);
        tmem_ld64(t0, v);
        tmem_wait(v);
        fold_batch<G, false>(lo, s2, 0, 0, 0, sum);
        fold_batch<G, false>(hi, s2, 0, 0, 0, sum);
        tmem_ld64(t0 + 64, v);
        tmem_wait(v);
        fold_batch<G, false>(lo, s2, 0, 0, 0, sum);
        fold_batch<G, false>(hi, s2, 0, 0, 0, sum);
      } else if (cb0 < cb1) {
        float va[32], vb[32];
        tmem_ld32(taddr + cb0 * 32, va);
        tmem_wait(va);
#pragma unroll 1
        for (int cb = cb0; cb < cb1; cb += 2) {
          if (cb + 1 < cb1) tmem_ld32(taddr + (cb + 1) * 32, vb);
          fold_batch<G, true>(va, s2, jc + cb * (32 / G), u.A, first_q, sum);
          if (cb + 1 < cb1) {
            tmem_wait(vb);
            if (cb + 2 < cb1) tmem_ld32(taddr + (cb + 2) * 32, va);
            fold_batch<G, true>(vb, s2, jc + (cb + 1) * (32 / G), u.A, first_q, sum);
            if (cb + 2 < cb1) tmem_wait(va);
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) arrive_cluster(aempty0 + buf * 8);
      ++acc_iter;
      return true;
    };
    // the two warpgroups' halves of a unit: the second to arrive adds them (0 + 1) and writes
    auto finish_unit = [&](const Unit& u, float sum) {
      const int t = u.tile * kTile + row_off;
      const int first_q = t - (u.S - u.A);
      if (u.nch == 0) {
        if (wg == 0 && t < u.S) {
          float* o = a.out + (a.out_off ? a.out_off[u.r] : u.r * a.out_stride_r) + u.l * a.out_stride_l +
                     u.h * a.out_stride_h + t;
          *o = finalize_score(0.0f, u.A, first_q, o, a.n_seen ? a.n_seen[u.r] : -1);
        }
        return;
      }
      const uint32_t slot = exch_iter++ % kPartSlots;
      float* ps = part + slot * 256;
      uint32_t* pc = part_cnt + slot * 128 + row;
      ps[wg * 128 + row] = sum;
      __threadfence_block();
      if (atomicAdd(pc, 1u) == 1u) {
        __threadfence_block();
        const float total = ps[row] + ps[128 + row];
        atomicExch(pc, 0u);
        if (t < u.S) {
          float* o = a.out + (a.out_off ? a.out_off[u.r] : u.r * a.out_stride_r) + u.l * a.out_stride_l +
                     u.h * a.out_stride_h + t;
          *o = finalize_score(total, u.A, first_q, o, a.n_seen ? a.n_seen[u.r] : -1);
        }
      }
    };
    for (int g = 0; g < n_lg && ok; ++g) {
      start_group(g);
      if constexpr (!WIDE) {
        while (ok && wk.next(x)) {
          float sum = 0.0f;
          if (x.nch > QS) {
            if (threadIdx.x == 64) flag(a.status, ACTKV_DEV_BAD_INDEX);
            continue;
          }
          for (int c = 0; c < x.nch && ok; ++c) ok = fold_chunk(x, c, sum);
          if (!ok) break;
          finish_unit(x, sum);
        }
      } else {
        Unit nx;
        bool have = wk.next(x);
        while (ok && have) {
          const Unit first = x;
          int nb = 0;
          bool nhave;
          while (true) {
            ++nb;
            nhave = wk.next(nx);
            if (first.nch <= QS || !(nhave && nb < kBlockTiles && same_block<QS>(nx, first, nb))) break;
            x = nx;
          }
          // per tile of the block, the chunks are folded in chunk order (groups outer, as the MMAs come)
          float sums[kBlockTiles];
  #pragma unroll
          for (int b = 0; b < kBlockTiles; ++b) sums[b] = 0.0f;
          for (int p = 0; p * QS < first.nch && ok; ++p)
            for (int b = 0; b < nb && ok; ++b) {
              Unit u = first;
              u.tile = first.tile + b;
              for (int sl = 0; sl < QS && p * QS + sl < first.nch && ok; ++sl) ok = fold_chunk(u, p * QS + sl, sums[b]);
            }
          if (!ok) break;
          // not unrolled: eight copies of finish_unit overflow the instruction cache the epilogue,
          // MMA and producer warps share (measured: the block path's scoring 3% slower unrolled)
  #pragma unroll 1
          for (int b = 0; b < kBlockTiles; ++b) {
            if (b >= nb) break;
            Unit u = first;
            u.tile = first.tile + b;
            finish_unit(u, sums[b]);
          }
          x = nx;
          have = nhave;
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  cluster_sync();                               // no MMA of the pair reads this CTA's memory any more
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// -lse/scale of every (layer, action row, query head) as the three-term bf16 split, one 16-byte
// row each: the query-side operand of the lse step.
__global__ void lse_split_kernel(const float* lse, int64_t stride_l, int64_t stride_a, int L, int sum_A, int Hq,
                                 float scale, uint4* out) {
  const int64_t n = int64_t(L) * sum_A * Hq;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int h = int(i % Hq);
    const int64_t la = i / Hq;
    const int aa = int(la % sum_A), l = int(la / sum_A);
    out[i] = lse_split_row(-lse[l * stride_l + aa * stride_a + h] / scale);
  }
}

}  // namespace pair

// ------------------------------------------------------------------------------------ host side
size_t pair_workspace_bytes(int L, int sum_A, int Hq) {
  return L > 0 && sum_A > 0 && Hq > 0 ? align256(size_t(L) * sum_A * Hq * 16) : 256;
}

bool pair_supported(const ScoreArgs& a, int max_A) {
  (void)max_A;                                  // wider regions take the block path
  return a.BS <= pair::kHalfM && pair::kHalfM % a.BS == 0 && pair::kHalfM / a.BS <= 16;
}

template <int G, bool BF16, int QS, bool WIDE>
static cudaError_t launch_pair_g(const CUtensorMap& mk, const CUtensorMap& mq, const CUtensorMap& ml,
                                 const ScoreArgs& a, cudaStream_t st) {
  auto k = a.n_lgroups > 0 ? pair::score_pair_kernel<G, BF16, QS, WIDE, true>
                           : pair::score_pair_kernel<G, BF16, QS, WIDE, false>;
  constexpr uint32_t smem = pair::Layout<QS>::kSmemBytes;
  static int clusters_of[2][64] = {};           // co-resident clusters of each kernel per device
  int* clusters = clusters_of[a.n_lgroups > 0 ? 1 : 0];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(pair::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (clusters[dev] == 0) {
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(2);
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, k, &cfg);
    if (e != cudaSuccess) return e;
    if (n < 1) return cudaErrorInvalidConfiguration;
    clusters[dev] = n;
  }
  cfg.gridDim = dim3(2 * clusters[dev]);
  return cudaLaunchKernelEx(&cfg, k, mk, mq, ml, a);
}

template <bool BF16, int QS, bool WIDE>
static cudaError_t launch_pair_q(const CUtensorMap& mk, const CUtensorMap& mq, const CUtensorMap& ml,
                                 const ScoreArgs& a, cudaStream_t st) {
  switch (a.G) {
    case 1: return launch_pair_g<1, BF16, QS, WIDE>(mk, mq, ml, a, st);
    case 2: return launch_pair_g<2, BF16, QS, WIDE>(mk, mq, ml, a, st);
    case 4: return launch_pair_g<4, BF16, QS, WIDE>(mk, mq, ml, a, st);
    case 8: return launch_pair_g<8, BF16, QS, WIDE>(mk, mq, ml, a, st);
    default: return launch_pair_g<16, BF16, QS, WIDE>(mk, mq, ml, a, st);
  }
}

template <bool BF16>
static cudaError_t launch_pair_t(const CUtensorMap& mk, const CUtensorMap& mq, const CUtensorMap& ml,
                                 const ScoreArgs& a, int max_A, cudaStream_t st) {
  const int64_t cols = int64_t(max_A) * a.G;
  if (cols <= 512) return launch_pair_q<BF16, 2, false>(mk, mq, ml, a, st);
  if (a.R == 1) return cols <= 1024 ? launch_pair_q<BF16, 4, false>(mk, mq, ml, a, st)
                                    : launch_pair_q<BF16, 4, true>(mk, mq, ml, a, st);
  // regions of several widths: each class on the layout that fits it, so that the narrow ones keep
  // two query slots and four K stages (their scoring is bound by the K stream, which the deeper
  // prefetch keeps full) and only regions wider than four slots take the block path
  ScoreArgs b = a;
  b.filter = 1;
  b.cols_lo = 0;
  b.cols_hi = 512;
  cudaError_t e = launch_pair_q<BF16, 2, false>(mk, mq, ml, b, st);
  if (e != cudaSuccess) return e;
  b.cols_lo = 513;
  b.cols_hi = 1024;
  e = launch_pair_q<BF16, 4, false>(mk, mq, ml, b, st);
  if (e != cudaSuccess || cols <= 1024) return e;
  b.cols_lo = 1025;
  b.cols_hi = 0x7fffffff;
  return launch_pair_q<BF16, 4, true>(mk, mq, ml, b, st);
}

// The pair kernel for a.G in {1, 2, 4, 8, 16}, bf16/fp16 q and cache (umma_supported), max_A * G
// (pair_supported); workspace: pair_workspace_bytes(L, sum_A, Hq) bytes, 16-byte aligned.
cudaError_t launch_score_pair(const ScoreArgs& a, int dtype, int sum_A, int max_A, void* workspace,
                              cudaStream_t st, const char** why) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    if (why) *why = "cuTensorMapEncodeTiled unavailable";
    return cudaErrorNotSupported;
  }
  // 1. the lse step's query-side rows
  {
    const int64_t n = int64_t(a.L) * sum_A * a.Hq;
    const int grid = int(std::min<int64_t>((n + 255) / 256, int64_t(device_sm_count()) * 8));
    pair::lse_split_kernel<<<grid > 0 ? grid : 1, 256, 0, st>>>(a.lse, a.lse_stride_l, a.lse_stride_a, a.L, sum_A,
                                                                 a.Hq, a.scale, static_cast<uint4*>(workspace));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const CUtensorMapDataType dt = dtype == ACTKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mk, mq, ml;
  const int qpc = 256 / a.G;
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
    const cuuint64_t dims[4] = {cuuint64_t(a.D), cuuint64_t(a.Hq), cuuint64_t(sum_A), cuuint64_t(a.L)};
    const cuuint64_t strides[3] = {cuuint64_t(a.q_stride_h) * 2, cuuint64_t(a.q_stride_a) * 2,
                                   cuuint64_t(a.q_stride_l) * 2};
    const cuuint32_t box[4] = {64, cuuint32_t(a.G), cuuint32_t(qpc / 2), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&mq, dt, 4, const_cast<void*>(a.q), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      if (why) *why = "cuTensorMapEncodeTiled rejected the query layout";
      return cudaErrorInvalidValue;
    }
  }
  {
    const cuuint64_t dims[4] = {8, cuuint64_t(a.Hq), cuuint64_t(sum_A), cuuint64_t(a.L)};
    const cuuint64_t strides[3] = {16, cuuint64_t(a.Hq) * 16, cuuint64_t(sum_A) * a.Hq * 16};
    const cuuint32_t box[4] = {8, cuuint32_t(a.G), cuuint32_t(qpc / 2), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&ml, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, workspace, dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      if (why) *why = "cuTensorMapEncodeTiled rejected the lse workspace";
      return cudaErrorInvalidValue;
    }
  }
  return dtype == ACTKV_BF16 ? launch_pair_t<true>(mk, mq, ml, a, max_A, st)
                             : launch_pair_t<false>(mk, mq, ml, a, max_A, st);
}

}  // namespace actkv
