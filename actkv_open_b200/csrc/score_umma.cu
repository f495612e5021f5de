// LSE-recovery scoring on the sm_100a tensor cores (tcgen05 + TMA + TMEM).
//
// For one (session r, layer l, KV head h) the action region's queries form a dense matrix
// Q_h [A*G, D] (row j*G+g = query head h*G+g of action token j) and the session's keys of head h
// form K_h [S, D].  Scores need X = K_h * Q_h^T [S, A*G]; the epilogue then folds each row
// (token) over the columns: max over the G heads of a group, exp(x*scale - lse), causal mask,
// sum over action tokens (Algorithm 3, actkv/kernels/lse_attn.py:63-78 / :85-130).
//
// Tiling: M = 128 tokens (8 paged blocks of 16, gathered through the block table with one TMA
// box per block and D-half), N = up to 256 query columns per MMA chunk, K = D = 128 (two 128-byte
// swizzle atoms).  Accumulators live in TMEM: two 128x256 fp32 buffers (512 columns), so the
// epilogue drains one chunk while the tensor core fills the other.
//
// The lse term rides on the tensor core: a ninth K=16 step multiplies a constant key-side tile
// (every token row = [1, 1, 1, 0, ...]) with a query-side tile whose row n is the three-term bf16
// split of -lse_n/scale, so the accumulator already holds x - lse/scale and the epilogue is
// max_g -> one multiply -> ex2 -> add, with no shared-memory reads.  (Reading per-column lse from
// shared memory in the epilogue competes with the tensor core's operand reads and measured ~2x
// slower than the MMAs themselves.)  The split is exact to fp32 precision: c1 = bf16(c),
// c2 = bf16(c - c1), c3 = bf16(c - c1 - c2).
//
// Warp roles (320 threads, one CTA per SM, persistent):
//   warp 0    TMA producer: K tiles through a 2-stage ring, lane b issuing paged block b's two
//             boxes (block ids read from the block table units ahead); Q chunks either resident for a whole (r, l, h) segment (A*G <= 512:
//             at most two chunks, one per slot), or, for wider action regions, loaded a pair at
//             a time for a block of up to kBlockTiles consecutive tiles, whose K tiles are then
//             re-read (mostly from L2) once per pair; its 32 lanes also write the lse split rows
//   warp 1    TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-9 epilogue, two warpgroups: warpgroup g folds columns [128g, 128g+128) of each chunk
//             (tcgen05.ld 32 columns at a time, the next load in flight while one is folded);
//             the second warpgroup to finish a unit adds both halves (always 0 + 1) and writes
//             the scores
// Work is a static, cost-balanced split of the flattened (r, l, h, tile) space over the grid,
// computed identically by every thread from seq_used / act_off (no host round trip).
//
// Wide regions: for each tile of a block, the chunks' sums are still added in chunk order (pair
// by pair), so the result is the same as folding the tile's chunks one after another; only the
// query traffic changes (a pair per block instead of every chunk per tile).
//
// Every wait is bounded: a wait that exceeds ~2^31 cycles sets ACTKV_DEV_TIMEOUT in `status`,
// raises a shared abort flag that every role polls, and the kernel unwinds (waiting, bounded, for
// its own copies and MMAs in flight) and frees its TMEM.  No trap, no unbounded spin.  Waiting
// threads sleep in mbarrier.try_wait (suspend hint) instead of spinning.
#include <cuda.h>

#include "common.cuh"
#include "score_common.cuh"
#include "score_tc.cuh"
#include "umma_common.cuh"

namespace actkv {

namespace umma {

constexpr int kThreads = 320;
constexpr int kTileM = 128;
constexpr int kKStages = 2;
constexpr int kIdsAhead = 4;                             // block ids read this many units ahead
constexpr uint32_t kQSlotBytes = 2 * 256 * 128;          // two D-halves of 256 rows x 128 B
constexpr uint32_t kKStageBytes = 2 * kTileM * 128;      // two D-halves of 128 rows x 128 B
// lse step operands, K-major without swizzle: 8-row x 16-byte core matrices, the two K halves
// (elements 0-7, 8-15) of an 8-row group 128 B apart, consecutive 8-row groups 256 B apart
constexpr uint32_t kExtRowGroupBytes = 256;
constexpr uint32_t kOnesBytes = (kTileM / 8) * kExtRowGroupBytes;   // 128 token rows
constexpr uint32_t kLseSlotBytes = (256 / 8) * kExtRowGroupBytes;   // 256 query rows per chunk
constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = 2 * kQSlotBytes;
constexpr uint32_t kOnesOff = kKOff + kKStages * kKStageBytes;
constexpr uint32_t kLseOff = kOnesOff + kOnesBytes;               // 2 slots, one per Q slot
constexpr int kBlockTiles = 8;                                     // tiles sharing one pass of a wide region's queries
constexpr int kPartSlots = 8;                                      // >= kBlockTiles units between the warpgroups
constexpr uint32_t kPartOff = kLseOff + 2 * kLseSlotBytes;         // [slot][warpgroup][128] fp32 partial sums
constexpr uint32_t kPartCntOff = kPartOff + kPartSlots * 2 * 128 * 4;  // [slot][128] u32 arrivals per row
constexpr uint32_t kBlkIdsOff = kPartCntOff + kPartSlots * 128 * 4;  // [kBlockTiles][16] block ids of a block
constexpr uint32_t kBarOff = kBlkIdsOff + kBlockTiles * 16 * 4;
// barriers: k_full[2] k_empty[2] q_full[2] q_empty[2] acc_full[2] acc_empty[2], then the TMEM
// address and the abort flag
constexpr uint32_t kNumBars = 2 * kKStages + 8;
constexpr uint32_t kSmemBytes = kBarOff + kNumBars * 8 + 16;
static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA can have");

// Descriptor of the lse step's operands: K-major, no swizzle (layout code 0), leading (K)
// core-matrix offset 128 B, stride (8-row group) offset 256 B, version 1.
__device__ __forceinline__ uint64_t plain_desc(uint32_t addr) {
  uint64_t d = uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(128 >> 4) << 16;
  d |= uint64_t(kExtRowGroupBytes >> 4) << 32;
  d |= uint64_t(1) << 46;
  return d;
}

// Byte offset of row n's first K half (elements 0-7) in a lse step operand tile.
__device__ __forceinline__ uint32_t ext_row(int n) {
  return uint32_t(n >> 3) * kExtRowGroupBytes + uint32_t(n & 7) * 16;
}

// Instruction descriptor of an M = kTileM (token rows) x N MMA.
__device__ __forceinline__ uint32_t instr_desc(int n, bool bf16) { return instr_desc_mn(kTileM, n, bf16); }

// u is the tile `nb` tiles after `first` in the same (session, layer, head) segment: it can join
// first's block of a wide action region.
__device__ __forceinline__ bool same_block(const Unit& u, const Unit& first, int nb) {
  return u.nch > 2 && u.r == first.r && u.l == first.l && u.h == first.h && u.tile == first.tile + nb;
}

// WIDE: some session's action region has more than two query chunks (A*G > 512); every unit then
// goes through the block path (a resident unit is a block of one tile).  Without it, the simpler
// per-unit loops of resident queries run: they measured faster, and both in one kernel exceed the
// register budget.
template <int G, bool BF16, bool WIDE>
__global__ void __launch_bounds__(kThreads, 1)
    score_umma_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_q,
                      ScoreArgs a) {
  constexpr int QPC = 256 / G;                  // queries per chunk
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kBarOff + kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kBarOff + kNumBars * 8 + 4);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int B_KFULL = 0, B_KEMPTY = kKStages, B_QFULL = 2 * kKStages, B_QEMPTY = 2 * kKStages + 2,
            B_AFULL = 2 * kKStages + 4, B_AEMPTY = 2 * kKStages + 6;
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_QFULL + i), 1 + 32);     // expect_tx by the TMA issuer + the 32 lse-row writers
      mbar_init(bar(B_QEMPTY + i), 1);
      mbar_init(bar(B_AFULL + i), 1);
      mbar_init(bar(B_AEMPTY + i), 8);         // one arrive per epilogue warp
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // lse step operands: the key-side tile (rows [1, 1, 1, 0, ...]) is constant; the second K half
  // of every query-side row stays zero, only the first half is rewritten per chunk
  for (int n = threadIdx.x; n < kTileM + 2 * 256; n += kThreads) {
    const bool ones = n < kTileM;
    uint8_t* row = smem + (ones ? kOnesOff + ext_row(n) : kLseOff + ((n - kTileM) >> 8) * kLseSlotBytes +
                                                            ext_row((n - kTileM) & 255));
    const __nv_bfloat16 one = __float2bfloat16_rn(1.0f), zero = __float2bfloat16_rn(0.0f);
    *reinterpret_cast<uint4*>(row) = ones ? make_uint4(pack_bf16x2(one, one), pack_bf16x2(one, zero), 0u, 0u)
                                          : make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(row + 128) = make_uint4(0u, 0u, 0u, 0u);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  for (int i = threadIdx.x; i < kPartSlots * 128; i += kThreads)
    reinterpret_cast<uint32_t*>(smem + kPartCntOff)[i] = 0u;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  Walker<kTileM> wk;
  wk.init(&a, QPC, blockIdx.x, gridDim.x);
  Unit x;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_k)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_q)) : "memory");
    }
    // Block ids are read from the block table units before they are used, so no global-load
    // latency sits between a freed stage and its TMA issue.  ids[i] holds this lane's block id
    // (lane b: paged block b of the tile) of the unit i ahead of the current one.  (Prefetching
    // those tiles into L2 as well measured slower: it doubles the TMA operations per tile.)
    const int bpt = kTileM / a.BS;
    auto read_id = [&](const Unit& y) -> int {
      if (y.nch == 0) return -2;
      const int first = y.tile * bpt;
      if (lane >= min(bpt, (y.S + a.BS - 1) / a.BS - first)) return -2;
      const int lb = first + lane;
      return lb < a.MB ? a.block_table[y.r * a.bt_stride_r + lb] : -1;
    };
    Walker<kTileM> ahead = wk;
    Unit y;
    int ids[kIdsAhead];
#pragma unroll
    for (int i = 0; i < kIdsAhead; ++i) ids[i] = ahead.next(y) ? read_id(y) : -2;
    auto pop_id = [&]() -> int {
      const int cur = ids[0];
#pragma unroll
      for (int i = 0; i + 1 < kIdsAhead; ++i) ids[i] = ids[i + 1];
      ids[kIdsAhead - 1] = ahead.next(y) ? read_id(y) : -2;
      return cur;
    };
    int* blk_ids = reinterpret_cast<int*>(smem + kBlkIdsOff);
    uint32_t kiter = 0;
    uint32_t quses[2] = {0, 0};
    bool ok = true;
    // Q chunk c of unit u's segment and its lse rows into slot: waits until the MMAs (q_empty) are
    // done with the slot's previous contents
    auto load_q = [&](const Unit& u, int slot, int c) -> bool {
      // the chunk's lse values first: their global loads overlap the wait for the slot
      const float* lrow = a.lse + u.l * a.lse_stride_l + u.h * G;
      float cn[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int n = lane + 32 * k, j = c * QPC + n / G, g = n % G;
        // padding columns (j >= A) get 0: the epilogue masks them
        cn[k] = j < u.A ? -__ldg(lrow + int64_t(u.a0 + j) * a.lse_stride_a + g) / a.scale : 0.0f;
      }
      const uint32_t par = (quses[slot] & 1u) ^ 1u;
      const bool w = mbar_wait(bar(B_QEMPTY + slot), par, abort_flag, a.status);
      if (!__all_sync(full, w)) return false;
      if (lane == 0) {
        const uint32_t dst = base + kQOff + slot * kQSlotBytes;
        mbar_expect_tx(bar(B_QFULL + slot), kQSlotBytes);
        for (int hf = 0; hf < 2; ++hf)
          tma_load_4d(dst + hf * (kQSlotBytes / 2), &tmap_q, bar(B_QFULL + slot), hf * 64, u.h * G,
                      u.a0 + c * QPC, u.l);
      }
      uint8_t* ls = smem + kLseOff + slot * kLseSlotBytes;
#pragma unroll
      for (int k = 0; k < 8; ++k) *reinterpret_cast<uint4*>(ls + ext_row(lane + 32 * k)) = lse_split_row(cn[k]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor core
      mbar_arrive(bar(B_QFULL + slot));
      ++quses[slot];
      return true;
    };
    // K tile of 128 tokens of tile u.tile into the next stage: one TMA box per paged block and
    // D-half; `id` is this lane's block id (lane b: paged block b of the tile)
    auto load_k = [&](const Unit& u, int id) -> bool {
      const int stage = kiter % kKStages;
      const bool w = mbar_wait(bar(B_KEMPTY + stage), ((kiter / kKStages) & 1u) ^ 1u, abort_flag, a.status);
      if (!__all_sync(full, w)) return false;
      const int first_blk = u.tile * bpt;
      const int nblk = min(bpt, (u.S + a.BS - 1) / a.BS - first_blk);
      int phys = 0;
      if (lane < nblk) {
        phys = id;
        if (phys < 0 || phys >= a.NB) {
          flag(a.status, ACTKV_DEV_BAD_INDEX);
          phys = 0;
        }
      }
      if (lane == 0) mbar_expect_tx(bar(B_KFULL + stage), uint32_t(nblk) * a.BS * 128u * 2u);
      __syncwarp();
      // lane b copies paged block b (both D-halves): the boxes go out in parallel, not one by one
      const uint32_t kdst = base + kKOff + stage * kKStageBytes;
      if (lane < nblk)
        for (int hf = 0; hf < 2; ++hf)
          tma_load_4d(kdst + hf * (kKStageBytes / 2) + lane * a.BS * 128, &tmap_k, bar(B_KFULL + stage), hf * 64,
                      u.h, phys * a.BS, u.l);
      ++kiter;
      return true;
    };
    if constexpr (!WIDE) {
      // resident queries (A*G <= 512): loaded once per segment, one K tile per unit (a wider
      // unit, which max_A should have excluded, is skipped by every role and flagged)
      while (ok && wk.next(x)) {
        const int id = pop_id();
        if (x.nch == 0 || x.nch > 2) continue;
        if (x.seg_first)
          for (int c = 0; c < x.nch && ok; ++c) ok = load_q(x, c, c);
        ok = ok && load_k(x, id);
      }
    } else {
      Unit nx;
      bool have = wk.next(x);
      int x_id = have ? pop_id() : -2;
      while (ok && have) {
        // WIDE: a unit of resident queries is a block of one tile; a wide region takes up to
        // kBlockTiles consecutive tiles of its segment, its query chunks go through the two slots a
        // pair at a time, and the block's K tiles are loaded once per pair
        const Unit first = x;
        const bool wide = first.nch > 2;
        int nb = 0;
        bool nhave;
        int nx_id;
        while (true) {
          if (lane < bpt) blk_ids[nb * bpt + lane] = x_id;
          ++nb;
          nhave = wk.next(nx);
          nx_id = nhave ? pop_id() : -2;
          if (!wide || !(nhave && nb < kBlockTiles && same_block(nx, first, nb))) break;
          x = nx;
          x_id = nx_id;
        }
        auto load_k_tile = [&](int b) -> bool {
          Unit u = first;
          u.tile = first.tile + b;
          return load_k(u, lane < bpt ? blk_ids[b * bpt + lane] : -2);
        };
        for (int p = 0; 2 * p < first.nch && ok; ++p) {
          if (wide || first.seg_first) {
            // the pair's query chunks as soon as their slots free up (the MMAs of the previous
            // pair's last tile), then its K tiles
            for (int s = 0; s < 2 && 2 * p + s < first.nch && ok; ++s) ok = load_q(first, s, 2 * p + s);
          }
          for (int b = 0; b < nb && ok; ++b) ok = load_k_tile(b);
        }
        x = nx;
        x_id = nx_id;
        have = nhave;
      }
    }
    if (*abort_flag && lane == 0) {
      // let copies already issued land before the CTA can exit (bounded)
      for (int s = 0; s < kKStages; ++s) {
        const uint32_t uses = kiter / kKStages + (uint32_t(s) < kiter % kKStages ? 1u : 0u);
        if (uses) mbar_drain(bar(B_KFULL + s), (uses - 1) & 1u);
      }
      for (int s = 0; s < 2; ++s)
        if (quses[s]) mbar_drain(bar(B_QFULL + s), (quses[s] - 1) & 1u);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------ MMA issuer
    uint32_t kiter = 0, acc_iter = 0;
    uint32_t quses[2] = {0, 0};
    int last_commit_bar = -1;
    uint32_t last_commit_parity = 0;
    bool ok = true;
    // chunk c of unit u from Q slot `slot` against the K stage in kaddr into the next accumulator
    auto mma_chunk = [&](const Unit& u, int c, int slot, uint32_t kaddr) -> bool {
      const int buf = acc_iter & 1;
      if (!mbar_wait(bar(B_AEMPTY + buf), ((acc_iter >> 1) & 1u) ^ 1u, abort_flag, a.status)) return false;
      fence_after();
      const int ncols = min(256, (u.A - c * QPC) * G);
      const uint32_t idesc = instr_desc((ncols + 15) & ~15, BF16);
      const uint32_t idesc_lse = instr_desc((ncols + 15) & ~15, true);
      const uint32_t qaddr = base + kQOff + slot * kQSlotBytes;
      // the descriptors' start-address field is addr >> 4 in the low 14 bits: shared memory is
      // below 256 KB, so a K step's byte offset adds to it without carrying out of the field
      const uint64_t dk = sw128_desc(kaddr), dq = sw128_desc(qaddr);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t koff = (k >> 2) * (kKStageBytes / 2) + (k & 3) * 32;
        const uint32_t qoff = (k >> 2) * (kQSlotBytes / 2) + (k & 3) * 32;
        mma_f16(tmem + buf * 256, dk + (koff >> 4), dq + (qoff >> 4), idesc, k > 0);
      }
      // lse step: ones x (c1, c2, c3) adds -lse/scale to every column (bf16 operands whatever
      // the cache dtype: one instruction, both operands of the same type)
      mma_f16(tmem + buf * 256, plain_desc(base + kOnesOff), plain_desc(base + kLseOff + slot * kLseSlotBytes),
              idesc_lse, 1);
      mma_commit(bar(B_AFULL + buf));
      last_commit_bar = B_AFULL + buf;
      last_commit_parity = (acc_iter >> 1) & 1u;
      ++acc_iter;
      return true;
    };
    auto wait_k = [&](uint32_t& kaddr) -> bool {
      const int stage = kiter % kKStages;
      if (!mbar_wait(bar(B_KFULL + stage), (kiter / kKStages) & 1u, abort_flag, a.status)) return false;
      kaddr = base + kKOff + stage * kKStageBytes;
      return true;
    };
    auto release_k = [&]() {
      mma_commit(bar(B_KEMPTY + kiter % kKStages));
      ++kiter;
    };
    auto wait_q = [&](int slot) -> bool {
      if (!mbar_wait(bar(B_QFULL + slot), quses[slot] & 1u, abort_flag, a.status)) return false;
      ++quses[slot];
      return true;
    };
    if constexpr (!WIDE) {                             // resident queries, one unit at a time
      while (ok && wk.next(x)) {
        if (x.nch == 0 || x.nch > 2) continue;
        uint32_t kaddr;
        ok = wait_k(kaddr);
        for (int c = 0; c < x.nch && ok; ++c) {
          if (x.seg_first) ok = wait_q(c);
          ok = ok && mma_chunk(x, c, c, kaddr);
          if (ok && x.seg_last) mma_commit(bar(B_QEMPTY + c));
        }
        if (ok) release_k();
      }
    } else {
      Unit nx;
      bool have = wk.next(x);
      while (ok && have) {
        // the same blocks as the producer's
        const Unit first = x;
        const bool wide = first.nch > 2;
        int nb = 0;
        bool nhave;
        while (true) {
          ++nb;
          nhave = wk.next(nx);
          if (!wide || !(nhave && nb < kBlockTiles && same_block(nx, first, nb))) break;
          x = nx;
        }
        for (int p = 0; 2 * p < first.nch && ok; ++p) {
          if (wide || first.seg_first)
            for (int s = 0; s < 2 && 2 * p + s < first.nch && ok; ++s) ok = wait_q(s);
          for (int b = 0; b < nb && ok; ++b) {
            uint32_t kaddr;
            ok = wait_k(kaddr);
            Unit u = first;
            u.tile = first.tile + b;
            for (int s = 0; s < 2 && 2 * p + s < first.nch && ok; ++s) {
              ok = mma_chunk(u, 2 * p + s, s, kaddr);
              // the last use of the chunk: the block's last tile (wide) or the segment's (resident)
              if (ok && (wide ? b == nb - 1 : first.seg_last)) mma_commit(bar(B_QEMPTY + s));
            }
            if (ok) release_k();
          }
        }
        x = nx;
        have = nhave;
      }
    }
    if (*abort_flag && last_commit_bar >= 0) mbar_drain(bar(last_commit_bar), last_commit_parity);
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ epilogue (2 x 4 warps)
    // Warpgroup wg folds columns [128 wg, 128 wg + 128) of every chunk; warp w reads TMEM lanes
    // 32 (w % 4) .. + 31, i.e. 32 tokens of the tile.
    const int wg = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const float s2 = a.scale * kLog2e;
    float* part = reinterpret_cast<float*>(smem + kPartOff);
    uint32_t* part_cnt = reinterpret_cast<uint32_t*>(smem + kPartCntOff);
    uint32_t acc_iter = 0, exch_iter = 0;
    bool ok = true;
    // Fold chunk c of unit u (the next accumulator) into sum_io and hand the accumulator back.
    // The running sum lives in a register while the chunk is folded (sum_io may be local memory).
    auto fold_chunk = [&](const Unit& u, int c, float& sum_io) -> bool {
      float sum = sum_io;
      const int t = u.tile * kTileM + row_in_tile;
      const int first_q = t - (u.S - u.A);
      // rows of this tile that some action token does not see yet need the causal test
      const bool causal_tile = u.tile * kTileM + kTileM - 1 > u.S - u.A;
      const int buf = acc_iter & 1;
      const bool w = mbar_wait(bar(B_AFULL + buf), (acc_iter >> 1) & 1u, abort_flag, a.status);
      if (!__all_sync(full, w)) return false;
      fence_after();
      const int ncols = min(256, (u.A - c * QPC) * G);
      const int cb0 = wg * 4, cb1 = min((ncols + 31) / 32, cb0 + 4);
      const int jc = c * QPC;
      const uint32_t taddr = lane_addr + buf * 256;
      const bool check = causal_tile || ncols < 256;
      if (!check) {
        // full chunk, no masking: this warpgroup's four 32-column batches, straight-line
        float va[32], vb[32];
        const uint32_t t0 = taddr + cb0 * 32;
        tmem_ld32(t0, va);
        tmem_wait(va);
        tmem_ld32(t0 + 32, vb);
        fold_batch<G, false>(va, s2, 0, 0, 0, sum);
        tmem_wait(vb);
        tmem_ld32(t0 + 64, va);
        fold_batch<G, false>(vb, s2, 0, 0, 0, sum);
        tmem_wait(va);
        tmem_ld32(t0 + 96, vb);
        fold_batch<G, false>(va, s2, 0, 0, 0, sum);
        tmem_wait(vb);
        fold_batch<G, false>(vb, s2, 0, 0, 0, sum);
      } else if (cb0 < cb1) {
        float va[32], vb[32];
        tmem_ld32(taddr + cb0 * 32, va);
        tmem_wait(va);
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
      if (lane == 0) mbar_arrive(bar(B_AEMPTY + buf));
      ++acc_iter;
      sum_io = sum;
      return true;
    };
    // combine the two warpgroups' halves of unit u without either waiting for the other: each
    // writes its partial into the unit's slot and counts itself in; the second to arrive adds them,
    // always as warpgroup 0 + warpgroup 1, and writes the score.  Slots are counted over units
    // that have chunks.  The warpgroups stay within a block (kBlockTiles units) of each other:
    // every accumulator must be released by both before the tensor core refills it, and a
    // warpgroup combines a block's units only after folding all of its chunks; kPartSlots >=
    // kBlockTiles slots are enough.  A unit without action tokens has nothing to combine.
    auto finish_unit = [&](const Unit& u, float sum) {
      const int t = u.tile * kTileM + row_in_tile;
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
      uint32_t* pc = part_cnt + slot * 128 + row_in_tile;
      ps[wg * 128 + row_in_tile] = sum;
      __threadfence_block();
      if (atomicAdd(pc, 1u) == 1u) {
        __threadfence_block();
        const float total = ps[row_in_tile] + ps[128 + row_in_tile];
        atomicExch(pc, 0u);
        if (t < u.S) {
          float* o = a.out + (a.out_off ? a.out_off[u.r] : u.r * a.out_stride_r) + u.l * a.out_stride_l +
                     u.h * a.out_stride_h + t;
          *o = finalize_score(total, u.A, first_q, o, a.n_seen ? a.n_seen[u.r] : -1);
        }
      }
    };
    if constexpr (!WIDE) {                             // resident queries, one unit at a time
      while (ok && wk.next(x)) {
        float sum = 0.0f;
        if (x.nch > 2) {
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
        // WIDE: the producer's blocks (a resident unit is a block of one tile)
        const Unit first = x;
        int nb = 0;
        bool nhave;
        while (true) {
          ++nb;
          nhave = wk.next(nx);
          if (first.nch <= 2 || !(nhave && nb < kBlockTiles && same_block(nx, first, nb))) break;
          x = nx;
        }
        // per tile of the block, the chunks are added in chunk order (pairs outer, as the MMAs come)
        float sums[kBlockTiles];
#pragma unroll
        for (int b = 0; b < kBlockTiles; ++b) sums[b] = 0.0f;
        if constexpr (G == 2 || G == 4) {
          // the block's running sums stay in registers: tile b's is selected into `cur`, folded and
          // written back with constant indices, so the fold is inlined once, not once per tile
          // (measured 7% faster at G=4; at G=1 and G=8 the extra live values spill, and at G=8 it
          // measured slower)
#pragma unroll 1
          for (int p = 0; 2 * p < first.nch && ok; ++p)
#pragma unroll 1
            for (int b = 0; b < nb && ok; ++b) {
              Unit u = first;
              u.tile = first.tile + b;
              float cur = sums[0];
#pragma unroll
              for (int i = 1; i < kBlockTiles; ++i) cur = b == i ? sums[i] : cur;
#pragma unroll 1
              for (int s = 0; s < 2 && 2 * p + s < first.nch && ok; ++s) ok = fold_chunk(u, 2 * p + s, cur);
#pragma unroll
              for (int i = 0; i < kBlockTiles; ++i) sums[i] = b == i ? cur : sums[i];
            }
        } else {
          for (int p = 0; 2 * p < first.nch && ok; ++p)
            for (int b = 0; b < nb && ok; ++b) {
              Unit u = first;
              u.tile = first.tile + b;
              for (int s = 0; s < 2 && 2 * p + s < first.nch && ok; ++s) ok = fold_chunk(u, 2 * p + s, sums[b]);
            }
        }
        if (!ok) break;
#pragma unroll
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
    fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace umma

// ------------------------------------------------------------------------------------ host side
bool umma_supported(const ScoreArgs& a, int kv_dtype, int q_dtype, const char** why) {
  auto no = [&](const char* w) {
    if (why) *why = w;
    return false;
  };
  if (kv_dtype != q_dtype || (kv_dtype != ACTKV_BF16 && kv_dtype != ACTKV_F16))
    return no("tcgen05 path needs bf16 or fp16 q and cache of the same dtype");
  if (a.D != 128) return no("tcgen05 path needs head_dim 128");
  if (!(a.G == 1 || a.G == 2 || a.G == 4 || a.G == 8 || a.G == 16)) return no("GQA group must be 1,2,4,8 or 16");
  if (a.BS % 8 != 0 || 128 % a.BS != 0) return no("block_size must divide 128 and be a multiple of 8");
  if (a.kv_stride_b != int64_t(a.BS) * a.kv_stride_s) return no("kv blocks must be contiguous slots");
  const int64_t es = 2;
  if ((reinterpret_cast<uintptr_t>(a.kv) | reinterpret_cast<uintptr_t>(a.q)) % 16)
    return no("q and kv must be 16-byte aligned");
  if ((a.kv_stride_h * es) % 16 || (a.kv_stride_s * es) % 16 || (a.kv_stride_l * es) % 16)
    return no("kv strides must be multiples of 16 bytes");
  if ((a.q_stride_h * es) % 16 || (a.q_stride_a * es) % 16 || (a.q_stride_l * es) % 16)
    return no("q strides must be multiples of 16 bytes");
  if (a.act_off == nullptr) return no("tcgen05 path needs act_off");
  return true;
}

template <int G, bool BF16, bool WIDE>
static cudaError_t launch_umma_g(const CUtensorMap& mk, const CUtensorMap& mq, const ScoreArgs& a, int grid,
                                 cudaStream_t st) {
  auto k = umma::score_umma_kernel<G, BF16, WIDE>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(umma::kSmemBytes));
  if (e != cudaSuccess) return e;
  k<<<grid, umma::kThreads, umma::kSmemBytes, st>>>(mk, mq, a);
  return cudaGetLastError();
}

template <bool BF16, bool WIDE>
static cudaError_t launch_umma_w(const CUtensorMap& mk, const CUtensorMap& mq, const ScoreArgs& a, int grid,
                                 cudaStream_t st) {
  switch (a.G) {
    case 1: return launch_umma_g<1, BF16, WIDE>(mk, mq, a, grid, st);
    case 2: return launch_umma_g<2, BF16, WIDE>(mk, mq, a, grid, st);
    case 4: return launch_umma_g<4, BF16, WIDE>(mk, mq, a, grid, st);
    case 8: return launch_umma_g<8, BF16, WIDE>(mk, mq, a, grid, st);
    default: return launch_umma_g<16, BF16, WIDE>(mk, mq, a, grid, st);
  }
}

template <bool BF16>
static cudaError_t launch_umma_t(const CUtensorMap& mk, const CUtensorMap& mq, const ScoreArgs& a, int grid,
                                 bool wide, cudaStream_t st) {
  return wide ? launch_umma_w<BF16, true>(mk, mq, a, grid, st) : launch_umma_w<BF16, false>(mk, mq, a, grid, st);
}

// Returns cudaErrorNotSupported when the driver entry point is missing.
cudaError_t launch_score_umma(const ScoreArgs& a, int dtype, int sum_A, int max_A, int grid, cudaStream_t st,
                              const char** why) {
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
    const int qpc = 256 / a.G;
    const cuuint64_t dims[4] = {cuuint64_t(a.D), cuuint64_t(a.Hq), cuuint64_t(sum_A), cuuint64_t(a.L)};
    const cuuint64_t strides[3] = {cuuint64_t(a.q_stride_h) * 2, cuuint64_t(a.q_stride_a) * 2,
                                   cuuint64_t(a.q_stride_l) * 2};
    const cuuint32_t box[4] = {64, cuuint32_t(a.G), cuuint32_t(qpc), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&mq, dt, 4, const_cast<void*>(a.q), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      if (why) *why = "cuTensorMapEncodeTiled rejected the query layout";
      return cudaErrorInvalidValue;
    }
  }
  // more than two 256-column query chunks in some session: the kernel with the block path
  const bool wide = int64_t(max_A) * a.G > 512;
  return dtype == ACTKV_BF16 ? launch_umma_t<true>(mk, mq, a, grid, wide, st)
                             : launch_umma_t<false>(mk, mq, a, grid, wide, st);
}

}  // namespace actkv
