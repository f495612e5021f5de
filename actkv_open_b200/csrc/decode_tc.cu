// Paged decode attention with its log-sum-exp on the sm_100a tensor cores (tcgen05 + TMA + TMEM):
// the same result as decode_attn.cu (the reference's paged_decode_attention_ref,
// actkv/kernels/lse_attn.py:42-60, for one query per session), for bf16 / fp16 caches with
// head_dim 128.
//
// A CTA takes one (session, KV head, token split) and streams the split's paged K and V in tiles of
// 128 tokens (TMA, one box per paged block and D-half, three stages of 64 KB):
//   S = K Q^T   tcgen05.mma M = 128 tokens, N = 16 (the G query heads, zero rows above), K = D,
//               into TMEM: lane t of the accumulator is token t's G logits
//   softmax     four warps, a thread per token: tile max per head (shuffles + shared memory),
//               online rescale, p = 2^(x - m), per-lane running sums; p is written to shared
//               memory as two bf16 / fp16 rows per head (p_hi = rn(p), p_lo = rn(p - p_hi)), so
//               the product below carries p to ~16 significant bits with no extra MMA
//   O += P V    tcgen05.mma M = 128 (dims of V), N = 16 (the hi and lo rows), K = 128 tokens, with
//               V read as an MN-major operand straight from the tile the TMA wrote; lane d of the
//               accumulator is output dimension d, folded into registers (o = o * alpha + hi + lo)
// Rows of tokens past the session end are zeroed in the V tile before P V (0 x stale bits could
// be NaN).  The P V of tile i is issued as soon as its P is written, before the S of tile i + 1
// waits for its data, so that tile's stage is refilled while the next one is still loading, and each
// tile's output fold waits until the next tile's softmax is done (one CTA per SM, up to 192 KB in
// flight).  Splits are
// merged by decode_combine_kernel (decode_attn.cu) from the same partial (m, l, acc) layout.
//
// Every wait is bounded (umma_common.cuh): a timeout sets ACTKV_DEV_TIMEOUT, raises the CTA's
// abort flag, drains what was issued and frees the TMEM.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"
#include "umma_common.cuh"

namespace actkv {
namespace dtc {

using namespace umma;

constexpr int kThreads = 192;                       // warp 0 TMA, warp 1 MMA, warps 2-5 softmax / output
constexpr int kTile = 128;
constexpr int kStages = 3;
constexpr uint32_t kHalf = 128 * 128;               // one D-half of 128 rows of 128 B
constexpr uint32_t kStageBytes = 4 * kHalf;         // K (two halves), V (two halves)
constexpr uint32_t kQOff = kStages * kStageBytes;   // Q: two halves of 16 rows (2 KB each)
constexpr uint32_t kPOff = kQOff + 2 * 16 * 128;    // P: two buffers of 16 rows x 128 tokens
constexpr uint32_t kPBytes = 16 * kTile * 2;
constexpr uint32_t kRedOff = kPOff + 2 * kPBytes;   // [4 warps][16] floats of cross-warp exchange
constexpr uint32_t kBarOff = kRedOff + 4 * 16 * 4;
// kv_full[3] kv_empty[3] q_full s_full[2] s_empty[2] p_full[2] o_full[2] o_empty[2]
constexpr int kNumBars = 2 * kStages + 1 + 10;
constexpr uint32_t kSmemBytes = kBarOff + kNumBars * 8 + 16;
static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA can have");
constexpr uint32_t kTmemCols = 64;                  // S[2] at columns 0, 16; O[2] at 32, 48

// P tile, K-major without swizzle: core matrices of 8 rows x 8 tokens (16 B per row), 8-row
// groups 128 B apart, 8-token groups 256 B apart; element (row n, token k) at
// (k / 8) * 256 + (n / 8) * 128 + (n % 8) * 16 + (k % 8) * 2.
__device__ __forceinline__ uint32_t p_offset(int n, int k) {
  return uint32_t(k >> 3) * 256 + uint32_t(n >> 3) * 128 + uint32_t(n & 7) * 16 + uint32_t(k & 7) * 2;
}
__device__ __forceinline__ uint64_t p_desc(uint32_t addr) {      // LBO 256 (next 8 tokens), SBO 128
  uint64_t d = uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(256 >> 4) << 16;
  d |= uint64_t(128 >> 4) << 32;
  d |= uint64_t(1) << 46;
  return d;
}
// V tile as the MN-major A operand (M = head dims, K = tokens), 128-byte swizzle: 64 dims per
// 128-byte row, the other 64 dims one D-half (16 KB) further (leading offset), 8-token groups
// 1024 B apart (stride offset).
__device__ __forceinline__ uint64_t v_desc(uint32_t addr) {
  uint64_t d = uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(kHalf >> 4) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

template <bool BF16> struct Elem;
template <> struct Elem<true> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ T from(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float to(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ uint16_t bits(T x) { return __bfloat16_as_ushort(x); }
};
template <> struct Elem<false> {
  using T = __half;
  static __device__ __forceinline__ T from(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float to(T x) { return __half2float(x); }
  static __device__ __forceinline__ uint16_t bits(T x) { return __half_as_ushort(x); }
};

// 16 consecutive TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t* u = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Barrier `id` over n threads that also ANDs their predicates: every thread gets the same answer,
// so the four softmax warps leave their loop together (a warp that left alone would strand the
// others at the next named barrier).
__device__ __forceinline__ bool named_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

template <int G, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tmap_kv, const __grid_constant__ CUtensorMap tmap_q,
                     DecodeArgs a) {
  using E = Elem<BF16>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kBarOff + kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kBarOff + kNumBars * 8 + 4);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int B_KVF = 0, B_KVE = kStages, B_QF = 2 * kStages, B_SF = B_QF + 1, B_SE = B_SF + 2, B_PF = B_SE + 2,
            B_OF = B_PF + 2, B_OE = B_OF + 2;
  const unsigned full = 0xffffffffu;                // the producer warp's votes
  const int sp = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int S = a.seq_used[r];
  const int tiles = (S + kTile - 1) / kTile;
  const int tps = (tiles + a.splits - 1) / a.splits;            // tiles per split
  const int j0 = min(tiles, sp * tps), j1 = min(tiles, j0 + tps);
  const int nt = j1 - j0;
  const int bpt = kTile / a.BS;

  if ((base & 1023u) != 0) {
    if (threadIdx.x == 0) flag(a.status, ACTKV_DEV_MISALIGNED);
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(B_KVF + i), 1);
      mbar_init(bar(B_KVE + i), 1);
    }
    mbar_init(bar(B_QF), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_SF + i), 1);
      mbar_init(bar(B_SE + i), 4);
      mbar_init(bar(B_PF + i), 4);
      mbar_init(bar(B_OF + i), 1);
      mbar_init(bar(B_OE + i), 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // zero the Q rows above G and both P buffers (their rows above 2G stay zero)
  for (int i = threadIdx.x; i < int(2 * 16 * 128 + 2 * kPBytes) / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem + kQOff)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (nt > 0) {
      if (lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_kv)) : "memory");
        mbar_expect_tx(bar(B_QF), 2 * G * 128);
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(base + kQOff + hf * 2048, &tmap_q, bar(B_QF), hf * 64, h * G, r);
      }
      const int nb_seq = (S + a.BS - 1) / a.BS;
      // lane b's block id of tile j (block b of the tile), read two tiles before its copies are
      // issued so that no table load sits between a freed stage and its refill
      auto read_id = [&](int j) -> int {
        if (j >= nt) return 0;
        const int lb = (j0 + j) * bpt + lane;
        if (lane >= bpt || lb >= nb_seq) return 0;
        return lb < a.MB ? a.block_table[r * a.bt_stride_r + lb] : -1;
      };
      int id0 = read_id(0), id1 = read_id(1);
      for (int j = 0; j < nt; ++j) {
        const int id2 = read_id(j + 2);
        const int stage = j % kStages;
        const bool w = mbar_wait(bar(B_KVE + stage), ((j / kStages) & 1u) ^ 1u, abort_flag, a.status);
        if (!__all_sync(full, w)) break;
        const int first = (j0 + j) * bpt;
        const int nblk = max(0, min(bpt, nb_seq - first));
        int phys = 0;
        if (lane < nblk) {
          phys = id0;
          if (phys < 0 || phys >= a.NB) {
            flag(a.status, ACTKV_DEV_BAD_INDEX);
            phys = 0;
          }
        }
        id0 = id1;
        id1 = id2;
        if (lane == 0) mbar_expect_tx(bar(B_KVF + stage), uint32_t(nblk) * a.BS * 128u * 4u);
        __syncwarp();
        const uint32_t dst = base + stage * kStageBytes + lane * a.BS * 128;
        if (lane < nblk)
          for (int kv = 0; kv < 2; ++kv)
            for (int hf = 0; hf < 2; ++hf)
              tma_load_4d(dst + (2 * kv + hf) * kHalf, &tmap_kv, bar(B_KVF + stage), hf * 64, h, phys * a.BS, kv);
      }
      if (*abort_flag && lane == 0) {
        mbar_drain(bar(B_QF), 0);
        for (int s = 0; s < kStages; ++s) {
          const int uses = nt / kStages + (s < nt % kStages ? 1 : 0);
          if (uses) mbar_drain(bar(B_KVF + s), (uses - 1) & 1u);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nt > 0) {
      const uint32_t idesc_s = instr_desc_mn(128, 16, BF16);
      const uint32_t idesc_o = instr_desc_mn(128, 16, BF16) | (1u << 15);      // A (V) MN-major
      bool ok = mbar_wait(bar(B_QF), 0, abort_flag, a.status);
      const uint64_t dq = sw128_desc(base + kQOff);
      int last_bar = -1;
      uint32_t last_par = 0;
      for (int j = 0; ok && j <= nt; ++j) {
        // the P V of tile j - 1 goes first: it frees its stage for the load of tile j + 2 while the
        // S of tile j still waits for its data (three tiles in flight with three stages)
        if (j >= 1) {                             // P V of tile j - 1
          const int i = j - 1, stage = i % kStages, pb = i & 1;
          ok = mbar_wait(bar(B_PF + pb), (i >> 1) & 1u, abort_flag, a.status) &&
               mbar_wait(bar(B_OE + pb), ((i >> 1) & 1u) ^ 1u, abort_flag, a.status);
          if (!ok) break;
          fence_after();
          const uint32_t vbase = base + stage * kStageBytes + 2 * kHalf;
#pragma unroll
          for (int k = 0; k < 8; ++k)           // 16 tokens per step: two 8-token groups of V and of P
            mma_f16(tmem + 32 + pb * 16, v_desc(vbase + k * 2048), p_desc(base + kPOff + pb * kPBytes + k * 512),
                    idesc_o, k > 0);
          mma_commit(bar(B_OF + pb));
          mma_commit(bar(B_KVE + stage));
          last_bar = B_OF + pb;
          last_par = (i >> 1) & 1u;
        }
        if (j < nt) {                             // S of tile j
          const int stage = j % kStages, sb = j & 1;
          ok = mbar_wait(bar(B_KVF + stage), (j / kStages) & 1u, abort_flag, a.status) &&
               mbar_wait(bar(B_SE + sb), ((j >> 1) & 1u) ^ 1u, abort_flag, a.status);
          if (!ok) break;
          fence_after();
          const uint64_t dk = sw128_desc(base + stage * kStageBytes);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
            const uint32_t qoff = (k >> 2) * 2048 + (k & 3) * 32;
            mma_f16(tmem + sb * 16, dk + (off >> 4), dq + (qoff >> 4), idesc_s, k > 0);
          }
          mma_commit(bar(B_SF + sb));
          last_bar = B_SF + sb;
          last_par = (j >> 1) & 1u;
        }
      }
      if (*abort_flag && last_bar >= 0) mbar_drain(bar(last_bar), last_par);
    }
  } else {
    // ------------------------------------------------------------------ softmax and output (warps 2-5)
    const int quad = warp & 3;                    // TMEM lanes 32 quad .. 32 quad + 31
    const int row = quad * 32 + lane;             // token of the tile (S), head dim (O)
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const int ew = warp - 2;                      // exchange slot
    float* red = reinterpret_cast<float*>(smem + kRedOff);
    const float c2 = a.scale * kLog2e;
    float m[G], l[G], acc[G], alpha_prev[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.0f;
      acc[g] = 0.0f;
      alpha_prev[g] = 0.0f;
    }
    bool ok = true;
    // fold the output of tile i (its P V in O buffer i & 1) with that tile's rescale factors
    auto fold_o = [&](int i, const float (&al)[G]) -> bool {
      const int pb = i & 1;
      const bool w = mbar_wait(bar(B_OF + pb), (i >> 1) & 1u, abort_flag, a.status);
      if (!named_and(2, 128, w)) return false;
      fence_after();
      float o[16];
      tmem_ld16(lane_addr + 32 + pb * 16, o);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_OE + pb));
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = fmaf(acc[g], al[g], o[g] + o[G + g]);
      return true;
    };
    for (int j = 0; j < nt && ok; ++j) {
      const int sb = j & 1;
      const bool w = mbar_wait(bar(B_SF + sb), (j >> 1) & 1u, abort_flag, a.status);
      if (!named_and(2, 128, w)) {
        ok = false;
        break;
      }
      fence_after();
      float s[16];
      tmem_ld16(lane_addr + sb * 16, s);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_SE + sb));
      const int t = (j0 + j) * kTile + row;
      const bool valid = t < S;
      if (!valid) {
        // a token past the session end (a free slot of the last paged block, or a row the TMA
        // did not write): its p is 0, but P V contracts over tokens, so its V row must hold
        // numbers: zero it (both D-halves) before P is published
        uint4* vr = reinterpret_cast<uint4*>(smem + (j % kStages) * kStageBytes + 2 * kHalf + row * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          vr[c] = make_uint4(0u, 0u, 0u, 0u);
          vr[kHalf / 16 + c] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      float x[G], tmax[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        x[g] = valid ? s[g] * c2 : -INFINITY;
        tmax[g] = warp_max(x[g]);
      }
      if (lane == 0)
#pragma unroll
        for (int g = 0; g < G; ++g) red[ew * 16 + g] = tmax[g];
      named_sync(1, 128);
      float al[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float tm = fmaxf(fmaxf(red[g], red[16 + g]), fmaxf(red[32 + g], red[48 + g]));
        const float mn = fmaxf(m[g], tm);
        al[g] = ex2(m[g] - mn);                   // 0 while m is -inf
        m[g] = mn;
      }
      named_sync(1, 128);                         // every warp read red before the next tile's writes
      // P of this tile (buffer sb): free once the output of tile j - 2 was folded (below, in the
      // previous iteration)
      uint8_t* pt = smem + kPOff + sb * kPBytes;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = valid ? ex2(x[g] - m[g]) : 0.0f;
        l[g] = fmaf(l[g], al[g], p);
        const typename E::T hi = E::from(p);
        const typename E::T lo = E::from(p - E::to(hi));
        *reinterpret_cast<uint16_t*>(pt + p_offset(g, row)) = E::bits(hi);
        *reinterpret_cast<uint16_t*>(pt + p_offset(G + g, row)) = E::bits(lo);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PF + sb));
      if (j >= 1) ok = fold_o(j - 1, alpha_prev);
#pragma unroll
      for (int g = 0; g < G; ++g) alpha_prev[g] = al[g];
    }
    if (ok && nt > 0) ok = fold_o(nt - 1, alpha_prev);
    // the split's partials: m (log2 units), l summed over the 128 token lanes, acc per head dim
    float L[G];
#pragma unroll
    for (int g = 0; g < G; ++g) L[g] = warp_sum(l[g]);
    named_sync(1, 128);
    if (lane == 0)
#pragma unroll
      for (int g = 0; g < G; ++g) red[ew * 16 + g] = L[g];
    named_sync(1, 128);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float lt = (red[g] + red[16 + g]) + (red[32 + g] + red[48 + g]);
      const int64_t pi = (int64_t(r) * a.Hq + h * G + g) * a.splits + sp;
      if (ok && nt > 0) {
        a.part_acc[pi * a.D + row] = acc[g];
        if (row == 0) {
          a.part_m[pi] = m[g];
          a.part_l[pi] = lt;
        }
      } else if (row == 0) {                      // an empty split (or an aborted one) adds nothing
        a.part_m[pi] = -INFINITY;
        a.part_l[pi] = 0.0f;
      }
      if (!(ok && nt > 0)) a.part_acc[pi * a.D + row] = 0.0f;
    }
    fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace dtc

// ------------------------------------------------------------------------------------ host side
bool decode_tc_supported(const DecodeArgs& a, int dtype) {
  if (dtype != ACTKV_BF16 && dtype != ACTKV_F16) return false;
  if (a.D != 128 || !(a.G == 1 || a.G == 2 || a.G == 4 || a.G == 8)) return false;
  if (a.BS % 8 != 0 || dtc::kTile % a.BS != 0) return false;
  if (a.kv_stride_b != int64_t(a.BS) * a.kv_stride_s || a.kv_stride_h * 2 % 16 || a.kv_stride_s * 2 % 16 ||
      a.kv_stride_kv * 2 % 16)
    return false;
  if ((reinterpret_cast<uintptr_t>(a.kv) | reinterpret_cast<uintptr_t>(a.q)) % 16) return false;
  if (a.q_stride_h * 2 % 16 || a.q_stride_r * 2 % 16) return false;
  return true;
}

// Token splits of the tensor-core kernel: one CTA per SM, one wave, whole tiles of 128 tokens.
int decode_tc_splits(int R, int Hkv, int64_t max_seq, int n_sm) {
  const int64_t want = int64_t(n_sm) / (int64_t(R) * Hkv);
  const int64_t cap = (max_seq + dtc::kTile - 1) / dtc::kTile;
  int64_t s = want < cap ? want : cap;
  return int(s < 1 ? 1 : (s > kDecodeMaxSplits ? kDecodeMaxSplits : s));
}

template <int G, bool BF16>
static cudaError_t launch_dtc_g(const CUtensorMap& mkv, const CUtensorMap& mq, const DecodeArgs& a, cudaStream_t st) {
  auto k = dtc::decode_tc_kernel<G, BF16>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(dtc::kSmemBytes));
  if (e != cudaSuccess) return e;
  k<<<dim3(a.splits, a.Hkv, a.R), dtc::kThreads, dtc::kSmemBytes, st>>>(mkv, mq, a);
  return cudaGetLastError();
}

template <bool BF16>
static cudaError_t launch_dtc_t(const CUtensorMap& mkv, const CUtensorMap& mq, const DecodeArgs& a, cudaStream_t st) {
  switch (a.G) {
    case 1: return launch_dtc_g<1, BF16>(mkv, mq, a, st);
    case 2: return launch_dtc_g<2, BF16>(mkv, mq, a, st);
    case 4: return launch_dtc_g<4, BF16>(mkv, mq, a, st);
    default: return launch_dtc_g<8, BF16>(mkv, mq, a, st);
  }
}

// The partials of every split (a.splits = decode_tc_splits); decode_combine_kernel merges them.
cudaError_t launch_decode_tc(const DecodeArgs& a, int dtype, cudaStream_t st, const char** why) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    if (why) *why = "cuTensorMapEncodeTiled unavailable";
    return cudaErrorNotSupported;
  }
  const CUtensorMapDataType dt = dtype == ACTKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mkv, mq;
  {
    const cuuint64_t dims[4] = {cuuint64_t(a.D), cuuint64_t(a.Hkv), cuuint64_t(a.NB) * a.BS, 2};
    const cuuint64_t strides[3] = {cuuint64_t(a.kv_stride_h) * 2, cuuint64_t(a.kv_stride_s) * 2,
                                   cuuint64_t(a.kv_stride_kv) * 2};
    const cuuint32_t box[4] = {64, 1, cuuint32_t(a.BS), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&mkv, dt, 4, const_cast<void*>(a.kv), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      if (why) *why = "cuTensorMapEncodeTiled rejected the K / V layout";
      return cudaErrorInvalidValue;
    }
  }
  {
    const cuuint64_t dims[3] = {cuuint64_t(a.D), cuuint64_t(a.Hq), cuuint64_t(a.R)};
    const cuuint64_t strides[2] = {cuuint64_t(a.q_stride_h) * 2, cuuint64_t(a.q_stride_r) * 2};
    const cuuint32_t box[3] = {64, cuuint32_t(a.G), 1};
    const cuuint32_t es[3] = {1, 1, 1};
    if (enc(&mq, dt, 3, const_cast<void*>(a.q), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      if (why) *why = "cuTensorMapEncodeTiled rejected the query layout";
      return cudaErrorInvalidValue;
    }
  }
  return dtype == ACTKV_BF16 ? launch_dtc_t<true>(mkv, mq, a, st) : launch_dtc_t<false>(mkv, mq, a, st);
}

}  // namespace actkv
