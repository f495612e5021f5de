// Conflict-free in-place paged compaction (ActKV Algorithm 4) for a batch of sessions.
//
// Mirrors actkv/kernels/compaction.py:44-69 (plan), :96-106 (copies) and actkv/paged.py:125-139
// (table / free-list update), re-organised for the GPU:
//   batched (actkv_compact): count_chunks / plan_chunks / copy_pairs / finish, below: the
//                  plan of every session spread over chunks of 4096 tokens, one CTA each.
//   one session (actkv_plan_compaction, the drop-in plan_compaction):
//   count_kernel   one CTA per session: B = #kept, drop = Y - X; the last CTA to finish (atomic
//                  ticket, no spinning) turns the drops into free-stack push offsets in session
//                  order and moves the stack top.
//   plan_kernel    one CTA per session: block-wide ballot scans rank the kept-outside-window tokens
//                  (sources) and the window's holes (destinations) in ascending order, write the
//                  (src, dst) physical-slot pairs and perm, then rewrite the table row and push the
//                  freed blocks (reversed) onto the free stack.
//   copy_kernel    persistent grid, one warp per (pair, plane) row, 16-byte vector loads/stores.
//   permute_kernel gathers per-token state (keep scores, pinned flags) through perm.
#include "kernels.cuh"

namespace actkv {

__device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------- count
// seq_used == nullptr: a single session of seq_const tokens.  free_top == nullptr: no free stack.
// One CTA of kCountThreads per session; each thread counts 16 consecutive bytes per step.
__global__ void __launch_bounds__(kCountThreads) count_kernel(const uint8_t* __restrict__ keep, int64_t keep_stride_r,
                                                              const int32_t* __restrict__ seq_used, int seq_const,
                                                              int BS, CompactWs ws, int32_t* free_top,
                                                              int64_t free_capacity, int32_t* kept_out, int R,
                                                              int32_t* status) {
  __shared__ int red[33];
  __shared__ bool last;
  const int r = blockIdx.x;
  const int n = seq_used ? seq_used[r] : seq_const;
  const uint8_t* row = keep + r * keep_stride_r;
  int c = 0;
  for (int t0 = threadIdx.x * 16; t0 < n; t0 += blockDim.x * 16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) c += (t0 + i < n) && row[t0 + i] != 0;
  }
  c = block_sum(c, red);
  if (threadIdx.x == 0) {
    ws.kept[r] = c;
    if (kept_out) kept_out[r] = c;
    ws.drop[r] = ceil_div(n, BS) - ceil_div(c, BS);
    __threadfence();
    last = atomicAdd(ws.ticket, 1) == R - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    int top = free_top ? *free_top : 0;
    for (int i = 0; i < R; ++i) {
      ws.push_off[i] = top;
      top += *((volatile int32_t*)&ws.drop[i]);
    }
    if (free_top) {
      if (top > free_capacity) flag(status, ACTKV_DEV_BAD_INDEX);
      else *free_top = top;
    }
    *ws.ticket = 0;
  }
}

// ---------------------------------------------------------------------------- plan
__device__ __forceinline__ int64_t phys_slot(const int32_t* table, int logical, int BS, int64_t n_slots,
                                             int32_t* status) {
  const int64_t s = int64_t(table[logical / BS]) * BS + logical % BS;
  if (s < 0 || s >= n_slots) {
    flag(status, ACTKV_DEV_BAD_INDEX);
    return -1;
  }
  return s;
}

// One CTA (1024 threads) per session.
// update_cache == false: plan only (no table / free-list / seq_used writes); counts (may be null)
// receives {B, n_pairs, drop_blocks, start} of session 0.
__global__ void __launch_bounds__(1024) plan_kernel(const uint8_t* __restrict__ keep, int64_t keep_stride_r,
                                                    int32_t* seq_used, int seq_const, int32_t* block_table,
                                                    int64_t bt_stride_r, int MB, int BS, int64_t n_slots,
                                                    int32_t* free_list, int64_t free_capacity,
                                                    int64_t* perm, int64_t perm_stride_r, CompactWs ws,
                                                    bool update_cache, int32_t* counts, int32_t* status) {
  __shared__ int red[33];
  const int r = blockIdx.x;
  const int n = seq_used ? seq_used[r] : seq_const;
  const int B = ws.kept[r];
  const int y = ceil_div(n, BS), x = ceil_div(B, BS);
  const int start = (y - x) * BS, end = start + B;
  const uint8_t* krow = keep + r * keep_stride_r;
  int32_t* table = block_table + r * bt_stride_r;
  int32_t* src_log = ws.src_logical + r * ws.cap;
  int64_t* psrc = ws.pair_src + r * ws.cap;
  int64_t* pdst = ws.pair_dst + r * ws.cap;
  int64_t* prow = perm ? perm + r * perm_stride_r : nullptr;
  if (y > MB) {                      // the table row cannot hold this session: refuse it
    if (threadIdx.x == 0) {
      ws.pair_count[r] = 0;
      flag(status, ACTKV_DEV_BAD_INDEX);
    }
    return;
  }
  // Each thread takes 16 consecutive positions per step; a block-wide exclusive sum of the
  // per-thread counts gives every position its rank in ascending order.
  constexpr int kPer = 16;
  const int step = blockDim.x * kPer;
  // pass A: rank the kept tokens outside the window, ascending
  int n_src = 0;
  for (int base = 0; base < n; base += step) {
    const int t0 = base + threadIdx.x * kPer;
    uint32_t bits = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int t = t0 + i;
      if (t < n && krow[t] && (t < start || t >= end)) bits |= 1u << i;
    }
    int tot;
    int rank = block_excl_sum(__popc(bits), red, &tot) + n_src;
    for (uint32_t b = bits; b; b &= b - 1) src_log[rank++] = t0 + __ffs(b) - 1;
    n_src += tot;
  }
  __syncthreads();
  // pass B: rank the holes inside the window, ascending, and pair them with the sources
  int n_dst = 0;
  for (int base = start; base < end; base += step) {
    const int t0 = base + threadIdx.x * kPer;
    uint32_t holes = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int t = t0 + i;
      if (t < end && !(t < n && krow[t])) holes |= 1u << i;
    }
    int tot;
    int rank = block_excl_sum(__popc(holes), red, &tot) + n_dst;
    for (int i = 0; i < kPer; ++i) {
      const int t = t0 + i;
      if (t >= end) break;
      if (holes & (1u << i)) {
        const int s = rank < n_src ? src_log[rank] : -1;
        if (s < 0) {
          flag(status, ACTKV_DEV_BAD_INDEX);
        } else {
          if (prow) prow[t - start] = s;
          psrc[rank] = phys_slot(table, s, BS, n_slots, status);
          pdst[rank] = phys_slot(table, t, BS, n_slots, status);
        }
        ++rank;
      } else if (prow) {
        prow[t - start] = t;
      }
    }
    n_dst += tot;
  }
  if (threadIdx.x == 0) {
    ws.pair_count[r] = n_src == n_dst ? n_src : 0;
    if (n_src != n_dst) flag(status, ACTKV_DEV_BAD_INDEX);
    if (counts && r == 0) {
      counts[0] = B;
      counts[1] = ws.pair_count[r];
      counts[2] = y - x;
      counts[3] = start;
    }
  }
  if (!update_cache) return;
  __syncthreads();
  // table rewrite: keep table[drop:y], push table[0:drop] reversed, zero the vacated tail
  const int drop = y - x;
  int32_t* tmp = src_log;            // free now: pairs are written
  for (int i = threadIdx.x; i < y; i += blockDim.x) tmp[i] = table[i];
  __syncthreads();
  for (int i = threadIdx.x; i < y; i += blockDim.x) table[i] = i < x ? tmp[drop + i] : 0;
  const int off = ws.push_off[r];
  for (int i = threadIdx.x; i < drop; i += blockDim.x) {
    const int64_t pos = int64_t(off) + i;
    if (pos < free_capacity) free_list[pos] = tmp[drop - 1 - i];
    else flag(status, ACTKV_DEV_BAD_INDEX);
  }
  if (threadIdx.x == 0) seq_used[r] = B;
}

// ---------------------------------------------------------------------------- chunked plan
// The batched compaction (actkv_compact) plans every session over chunks of kChunkTok tokens, one
// CTA each, so that a single long session is planned by many SMs:
//   count_chunks_kernel  kept tokens per chunk; the last CTA (ticket) turns them into per-session
//                        exclusive prefixes, B, drop and the free-stack push offsets
//   plan_chunks_kernel   each chunk ranks its sources (kept tokens outside the window) and holes
//                        (window positions not kept) from the prefixes, K(start) and K(end), and
//                        writes them as logical positions in ascending rank order; kept tokens
//                        inside the window keep their place (perm[t - start] = t)
//   copy_pairs_kernel    pair i = (i-th source, i-th hole): physical slots through the old table,
//                        perm[hole - start] = source, row copies over every plane
//   finish_kernel        table rewrite, freed blocks pushed (reversed), seq_used = B
// Every position of a session is in exactly one chunk, so the ranks are those of the one-CTA plan.

__device__ __forceinline__ uint32_t kept_bits16(const uint8_t* row, int t0, int n) {
  uint32_t b = 0;
  if (t0 + 16 <= n && (reinterpret_cast<uintptr_t>(row + t0) & 15u) == 0) {
    const uint4 v = *reinterpret_cast<const uint4*>(row + t0);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) b |= ((w[i >> 2] >> (8 * (i & 3))) & 0xFFu) ? 1u << i : 0u;
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) b |= (t0 + i < n && row[t0 + i]) ? 1u << i : 0u;
  }
  return b;
}

__global__ void __launch_bounds__(kChunkThreads) count_chunks_kernel(const uint8_t* __restrict__ keep,
                                                                     int64_t keep_stride_r,
                                                                     const int32_t* __restrict__ seq_used, int BS,
                                                                     ChunkWs ws, int32_t* free_top,
                                                                     int64_t free_capacity, int32_t* kept_out, int R,
                                                                     int32_t* status) {
  __shared__ int red[33];
  __shared__ bool last;
  const int r = blockIdx.y, c = blockIdx.x;
  const int n = seq_used[r];
  const uint8_t* row = keep + r * keep_stride_r;
  const int t0 = c * kChunkTok + threadIdx.x * 16;
  int cnt = t0 < n ? __popc(kept_bits16(row, t0, n)) : 0;
  cnt = block_sum(cnt, red);
  if (threadIdx.x == 0) {
    ws.cpre[r * (ws.nchunk + 1) + c] = cnt;
    __threadfence();
    last = atomicAdd(ws.ticket, 1) == int(gridDim.x * gridDim.y) - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int q = threadIdx.x; q < R; q += blockDim.x) {
    volatile int32_t* pre = ws.cpre + q * (ws.nchunk + 1);
    int acc = 0;
    for (int k = 0; k < ws.nchunk; ++k) {
      const int v = pre[k];
      pre[k] = acc;
      acc += v;
    }
    pre[ws.nchunk] = acc;
    ws.kept[q] = acc;
    if (kept_out) kept_out[q] = acc;
    ws.drop[q] = ceil_div(seq_used[q], BS) - ceil_div(acc, BS);
    ws.pair_count[q] = 0;                    // the plan's first chunk writes the real count
  }
  __syncthreads();
  int top = free_top ? *free_top : 0;
  for (int base = 0; base < R; base += blockDim.x) {
    const int q = base + threadIdx.x;
    int tot;
    const int ex = block_excl_sum(q < R ? *((volatile int32_t*)&ws.drop[q]) : 0, red, &tot);
    if (q < R) ws.push_off[q] = top + ex;
    top += tot;
  }
  if (threadIdx.x == 0) {
    if (free_top) {
      if (top > free_capacity) flag(status, ACTKV_DEV_BAD_INDEX);
      else *free_top = top;
    }
    *ws.ticket = 0;
  }
}

__global__ void __launch_bounds__(kChunkThreads) plan_chunks_kernel(const uint8_t* __restrict__ keep,
                                                                    int64_t keep_stride_r,
                                                                    const int32_t* __restrict__ seq_used, int MB,
                                                                    int BS, int64_t* perm, int64_t perm_stride_r,
                                                                    ChunkWs ws, int32_t* status) {
  pdl_wait();                                   // launched by launch_pdl: see common.cuh
  pdl_trigger();
  __shared__ int red[33];
  const int r = blockIdx.y, c = blockIdx.x;
  const int n = seq_used[r];
  const int B = ws.kept[r];
  const int y = ceil_div(n, BS), x = ceil_div(B, BS);
  const int start = (y - x) * BS, end = start + B, span = y * BS;
  if (y > MB) {                                // the table row cannot hold this session: refuse it
    if (c == 0 && threadIdx.x == 0) flag(status, ACTKV_DEV_BAD_INDEX);
    return;
  }
  const int lo = c * kChunkTok;
  if (lo >= span) return;                      // uniform over the CTA
  const int hi = min(lo + kChunkTok, span);
  const uint8_t* row = keep + r * keep_stride_r;
  const int32_t* pre = ws.cpre + r * (ws.nchunk + 1);
  // K(p): kept tokens before position p (the chunk prefix plus a count inside p's chunk)
  auto K = [&](int p) -> int {
    const int cp = p / kChunkTok;
    const int t0 = cp * kChunkTok + threadIdx.x * 16;
    int k = 0;
    if (t0 < p) {
      const uint32_t b = kept_bits16(row, t0, n);
      const int m = min(16, p - t0);
      k = __popc(m == 16 ? b : b & ((1u << m) - 1u));
    }
    return (cp < ws.nchunk ? pre[cp] : pre[ws.nchunk]) + block_sum(k, red);
  };
  const int Ks = K(start), Ke = K(end);
  const int Klo = pre[c];
  const int src_base = (lo <= start ? Klo : Ks) + (lo > end ? Klo - Ke : 0);
  const int dst_base = lo <= start ? 0 : (min(lo, end) - start) - ((lo <= end ? Klo : Ke) - Ks);
  const int t0 = lo + threadIdx.x * 16;
  uint32_t kb = 0, valid = 0, inwin = 0;
  if (t0 < hi) {
    kb = t0 < n ? kept_bits16(row, t0, n) : 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int t = t0 + i;
      valid |= t < hi ? 1u << i : 0u;
      inwin |= (t >= start && t < end) ? 1u << i : 0u;
    }
  }
  kb &= valid;
  const uint32_t srcb = kb & ~inwin, holeb = valid & inwin & ~kb, identb = kb & inwin;
  int tot;
  int rs = src_base + block_excl_sum(__popc(srcb), red, &tot);
  int rh = dst_base + block_excl_sum(__popc(holeb), red, &tot);
  int32_t* slog = ws.src_log + r * ws.cap;
  int32_t* dlog = ws.dst_log + r * ws.cap;
  int64_t* prow = perm ? perm + r * perm_stride_r : nullptr;
  for (uint32_t b = srcb; b; b &= b - 1) slog[rs++] = t0 + __ffs(b) - 1;
  for (uint32_t b = holeb; b; b &= b - 1) dlog[rh++] = t0 + __ffs(b) - 1;
  if (prow)
    for (uint32_t b = identb; b; b &= b - 1) {
      const int t = t0 + __ffs(b) - 1;
      prow[t - start] = t;
    }
  if (c == 0 && threadIdx.x == 0) ws.pair_count[r] = Ks + (B - Ke);
}

// ---------------------------------------------------------------------------- copy
__device__ __forceinline__ void copy_row(const char* __restrict__ s, char* __restrict__ d, int64_t row_bytes,
                                         int lane, bool vec16) {
  if (vec16) {
    int64_t off = int64_t(lane) * 16;
    for (; off + 3 * 512 < row_bytes; off += 4 * 512) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(s + off));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(s + off + 512));
      const uint4 c = __ldg(reinterpret_cast<const uint4*>(s + off + 1024));
      const uint4 e = __ldg(reinterpret_cast<const uint4*>(s + off + 1536));
      *reinterpret_cast<uint4*>(d + off) = a;
      *reinterpret_cast<uint4*>(d + off + 512) = b;
      *reinterpret_cast<uint4*>(d + off + 1024) = c;
      *reinterpret_cast<uint4*>(d + off + 1536) = e;
    }
    for (; off < row_bytes; off += 512)
      *reinterpret_cast<uint4*>(d + off) = __ldg(reinterpret_cast<const uint4*>(s + off));
  } else {
    for (int64_t off = lane; off < row_bytes; off += 32) d[off] = s[off];
  }
}

// Persistent: warp w copies rows w, w + n_warps, ... of the flattened (pair, plane) space.
// Pairs of session r live at pair_src/dst[r * pair_stride + i], i < pair_count[r]
// (pair_count == nullptr: one session with single_count pairs).
__global__ void __launch_bounds__(256) copy_kernel(char* __restrict__ kv, int n_planes, int64_t plane_stride,
                                                   int64_t slot_stride, int64_t row_bytes, int64_t n_slots,
                                                   const int64_t* __restrict__ pair_src,
                                                   const int64_t* __restrict__ pair_dst, int64_t pair_stride,
                                                   const int32_t* __restrict__ pair_count, int64_t single_count,
                                                   int R, bool vec16, int32_t* status) {
  extern __shared__ int64_t prefix[];            // [R + 1]
  if (pair_count) {
    if (threadIdx.x == 0) {
      int64_t acc = 0;
      for (int i = 0; i < R; ++i) {
        prefix[i] = acc;
        acc += pair_count[i];
      }
      prefix[R] = acc;
    }
  } else if (threadIdx.x == 0) {
    prefix[0] = 0;
    prefix[1] = single_count;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t total = prefix[R] * n_planes;
  int r = 0;
  for (int64_t item = warp; item < total; item += n_warps) {
    const int64_t pg = item / n_planes;
    const int plane = int(item - pg * n_planes);
    while (r + 1 <= R && prefix[r + 1] <= pg) ++r;        // items ascend per warp
    const int64_t i = pg - prefix[r];
    const int64_t s = pair_src[r * pair_stride + i];
    const int64_t d = pair_dst[r * pair_stride + i];
    if (s < 0 || d < 0 || s >= n_slots || d >= n_slots) {
      if (lane == 0) flag(status, ACTKV_DEV_BAD_INDEX);
      continue;
    }
    const char* sp = kv + plane * plane_stride + s * slot_stride;
    char* dp = kv + plane * plane_stride + d * slot_stride;
    copy_row(sp, dp, row_bytes, lane, vec16);
  }
}

// Persistent: warp w copies rows w, w + n_warps, ... of the flattened (pair, plane) space; pair i
// of session r is (src_log[i], dst_log[i]), mapped to physical slots through the (old) table.
__global__ void __launch_bounds__(256) copy_pairs_kernel(char* __restrict__ kv, int n_planes, int64_t plane_stride,
                                                         int64_t slot_stride, int64_t row_bytes, int64_t n_slots,
                                                         const int32_t* __restrict__ seq_used,
                                                         const int32_t* __restrict__ block_table, int64_t bt_stride_r,
                                                         int BS, int64_t* perm, int64_t perm_stride_r, ChunkWs ws,
                                                         int R, bool vec16, int32_t* status) {
  pdl_wait();                                   // launched by launch_pdl: see common.cuh
  pdl_trigger();
  extern __shared__ int64_t cp_smem[];           // prefix [R + 1], then start [R] (int32)
  int64_t* prefix = cp_smem;
  int32_t* start = reinterpret_cast<int32_t*>(cp_smem + R + 1);
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int i = 0; i < R; ++i) {
      prefix[i] = acc;
      acc += ws.pair_count[i];
    }
    prefix[R] = acc;
  }
  for (int i = threadIdx.x; i < R; i += blockDim.x)
    start[i] = (ceil_div(seq_used[i], BS) - ceil_div(ws.kept[i], BS)) * BS;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t total = prefix[R] * n_planes;
  int r = 0;
  for (int64_t item = warp; item < total; item += n_warps) {
    const int64_t pg = item / n_planes;
    const int plane = int(item - pg * n_planes);
    while (r + 1 <= R && prefix[r + 1] <= pg) ++r;        // items ascend per warp
    const int64_t i = pg - prefix[r];
    const int sl = ws.src_log[r * ws.cap + i], dl = ws.dst_log[r * ws.cap + i];
    const int32_t* table = block_table + r * bt_stride_r;
    const int64_t s = int64_t(table[sl / BS]) * BS + sl % BS;
    const int64_t d = int64_t(table[dl / BS]) * BS + dl % BS;
    if (s < 0 || d < 0 || s >= n_slots || d >= n_slots) {
      if (lane == 0) flag(status, ACTKV_DEV_BAD_INDEX);
      continue;
    }
    if (plane == 0 && lane == 0 && perm) perm[r * perm_stride_r + (dl - start[r])] = sl;
    copy_row(kv + plane * plane_stride + s * slot_stride, kv + plane * plane_stride + d * slot_stride, row_bytes,
             lane, vec16);
  }
}

// One CTA per session, after the copies: the table keeps blocks [drop, y) at its front (the rest
// zeroed), blocks [0, drop) go onto the free stack reversed at the session's push offset, and
// seq_used becomes B (actkv/paged.py:135-139).
__global__ void __launch_bounds__(256) finish_kernel(int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r,
                                                     int MB, int BS, int32_t* free_list, int64_t free_capacity,
                                                     ChunkWs ws, int32_t* status) {
  pdl_wait();                                   // launched by launch_pdl: see common.cuh
  pdl_trigger();
  const int r = blockIdx.x;
  const int n = seq_used[r];
  const int B = ws.kept[r];
  const int y = ceil_div(n, BS), x = ceil_div(B, BS), drop = y - x;
  if (y > MB) return;                           // refused by the plan
  int32_t* table = block_table + r * bt_stride_r;
  int32_t* tmp = ws.src_log + r * ws.cap;       // free now: the copies are done
  for (int i = threadIdx.x; i < y; i += blockDim.x) tmp[i] = table[i];
  __syncthreads();
  for (int i = threadIdx.x; i < y; i += blockDim.x) table[i] = i < x ? tmp[drop + i] : 0;
  const int off = ws.push_off[r];
  for (int i = threadIdx.x; i < drop; i += blockDim.x) {
    const int64_t pos = int64_t(off) + i;
    if (pos < free_capacity) free_list[pos] = tmp[drop - 1 - i];
    else flag(status, ACTKV_DEV_BAD_INDEX);
  }
  if (threadIdx.x == 0) seq_used[r] = B;
}

// ---------------------------------------------------------------------------- permute
// grid (ceil(width / 256), R, ceil(L / 8)): CTA z moves layers [8z, 8z + 8); dst rows are written for
// every j < width; the pins go with z = 0.
__global__ void __launch_bounds__(256) permute_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                      int64_t stride_r, int64_t stride_l, int L,
                                                      const uint8_t* __restrict__ pin_src,
                                                      uint8_t* __restrict__ pin_dst, int64_t pin_stride_r,
                                                      const int64_t* __restrict__ perm, int64_t perm_stride_r,
                                                      const int32_t* __restrict__ new_len, int width,
                                                      int32_t* status) {
  pdl_wait();                                   // launched by launch_pdl: see common.cuh
  pdl_trigger();
  const int r = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= width) return;
  const int len = new_len[r];
  int64_t p = -1;
  if (j < len) {
    p = perm[r * perm_stride_r + j];
    if (p < 0 || p >= width) {
      if (blockIdx.z == 0) flag(status, ACTKV_DEV_BAD_INDEX);
      p = -1;
    }
  }
  if (src) {
    // this CTA's 8 layers (grid z): their loads in flight together, then their stores
    int l = blockIdx.z * 8;
    const int l_end = min(L, l + 8);
    for (; l + 8 <= l_end; l += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = p >= 0 ? __ldg(src + r * stride_r + (l + k) * stride_l + p) : 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) dst[r * stride_r + (l + k) * stride_l + j] = v[k];
    }
    for (; l < l_end; ++l) {
      const int64_t o = r * stride_r + l * stride_l;
      dst[o + j] = p >= 0 ? src[o + p] : 0.0f;
    }
  }
  if (pin_src && blockIdx.z == 0) pin_dst[r * pin_stride_r + j] = p >= 0 ? pin_src[r * pin_stride_r + p] : 0;
}

__global__ void add_kernel(int32_t* n, const int32_t* act_off, int R) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < R) n[i] += act_off ? act_off[i + 1] - act_off[i] : 1;
}

}  // namespace actkv
