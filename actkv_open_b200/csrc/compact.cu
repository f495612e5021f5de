// Conflict-free in-place paged compaction (ActKV Algorithm 4) for a batch of sessions.
//
// Mirrors actkv/kernels/compaction.py:44-69 (plan), :96-106 (copies) and actkv/paged.py:125-139
// (table / free-list update), re-organised for the GPU:
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

// ---------------------------------------------------------------------------- permute
// grid (ceil(width / 256), R); dst rows are written for every j < width.
__global__ void __launch_bounds__(256) permute_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                      int64_t stride_r, int64_t stride_l, int L,
                                                      const uint8_t* __restrict__ pin_src,
                                                      uint8_t* __restrict__ pin_dst, int64_t pin_stride_r,
                                                      const int64_t* __restrict__ perm, int64_t perm_stride_r,
                                                      const int32_t* __restrict__ new_len, int width,
                                                      int32_t* status) {
  const int r = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= width) return;
  const int len = new_len[r];
  int64_t p = -1;
  if (j < len) {
    p = perm[r * perm_stride_r + j];
    if (p < 0 || p >= width) {
      flag(status, ACTKV_DEV_BAD_INDEX);
      p = -1;
    }
  }
  if (src) {
    for (int l = 0; l < L; ++l) {
      const int64_t o = r * stride_r + l * stride_l;
      dst[o + j] = p >= 0 ? src[o + p] : 0.0f;
    }
  }
  if (pin_src) pin_dst[r * pin_stride_r + j] = p >= 0 ? pin_src[r * pin_stride_r + p] : 0;
}

__global__ void add_kernel(int32_t* n, const int32_t* act_off, int R) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < R) n[i] += act_off ? act_off[i + 1] - act_off[i] : 1;
}

}  // namespace actkv
