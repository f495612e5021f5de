// Device-resident block allocation for a batch of sessions: batched append and release on the
// device block tables and free stack (actkv/paged.py:67-90: _ensure / append / release), so an
// agent loop never round-trips its tables through the host.
//
// append (sessions 0..R-1 in order, as the reference's per-request calls would run):
//   plan     one CTA: blocks needed per session (tables hold ceil(seq/BS) blocks), exclusive scan in
//            session order; session r fits when the blocks of sessions 0..r fit on the free stack
//            and in its table row.  Fitting sessions advance seq_used, free_top drops by their
//            total; from the first session that does not fit on, nothing changes and
//            ACTKV_DEV_OUT_OF_BLOCKS is raised (where the reference raises OutOfBlocks).
//   tables   one CTA per session: the popped blocks, free[top0-1-(pre_r+i)], go to the table row.
//   rows     one warp per (new token, 8 planes): slot looked up once, 8 rows in flight, 16-byte copies.
// release (sessions with release[r] != 0, in order): each pushes its blocks reversed onto the free
//   stack (free.extend(reversed(table))), then its table row, length and pinned row are cleared.
#include "kernels.cuh"

namespace actkv {

namespace {

struct BlockWs {            // carved out of the caller's workspace
  int32_t* need;            // [R] blocks to pop (append) / to push (release)
  int32_t* pre;             // [R] exclusive prefix of need in session order
  int32_t* start;           // [R] old seq_used
  int32_t* ok;              // [R] session takes part
  int32_t* top0;            // [1] free_top before the call
};

BlockWs carve_blocks(void* ws, int R) {
  char* p = static_cast<char*>(ws);
  BlockWs w;
  w.need = reinterpret_cast<int32_t*>(p);
  w.pre = w.need + R;
  w.start = w.pre + R;
  w.ok = w.start + R;
  w.top0 = w.ok + R;
  return w;
}

constexpr int kPlanThreads = 1024;

__global__ void append_plan_kernel(const int32_t* new_off, int32_t* seq_used, int MB, int BS, int32_t* free_top,
                                   int64_t free_capacity, BlockWs w, int R, int32_t* status) {
  __shared__ int red[33];
  __shared__ int carry, first_bad;
  const int top = *free_top;
  if (threadIdx.x == 0) {
    carry = 0;
    first_bad = R;
    *w.top0 = top;
  }
  __syncthreads();
  // blocks each session needs, their exclusive prefix in session order, and the first session
  // that does not fit (the free stack cannot give it its blocks, or its table row is full)
  for (int base = 0; base < R; base += kPlanThreads) {
    const int r = base + threadIdx.x;
    int need = 0, start = 0, n = 0;
    if (r < R) {
      start = seq_used[r];
      n = new_off[r + 1] - new_off[r];
      if (n < 0 || start < 0) {
        flag(status, ACTKV_DEV_BAD_INDEX);
        n = 0;
        start = start < 0 ? 0 : start;
      }
      need = (start + n + BS - 1) / BS - (start + BS - 1) / BS;
    }
    int total;
    const int pre = carry + block_excl_sum(need, red, &total);
    if (r < R) {
      w.need[r] = need;
      w.pre[r] = pre;
      w.start[r] = start;
      w.ok[r] = n;                                   // token count for now, the flag below
      if (pre + need > top || (start + n + BS - 1) / BS > MB) atomicMin(&first_bad, r);
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += total;
    __syncthreads();
  }
  // sessions before the first failure are appended, the rest untouched (the reference's loop
  // raises at the first failure); what they popped is the failing session's prefix
  const int F = first_bad;
  for (int r = threadIdx.x; r < R; r += kPlanThreads) {
    const int n = w.ok[r];
    const bool ok = r < F;
    w.ok[r] = ok;
    if (ok) seq_used[r] = w.start[r] + n;
  }
  if (threadIdx.x == 0) {
    *free_top = top - (F < R ? w.pre[F] : carry);
    if (F < R) flag(status, ACTKV_DEV_OUT_OF_BLOCKS);
    if (int64_t(top) > free_capacity) flag(status, ACTKV_DEV_BAD_INDEX);
  }
}

__global__ void append_tables_kernel(int32_t* block_table, int64_t bt_stride_r, int BS, const int32_t* free_list,
                                     BlockWs w, int32_t* status) {
  const int r = blockIdx.x;
  if (!w.ok[r]) return;
  const int need = w.need[r], pre = w.pre[r], top0 = *w.top0;
  const int have = (w.start[r] + BS - 1) / BS;
  int32_t* row = block_table + r * bt_stride_r;
  for (int i = threadIdx.x; i < need; i += blockDim.x) {
    const int idx = top0 - 1 - (pre + i);
    if (idx < 0) {
      flag(status, ACTKV_DEV_BAD_INDEX);
      continue;
    }
    row[have + i] = free_list[idx];
  }
}

// grid (chunks, R); one warp per (new token of session r, group of kPlaneGroup planes): the slot is
// looked up once per warp, and the group's rows are loaded (16-byte lanes) before any is stored, so
// a lane has kPlaneGroup loads in flight
constexpr int kPlaneGroup = 8;
__global__ void append_rows_kernel(char* kv, int L, int64_t plane_stride, int64_t slot_stride, int64_t row_bytes,
                                   int64_t n_slots, const char* k_new, const char* v_new, int64_t new_layer_stride,
                                   int64_t new_row_stride, const int32_t* new_off, const int32_t* block_table,
                                   int64_t bt_stride_r, int BS, BlockWs w, bool vec16, int32_t* status) {
  const int r = blockIdx.y;
  if (!w.ok[r]) return;
  const int n = new_off[r + 1] - new_off[r], start = w.start[r], off = new_off[r];
  const int lane = threadIdx.x & 31;
  const int groups = (2 * L + kPlaneGroup - 1) / kPlaneGroup;
  const int warp = int((int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int nwarps = int((int64_t(gridDim.x) * blockDim.x) >> 5);
  const int32_t* table = block_table + r * bt_stride_r;
  for (int item = warp; item < n * groups; item += nwarps) {
    const int j = item / groups, g0 = (item - j * groups) * kPlaneGroup;
    const int pos = start + j;
    const int64_t slot = int64_t(table[pos / BS]) * BS + pos % BS;
    if (slot < 0 || slot >= n_slots) {
      if (lane == 0) flag(status, ACTKV_DEV_BAD_INDEX);
      continue;
    }
    const int64_t src_row = int64_t(off + j) * new_row_stride;
    char* dst_slot = kv + slot * slot_stride;
    const int np = min(kPlaneGroup, 2 * L - g0);
    if (vec16) {
      for (int64_t b = int64_t(lane) * 16; b < row_bytes; b += 32 * 16) {
        int4 t[kPlaneGroup];
#pragma unroll
        for (int g = 0; g < kPlaneGroup; ++g) {
          const int lp = g0 + g;
          if (g < np)
            t[g] = *reinterpret_cast<const int4*>(((lp & 1) ? v_new : k_new) + (lp >> 1) * new_layer_stride +
                                                  src_row + b);
        }
#pragma unroll
        for (int g = 0; g < kPlaneGroup; ++g)
          if (g < np) *reinterpret_cast<int4*>(dst_slot + int64_t(g0 + g) * plane_stride + b) = t[g];
      }
    } else {
      for (int g = 0; g < np; ++g) {
        const int lp = g0 + g;
        const char* src = ((lp & 1) ? v_new : k_new) + (lp >> 1) * new_layer_stride + src_row;
        char* dst = dst_slot + int64_t(lp) * plane_stride;
        for (int64_t b = lane; b < row_bytes; b += 32) dst[b] = src[b];
      }
    }
  }
}

__global__ void release_plan_kernel(const uint8_t* release, const int32_t* seq_used, int BS, int32_t* free_top,
                                    int64_t free_capacity, BlockWs w, int R, int32_t* status) {
  __shared__ int red[33];
  __shared__ int carry;
  const int top = *free_top;
  if (threadIdx.x == 0) {
    carry = 0;
    *w.top0 = top;
  }
  __syncthreads();
  for (int base = 0; base < R; base += kPlanThreads) {
    const int r = base + threadIdx.x;
    const bool rel = r < R && release[r] != 0;
    const int n = rel ? (seq_used[r] + BS - 1) / BS : 0;
    int total;
    const int ex = block_excl_sum(n, red, &total);
    if (r < R) {
      w.need[r] = n;
      w.pre[r] = carry + ex;
      w.ok[r] = rel;
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (int64_t(top) + carry > free_capacity) flag(status, ACTKV_DEV_BAD_INDEX);
    else *free_top = top + carry;
  }
}

__global__ void release_push_kernel(int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r, int32_t* free_list,
                                    int64_t free_capacity, uint8_t* pinned, int64_t pinned_stride_r,
                                    int pinned_width, BlockWs w, int32_t* status) {
  const int r = blockIdx.x;
  if (!w.ok[r]) return;
  const int n = w.need[r], pre = w.pre[r], top0 = *w.top0;
  if (int64_t(top0) + pre + n > free_capacity) return;      // flagged by the plan
  int32_t* row = block_table + r * bt_stride_r;
  for (int i = threadIdx.x; i < n; i += blockDim.x) free_list[top0 + pre + i] = row[n - 1 - i];
  __syncthreads();                                           // every read of the row is done
  for (int i = threadIdx.x; i < n; i += blockDim.x) row[i] = 0;
  if (pinned)
    for (int i = threadIdx.x; i < pinned_width; i += blockDim.x) pinned[r * pinned_stride_r + i] = 0;
  if (threadIdx.x == 0) seq_used[r] = 0;
}

}  // namespace

size_t blocks_workspace_bytes(int R) { return align256(size_t(R > 0 ? R : 1) * 4 * 4 + 16); }

cudaError_t launch_append(char* kv, int L, int64_t plane_stride, int64_t slot_stride, int64_t row_bytes,
                          int64_t n_slots, const char* k_new, const char* v_new, int64_t new_layer_stride,
                          int64_t new_row_stride, const int32_t* new_off, int max_new, int32_t* seq_used,
                          int32_t* block_table, int64_t bt_stride_r, int MB, int BS, const int32_t* free_list,
                          int32_t* free_top, int64_t free_capacity, int R, void* workspace, int32_t* status,
                          cudaStream_t st) {
  BlockWs w = carve_blocks(workspace, R);
  append_plan_kernel<<<1, kPlanThreads, 0, st>>>(new_off, seq_used, MB, BS, free_top, free_capacity, w, R, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  append_tables_kernel<<<R, 256, 0, st>>>(block_table, bt_stride_r, BS, free_list, w, status);
  if ((e = cudaGetLastError()) != cudaSuccess || max_new <= 0) return e;
  const bool vec16 = row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(kv) | reinterpret_cast<uintptr_t>(k_new) |
                                              reinterpret_cast<uintptr_t>(v_new)) % 16 == 0 &&
                     plane_stride % 16 == 0 && slot_stride % 16 == 0 && new_layer_stride % 16 == 0 &&
                     new_row_stride % 16 == 0;
  const int threads = 256, warps_per_cta = threads / 32;
  const int64_t items = int64_t(max_new) * ((2 * L + kPlaneGroup - 1) / kPlaneGroup);
  const int64_t ctas = (items + warps_per_cta - 1) / warps_per_cta;      // a warp per (token, plane group)
  const int gx = int(ctas < 1184 ? ctas : 1184);
  if (gx <= 0) return cudaSuccess;
  append_rows_kernel<<<dim3(gx, R), threads, 0, st>>>(kv, L, plane_stride, slot_stride, row_bytes, n_slots, k_new,
                                                      v_new, new_layer_stride, new_row_stride, new_off, block_table,
                                                      bt_stride_r, BS, w, vec16, status);
  return cudaGetLastError();
}

cudaError_t launch_release(const uint8_t* release, int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r,
                           int BS, int32_t* free_list, int32_t* free_top, int64_t free_capacity, uint8_t* pinned,
                           int64_t pinned_stride_r, int pinned_width, int R, void* workspace, int32_t* status,
                           cudaStream_t st) {
  BlockWs w = carve_blocks(workspace, R);
  release_plan_kernel<<<1, kPlanThreads, 0, st>>>(release, seq_used, BS, free_top, free_capacity, w, R, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  release_push_kernel<<<R, 256, 0, st>>>(seq_used, block_table, bt_stride_r, free_list, free_capacity, pinned,
                                         pinned_stride_r, pinned_width, w, status);
  return cudaGetLastError();
}

}  // namespace actkv
