// Declarations shared by the kernel translation units and the C-ABI layer.
#pragma once
#include "common.cuh"
#include "score_common.cuh"

namespace actkv {

// SM count of the current device (148 on a B200; 148 if the query fails).
int device_sm_count();

// Launch with programmatic stream serialization (see pdl_wait): the kernel may be scheduled while
// the previous kernel in the stream finishes, and must call pdl_wait() before it touches global
// memory.  Grids of kernels declared with __cluster_dims__ keep their clusters.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------- compaction (compact.cu)
struct CompactWs {           // carved out of the caller's workspace
  int32_t* kept;             // [R] kept tokens per session
  int32_t* drop;             // [R] blocks freed per session
  int32_t* push_off;         // [R] where session r's freed blocks go on the free stack
  int32_t* pair_count;       // [R] copy pairs per session
  int32_t* ticket;           // [1] CTAs of count_kernel done (reset by the last one)
  int64_t* pair_src;         // [R * cap] physical source slots
  int64_t* pair_dst;         // [R * cap] physical destination slots
  int32_t* src_logical;      // [R * cap] ranked source positions; later the table scratch
  int64_t cap;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
constexpr int kCountThreads = 1024;
inline size_t compact_header_bytes(int R) { return align256(size_t(R) * 4 * 4 + 16); }

// chunked batch plan (actkv_compact)
constexpr int kChunkTok = 4096;          // tokens per CTA of the chunked count / plan
constexpr int kChunkThreads = 256;       // 16 tokens (one 16-byte mask load) per thread
struct ChunkWs {
  int32_t* kept;             // [R]
  int32_t* drop;             // [R]
  int32_t* push_off;         // [R]
  int32_t* pair_count;       // [R]
  int32_t* ticket;           // [1]
  int32_t* cpre;             // [R][nchunk + 1] kept tokens before each chunk, then the total
  int32_t* src_log;          // [R * cap] sources (logical positions) in rank order; later the table scratch
  int32_t* dst_log;          // [R * cap] holes (logical positions) in rank order
  int64_t cap;
  int nchunk;
};
inline int chunk_count(int64_t max_seq, int BS) {
  const int64_t span = (max_seq + BS - 1) / BS * BS;
  return int(span > 0 ? (span + kChunkTok - 1) / kChunkTok : 1);
}
__global__ void count_chunks_kernel(const uint8_t* keep, int64_t keep_stride_r, const int32_t* seq_used, int BS,
                                    ChunkWs ws, int32_t* free_top, int64_t free_capacity, int32_t* kept_out, int R,
                                    int32_t* status);
__global__ void plan_chunks_kernel(const uint8_t* keep, int64_t keep_stride_r, const int32_t* seq_used, int MB,
                                   int BS, int64_t* perm, int64_t perm_stride_r, ChunkWs ws, int32_t* status);
__global__ void copy_pairs_kernel(char* kv, int n_planes, int64_t plane_stride, int64_t slot_stride, int64_t row_bytes,
                                  int64_t n_slots, const int32_t* seq_used, const int32_t* block_table,
                                  int64_t bt_stride_r, int BS, int64_t* perm, int64_t perm_stride_r, ChunkWs ws, int R,
                                  bool vec16, int32_t* status);
__global__ void finish_kernel(int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r, int MB, int BS,
                              int32_t* free_list, int64_t free_capacity, ChunkWs ws, int32_t* status);

__global__ void count_kernel(const uint8_t* keep, int64_t keep_stride_r, const int32_t* seq_used, int seq_const,
                             int BS, CompactWs ws, int32_t* free_top, int64_t free_capacity, int32_t* kept_out,
                             int R, int32_t* status);
__global__ void plan_kernel(const uint8_t* keep, int64_t keep_stride_r, int32_t* seq_used, int seq_const,
                            int32_t* block_table, int64_t bt_stride_r, int MB, int BS, int64_t n_slots,
                            int32_t* free_list, int64_t free_capacity, int64_t* perm, int64_t perm_stride_r,
                            CompactWs ws, bool update_cache, int32_t* counts, int32_t* status);
__global__ void copy_kernel(char* kv, int n_planes, int64_t plane_stride, int64_t slot_stride, int64_t row_bytes,
                            int64_t n_slots, const int64_t* pair_src, const int64_t* pair_dst, int64_t pair_stride,
                            const int32_t* pair_count, int64_t single_count, int R, bool vec16, int32_t* status);
__global__ void permute_kernel(const float* src, float* dst, int64_t stride_r, int64_t stride_l, int L,
                               const uint8_t* pin_src, uint8_t* pin_dst, int64_t pin_stride_r, const int64_t* perm,
                               int64_t perm_stride_r, const int32_t* new_len, int width, int32_t* status);
__global__ void add_kernel(int32_t* n, const int32_t* act_off, int R);

// ---------------------------------------------------------------- block allocation (blocks.cu)
size_t blocks_workspace_bytes(int R);
cudaError_t launch_append(char* kv, int L, int64_t plane_stride, int64_t slot_stride, int64_t row_bytes,
                          int64_t n_slots, const char* k_new, const char* v_new, int64_t new_layer_stride,
                          int64_t new_row_stride, const int32_t* new_off, int max_new, int32_t* seq_used,
                          int32_t* block_table, int64_t bt_stride_r, int MB, int BS, const int32_t* free_list,
                          int32_t* free_top, int64_t free_capacity, int R, void* workspace, int32_t* status,
                          cudaStream_t st);
cudaError_t launch_release(const uint8_t* release, int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r,
                           int BS, int32_t* free_list, int32_t* free_top, int64_t free_capacity, uint8_t* pinned,
                           int64_t pinned_stride_r, int pinned_width, int R, void* workspace, int32_t* status,
                           cudaStream_t st);

// ---------------------------------------------------------------- selection (select.cu)
struct KeepMaskArgs {
  const float* scores;
  const int64_t* scores_off;
  int64_t stride_r, stride_l, stride_x;
  int n_lead, n_red, reduce;
  const uint8_t* pinned;
  int64_t pinned_stride_r;
  int protected_prefix;
  const int32_t* seq_used;
  const int32_t* budget;
  int evict_semantics;
  uint8_t* keep;
  int64_t keep_stride_r;
  int32_t* kept;
  float* s_ws;               // [R * max_seq] reduced per-token scores
  int64_t max_seq;
  int32_t* status;
};

struct LrfuArgs {
  const float* src;
  const int64_t* src_off;
  int64_t src_stride_r, src_stride_l, src_stride_h;
  int H, reduce;
  float* ks;
  int64_t ks_stride_r, ks_stride_l;
  float* act;
  int64_t act_stride_r, act_stride_l;
  const uint8_t* pinned;
  int64_t pinned_stride_r;
  int protected_prefix;
  const int32_t* seq_used;
  const int32_t* n_act;
  float decay, top_p;
  int32_t* status;
  int64_t max_seq;           // >= every row length; 0 = unknown
};

// reduce + select launches of the keep mask (R sessions) and of the ActionLRFU update (R x L rows)
cudaError_t launch_keep_mask(const KeepMaskArgs& a, int R, cudaStream_t st);
cudaError_t launch_lrfu(const LrfuArgs& a, int R, int L, cudaStream_t st);

// ---------------------------------------------------------------- scoring (score_umma.cu)
bool umma_supported(const ScoreArgs& a, int kv_dtype, int q_dtype, const char** why);
cudaError_t launch_score_umma(const ScoreArgs& a, int dtype, int sum_A, int max_A, int grid, cudaStream_t st,
                              const char** why);
// CTA-pair kernel (score_pair.cu)
size_t pair_workspace_bytes(int L, int sum_A, int Hq);
bool pair_supported(const ScoreArgs& a, int max_A);
cudaError_t launch_score_pair(const ScoreArgs& a, int dtype, int sum_A, int max_A, void* workspace,
                              cudaStream_t st, const char** why);

// ---------------------------------------------------------------- region lse (lse_umma.cu)
constexpr int kLseTileTokens = 128;        // tokens per key tile (one MMA of N = 128 per row block)
constexpr int kLseSplitTiles = 32;         // key tiles per unit at most (4096 tokens)
constexpr int kLseParts = 4;               // partial (max, sum) pairs per row and split

// Splits a session of max_seq tokens can need (the workspace holds this many per row).
inline int lse_nsplit(int64_t max_seq) {
  const int64_t t = (max_seq + kLseTileTokens - 1) / kLseTileTokens;
  return int(t > 0 ? (t + kLseSplitTiles - 1) / kLseSplitTiles : 1);
}

struct LseArgs {
  const void* q;
  int64_t q_stride_l, q_stride_a, q_stride_h;
  const int32_t* act_off;
  const void* kv;
  int64_t kv_stride_l, kv_stride_kv, kv_stride_b, kv_stride_s, kv_stride_h;
  const int32_t* block_table;
  int64_t bt_stride_r;
  const int32_t* seq_used;
  float* lse;
  int64_t lse_stride_l, lse_stride_a;
  float2* part;              // [L][sum_A][Hq][nsplit][kLseParts] partial (max, sum) in log2 units
  int R, L, MB, NB, BS, Hq, Hkv, G, D, sum_A, nsplit;
  float scale;
  int32_t* status;
};

bool lse_umma_supported(const LseArgs& a, int kv_dtype, int q_dtype, const char** why);

// ---------------------------------------------------------------- adaptive budget (budget.cu)
constexpr int kBudgetMaxPooled = 16384;    // min-pooled windows per trace (shared memory of one CTA)

struct ConfidenceArgs {
  const void* logits;
  int64_t row_stride;
  int V, k;
  const int32_t* sessions;   // row b -> session (nullptr: row b is session b)
  float* trace;              // [R][capacity]
  int64_t capacity;
  int32_t* trace_len;        // [R], advanced by one per recorded row
  int32_t* status;
};

struct BudgetArgs {
  const float* trace;
  int64_t capacity;
  const int32_t* trace_len;
  int window, stride;
  double bottom_pct, scale_up, shrink_slope, scale_down;
  int upper, lower, bidirectional, shrink_patience;
  const int32_t* seq_used;   // nullptr: step every session
  int protected_tokens;
  int32_t* budget;           // [R] in/out
  int32_t* rising;           // [R] in/out
  double* slope;             // [R] out, NaN where not stepped (nullable)
  int32_t* budget_out;       // [R] copy of the new budget (nullable)
  int32_t* status;
};

cudaError_t launch_confidence(const ConfidenceArgs& a, int dtype, int B, cudaStream_t st);

// ---------------------------------------------------------------- baseline policies (policies.cu)
constexpr int kSnapMaxRows = 64;           // observed rows one SnapKV selection can sum
constexpr int kSnapMaxPool = 64;

struct SnapScoreArgs {
  const float* rows;         // ring [slot][layer][W] of observed attention rows
  int64_t stride_slot, stride_l;
  const int32_t* lens;       // [slot][layer] row lengths
  int64_t lens_stride_slot;
  int slots[kSnapMaxRows];   // the w rows to sum, oldest first
  int w, length, pool, rest;  // rest = budget - w
  float* scores;             // [L][stride_out]
  uint8_t* pinned;           // [L][stride_out] observation window
  int64_t stride_out;
  int32_t* seq;              // [L] = length
  int32_t* budget_rest;      // [L] = rest
};

struct SnapGatherArgs {
  const float* src;
  float* dst;
  int64_t stride_slot, stride_l;
  int32_t* lens;
  int64_t lens_stride_slot;
  int slots[kSnapMaxRows];
  const int64_t* keep;       // [L][keep_stride] sorted keep indices
  int64_t keep_stride;
  int K;
};

cudaError_t launch_snapkv_scores(const SnapScoreArgs& a, int L, cudaStream_t st);
cudaError_t launch_keep_indices(const uint8_t* keep, int64_t keep_stride, int length, int64_t* out,
                                int64_t out_stride, int K, int L, int32_t* status, cudaStream_t st);
cudaError_t launch_streaming_keep(int64_t* out, int64_t out_stride, int L, int length, int protected_tokens,
                                  int budget, cudaStream_t st);
cudaError_t launch_snapkv_gather(const SnapGatherArgs& a, int n, int L, cudaStream_t st);

// ---------------------------------------------------------------- decode attention (decode_attn.cu)
struct DecodeArgs {
  const void* q;
  int64_t q_stride_r, q_stride_h;
  const void* kv;            // one layer [2][NB][BS][Hkv][D]
  int64_t kv_stride_kv, kv_stride_b, kv_stride_s, kv_stride_h;
  const int32_t* block_table;
  int64_t bt_stride_r;
  const int32_t* seq_used;
  float* out;
  int64_t out_stride_r, out_stride_h;
  float* lse;
  int64_t lse_stride_r;
  float* part_m;             // [R][Hq][splits]
  float* part_l;
  float* part_acc;           // [R][Hq][splits][D]
  int R, MB, NB, BS, Hq, Hkv, G, D, splits;
  float scale;
  int32_t* status;
};

// Resident decode CTAs per SM (the kernel's launch bounds): a GQA group of 8 carries twice the
// registers.
constexpr int decode_ctas_per_sm(int G) { return G >= 8 ? 2 : 3; }
constexpr int kDecodeMaxSplits = 128;   // the combine kernel's threads

// Token splits per (session, KV head): as many as one wave of resident CTAs on the device's n_sm
// SMs holds (rounded down, so the grid does not spill a few CTAs into a second wave), at least 128
// tokens each, between 1 and kDecodeMaxSplits.  The workspace size and the launch both call this
// with the current device's SM count, so they agree.
inline int decode_splits(int R, int Hkv, int G, int64_t max_seq, int n_sm) {
  const int64_t slots = int64_t(n_sm) * decode_ctas_per_sm(G);
  const int64_t want = slots / (int64_t(R) * Hkv);
  const int64_t cap = (max_seq + 127) / 128;
  int64_t s = want < cap ? want : cap;
  return int(s < 1 ? 1 : (s > kDecodeMaxSplits ? kDecodeMaxSplits : s));
}

bool decode_supported(int D, int G);
// a.splits must be decode_tc_splits(...) when decode_tc_supported(a, dtype), else decode_splits(...)
cudaError_t launch_decode_attention(const DecodeArgs& a, int dtype, cudaStream_t st);
// tensor-core decode (decode_tc.cu): bf16 / fp16, head_dim 128, G in {1, 2, 4, 8}, 16-byte rows
bool decode_tc_supported(const DecodeArgs& a, int dtype);
int decode_tc_splits(int R, int Hkv, int64_t max_seq, int n_sm);
cudaError_t launch_decode_tc(const DecodeArgs& a, int dtype, cudaStream_t st, const char** why);

// ---------------------------------------------------------------- failure-path self-test (selftest.cu)
cudaError_t launch_bounded_wait_probe(int32_t* status, long long* waited, cudaStream_t st);
cudaError_t launch_kv_gather(const void* kv, int64_t n_blocks, int BS, int row_bytes, int head_bytes, int mode,
                             unsigned long long* sink, cudaStream_t st);
cudaError_t launch_budget(const BudgetArgs& a, int R, cudaStream_t st);
cudaError_t launch_region_lse(const LseArgs& a, int dtype, int grid, cudaStream_t st, const char** why);

}  // namespace actkv
