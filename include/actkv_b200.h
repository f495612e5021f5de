/*
 * actkv_b200.h - C ABI of the B200 (sm_100a) kernels for actkv-open's eviction hot path:
 * LSE-recovery scoring -> ActionLRFU keep-score update -> keep mask -> conflict-free in-place
 * paged compaction.
 *
 * Conventions (every entry point):
 *   - plain pointers to DEVICE memory unless a parameter says "host"; sizes and strides are in
 *     ELEMENTS of the pointed-to type unless the name ends in _bytes;
 *   - work is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream) and the call
 *     returns without synchronising;
 *   - the return value is an actkv_status; on failure actkv_last_error() gives a message for the
 *     calling thread.  Argument errors are detected on the host before anything is launched;
 *   - `status` (may be NULL) is a device int32 that kernels OR an ACTKV_DEV_* bit into when a
 *     device-side check fails (an index out of range, a bounded wait that gave up); the kernels
 *     never trap, so the context stays usable and the host can read the word after a sync;
 *   - no entry point allocates device memory; those that need scratch take a caller-provided
 *     `workspace` sized by the matching *_workspace_bytes() query.
 *
 * Layout of the paged cache (the reference's vLLM layout, actkv/paged.py:54):
 *   kv [L][2][NB][BS][Hkv][D], last dim contiguous; plane p = 2*layer + (0: K, 1: V).
 */
#ifndef ACTKV_B200_H
#define ACTKV_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ACTKV_API __attribute__((visibility("default")))
#else
#define ACTKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  ACTKV_OK = 0,
  ACTKV_ERR_INVALID = -1,        /* bad shape / stride / alignment (reference: assert)        */
  ACTKV_ERR_OUT_TOO_NARROW = -2, /* `out` narrower than the block table (reference: ValueError)*/
  ACTKV_ERR_UNSUPPORTED = -3,    /* a valid case this build has no kernel for                 */
  ACTKV_ERR_CUDA = -4,           /* a CUDA runtime call failed                                */
  ACTKV_ERR_BUDGET = -5,         /* plan: kept count != budget (reference: assert)            */
  ACTKV_ERR_WORKSPACE = -6,      /* workspace smaller than *_workspace_bytes()                */
  ACTKV_ERR_HEAD_REDUCE = -7     /* head_reduce not mean/max (reference: ValueError)          */
} actkv_status;

typedef enum { ACTKV_F32 = 0, ACTKV_F16 = 1, ACTKV_BF16 = 2 } actkv_dtype;
typedef enum { ACTKV_REDUCE_MEAN = 0, ACTKV_REDUCE_MAX = 1 } actkv_reduce;

/* device status bits */
#define ACTKV_DEV_BAD_INDEX 1    /* a block id / slot / perm entry out of range: access skipped */
#define ACTKV_DEV_TIMEOUT 2      /* a bounded wait in a pipelined kernel gave up                */
#define ACTKV_DEV_MISALIGNED 4   /* shared memory not aligned as the kernel needs: no work done */
#define ACTKV_DEV_OUT_OF_BLOCKS 8 /* append: a session's blocks did not fit (reference: OutOfBlocks) */

/* scoring-path selector for actkv_score_region */
#define ACTKV_PATH_AUTO 0
#define ACTKV_PATH_SIMT 1        /* CUDA-core path: any dtype, any head_dim <= 256              */
#define ACTKV_PATH_TCGEN05 2     /* tcgen05, one CTA per 128-token tile: bf16/fp16, head_dim 128  */
#define ACTKV_PATH_TCGEN05_PAIR 3 /* tcgen05 on CTA pairs (cta_group::2), 256-token tiles: bf16/fp16,
                                     head_dim 128, needs the workspace                            */

ACTKV_API const char* actkv_last_error(void);
ACTKV_API int actkv_abi_version(void);

/*
 * Fold ONE action query per request into the running mean `out` and add 1 to n_seen.
 * Replaces actkv/kernels/lse_attn.py:133-163 (action_scores; the Triton kernel at :85-130):
 *   best[r,h,t] = max_{g<G} exp(scale * <q[r,h*G+g], k[t,h]> - lse[r,h*G+g])
 *   out[r,h,t] += (best - out[r,h,t]) / (n_seen[r] + 1)        for t < seq_used[r]
 * q [R][Hq][D] (q_stride_r, q_stride_h), kv one layer [2][NB][BS][Hkv][D] (kv_stride_* for the
 * K/V, block, slot and head dims), block_table [R][MB] int32, seq_used [R] int32,
 * lse [R][Hq] fp32, out [R][Hkv][out_width] fp32, n_seen [R] int32.
 * Errors: ACTKV_ERR_OUT_TOO_NARROW when out_width < MB*BS (lse_attn.py:139-142).
 */
ACTKV_API int actkv_action_scores(const void* q, int q_dtype, int64_t q_stride_r, int64_t q_stride_h,
                        const void* kv, int kv_dtype, int64_t kv_stride_kv, int64_t kv_stride_b,
                        int64_t kv_stride_s, int64_t kv_stride_h,
                        const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used,
                        const float* lse, int64_t lse_stride_r,
                        float* out, int64_t out_stride_r, int64_t out_stride_h, int64_t out_width,
                        int32_t* n_seen,
                        int R, int MB, int NB, int BS, int Hq, int Hkv, int D, float scale,
                        int32_t* status, void* stream);

/*
 * Score every layer of R sessions against each session's causal action region in one pass.
 * Session r owns query rows a in [act_off[r], act_off[r+1]) (A_r = act_off[r+1]-act_off[r]);
 * action token j of the region sees the first seq_used[r] - A_r + j + 1 tokens.  The result
 * equals A_r calls of actkv_action_scores (lse_attn.py:133) on a zeroed `out`, token j with
 * seq_used = seq_used[r] - A_r + j + 1, i.e. for t < seq_used[r]:
 *   out(r,l,h,t) = (1/A_r) * sum_{j : t <= seq_used[r]-A_r+j} max_g exp(scale<q,k> - lse)
 * If n_seen is not NULL the region continues a running mean that already folded n_seen[r]
 * tokens (out is read, then rewritten) and n_seen[r] += A_r afterwards.
 * q    [L][sumA][Hq][D]       element (l,a,hq,d) at q + l*q_stride_l + a*q_stride_a + hq*q_stride_h + d
 * lse  [L][sumA][Hq] fp32     element (l,a,hq)   at lse + l*lse_stride_l + a*lse_stride_a + hq
 * kv   [L][2][NB][BS][Hkv][D] with element strides kv_stride_l, kv_stride_kv, kv_stride_b,
 *                             kv_stride_s, kv_stride_h
 * out  fp32, element (r,l,h,t) at out + out_off[r] + l*out_stride_l + h*out_stride_h + t
 *      (out_off: device int64 [R]; when NULL, r*out_stride_r is used instead)
 * block_table [R][MB] int32 (bt_stride_r), seq_used [R] int32, act_off [R+1] int32 (device).
 * `path` is one of ACTKV_PATH_*; AUTO takes the CTA-pair kernel when it applies and the
 * workspace is large enough, else the one-CTA tcgen05 kernel, else (fp32, other head dims, tiny
 * regions) the CUDA-core kernel.
 * New entry point (no reference counterpart: the reference folds one token per call).
 */
ACTKV_API int actkv_score_region(const void* q, int q_dtype, int64_t q_stride_l, int64_t q_stride_a,
                       int64_t q_stride_h,
                       const float* lse, int64_t lse_stride_l, int64_t lse_stride_a,
                       const int32_t* act_off,
                       const void* kv, int kv_dtype, int64_t kv_stride_l, int64_t kv_stride_kv,
                       int64_t kv_stride_b, int64_t kv_stride_s, int64_t kv_stride_h,
                       const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used,
                       float* out, const int64_t* out_off, int64_t out_stride_r,
                       int64_t out_stride_l, int64_t out_stride_h,
                       int32_t* n_seen,
                       int R, int L, int MB, int NB, int BS, int Hq, int Hkv, int D,
                       int sum_A, int max_A, float scale, int path,
                       void* workspace, size_t workspace_bytes,
                       int32_t* status, void* stream);

/*
 * actkv_score_region with the queries streamed in by layer groups, for callers whose queries
 * arrive from host memory: group g is layers [group_layers[g], group_layers[g+1]) (host array of
 * n_groups + 1 increasing entries from 0 to L, 1 <= n_groups <= 16), and the kernel reads a
 * group's queries only once the device word *ready has advanced to ready_base + g + 1 (modulo
 * 2^32), e.g. by actkv_stream_signal on the copy stream after that group's copy.  One launch scores
 * all groups: each CTA pair takes its share of group 0, then of group 1, and so on, so scoring
 * starts with the first group while the later ones are still being copied.  lse must be resident
 * when this is called (its operand rows are formed first).  CTA-pair path only: returns
 * ACTKV_ERR_UNSUPPORTED, before any launch, where actkv_score_region would take another path.
 * A wait that exceeds about a second sets ACTKV_DEV_TIMEOUT in *status and ends the launch.
 * New entry point (no reference counterpart).
 */
ACTKV_API int actkv_score_region_streamed(const void* q, int q_dtype, int64_t q_stride_l,
                       int64_t q_stride_a, int64_t q_stride_h,
                       const float* lse, int64_t lse_stride_l, int64_t lse_stride_a,
                       const int32_t* act_off,
                       const void* kv, int kv_dtype, int64_t kv_stride_l, int64_t kv_stride_kv,
                       int64_t kv_stride_b, int64_t kv_stride_s, int64_t kv_stride_h,
                       const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used,
                       float* out, const int64_t* out_off, int64_t out_stride_r,
                       int64_t out_stride_l, int64_t out_stride_h,
                       int32_t* n_seen,
                       int R, int L, int MB, int NB, int BS, int Hq, int Hkv, int D,
                       int sum_A, int max_A, float scale, int path,
                       void* workspace, size_t workspace_bytes,
                       const uint32_t* ready, uint32_t ready_base, int n_groups,
                       const int32_t* group_layers,
                       int32_t* status, void* stream);

/* Stream-ordered write of `value` into the device word `word` (cuStreamWriteValue32: executed by
 * the stream's front end after the stream's earlier work, no kernel launch), the signal that
 * actkv_score_region_streamed waits for.  ACTKV_ERR_UNSUPPORTED when the driver offers no stream
 * memory operations.  New entry point (no reference counterpart). */
ACTKV_API int actkv_stream_signal(uint32_t* word, uint32_t value, void* stream);

/* The copies and signals actkv_score_region_streamed waits for, queued in one call: for each layer
 * group g in [g0, g1), a host->device copy of layers [bounds[g], bounds[g+1]) of the layer-major
 * array src (pinned host memory, layer_bytes per layer) into dst on `stream`, then the stream
 * signal *ready := ready_base + g + 1.  New entry point (no reference counterpart). */
ACTKV_API int actkv_stream_copy_groups(void* dst, const void* src, size_t layer_bytes,
                       const int32_t* bounds, int g0, int g1, uint32_t* ready,
                       uint32_t ready_base, void* stream);

/* Workspace of actkv_score_region: the lse step's operand rows of the CTA-pair kernel
 * (L * sum_A * Hq rows of 16 bytes).  With less (or NULL), ACTKV_PATH_AUTO uses the one-CTA
 * kernel and ACTKV_PATH_TCGEN05_PAIR fails with ACTKV_ERR_WORKSPACE. */
ACTKV_API size_t actkv_score_region_workspace_bytes(int L, int sum_A, int Hq);

/*
 * ActionLRFU keep-score update for R sessions x L layers, in place.
 * Replaces actkv/eviction.py:198-210 (ActionLRFU.update_scores) together with top_p_mask
 * (:36-50) and the head reduction of reduce_heads (:20-33):
 *   a[t]   = reduce_{h<H} src(r,l,h,t)                 (H=1: src already is the action mean)
 *   hit    = nucleus of a over the non-protected tokens t < seq_used[r]: the fewest largest
 *            entries whose sum reaches top_p * sum(a) (the crossing entry included), a > 0;
 *            empty when n_act[r] == 0 or sum(a) <= 0
 *   ks[t]  = fl(fl(decay * ks[t]) + a[t])  if hit,  fl(decay * ks[t])  otherwise
 * Protected tokens (t < protected_prefix, or pinned[r][t] != 0) are left out: ks unchanged.
 * The per-layer a[t] is written to act (r,l,t) (the reference's ActionLRFU.act after the round).
 * src  element (r,l,h,t) at src + src_off[r] (or r*src_stride_r) + l*src_stride_l + h*src_stride_h + t
 * ks   element (r,l,t)   at ks  + r*ks_stride_r  + l*ks_stride_l  + t   (fp32)
 * act  element (r,l,t)   at act + r*act_stride_r + l*act_stride_l + t  (fp32)
 * pinned [R][pinned_stride_r] uint8 (may be NULL); n_act [R] int32 (may be NULL = every session
 * had action tokens).  Ties at the nucleus boundary go to the lowest index.  max_seq >= every
 * seq_used[r] bounds the launch (rows longer than it are flagged ACTKV_DEV_BAD_INDEX and left
 * alone; 0 = unknown, which takes a slower one-CTA-per-row path).
 */
ACTKV_API int actkv_lrfu_update(const float* src, const int64_t* src_off, int64_t src_stride_r,
                      int64_t src_stride_l, int64_t src_stride_h, int H, int head_reduce,
                      float* ks, int64_t ks_stride_r, int64_t ks_stride_l,
                      float* act, int64_t act_stride_r, int64_t act_stride_l,
                      const uint8_t* pinned, int64_t pinned_stride_r, int protected_prefix,
                      const int32_t* seq_used, const int32_t* n_act,
                      int R, int L, int max_seq, float decay, float top_p,
                      int32_t* status, void* stream);

/*
 * Keep masks for R sessions: protected tokens plus the top-budget others.
 * Replaces actkv/paged.py:23-46 (keep_mask_from_scores) and, with evict_semantics=1, the
 * within-budget early exit of PagedKVCache.evict (paged.py:153-154: keep everything when
 * n - #protected <= budget).  Scores of session r: element (r,l,x,t) at
 * scores + scores_off[r] (or r*scores_stride_r) + l*scores_stride_l + x*scores_stride_x + t,
 * l < n_lead, x < n_red: x is reduced with head_reduce (dim -2 of the reference's tensor), then
 * the n_lead rows are averaged.  Tokens t < seq_used[r]; protected = t < protected_prefix or
 * pinned[r][t].  budget [R] int32.  Output keep [R][keep_stride_r] uint8 (1 = keep) for
 * t < seq_used[r], kept[r] = number kept (may be NULL).  Ties at the threshold go to the lowest
 * index.  Needs workspace of actkv_keep_mask_workspace_bytes(R, max_seq) bytes.
 */
ACTKV_API size_t actkv_keep_mask_workspace_bytes(int R, int max_seq);
ACTKV_API int actkv_keep_mask(const float* scores, const int64_t* scores_off, int64_t scores_stride_r,
                    int64_t scores_stride_l, int64_t scores_stride_x, int n_lead, int n_red,
                    int head_reduce,
                    const uint8_t* pinned, int64_t pinned_stride_r, int protected_prefix,
                    const int32_t* seq_used, const int32_t* budget, int evict_semantics,
                    uint8_t* keep, int64_t keep_stride_r, int32_t* kept,
                    int R, int max_seq, void* workspace, size_t workspace_bytes,
                    int32_t* status, void* stream);

/*
 * actkv_keep_mask without a workspace argument: the same keep masks, for callers that cannot
 * allocate device memory -- a host runtime with no device allocator of its own, a serving engine
 * whose memory pool is fully carved up before requests arrive, or a plugin whose host forbids
 * cudaMalloc while it serves.  No counterpart in the reference (it has no allocation-free entry).
 * The scratch is a static device array of 1,048,576 floats (4 MiB) inside this library, which
 * every GPU that loads the library holds until the process exits; calls with R * max_seq above
 * that return ACTKV_ERR_WORKSPACE and launch nothing.  The first call on a device looks up the
 * array's device address (set-up, once per device, with that device current), so make that first
 * call before any stream capture.  Every call uses the same array: calls that can overlap on the
 * GPU (different streams, or several host threads) race and must be serialised by the caller.
 * The kernel writes every scratch entry before reading it, so no clearing between calls is
 * needed.  Arguments mean what they mean for actkv_keep_mask.
 */
ACTKV_API int actkv_keep_mask_static(const float* scores, const int64_t* scores_off, int64_t scores_stride_r,
                           int64_t scores_stride_l, int64_t scores_stride_x, int n_lead, int n_red,
                           int head_reduce,
                           const uint8_t* pinned, int64_t pinned_stride_r, int protected_prefix,
                           const int32_t* seq_used, const int32_t* budget, int evict_semantics,
                           uint8_t* keep, int64_t keep_stride_r, int32_t* kept,
                           int R, int max_seq, int32_t* status, void* stream);

/*
 * Conflict-free in-place compaction of R sessions of a paged cache (Algorithm 4).
 * Replaces actkv/paged.py:125-139 (PagedKVCache.compact) with actkv/kernels/compaction.py:44-69
 * (plan_compaction) and :96-106 (apply_copies) for a whole batch:
 *   B = #kept, Y = ceil(n/BS), X = ceil(B/BS), window [start, start+B) with start = (Y-X)*BS;
 *   kept tokens outside the window move, ascending, into the window's holes, ascending, in every
 *   one of the n_planes planes; perm[j] (new logical j -> old logical) is written;
 *   the table row becomes table[Y-X:Y] (zero padded), the freed blocks table[0:Y-X] are pushed
 *   onto the free stack in reverse order (free.extend(reversed(freed))), sessions in order
 *   r = 0..R-1; seq_used[r] = B.
 * keep [R][keep_stride_r] uint8, seq_used [R] int32 (in/out), block_table [R][MB] int32 (in/out),
 * free_list [NB] int32 with free_top [1] int32 = its length (in/out; the stack grows upward),
 * perm [R][perm_stride_r] int64 (may be NULL), kept [R] int32 out (may be NULL).
 * kv: base of plane 0, plane p starts at kv + p*plane_stride_bytes, slot s at
 * + s*slot_stride_bytes, row_bytes contiguous bytes per slot.
 * Needs workspace of actkv_compact_workspace_bytes(R, max_seq).
 */
ACTKV_API size_t actkv_compact_workspace_bytes(int R, int max_seq);
ACTKV_API int actkv_compact(void* kv, int n_planes, int64_t plane_stride_bytes, int64_t slot_stride_bytes,
                  int64_t row_bytes, int64_t n_slots,
                  const uint8_t* keep, int64_t keep_stride_r,
                  int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r, int MB, int BS,
                  int32_t* free_list, int32_t* free_top, int64_t free_capacity,
                  int64_t* perm, int64_t perm_stride_r, int32_t* kept,
                  int R, int max_seq, void* workspace, size_t workspace_bytes,
                  int32_t* status, void* stream);

/*
 * Plan only, one request.  Replaces actkv/kernels/compaction.py:44-69 (plan_compaction):
 * writes src_slots/dst_slots (int64, physical slots, n_pairs of them), perm [B] int64 and
 * counts[0..3] = {B, n_pairs, drop_blocks, start} (int32, device).  src/dst/perm need room for
 * seq_used entries.  Needs workspace of actkv_plan_workspace_bytes(seq_used).
 */
ACTKV_API size_t actkv_plan_workspace_bytes(int seq_used);
ACTKV_API int actkv_plan_compaction(const uint8_t* keep, int seq_used, const int32_t* table_row,
                          int n_table, int BS, int64_t* src_slots, int64_t* dst_slots,
                          int64_t* perm, int32_t* counts, void* workspace,
                          size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Copy rows between slots of every plane: kv[p][dst[i]] = kv[p][src[i]] for i < n_pairs,
 * p < n_planes.  src and dst must be disjoint (the plan guarantees it).
 * Replaces actkv/kernels/compaction.py:96-106 (apply_copies, Triton kernel :79-93).
 * Offsets are 64-bit throughout (planes past 2^31 elements are fine).
 */
ACTKV_API int actkv_apply_copies(void* kv, int n_planes, int64_t plane_stride_bytes,
                       int64_t slot_stride_bytes, int64_t row_bytes, int64_t n_slots,
                       const int64_t* src, const int64_t* dst, int64_t n_pairs,
                       int32_t* status, void* stream);

/*
 * Permute per-token state after a compaction: for each session r and j < new_len[r]:
 *   dst(r,l,j) = src(r,l,perm[r][j]) for l < L     (fp32 rows, e.g. ActionLRFU ks/act)
 *   pin_dst[r][j] = pin_src[r][perm[r][j]]          (uint8, may be NULL)
 * and zero for new_len[r] <= j < width.  Out of place.  Replaces ActionLRFU.apply_keep
 * (actkv/eviction.py:222-224) and the pinned permutation of PagedKVCache.evict (paged.py:156).
 */
ACTKV_API int actkv_permute_tokens(const float* src, float* dst, int64_t stride_r, int64_t stride_l, int L,
                         const uint8_t* pin_src, uint8_t* pin_dst, int64_t pin_stride_r,
                         const int64_t* perm, int64_t perm_stride_r, const int32_t* new_len,
                         int R, int width, int32_t* status, void* stream);

/* n[i] += inc[i] (inc may be NULL: += 1) for i < R.  The n_seen bump of lse_attn.py:162. */
ACTKV_API int actkv_add_i32(int32_t* n, const int32_t* act_off, int R, void* stream);

/*
 * Device-resident block allocation.  Replaces PagedKVCache._ensure / append / release
 * (actkv/paged.py:67-90) for a batch of sessions whose tables, lengths and free stack live on
 * the device (tables hold ceil(seq_used/BS) blocks; the free stack is free_list[0..*free_top),
 * popped from the top).  Both need workspace of actkv_blocks_workspace_bytes(R).
 *
 * actkv_append: session r gets new_off[r+1]-new_off[r] tokens whose K and V rows are
 *   k_new/v_new + l*new_layer_stride + (new_off[r]+j)*new_row_stride (row_bytes each, layers
 *   l < L).  As the reference's per-request calls in session order would: blocks are popped from
 *   the top of the free stack, session 0 first, and appended to each table row; the rows are
 *   written into the new slots of plane 2l (K) and 2l+1 (V) of the kv view
 *   [2L][n_slots][row]; seq_used advances.  Sessions from the first one whose blocks do not fit
 *   (free stack, or MB table columns) on are left untouched and ACTKV_DEV_OUT_OF_BLOCKS is set
 *   in status (the reference raises OutOfBlocks there, after appending the earlier requests).
 *   max_new >= every session's new-token count (a launch-size bound, no host sync).
 */
ACTKV_API size_t actkv_blocks_workspace_bytes(int R);
ACTKV_API int actkv_append(void* kv, int L, int64_t plane_stride_bytes, int64_t slot_stride_bytes,
                           int64_t row_bytes, int64_t n_slots,
                           const void* k_new, const void* v_new, int64_t new_layer_stride_bytes,
                           int64_t new_row_stride_bytes, const int32_t* new_off, int max_new,
                           int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r, int MB, int BS,
                           const int32_t* free_list, int32_t* free_top, int64_t free_capacity,
                           int R, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * actkv_release: every session r with release[r] != 0, in session order, pushes its blocks onto
 *   the free stack in reverse table order (free.extend(reversed(table)), paged.py:87-90); its
 *   table row, seq_used and (if pinned is not NULL) its pinned row of pinned_width bytes are
 *   cleared.
 */
ACTKV_API int actkv_release(const uint8_t* release, int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r,
                            int MB, int BS, int32_t* free_list, int32_t* free_top, int64_t free_capacity,
                            uint8_t* pinned, int64_t pinned_stride_r, int pinned_width,
                            int R, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Causal log-sum-exp of every session's action region, all layers, from the paged cache: the LSE
 * by-product that the reference takes from paged_decode_attention_ref (actkv/kernels/lse_attn.py
 * :42-60), called for action token j with seq_used = seq_used[r] - A_r + j + 1:
 *   lse(l, a, hq) = log sum_{t <= seq_used[r] - A_r + j} exp(scale * <q(l, a, hq), k(l, t, hq / G)>)
 * for a = act_off[r] + j.  q, act_off, kv, block_table, seq_used as in actkv_score_region; lse
 * fp32 at lse + l*lse_stride_l + a*lse_stride_a + hq.  bf16 or fp16 q and cache, head_dim 128,
 * G in {1, 2, 4, 8, 16}, block_size a multiple of 8 dividing 128 (else ACTKV_ERR_UNSUPPORTED);
 * scale > 0.
 * max_seq bounds every seq_used[r] (it sizes the workspace; a longer session sets
 * ACTKV_DEV_BAD_INDEX, as does a row that sees no token).  Replaces the untimed torch reference
 * pass (lse_attn.py:42-60) on the eviction path.
 */
ACTKV_API size_t actkv_region_lse_workspace_bytes(int L, int sum_A, int Hq, int64_t max_seq);
ACTKV_API int actkv_region_lse(const void* q, int q_dtype, int64_t q_stride_l, int64_t q_stride_a,
                               int64_t q_stride_h, const int32_t* act_off,
                               const void* kv, int kv_dtype, int64_t kv_stride_l, int64_t kv_stride_kv,
                               int64_t kv_stride_b, int64_t kv_stride_s, int64_t kv_stride_h,
                               const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used,
                               float* lse, int64_t lse_stride_l, int64_t lse_stride_a,
                               int R, int L, int MB, int NB, int BS, int Hq, int Hkv, int D,
                               int sum_A, int64_t max_seq, float scale,
                               void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Adaptive budget (ActKV Algorithm 2, actkv/budget.py:9-104) on the device.
 *
 * actkv_token_confidence: for each of B logit rows (V values, row b at logits + b*row_stride,
 *   f32/f16/bf16), T = -(1/k) * sum of the k largest log-softmax values (token_confidence,
 *   budget.py:9-17; k is capped at V), appended to its session's trace:
 *   trace[r*capacity + trace_len[r]] = T, trace_len[r] += 1, r = sessions ? sessions[b] : b.
 *   A session appears at most once per call.  A full trace sets ACTKV_DEV_BAD_INDEX.
 * actkv_budget_update: for each of R sessions, ConfidenceBudget.next_budget (budget.py:83-104)
 *   on its whole trace: min pooling (window, stride), bottom_pct quantile, least-squares slope;
 *   budget[r] grows to min(int(budget * scale_up), upper) on a negative slope; with bidirectional
 *   it shrinks to max(int(budget / scale_down), lower) after shrink_patience consecutive slopes
 *   above shrink_slope (rising[r] counts them).  slope[r] (nullable) receives the slope.  With
 *   seq_used not NULL only sessions with seq_used[r] - protected_tokens > budget[r] are stepped
 *   (actkv/hf/session.py:186-193), the others get slope NaN.  budget_out (nullable) receives the
 *   new budgets, e.g. the eviction step's budget array.  A trace longer than
 *   window + stride * 16383 values sets ACTKV_DEV_BAD_INDEX and leaves the session unchanged.
 */
ACTKV_API int actkv_token_confidence(const void* logits, int dtype, int64_t row_stride, int B, int V, int k,
                                     const int32_t* sessions, float* trace, int64_t capacity,
                                     int32_t* trace_len, int32_t* status, void* stream);
ACTKV_API int actkv_budget_update(const float* trace, int64_t capacity, const int32_t* trace_len, int R,
                                  int window, int stride, double bottom_pct, double scale_up, int upper,
                                  int bidirectional, int shrink_patience, double shrink_slope,
                                  double scale_down, int lower, const int32_t* seq_used, int protected_tokens,
                                  int32_t* budget, int32_t* rising, double* slope, int32_t* budget_out,
                                  int32_t* status, void* stream);

/*
 * Baseline policies of the reference on the device (actkv/eviction.py:89-149); keep indices are
 * int64 [L][keep_stride], sorted, protected_tokens + budget per layer.  Callers skip these when
 * length - protected_tokens <= budget (the reference's select returns None there).
 *
 * actkv_streaming_keep: StreamingLLM.select (eviction.py:89-100): the protected prefix and the
 *   last `budget` tokens, every layer.
 * actkv_snapkv_select: SnapKV.select (eviction.py:103-141).  rows: a ring of observed attention
 *   rows, element (slot, layer, t) at rows + slot*row_stride_slot + layer*row_stride_l + t, the
 *   row of (slot, layer) lens[slot*lens_stride_slot + layer] long; slots (HOST memory) lists the
 *   w <= 64 rows to sum, oldest first (w = min(rows observed, budget)).  The sum is
 *   average-pooled with kernel pool <= 64 (stride 1, zero padding pool/2); the window
 *   [length - w, length) and the protected prefix are kept, plus the top budget - w of the other
 *   tokens of each layer (ties to the lowest index).  W >= length; the workspace is
 *   actkv_snapkv_workspace_bytes(L, W) bytes.
 * actkv_snapkv_compact_rows: SnapKV.apply_keep (eviction.py:143-149): for each of the n slots
 *   (HOST memory), each layer's row is gathered by that layer's K keep indices (those < its
 *   length) from src into dst (same layout, another buffer), and its length updated.
 */
ACTKV_API int actkv_streaming_keep(int64_t* keep, int64_t keep_stride, int L, int length, int protected_tokens,
                                   int budget, void* stream);
ACTKV_API size_t actkv_snapkv_workspace_bytes(int L, int W);
ACTKV_API int actkv_snapkv_select(const float* rows, int64_t row_stride_slot, int64_t row_stride_l,
                                  const int32_t* lens, int64_t lens_stride_slot, const int32_t* slots, int w,
                                  int L, int W, int length, int protected_tokens, int budget, int pool,
                                  int64_t* keep, int64_t keep_stride, void* workspace, size_t workspace_bytes,
                                  int32_t* status, void* stream);
ACTKV_API int actkv_snapkv_compact_rows(const float* src, float* dst, int64_t row_stride_slot, int64_t row_stride_l,
                                        int32_t* lens, int64_t lens_stride_slot, const int32_t* slots, int n,
                                        int L, const int64_t* keep, int64_t keep_stride, int K,
                                        int32_t* status, void* stream);

/*
 * Paged decode attention with its lse (paged_decode_attention_ref, actkv/kernels/lse_attn.py:42-60)
 * for one query per session, one layer: out[r, hq, :] = softmax(scale * q . k) @ v and
 * lse[r, hq] over the first seq_used[r] tokens (out 0 and lse -inf for an empty session).
 * q [R][Hq][D] (q + r*q_stride_r + hq*q_stride_h + d), kv [2][NB][BS][Hkv][D] with element strides
 * kv_stride_kv, kv_stride_b, kv_stride_s, kv_stride_h (D contiguous), q and kv of one dtype;
 * out fp32 [R][Hq][D] (out_stride_r, out_stride_h), lse fp32 [R][Hq] (lse_stride_r).  D 64 or 128,
 * G = Hq / Hkv in {1, 2, 4, 8}, kv and its strides aligned to 16 bytes (rows are fetched as
 * 16-byte copies) (else ACTKV_ERR_UNSUPPORTED).  Workspace:
 * actkv_decode_workspace_bytes(R, Hq, Hkv, D, MB * BS) bytes.
 */
ACTKV_API size_t actkv_decode_workspace_bytes(int R, int Hq, int Hkv, int D, int64_t max_seq);
ACTKV_API int actkv_decode_attention(const void* q, int dtype, int64_t q_stride_r, int64_t q_stride_h,
                                     const void* kv, int64_t kv_stride_kv, int64_t kv_stride_b, int64_t kv_stride_s,
                                     int64_t kv_stride_h, const int32_t* block_table, int64_t bt_stride_r,
                                     const int32_t* seq_used, float* out, int64_t out_stride_r, int64_t out_stride_h,
                                     float* lse, int64_t lse_stride_r, int R, int MB, int NB, int BS, int Hq, int Hkv,
                                     int D, float scale, void* workspace, size_t workspace_bytes,
                                     int32_t* status, void* stream);

/*
 * Self-test of the kernels' failure path (no counterpart in the reference): one block waits, with
 * the bounded mbarrier wait that every pipelined kernel here uses, on a barrier that nothing
 * completes.  The wait gives up after ~2^31 cycles (about a second), sets ACTKV_DEV_TIMEOUT in
 * *status and the kernel returns; *waited_cycles (device int64) receives the cycles it waited
 * (-1 if the wait had completed).  The context stays usable afterwards.
 */
ACTKV_API int actkv_selftest_bounded_wait(int32_t* status, long long* waited_cycles, void* stream);

/*
 * Measurement aid (no counterpart in the reference): one read of a paged cache's blocks in the two
 * patterns its kernels can use, for the caller to time on `stream`.  kv holds n_blocks consecutive
 * blocks of BS token rows of row_bytes (Hkv heads of head_bytes each: row_bytes = Hkv * head_bytes;
 * the whole [L][2][NB][BS][Hkv][D] cache is L * 2 * NB such blocks).  mode 0: one head per CTA, BS
 * pieces of head_bytes per block, row_bytes apart (how the scoring and decode kernels read);
 * mode 1: whole blocks.  Reads only (a checksum is written to *sink, device uint64, only in a case
 * real data never meets).  kv 16-byte aligned, head_bytes a multiple of 16 dividing row_bytes.
 */
ACTKV_API int actkv_measure_kv_gather(const void* kv, int64_t n_blocks, int BS, int row_bytes, int head_bytes,
                                      int mode, unsigned long long* sink, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ACTKV_B200_H */
