// extern "C" entry points declared in include/actkv_b200.h: host-side validation (the reference's
// asserts and ValueErrors become status codes), launch configuration and dispatch.
#include <cuda.h>
#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <string>

#include "kernels.cuh"

using namespace actkv;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(ACTKV_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

int ok() {
  g_err.clear();
  return ACTKV_OK;
}

int sm_count() { return device_sm_count(); }

bool dtype_ok(int d) { return d == ACTKV_F32 || d == ACTKV_F16 || d == ACTKV_BF16; }

size_t a256(size_t x) { return align256(x); }

CompactWs carve(void* base, int R, int64_t cap, bool with_pairs) {
  char* p = static_cast<char*>(base);
  CompactWs w;
  w.kept = reinterpret_cast<int32_t*>(p);
  w.drop = w.kept + R;
  w.push_off = w.drop + R;
  w.pair_count = w.push_off + R;
  w.ticket = w.pair_count + R;
  p += compact_header_bytes(R);
  w.pair_src = w.pair_dst = nullptr;
  if (with_pairs) {
    w.pair_src = reinterpret_cast<int64_t*>(p);
    p += a256(size_t(R) * cap * 8);
    w.pair_dst = reinterpret_cast<int64_t*>(p);
    p += a256(size_t(R) * cap * 8);
  }
  w.src_logical = reinterpret_cast<int32_t*>(p);
  w.cap = cap;
  return w;
}

// The chunked plan's workspace: the same header as carve() (kept, drop, push offsets, pair counts,
// ticket), then the chunk prefixes and the ranked sources / holes.  Fits in
// actkv_compact_workspace_bytes(R, cap) for every cap (it needs 8 bytes per token, that gives 20).
ChunkWs carve_chunked(void* base, int R, int64_t cap, int nchunk) {
  char* p = static_cast<char*>(base);
  ChunkWs w;
  w.kept = reinterpret_cast<int32_t*>(p);
  w.drop = w.kept + R;
  w.push_off = w.drop + R;
  w.pair_count = w.push_off + R;
  w.ticket = w.pair_count + R;
  p += compact_header_bytes(R);
  w.cpre = reinterpret_cast<int32_t*>(p);
  p += a256(size_t(R) * (nchunk + 1) * 4);
  w.src_log = reinterpret_cast<int32_t*>(p);
  p += a256(size_t(R) * cap * 4);
  w.dst_log = reinterpret_cast<int32_t*>(p);
  w.cap = cap;
  w.nchunk = nchunk;
  return w;
}

constexpr int kCopyThreads = 256;

cudaError_t launch_copy(char* kv, int n_planes, int64_t plane_stride, int64_t slot_stride, int64_t row_bytes,
                        int64_t n_slots, const int64_t* src, const int64_t* dst, int64_t pair_stride,
                        const int32_t* pair_count, int64_t single_count, int R, int32_t* status,
                        cudaStream_t st) {
  const bool vec16 = (reinterpret_cast<uintptr_t>(kv) % 16 == 0) && plane_stride % 16 == 0 &&
                     slot_stride % 16 == 0 && row_bytes % 16 == 0;
  const int grid = sm_count() * 8;
  const size_t sm = size_t(R + 1) * sizeof(int64_t);
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    if (e != cudaSuccess) return e;
  }
  copy_kernel<<<grid, kCopyThreads, sm, st>>>(kv, n_planes, plane_stride, slot_stride, row_bytes, n_slots, src,
                                               dst, pair_stride, pair_count, single_count, R, vec16, status);
  return cudaGetLastError();
}

}  // namespace

namespace actkv {
// Lets the other entry-point file report its errors through actkv_last_error().
void set_last_error(const char* msg) { g_err = msg; }

int device_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    n = 0;
  return n > 0 ? n : 148;
}
}  // namespace actkv

extern "C" {

const char* actkv_last_error(void) { return g_err.c_str(); }

int actkv_abi_version(void) { return 2; }

size_t actkv_score_region_workspace_bytes(int L, int sum_A, int Hq) { return pair_workspace_bytes(L, sum_A, Hq); }

int actkv_action_scores(const void* q, int q_dtype, int64_t q_stride_r, int64_t q_stride_h, const void* kv,
                        int kv_dtype, int64_t kv_stride_kv, int64_t kv_stride_b, int64_t kv_stride_s,
                        int64_t kv_stride_h, const int32_t* block_table, int64_t bt_stride_r,
                        const int32_t* seq_used, const float* lse, int64_t lse_stride_r, float* out,
                        int64_t out_stride_r, int64_t out_stride_h, int64_t out_width, int32_t* n_seen, int R,
                        int MB, int NB, int BS, int Hq, int Hkv, int D, float scale, int32_t* status,
                        void* stream) {
  if (out_width < int64_t(MB) * BS)
    return fail(ACTKV_ERR_OUT_TOO_NARROW,
                "out is %lld wide but the block table spans %lld slots; allocate it as "
                "[R, Hkv, max_blocks * block_size]",
                (long long)out_width, (long long)MB * BS);
  if (!dtype_ok(q_dtype) || !dtype_ok(kv_dtype)) return fail(ACTKV_ERR_INVALID, "unknown dtype code");
  if (Hkv <= 0 || Hq % Hkv != 0) return fail(ACTKV_ERR_INVALID, "n_q_heads %% n_kv_heads != 0");
  if (D <= 0 || D > 256) return fail(ACTKV_ERR_UNSUPPORTED, "head_dim %d: supported up to 256", D);
  if (BS <= 0 || MB <= 0 || NB <= 0 || R < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (R == 0) return ok();
  ScoreArgs a{};
  a.q = q;
  a.q_stride_l = 0;
  a.q_stride_a = q_stride_r;
  a.q_stride_h = q_stride_h;
  a.lse = lse;
  a.lse_stride_l = 0;
  a.lse_stride_a = lse_stride_r;
  a.act_off = nullptr;
  a.kv = kv;
  a.kv_stride_l = 0;
  a.kv_stride_kv = kv_stride_kv;
  a.kv_stride_b = kv_stride_b;
  a.kv_stride_s = kv_stride_s;
  a.kv_stride_h = kv_stride_h;
  a.block_table = block_table;
  a.bt_stride_r = bt_stride_r;
  a.seq_used = seq_used;
  a.out = out;
  a.out_off = nullptr;
  a.out_stride_r = out_stride_r;
  a.out_stride_l = 0;
  a.out_stride_h = out_stride_h;
  a.n_seen = n_seen;
  a.R = R;
  a.L = 1;
  a.MB = MB;
  a.NB = NB;
  a.BS = BS;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.D = D;
  a.qrows = a.G > 64 ? a.G : (64 / a.G) * a.G;
  a.scale = scale;
  a.status = status;
  cudaError_t e = launch_score_simt(a, kv_dtype, q_dtype, MB * BS, 1, st);
  if (e != cudaSuccess) return cuda_fail(e, "action_scores");
  add_kernel<<<(R + 255) / 256, 256, 0, st>>>(n_seen, nullptr, R);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "n_seen += 1");
  return ok();
}

namespace {
// The layer groups of a streamed call (actkv_score_region_streamed); nullptr: all layers resident.
struct StreamSpec {
  const uint32_t* ready;
  uint32_t ready_base;
  int n_groups;
  const int32_t* group_layers;
};

int score_region_impl(const void* q, int q_dtype, int64_t q_stride_l, int64_t q_stride_a, int64_t q_stride_h,
                      const float* lse, int64_t lse_stride_l, int64_t lse_stride_a, const int32_t* act_off,
                      const void* kv, int kv_dtype, int64_t kv_stride_l, int64_t kv_stride_kv, int64_t kv_stride_b,
                      int64_t kv_stride_s, int64_t kv_stride_h, const int32_t* block_table, int64_t bt_stride_r,
                      const int32_t* seq_used, float* out, const int64_t* out_off, int64_t out_stride_r,
                      int64_t out_stride_l, int64_t out_stride_h, int32_t* n_seen, int R, int L, int MB, int NB,
                      int BS, int Hq, int Hkv, int D, int sum_A, int max_A, float scale, int path, void* workspace,
                      size_t workspace_bytes, const StreamSpec* sp, int32_t* status, void* stream) {
  if (!dtype_ok(q_dtype) || !dtype_ok(kv_dtype)) return fail(ACTKV_ERR_INVALID, "unknown dtype code");
  if (Hkv <= 0 || Hq % Hkv != 0) return fail(ACTKV_ERR_INVALID, "n_q_heads %% n_kv_heads != 0");
  if (D <= 0 || D > 256) return fail(ACTKV_ERR_UNSUPPORTED, "head_dim %d: supported up to 256", D);
  if (BS <= 0 || MB <= 0 || NB <= 0 || R < 0 || L <= 0 || sum_A < 0 || max_A < 0)
    return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (act_off == nullptr) return fail(ACTKV_ERR_INVALID, "act_off is required");
  if (path != ACTKV_PATH_AUTO && path != ACTKV_PATH_SIMT && path != ACTKV_PATH_TCGEN05 &&
      path != ACTKV_PATH_TCGEN05_PAIR)
    return fail(ACTKV_ERR_INVALID, "unknown path %d", path);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (R == 0) return ok();
  ScoreArgs a{};
  a.q = q;
  a.q_stride_l = q_stride_l;
  a.q_stride_a = q_stride_a;
  a.q_stride_h = q_stride_h;
  a.lse = lse;
  a.lse_stride_l = lse_stride_l;
  a.lse_stride_a = lse_stride_a;
  a.act_off = act_off;
  a.kv = kv;
  a.kv_stride_l = kv_stride_l;
  a.kv_stride_kv = kv_stride_kv;
  a.kv_stride_b = kv_stride_b;
  a.kv_stride_s = kv_stride_s;
  a.kv_stride_h = kv_stride_h;
  a.block_table = block_table;
  a.bt_stride_r = bt_stride_r;
  a.seq_used = seq_used;
  a.out = out;
  a.out_off = out_off;
  a.out_stride_r = out_stride_r;
  a.out_stride_l = out_stride_l;
  a.out_stride_h = out_stride_h;
  a.n_seen = n_seen;
  a.R = R;
  a.L = L;
  a.MB = MB;
  a.NB = NB;
  a.BS = BS;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.D = D;
  a.qrows = a.G > 64 ? a.G : (64 / a.G) * a.G;
  a.scale = scale;
  a.status = status;
  const char* why = nullptr;
  const bool umma_ok = umma_supported(a, kv_dtype, q_dtype, &why);
  const bool tc = path == ACTKV_PATH_TCGEN05 || path == ACTKV_PATH_TCGEN05_PAIR;
  bool use_umma = tc || (path == ACTKV_PATH_AUTO && umma_ok && max_A * a.G >= 32);
  if (tc && !umma_ok) return fail(ACTKV_ERR_UNSUPPORTED, "tcgen05 path: %s", why);
  const bool ws_ok = workspace != nullptr && workspace_bytes >= pair_workspace_bytes(L, sum_A, Hq) &&
                     reinterpret_cast<uintptr_t>(workspace) % 16 == 0;
  if (path == ACTKV_PATH_TCGEN05_PAIR) {
    if (!pair_supported(a, max_A))
      return fail(ACTKV_ERR_UNSUPPORTED, "CTA-pair path: block_size %d must divide 128 and be at least 8", BS);
    if (!ws_ok)
      return fail(ACTKV_ERR_WORKSPACE, "CTA-pair path: workspace of %zu bytes (16-byte aligned) is smaller than %zu",
                  workspace_bytes, pair_workspace_bytes(L, sum_A, Hq));
  }
  const bool use_pair = use_umma && path != ACTKV_PATH_TCGEN05 && ws_ok && pair_supported(a, max_A);
  if (sp) {
    if (!use_pair) return fail(ACTKV_ERR_UNSUPPORTED, "streamed layer groups need the CTA-pair path");
    if (!sp->ready || sp->n_groups < 1 || sp->n_groups > kMaxLayerGroups || !sp->group_layers)
      return fail(ACTKV_ERR_INVALID, "streamed scoring: ready word and 1..%d layer groups required", kMaxLayerGroups);
    if (sp->group_layers[0] != 0 || sp->group_layers[sp->n_groups] != L)
      return fail(ACTKV_ERR_INVALID, "layer groups must cover layers 0..%d", L);
    for (int g = 0; g < sp->n_groups; ++g)
      if (sp->group_layers[g + 1] <= sp->group_layers[g])
        return fail(ACTKV_ERR_INVALID, "layer group %d is empty or out of order", g);
    a.ready = sp->ready;
    a.ready_base = sp->ready_base;
    a.n_lgroups = sp->n_groups;
    for (int g = 0; g <= sp->n_groups; ++g) a.lgrp[g] = sp->group_layers[g];
  }
  cudaError_t e;
  if (use_pair) {
    e = launch_score_pair(a, kv_dtype, sum_A, max_A, workspace, st, &why);
    if (e != cudaSuccess) return cuda_fail(e, why ? why : "score_region (tcgen05, CTA pairs)");
  } else if (use_umma) {
    e = launch_score_umma(a, kv_dtype, sum_A, max_A, sm_count(), st, &why);
    if (e != cudaSuccess) return cuda_fail(e, why ? why : "score_region (tcgen05)");
  } else {
    e = launch_score_simt(a, kv_dtype, q_dtype, MB * BS, max_A, st);
    if (e != cudaSuccess) return cuda_fail(e, "score_region (simt)");
  }
  if (n_seen) {
    add_kernel<<<(R + 255) / 256, 256, 0, st>>>(n_seen, act_off, R);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "n_seen += A");
  }
  return ok();
}

using StreamWriteValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
StreamWriteValue32Fn get_write_value_fn() {
  static StreamWriteValue32Fn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<StreamWriteValue32Fn>(p);
  }
  return fn;
}
}  // namespace

int actkv_score_region(const void* q, int q_dtype, int64_t q_stride_l, int64_t q_stride_a, int64_t q_stride_h,
                       const float* lse, int64_t lse_stride_l, int64_t lse_stride_a, const int32_t* act_off,
                       const void* kv, int kv_dtype, int64_t kv_stride_l, int64_t kv_stride_kv,
                       int64_t kv_stride_b, int64_t kv_stride_s, int64_t kv_stride_h,
                       const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used, float* out,
                       const int64_t* out_off, int64_t out_stride_r, int64_t out_stride_l,
                       int64_t out_stride_h, int32_t* n_seen, int R, int L, int MB, int NB, int BS, int Hq,
                       int Hkv, int D, int sum_A, int max_A, float scale, int path, void* workspace,
                       size_t workspace_bytes, int32_t* status, void* stream) {
  return score_region_impl(q, q_dtype, q_stride_l, q_stride_a, q_stride_h, lse, lse_stride_l, lse_stride_a, act_off,
                           kv, kv_dtype, kv_stride_l, kv_stride_kv, kv_stride_b, kv_stride_s, kv_stride_h,
                           block_table, bt_stride_r, seq_used, out, out_off, out_stride_r, out_stride_l,
                           out_stride_h, n_seen, R, L, MB, NB, BS, Hq, Hkv, D, sum_A, max_A, scale, path, workspace,
                           workspace_bytes, nullptr, status, stream);
}

int actkv_score_region_streamed(const void* q, int q_dtype, int64_t q_stride_l, int64_t q_stride_a,
                                int64_t q_stride_h, const float* lse, int64_t lse_stride_l, int64_t lse_stride_a,
                                const int32_t* act_off, const void* kv, int kv_dtype, int64_t kv_stride_l,
                                int64_t kv_stride_kv, int64_t kv_stride_b, int64_t kv_stride_s, int64_t kv_stride_h,
                                const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used, float* out,
                                const int64_t* out_off, int64_t out_stride_r, int64_t out_stride_l,
                                int64_t out_stride_h, int32_t* n_seen, int R, int L, int MB, int NB, int BS, int Hq,
                                int Hkv, int D, int sum_A, int max_A, float scale, int path, void* workspace,
                                size_t workspace_bytes, const uint32_t* ready, uint32_t ready_base, int n_groups,
                                const int32_t* group_layers, int32_t* status, void* stream) {
  const StreamSpec sp{ready, ready_base, n_groups, group_layers};
  return score_region_impl(q, q_dtype, q_stride_l, q_stride_a, q_stride_h, lse, lse_stride_l, lse_stride_a, act_off,
                           kv, kv_dtype, kv_stride_l, kv_stride_kv, kv_stride_b, kv_stride_s, kv_stride_h,
                           block_table, bt_stride_r, seq_used, out, out_off, out_stride_r, out_stride_l,
                           out_stride_h, n_seen, R, L, MB, NB, BS, Hq, Hkv, D, sum_A, max_A, scale, path, workspace,
                           workspace_bytes, &sp, status, stream);
}

int actkv_stream_copy_groups(void* dst, const void* src, size_t layer_bytes, const int32_t* bounds, int g0, int g1,
                             uint32_t* ready, uint32_t ready_base, void* stream) {
  if (!dst || !src || !bounds || !ready || g0 < 0 || g1 < g0) return fail(ACTKV_ERR_INVALID, "bad arguments");
  StreamWriteValue32Fn fn = get_write_value_fn();
  if (!fn) return fail(ACTKV_ERR_UNSUPPORTED, "cuStreamWriteValue32 unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int g = g0; g < g1; ++g) {
    if (bounds[g + 1] < bounds[g]) return fail(ACTKV_ERR_INVALID, "layer group %d out of order", g);
    const size_t off = size_t(bounds[g]) * layer_bytes, n = size_t(bounds[g + 1] - bounds[g]) * layer_bytes;
    const cudaError_t e = cudaMemcpyAsync(static_cast<char*>(dst) + off, static_cast<const char*>(src) + off, n,
                                          cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "stream_copy_groups");
    const CUresult r = fn(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(ready),
                          ready_base + uint32_t(g) + 1u, 0);
    if (r != CUDA_SUCCESS) return fail(ACTKV_ERR_UNSUPPORTED, "cuStreamWriteValue32 failed (%d)", int(r));
  }
  return ok();
}

int actkv_stream_signal(uint32_t* word, uint32_t value, void* stream) {
  if (!word) return fail(ACTKV_ERR_INVALID, "null word");
  StreamWriteValue32Fn fn = get_write_value_fn();
  if (!fn) return fail(ACTKV_ERR_UNSUPPORTED, "cuStreamWriteValue32 unavailable");
  const CUresult r = fn(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(word), value, 0);
  if (r != CUDA_SUCCESS) return fail(ACTKV_ERR_UNSUPPORTED, "cuStreamWriteValue32 failed (%d)", int(r));
  return ok();
}

int actkv_lrfu_update(const float* src, const int64_t* src_off, int64_t src_stride_r, int64_t src_stride_l,
                      int64_t src_stride_h, int H, int head_reduce, float* ks, int64_t ks_stride_r,
                      int64_t ks_stride_l, float* act, int64_t act_stride_r, int64_t act_stride_l,
                      const uint8_t* pinned, int64_t pinned_stride_r, int protected_prefix,
                      const int32_t* seq_used, const int32_t* n_act, int R, int L, int max_seq, float decay,
                      float top_p, int32_t* status, void* stream) {
  if (head_reduce != ACTKV_REDUCE_MEAN && head_reduce != ACTKV_REDUCE_MAX)
    return fail(ACTKV_ERR_HEAD_REDUCE, "head_reduce must be mean or max");
  if (H <= 0 || L <= 0 || R < 0 || max_seq < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (!src || !ks || !act || !seq_used) return fail(ACTKV_ERR_INVALID, "null pointer");
  if (R == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LrfuArgs a{src, src_off, src_stride_r, src_stride_l, src_stride_h, H, head_reduce, ks, ks_stride_r,
             ks_stride_l, act, act_stride_r, act_stride_l, pinned, pinned_stride_r, protected_prefix,
             seq_used, n_act, decay, top_p, status, max_seq};
  cudaError_t e = launch_lrfu(a, R, L, st);
  if (e != cudaSuccess) return cuda_fail(e, "lrfu_update");
  return ok();
}

size_t actkv_keep_mask_workspace_bytes(int R, int max_seq) {
  return a256(size_t(R > 0 ? R : 0) * size_t(max_seq > 0 ? max_seq : 0) * sizeof(float));
}

int actkv_keep_mask(const float* scores, const int64_t* scores_off, int64_t scores_stride_r,
                    int64_t scores_stride_l, int64_t scores_stride_x, int n_lead, int n_red, int head_reduce,
                    const uint8_t* pinned, int64_t pinned_stride_r, int protected_prefix,
                    const int32_t* seq_used, const int32_t* budget, int evict_semantics, uint8_t* keep,
                    int64_t keep_stride_r, int32_t* kept, int R, int max_seq, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream) {
  if (head_reduce != ACTKV_REDUCE_MEAN && head_reduce != ACTKV_REDUCE_MAX)
    return fail(ACTKV_ERR_HEAD_REDUCE, "head_reduce must be mean or max");
  if (n_lead <= 0 || n_red <= 0 || R < 0 || max_seq < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (workspace_bytes < actkv_keep_mask_workspace_bytes(R, max_seq))
    return fail(ACTKV_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes,
                actkv_keep_mask_workspace_bytes(R, max_seq));
  if (R == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KeepMaskArgs a{scores, scores_off, scores_stride_r, scores_stride_l, scores_stride_x, n_lead, n_red,
                 head_reduce, pinned, pinned_stride_r, protected_prefix, seq_used, budget, evict_semantics,
                 keep, keep_stride_r, kept, static_cast<float*>(workspace), max_seq, status};
  cudaError_t e = launch_keep_mask(a, R, st);
  if (e != cudaSuccess) return cuda_fail(e, "keep_mask");
  return ok();
}

size_t actkv_compact_workspace_bytes(int R, int max_seq) {
  const size_t r = R > 0 ? R : 0, c = max_seq > 0 ? max_seq : 1;
  return compact_header_bytes(int(r)) + 2 * a256(r * c * 8) + a256(r * c * 4);
}

int actkv_compact(void* kv, int n_planes, int64_t plane_stride_bytes, int64_t slot_stride_bytes,
                  int64_t row_bytes, int64_t n_slots, const uint8_t* keep, int64_t keep_stride_r,
                  int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r, int MB, int BS,
                  int32_t* free_list, int32_t* free_top, int64_t free_capacity, int64_t* perm,
                  int64_t perm_stride_r, int32_t* kept, int R, int max_seq, void* workspace,
                  size_t workspace_bytes, int32_t* status, void* stream) {
  if (n_planes <= 0 || row_bytes <= 0 || n_slots <= 0 || BS <= 0 || MB <= 0 || R < 0 || max_seq < 0)
    return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (!free_list || !free_top) return fail(ACTKV_ERR_INVALID, "free list required");
  if (workspace_bytes < actkv_compact_workspace_bytes(R, max_seq))
    return fail(ACTKV_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes,
                actkv_compact_workspace_bytes(R, max_seq));
  if (R == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t cap = max_seq > 0 ? max_seq : 1;
  ChunkWs w = carve_chunked(workspace, R, cap, chunk_count(cap, BS));
  cudaError_t e = cudaMemsetAsync(workspace, 0, compact_header_bytes(R), st);
  if (e != cudaSuccess) return cuda_fail(e, "workspace clear");
  const dim3 grid(w.nchunk, R);
  count_chunks_kernel<<<grid, kChunkThreads, 0, st>>>(keep, keep_stride_r, seq_used, BS, w, free_top, free_capacity,
                                                      kept, R, status);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "count");
  e = launch_pdl(plan_chunks_kernel, grid, dim3(kChunkThreads), 0, st, keep, keep_stride_r, seq_used, MB, BS, perm,
                 perm_stride_r, w, status);
  if (e != cudaSuccess) return cuda_fail(e, "plan");
  {
    const bool vec16 = (reinterpret_cast<uintptr_t>(kv) % 16 == 0) && plane_stride_bytes % 16 == 0 &&
                       slot_stride_bytes % 16 == 0 && row_bytes % 16 == 0;
    const size_t sm = size_t(R + 1) * sizeof(int64_t) + size_t(R) * sizeof(int32_t);
    if (sm > 48 * 1024) {
      e = cudaFuncSetAttribute(copy_pairs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
      if (e != cudaSuccess) return cuda_fail(e, "copy");
    }
    e = launch_pdl(copy_pairs_kernel, dim3(sm_count() * 8), dim3(kCopyThreads), sm, st, static_cast<char*>(kv),
                   n_planes, plane_stride_bytes, slot_stride_bytes, row_bytes, n_slots, seq_used, block_table,
                   bt_stride_r, BS, perm, perm_stride_r, w, R, vec16, status);
    if (e != cudaSuccess) return cuda_fail(e, "copy");
  }
  e = launch_pdl(finish_kernel, dim3(R), dim3(256), 0, st, seq_used, block_table, bt_stride_r, MB, BS, free_list,
                 free_capacity, w, status);
  if (e != cudaSuccess) return cuda_fail(e, "finish");
  return ok();
}

size_t actkv_plan_workspace_bytes(int seq_used) {
  return compact_header_bytes(1) + a256(size_t(seq_used > 0 ? seq_used : 1) * 4);
}

int actkv_plan_compaction(const uint8_t* keep, int seq_used, const int32_t* table_row, int n_table, int BS,
                          int64_t* src_slots, int64_t* dst_slots, int64_t* perm, int32_t* counts,
                          void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (seq_used < 0 || BS <= 0 || n_table < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if ((seq_used + BS - 1) / BS > n_table)
    return fail(ACTKV_ERR_INVALID, "table row of %d blocks cannot hold %d tokens", n_table, seq_used);
  if (workspace_bytes < actkv_plan_workspace_bytes(seq_used))
    return fail(ACTKV_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes,
                actkv_plan_workspace_bytes(seq_used));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t cap = seq_used > 0 ? seq_used : 1;
  CompactWs w = carve(workspace, 1, cap, false);
  w.pair_src = src_slots;
  w.pair_dst = dst_slots;
  cudaError_t e = cudaMemsetAsync(workspace, 0, compact_header_bytes(1), st);
  if (e != cudaSuccess) return cuda_fail(e, "workspace clear");
  count_kernel<<<1, kCountThreads, 0, st>>>(keep, 0, nullptr, seq_used, BS, w, nullptr, 0, nullptr, 1, status);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "count");
  plan_kernel<<<1, 1024, 0, st>>>(keep, 0, nullptr, seq_used, const_cast<int32_t*>(table_row), 0,
                                  n_table > 0 ? n_table : 1, BS, int64_t(1) << 62, nullptr, 0, perm, 0, w,
                                  false, counts, status);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "plan");
  return ok();
}

int actkv_apply_copies(void* kv, int n_planes, int64_t plane_stride_bytes, int64_t slot_stride_bytes,
                       int64_t row_bytes, int64_t n_slots, const int64_t* src, const int64_t* dst, int64_t n_pairs,
                       int32_t* status, void* stream) {
  if (n_planes < 0 || row_bytes < 0 || n_pairs < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (n_pairs == 0 || n_planes == 0 || row_bytes == 0) return ok();
  cudaError_t e = launch_copy(static_cast<char*>(kv), n_planes, plane_stride_bytes, slot_stride_bytes,
                              row_bytes, n_slots, src, dst, 0, nullptr, n_pairs, 1, status,
                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "apply_copies");
  return ok();
}

int actkv_permute_tokens(const float* src, float* dst, int64_t stride_r, int64_t stride_l, int L,
                         const uint8_t* pin_src, uint8_t* pin_dst, int64_t pin_stride_r, const int64_t* perm,
                         int64_t perm_stride_r, const int32_t* new_len, int R, int width, int32_t* status,
                         void* stream) {
  if (R < 0 || width < 0 || L < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if ((src == nullptr) != (dst == nullptr) || (pin_src == nullptr) != (pin_dst == nullptr))
    return fail(ACTKV_ERR_INVALID, "src/dst must both be given or both be null");
  if (src && (src == dst)) return fail(ACTKV_ERR_INVALID, "permute is out of place: src == dst");
  if (pin_src && pin_src == pin_dst) return fail(ACTKV_ERR_INVALID, "permute is out of place: pin_src == pin_dst");
  if (R == 0 || width == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_pdl(permute_kernel, dim3((width + 255) / 256, R, src && L > 0 ? (L + 7) / 8 : 1), dim3(256), 0,
                             st, src, dst, stride_r, stride_l, L, pin_src, pin_dst, pin_stride_r, perm,
                             perm_stride_r, new_len, width, status);
  if (e != cudaSuccess) return cuda_fail(e, "permute");
  return ok();
}

int actkv_add_i32(int32_t* n, const int32_t* act_off, int R, void* stream) {
  if (R <= 0) return ok();
  add_kernel<<<(R + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(n, act_off, R);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "add");
  return ok();
}

size_t actkv_blocks_workspace_bytes(int R) { return blocks_workspace_bytes(R); }

int actkv_append(void* kv, int L, int64_t plane_stride_bytes, int64_t slot_stride_bytes, int64_t row_bytes,
                 int64_t n_slots, const void* k_new, const void* v_new, int64_t new_layer_stride_bytes,
                 int64_t new_row_stride_bytes, const int32_t* new_off, int max_new, int32_t* seq_used,
                 int32_t* block_table, int64_t bt_stride_r, int MB, int BS, const int32_t* free_list,
                 int32_t* free_top, int64_t free_capacity, int R, void* workspace, size_t workspace_bytes,
                 int32_t* status, void* stream) {
  if (L <= 0 || row_bytes <= 0 || n_slots <= 0 || BS <= 0 || MB <= 0 || R < 0 || max_new < 0)
    return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (!kv || !new_off || !seq_used || !block_table || !free_list || !free_top)
    return fail(ACTKV_ERR_INVALID, "kv, new_off, seq_used, block_table and the free stack are required");
  if (max_new > 0 && (!k_new || !v_new)) return fail(ACTKV_ERR_INVALID, "k_new and v_new are required");
  if (workspace_bytes < blocks_workspace_bytes(R))
    return fail(ACTKV_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes, blocks_workspace_bytes(R));
  if (R == 0) return ok();
  cudaError_t e = launch_append(static_cast<char*>(kv), L, plane_stride_bytes, slot_stride_bytes, row_bytes, n_slots,
                                static_cast<const char*>(k_new), static_cast<const char*>(v_new),
                                new_layer_stride_bytes, new_row_stride_bytes, new_off, max_new, seq_used,
                                block_table, bt_stride_r, MB, BS, free_list, free_top, free_capacity, R, workspace,
                                status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "append");
  return ok();
}

int actkv_release(const uint8_t* release, int32_t* seq_used, int32_t* block_table, int64_t bt_stride_r, int MB,
                  int BS, int32_t* free_list, int32_t* free_top, int64_t free_capacity, uint8_t* pinned,
                  int64_t pinned_stride_r, int pinned_width, int R, void* workspace, size_t workspace_bytes,
                  int32_t* status, void* stream) {
  if (BS <= 0 || MB <= 0 || R < 0 || pinned_width < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (!release || !seq_used || !block_table || !free_list || !free_top)
    return fail(ACTKV_ERR_INVALID, "release mask, seq_used, block_table and the free stack are required");
  if (workspace_bytes < blocks_workspace_bytes(R))
    return fail(ACTKV_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes, blocks_workspace_bytes(R));
  if (R == 0) return ok();
  cudaError_t e = launch_release(release, seq_used, block_table, bt_stride_r, BS, free_list, free_top, free_capacity,
                                 pinned, pinned_stride_r, pinned_width, R, workspace, status,
                                 static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "release");
  return ok();
}

}  // extern "C"

size_t actkv_region_lse_workspace_bytes(int L, int sum_A, int Hq, int64_t max_seq) {
  if (L <= 0 || sum_A <= 0 || Hq <= 0) return 256;
  return a256(size_t(L) * sum_A * Hq * lse_nsplit(max_seq) * kLseParts * sizeof(float2));
}

int actkv_region_lse(const void* q, int q_dtype, int64_t q_stride_l, int64_t q_stride_a, int64_t q_stride_h,
                     const int32_t* act_off, const void* kv, int kv_dtype, int64_t kv_stride_l,
                     int64_t kv_stride_kv, int64_t kv_stride_b, int64_t kv_stride_s, int64_t kv_stride_h,
                     const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used, float* lse,
                     int64_t lse_stride_l, int64_t lse_stride_a, int R, int L, int MB, int NB, int BS, int Hq,
                     int Hkv, int D, int sum_A, int64_t max_seq, float scale, void* workspace,
                     size_t workspace_bytes, int32_t* status, void* stream) {
  if (!dtype_ok(q_dtype) || !dtype_ok(kv_dtype)) return fail(ACTKV_ERR_INVALID, "unknown dtype code");
  if (Hkv <= 0 || Hq % Hkv != 0) return fail(ACTKV_ERR_INVALID, "n_q_heads %% n_kv_heads != 0");
  if (BS <= 0 || MB <= 0 || NB <= 0 || R < 0 || L <= 0 || sum_A < 0 || max_seq < 0 || D <= 0)
    return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (act_off == nullptr) return fail(ACTKV_ERR_INVALID, "act_off is required");
  if (!(scale > 0.0f)) return fail(ACTKV_ERR_INVALID, "scale must be positive");
  if (R == 0 || sum_A == 0) return ok();
  if (workspace_bytes < actkv_region_lse_workspace_bytes(L, sum_A, Hq, max_seq))
    return fail(ACTKV_ERR_WORKSPACE, "region_lse workspace of %zu bytes is smaller than %zu", workspace_bytes,
                actkv_region_lse_workspace_bytes(L, sum_A, Hq, max_seq));
  LseArgs a{};
  a.q = q;
  a.q_stride_l = q_stride_l;
  a.q_stride_a = q_stride_a;
  a.q_stride_h = q_stride_h;
  a.act_off = act_off;
  a.kv = kv;
  a.kv_stride_l = kv_stride_l;
  a.kv_stride_kv = kv_stride_kv;
  a.kv_stride_b = kv_stride_b;
  a.kv_stride_s = kv_stride_s;
  a.kv_stride_h = kv_stride_h;
  a.block_table = block_table;
  a.bt_stride_r = bt_stride_r;
  a.seq_used = seq_used;
  a.lse = lse;
  a.lse_stride_l = lse_stride_l;
  a.lse_stride_a = lse_stride_a;
  a.part = static_cast<float2*>(workspace);
  a.R = R;
  a.L = L;
  a.MB = MB;
  a.NB = NB;
  a.BS = BS;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.D = D;
  a.sum_A = sum_A;
  a.nsplit = lse_nsplit(max_seq);
  a.scale = scale;
  a.status = status;
  const char* why = nullptr;
  if (!lse_umma_supported(a, kv_dtype, q_dtype, &why)) return fail(ACTKV_ERR_UNSUPPORTED, "region_lse: %s", why);
  cudaError_t e = launch_region_lse(a, kv_dtype, sm_count(), static_cast<cudaStream_t>(stream), &why);
  if (e != cudaSuccess) return cuda_fail(e, why ? why : "region_lse");
  return ok();
}

int actkv_token_confidence(const void* logits, int dtype, int64_t row_stride, int B, int V, int k,
                           const int32_t* sessions, float* trace, int64_t capacity, int32_t* trace_len,
                           int32_t* status, void* stream) {
  if (!dtype_ok(dtype)) return fail(ACTKV_ERR_INVALID, "unknown dtype code");
  if (B < 0 || V <= 0 || k <= 0 || capacity <= 0 || row_stride < V) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (!trace || !trace_len || !logits) return fail(ACTKV_ERR_INVALID, "logits, trace and trace_len are required");
  ConfidenceArgs a{};
  a.logits = logits;
  a.row_stride = row_stride;
  a.V = V;
  a.k = k;
  a.sessions = sessions;
  a.trace = trace;
  a.capacity = capacity;
  a.trace_len = trace_len;
  a.status = status;
  cudaError_t e = launch_confidence(a, dtype, B, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "token_confidence");
  return ok();
}

int actkv_budget_update(const float* trace, int64_t capacity, const int32_t* trace_len, int R, int window,
                        int stride, double bottom_pct, double scale_up, int upper, int bidirectional,
                        int shrink_patience, double shrink_slope, double scale_down, int lower,
                        const int32_t* seq_used, int protected_tokens, int32_t* budget, int32_t* rising,
                        double* slope, int32_t* budget_out, int32_t* status, void* stream) {
  if (R < 0 || capacity <= 0 || window <= 0 || stride <= 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (!(bottom_pct >= 0.0 && bottom_pct <= 100.0)) return fail(ACTKV_ERR_INVALID, "bottom_pct must be in [0, 100]");
  if (!trace || !trace_len || !budget || !rising) return fail(ACTKV_ERR_INVALID, "trace, trace_len, budget and rising are required");
  BudgetArgs a{};
  a.trace = trace;
  a.capacity = capacity;
  a.trace_len = trace_len;
  a.window = window;
  a.stride = stride;
  a.bottom_pct = bottom_pct;
  a.scale_up = scale_up;
  a.shrink_slope = shrink_slope;
  a.scale_down = scale_down;
  a.upper = upper;
  a.lower = lower;
  a.bidirectional = bidirectional;
  a.shrink_patience = shrink_patience;
  a.seq_used = seq_used;
  a.protected_tokens = protected_tokens;
  a.budget = budget;
  a.rising = rising;
  a.slope = slope;
  a.budget_out = budget_out;
  a.status = status;
  cudaError_t e = launch_budget(a, R, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "budget_update");
  return ok();
}

int actkv_streaming_keep(int64_t* keep, int64_t keep_stride, int L, int length, int protected_tokens, int budget,
                         void* stream) {
  if (!keep || L < 0 || protected_tokens < 0 || budget < 0 || protected_tokens + budget > length ||
      keep_stride < protected_tokens + budget)
    return fail(ACTKV_ERR_INVALID, "bad sizes");
  cudaError_t e = launch_streaming_keep(keep, keep_stride, L, length, protected_tokens, budget,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "streaming_keep");
  return ok();
}

namespace {
struct SnapWs {
  float* scores;
  uint8_t* pinned;
  uint8_t* keep;
  int32_t* seq;
  int32_t* rest;
  void* keep_ws;
  size_t keep_ws_bytes;
};
SnapWs snap_carve(void* base, int L, int W) {
  char* p = static_cast<char*>(base);
  SnapWs w;
  const size_t lw = size_t(L) * W;
  w.scores = reinterpret_cast<float*>(p);
  p += a256(lw * 4);
  w.pinned = reinterpret_cast<uint8_t*>(p);
  p += a256(lw);
  w.keep = reinterpret_cast<uint8_t*>(p);
  p += a256(lw);
  w.seq = reinterpret_cast<int32_t*>(p);
  w.rest = w.seq + L;
  p += a256(size_t(2) * L * 4);
  w.keep_ws = p;
  w.keep_ws_bytes = actkv_keep_mask_workspace_bytes(L, W);
  return w;
}
}  // namespace

size_t actkv_snapkv_workspace_bytes(int L, int W) {
  if (L <= 0 || W <= 0) return 256;
  const size_t lw = size_t(L) * W;
  return a256(lw * 4) + 2 * a256(lw) + a256(size_t(2) * L * 4) + actkv_keep_mask_workspace_bytes(L, W);
}

int actkv_snapkv_select(const float* rows, int64_t row_stride_slot, int64_t row_stride_l, const int32_t* lens,
                        int64_t lens_stride_slot, const int32_t* slots, int w, int L, int W, int length,
                        int protected_tokens, int budget, int pool, int64_t* keep, int64_t keep_stride,
                        void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (L <= 0 || W <= 0 || length <= 0 || length > W || protected_tokens < 0 || budget < 0)
    return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (w < 0 || w > kSnapMaxRows || w > budget) return fail(ACTKV_ERR_INVALID, "w must be in [0, min(64, budget)]");
  if (pool < 1 || pool > kSnapMaxPool) return fail(ACTKV_ERR_INVALID, "pool must be in [1, 64]");
  if (length - protected_tokens <= budget)
    return fail(ACTKV_ERR_INVALID, "within budget: nothing to select (the reference returns None)");
  if (keep_stride < protected_tokens + budget) return fail(ACTKV_ERR_INVALID, "keep rows too narrow");
  if (w > 0 && (!rows || !lens || !slots)) return fail(ACTKV_ERR_INVALID, "rows, lens and slots are required");
  if (workspace_bytes < actkv_snapkv_workspace_bytes(L, W))
    return fail(ACTKV_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes,
                actkv_snapkv_workspace_bytes(L, W));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SnapWs ws = snap_carve(workspace, L, W);
  SnapScoreArgs a{};
  a.rows = rows;
  a.stride_slot = row_stride_slot;
  a.stride_l = row_stride_l;
  a.lens = lens;
  a.lens_stride_slot = lens_stride_slot;
  for (int i = 0; i < w; ++i) a.slots[i] = slots[i];
  a.w = w;
  a.length = length;
  a.pool = pool;
  a.rest = budget - w;
  a.scores = ws.scores;
  a.pinned = ws.pinned;
  a.stride_out = W;
  a.seq = ws.seq;
  a.budget_rest = ws.rest;
  cudaError_t e = launch_snapkv_scores(a, L, st);
  if (e != cudaSuccess) return cuda_fail(e, "snapkv scores");
  KeepMaskArgs k{ws.scores, nullptr, W, 0, 0, 1, 1, ACTKV_REDUCE_MEAN, ws.pinned, W, protected_tokens, ws.seq,
                 ws.rest, 0, ws.keep, W, nullptr, static_cast<float*>(ws.keep_ws), W, status};
  e = launch_keep_mask(k, L, st);
  if (e != cudaSuccess) return cuda_fail(e, "snapkv keep mask");
  e = launch_keep_indices(ws.keep, W, length, keep, keep_stride, protected_tokens + budget, L, status, st);
  if (e != cudaSuccess) return cuda_fail(e, "snapkv keep indices");
  return ok();
}

int actkv_snapkv_compact_rows(const float* src, float* dst, int64_t row_stride_slot, int64_t row_stride_l,
                              int32_t* lens, int64_t lens_stride_slot, const int32_t* slots, int n, int L,
                              const int64_t* keep, int64_t keep_stride, int K, int32_t* status, void* stream) {
  if (n < 0 || n > kSnapMaxRows || L <= 0 || K < 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (n == 0) return ok();
  if (!src || !dst || !lens || !slots || !keep || src == dst)
    return fail(ACTKV_ERR_INVALID, "src, dst (another buffer), lens, slots and keep are required");
  SnapGatherArgs a{};
  a.src = src;
  a.dst = dst;
  a.stride_slot = row_stride_slot;
  a.stride_l = row_stride_l;
  a.lens = lens;
  a.lens_stride_slot = lens_stride_slot;
  for (int i = 0; i < n; ++i) a.slots[i] = slots[i];
  a.keep = keep;
  a.keep_stride = keep_stride;
  a.K = K;
  cudaError_t e = launch_snapkv_gather(a, n, L, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "snapkv compact rows");
  return ok();
}

int actkv_selftest_bounded_wait(int32_t* status, long long* waited_cycles, void* stream) {
  if (!status || !waited_cycles) return fail(ACTKV_ERR_INVALID, "status and waited_cycles are required");
  cudaError_t e = launch_bounded_wait_probe(status, waited_cycles, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "selftest_bounded_wait");
  return ok();
}

int actkv_measure_kv_gather(const void* kv, int64_t n_blocks, int BS, int row_bytes, int head_bytes, int mode,
                            unsigned long long* sink, void* stream) {
  if (!kv || reinterpret_cast<uintptr_t>(kv) % 16) return fail(ACTKV_ERR_INVALID, "kv must be 16-byte aligned");
  if (n_blocks < 0 || BS <= 0 || head_bytes <= 0 || head_bytes % 16 || row_bytes % head_bytes ||
      row_bytes / head_bytes > 1024 || (mode != 0 && mode != 1))
    return fail(ACTKV_ERR_INVALID, "bad sizes: head_bytes a multiple of 16 dividing row_bytes, mode 0 or 1");
  if (n_blocks == 0) return ok();
  cudaError_t e = launch_kv_gather(kv, n_blocks, BS, row_bytes, head_bytes, mode, sink,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "measure_kv_gather");
  return ok();
}

size_t actkv_decode_workspace_bytes(int R, int Hq, int Hkv, int D, int64_t max_seq) {
  if (R <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0) return 256;
  const int sp = std::max(decode_splits(R, Hkv, Hq / Hkv, max_seq, sm_count()), decode_tc_splits(R, Hkv, max_seq, sm_count()));
  const size_t n = size_t(R) * Hq * sp;
  return 2 * a256(n * 4) + a256(n * D * 4);
}

int actkv_decode_attention(const void* q, int dtype, int64_t q_stride_r, int64_t q_stride_h, const void* kv,
                           int64_t kv_stride_kv, int64_t kv_stride_b, int64_t kv_stride_s, int64_t kv_stride_h,
                           const int32_t* block_table, int64_t bt_stride_r, const int32_t* seq_used, float* out,
                           int64_t out_stride_r, int64_t out_stride_h, float* lse, int64_t lse_stride_r, int R,
                           int MB, int NB, int BS, int Hq, int Hkv, int D, float scale, void* workspace,
                           size_t workspace_bytes, int32_t* status, void* stream) {
  if (!dtype_ok(dtype)) return fail(ACTKV_ERR_INVALID, "unknown dtype code");
  if (Hkv <= 0 || Hq % Hkv != 0) return fail(ACTKV_ERR_INVALID, "n_q_heads %% n_kv_heads != 0");
  if (R < 0 || MB <= 0 || NB <= 0 || BS <= 0 || D <= 0) return fail(ACTKV_ERR_INVALID, "bad sizes");
  if (!decode_supported(D, Hq / Hkv))
    return fail(ACTKV_ERR_UNSUPPORTED, "decode attention: head_dim 64 or 128 and GQA group 1, 2, 4 or 8");
  if (R == 0) return ok();
  {
    // K / V rows are fetched as 16-byte copies
    const int64_t vec = 16;
    const int64_t es = dtype == ACTKV_F32 ? 4 : 2;
    if (reinterpret_cast<uintptr_t>(kv) % vec != 0 || (kv_stride_kv * es) % vec != 0 ||
        (kv_stride_b * es) % vec != 0 || (kv_stride_s * es) % vec != 0 || (kv_stride_h * es) % vec != 0)
      return fail(ACTKV_ERR_UNSUPPORTED, "decode attention: K / V rows must be aligned to %lld bytes",
                  static_cast<long long>(vec));
  }
  const int64_t max_seq = int64_t(MB) * BS;
  if (workspace_bytes < actkv_decode_workspace_bytes(R, Hq, Hkv, D, max_seq))
    return fail(ACTKV_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes,
                actkv_decode_workspace_bytes(R, Hq, Hkv, D, max_seq));
  DecodeArgs a{};
  a.q = q;
  a.q_stride_r = q_stride_r;
  a.q_stride_h = q_stride_h;
  a.kv = kv;
  a.kv_stride_kv = kv_stride_kv;
  a.kv_stride_b = kv_stride_b;
  a.kv_stride_s = kv_stride_s;
  a.kv_stride_h = kv_stride_h;
  a.block_table = block_table;
  a.bt_stride_r = bt_stride_r;
  a.seq_used = seq_used;
  a.out = out;
  a.out_stride_r = out_stride_r;
  a.out_stride_h = out_stride_h;
  a.lse = lse;
  a.lse_stride_r = lse_stride_r;
  a.R = R;
  a.MB = MB;
  a.NB = NB;
  a.BS = BS;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.D = D;
  a.splits = decode_tc_supported(a, dtype) ? decode_tc_splits(R, Hkv, max_seq, sm_count())
                                           : decode_splits(R, Hkv, Hq / Hkv, max_seq, sm_count());
  const size_t n = size_t(R) * Hq * a.splits;
  char* p = static_cast<char*>(workspace);
  a.part_m = reinterpret_cast<float*>(p);
  a.part_l = reinterpret_cast<float*>(p + a256(n * 4));
  a.part_acc = reinterpret_cast<float*>(p + 2 * a256(n * 4));
  a.scale = scale;
  a.status = status;
  cudaError_t e = launch_decode_attention(a, dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode_attention");
  return ok();
}
