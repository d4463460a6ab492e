// C ABI (include/w8a8.h): contexts, linears, boundary stages, LM-head top-k and merge.
//
// The objects here replace the per-die NPU plumbing of the reference: the loaded subgraph
// (weights + QuantM blob + quant_scales.json entry, lfm3_v2.cpp:3743-3826), the DmaBuffer
// staging of activations (lfm3_v2.cpp:1186-1225) and WorkerPool::submit_task
// (worker_pool.hpp:232-254).  Everything runs in-process on CUDA streams; no call allocates
// device memory after create, except a forward with T above the preallocated token budget and
// the first tensor-core forward of a linear (its tile-ordered weight copy and split-K scratch),
// both of which w8a8_linear_reserve allocates ahead at set-up.
#include "../../include/w8a8.h"
#include "kernels.h"
#include "linear_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

using namespace w8a8;

namespace {

thread_local std::string g_last_error;

w8a8_status fail(w8a8_status st, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

w8a8_status cuda_fail(cudaError_t e, const char *what) {
  return fail(W8A8_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define W8A8_CUDA(call)                                    \
  do {                                                     \
    cudaError_t e_ = (call);                               \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);    \
  } while (0)

constexpr int kPreallocTokens = 64;  // activation staging preallocated for T <= 64

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace w8a8 {
void set_last_error(const char *msg) { g_last_error = msg ? msg : ""; }
}  // namespace w8a8

struct w8a8_ctx {
  int device = 0;
  int sm_count = 0;
  int *d_err = nullptr;
};

struct w8a8_linear {
  w8a8_ctx *ctx = nullptr;
  int K = 0, N = 0, k_pad = 0;
  int8_t *w = nullptr;          // [N, k_pad]
  int16_t *quant_m = nullptr;   // [N]
  int32_t *quant_m32 = nullptr; // [N] widened copy
  float *out_step = nullptr;    // [N]
  float *acc_step = nullptr;    // [N]
  float *inv_smooth = nullptr;  // [K] or null
  bool has_quant_m = false, has_acc_step = false;
  int trunc = 0, qmax = 127, out_i16 = 0;
  float inv_step = 0.0f, safe_thresh = 1e-8f;
  // RMSNorm folded into the STATIC pack of the top-k forward (w8a8_linear_set_input_norm)
  const float *emb_norm = nullptr;
  float norm_eps = 0.0f;
  // scratch
  int8_t *xq = nullptr;         // [xq_tokens, k_pad]
  int xq_tokens = 0;
  float *ratio = nullptr;       // [xq_tokens]
  uint64_t *lists = nullptr;    // top-k per-CTA candidate lists
  size_t lists_keys = 0;
  unsigned *counter = nullptr;
  // 16+ token top-k: logits (when the caller passes none) and per-CTA row lists, grown on use
  // (kept apart from `lists`, whose address a built decode chain holds)
  float *logit_ws = nullptr;    // [T, N]
  size_t logit_ws_elems = 0;
  uint64_t *row_lists = nullptr;
  size_t row_lists_keys = 0;
  // tensor-core path: tile-ordered weights, split-K accumulation plane, per-tile arrival counters
  int path = W8A8_PATH_AUTO;
  int8_t *w_tiles = nullptr;    // weights in tensor-core tile order (built on first use)
  unsigned long long *tc_trace = nullptr;  // optional per-CTA timeline of tensor-core launches
  int32_t *tc_ws = nullptr;
  size_t tc_ws_elems = 0;
  unsigned *tc_count = nullptr;
  size_t tc_count_n = 0;
  size_t device_bytes = 0;
};

namespace {

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
    dev_ = dev;
  }
  ~DeviceGuard() {
    if (prev_ != dev_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0, dev_ = 0;
};

template <typename T>
w8a8_status dev_alloc(T **p, size_t count, size_t *acc) {
  if (count == 0) count = 1;
  cudaError_t e = cudaMalloc(reinterpret_cast<void **>(p), count * sizeof(T));
  if (e != cudaSuccess) return fail(W8A8_ERR_NO_MEMORY, "cudaMalloc(%zu): %s", count * sizeof(T), cudaGetErrorString(e));
  if (acc) *acc += count * sizeof(T);
  return W8A8_SUCCESS;
}

void linear_free(w8a8_linear *l) {
  if (!l) return;
  DeviceGuard g(l->ctx ? l->ctx->device : 0);
  cudaFree(l->w);
  cudaFree(l->quant_m);
  cudaFree(l->quant_m32);
  cudaFree(l->out_step);
  cudaFree(l->acc_step);
  cudaFree(l->inv_smooth);
  cudaFree(l->xq);
  cudaFree(l->ratio);
  cudaFree(l->lists);
  cudaFree(l->counter);
  cudaFree(l->logit_ws);
  cudaFree(l->row_lists);
  cudaFree(l->w_tiles);
  cudaFree(l->tc_ws);
  cudaFree(l->tc_count);
  delete l;
}

// Builds the tensor-core tile copy of the weights on the first tensor-core launch (stream
// ordered before it).  It doubles the linear's weight bytes, so decode-only linears never pay it.
w8a8_status ensure_tc_weights(w8a8_linear *l, cudaStream_t st, bool *built) {
  *built = false;
  if (l->w_tiles) return W8A8_SUCCESS;
  *built = true;
  const size_t bytes = tc_tile_bytes(l->N, l->k_pad);
  w8a8_status s = dev_alloc(&l->w_tiles, bytes, &l->device_bytes);
  if (s != W8A8_SUCCESS) return s;
  W8A8_CUDA(launch_tile_weights(l->w, l->k_pad, l->N, l->k_pad, l->w_tiles, st));
  return W8A8_SUCCESS;
}

// Grows the split-K accumulation plane / per-tile arrival counters of the tensor-core path (both
// start at zero and the kernel leaves them zero again).
w8a8_status ensure_tc_scratch(w8a8_linear *l, size_t ws_elems, size_t count_n) {
  if (ws_elems > l->tc_ws_elems) {
    cudaFree(l->tc_ws);
    l->tc_ws = nullptr;
    l->tc_ws_elems = 0;
    w8a8_status st = dev_alloc(&l->tc_ws, ws_elems, nullptr);
    if (st != W8A8_SUCCESS) return st;
    W8A8_CUDA(cudaMemset(l->tc_ws, 0, ws_elems * sizeof(int32_t)));
    l->tc_ws_elems = ws_elems;
  }
  if (count_n > l->tc_count_n) {
    cudaFree(l->tc_count);
    l->tc_count = nullptr;
    l->tc_count_n = 0;
    w8a8_status st = dev_alloc(&l->tc_count, count_n, nullptr);
    if (st != W8A8_SUCCESS) return st;
    W8A8_CUDA(cudaMemset(l->tc_count, 0, count_n * sizeof(unsigned)));
    l->tc_count_n = count_n;
  }
  return W8A8_SUCCESS;
}

// Grows a device scratch array to at least `need` elements (the old contents are dropped).
template <typename E>
w8a8_status grow_scratch(E **p, size_t *have, size_t need) {
  if (need <= *have) return W8A8_SUCCESS;
  cudaFree(*p);
  *p = nullptr;
  *have = 0;
  w8a8_status st = dev_alloc(p, need, nullptr);
  if (st != W8A8_SUCCESS) return st;
  *have = need;
  return W8A8_SUCCESS;
}

// Grows the activation staging buffers to hold T tokens (allocates only when T exceeds the
// preallocated budget).
w8a8_status ensure_tokens(w8a8_linear *l, int T) {
  if (T <= l->xq_tokens) return W8A8_SUCCESS;
  cudaFree(l->xq);
  cudaFree(l->ratio);
  l->xq = nullptr;
  l->ratio = nullptr;
  w8a8_status st = dev_alloc(&l->xq, static_cast<size_t>(T) * l->k_pad, nullptr);
  if (st != W8A8_SUCCESS) return st;
  st = dev_alloc(&l->ratio, static_cast<size_t>(T), nullptr);
  if (st != W8A8_SUCCESS) return st;
  W8A8_CUDA(cudaMemset(l->xq, 0, static_cast<size_t>(T) * l->k_pad));
  l->xq_tokens = T;
  return W8A8_SUCCESS;
}

Epilogue make_epilogue(const w8a8_linear *l, int out_mode, int act_mode, const float *ratio,
                       void *y, int64_t ldy) {
  Epilogue ep;
  ep.out_mode = out_mode;
  ep.act_mode = act_mode;
  ep.quant_m = l->quant_m;
  ep.trunc = l->trunc;
  ep.qmax = l->qmax;
  ep.out_i16 = l->out_i16;
  ep.out_step = l->out_step;
  ep.acc_step = l->acc_step;
  ep.ratio = ratio;
  ep.y = y;
  ep.ldy = ldy;
  return ep;
}

w8a8_status check_modes(const w8a8_linear *l, int act_mode, int out_mode) {
  if (act_mode != W8A8_ACT_STATIC && act_mode != W8A8_ACT_DYNTOK)
    return fail(W8A8_ERR_INVALID_ARG, "act_mode %d is not STATIC or DYNTOK", act_mode);
  if (out_mode < W8A8_OUT_ACC_I32 || out_mode > W8A8_OUT_F32_ACC)
    return fail(W8A8_ERR_INVALID_ARG, "out_mode %d is not a w8a8_out_mode", out_mode);
  if ((out_mode == W8A8_OUT_QUANT || out_mode == W8A8_OUT_F32) && !l->has_quant_m)
    return fail(W8A8_ERR_NOT_SUPPORTED, "requant output needs quant_m at create");
  if (out_mode == W8A8_OUT_F32_ACC && !l->has_acc_step)
    return fail(W8A8_ERR_NOT_SUPPORTED, "F32_ACC output needs acc_step at create");
  return W8A8_SUCCESS;
}

// Runs the contraction over int8 activations xq [T, ldx] (16-byte aligned rows, k_pad
// readable), in groups of at most 8 tokens.
w8a8_status run_gemv(w8a8_linear *l, const int8_t *xq, int64_t ldx, int T, int act_mode,
                     const float *ratio, int out_mode, void *y, int64_t ldy, bool pdl,
                     cudaStream_t st) {
  const bool tensor = l->path == W8A8_PATH_TENSOR || l->path == W8A8_PATH_TENSOR_PAIR ||
                      (l->path == W8A8_PATH_AUTO && T >= W8A8_TC_MIN_TOKENS);
  if (tensor) {
    TcPlan plan;
    if (!plan_tc(T, l->N, l->k_pad, l->ctx->sm_count, &plan, l->path == W8A8_PATH_TENSOR_PAIR))
      return fail(W8A8_ERR_NOT_SUPPORTED, "no tensor-core plan for T=%d N=%d K=%d", T, l->N, l->K);
    if (plan.splits > 1) {
      w8a8_status s = ensure_tc_scratch(l, static_cast<size_t>(T) * l->N,
                                        static_cast<size_t>(plan.tiles_n) * plan.tiles_t);
      if (s != W8A8_SUCCESS) return s;
    }
    bool built = false;
    w8a8_status s = ensure_tc_weights(l, st, &built);
    if (s != W8A8_SUCCESS) return s;
    TcLaunch L = {};
    L.w_tiles = l->w_tiles;
    L.x = xq;
    L.ldx = ldx;
    L.k_extent_x = l->k_pad;
    L.T = T;
    L.N = l->N;
    L.ep = make_epilogue(l, out_mode, act_mode, ratio, y, ldy);
    L.ws = l->tc_ws;
    L.tile_count = l->tc_count;
    L.err = l->ctx->d_err;
    L.trace = l->tc_trace;
    // The GEMM reads weight tiles before its dependency wait: not right after they were built.
    L.pdl = pdl && !built;
    W8A8_CUDA(launch_tc(L, plan, st));
    return W8A8_SUCCESS;
  }
  const size_t out_elem = out_mode == W8A8_OUT_ACC_I32 ? 4
                          : out_mode == W8A8_OUT_QUANT ? (l->out_i16 ? 2 : 1)
                                                        : 4;
  for (int t0 = 0; t0 < T; t0 += 8) {
    const int tg = std::min(8, T - t0);
    GemvPlan plan;
    if (!plan_gemv(tg, l->N, l->k_pad, false, 0, l->ctx->sm_count, &plan))
      return fail(W8A8_ERR_NOT_SUPPORTED, "no GEMV plan for T=%d N=%d K=%d", tg, l->N, l->K);
    GemvLaunch L = {};
    L.w = l->w;
    L.ldw = l->k_pad;
    L.x = xq + t0 * ldx;
    L.ldx = ldx;
    L.T = tg;
    L.N = l->N;
    L.k_pad = l->k_pad;
    L.ep = make_epilogue(l, out_mode, act_mode, ratio ? ratio + t0 : nullptr,
                         static_cast<char *>(y) + static_cast<size_t>(t0) * ldy * out_elem, ldy);
    L.topk = false;
    L.err = l->ctx->d_err;
    L.sm_count = l->ctx->sm_count;
    L.pdl = pdl;
    L.trace = plan.grid <= 2 * l->ctx->sm_count ? l->tc_trace : nullptr;
    W8A8_CUDA(launch_gemv(L, plan, st));
  }
  return W8A8_SUCCESS;
}

}  // namespace

namespace w8a8 {

w8a8_status linear_quant_input(w8a8_linear *l, const float *x, int64_t ldx, int T, int act_mode,
                               const PublishPeer *peers, int n_peers, unsigned *pub_seq,
                               unsigned *pub_arrive, cudaStream_t s, unsigned long long *trace,
                               int8_t *q_rows, int pub_row0, const float *emb_norm, float eps) {
  ActQuantLaunch A = {};
  A.x = x;
  A.ldx = ldx;
  A.T = T;
  A.K = l->K;
  A.k_fill = l->k_pad;
  A.inv_smooth = l->inv_smooth;
  A.act_mode = act_mode;
  A.inv_step = l->inv_step;
  A.safe_thresh = l->safe_thresh;
  A.q = q_rows ? q_rows : l->xq;
  A.ldq = l->k_pad;
  A.ratio = l->ratio;
  A.pdl = true;
  A.pub_row0 = pub_row0;
  A.emb_norm = emb_norm;
  A.eps = eps;
  A.peers = peers;
  A.n_peers = n_peers;
  A.pub_seq = pub_seq;
  A.pub_arrive = pub_arrive;
  A.trace = trace;
  W8A8_CUDA(launch_act_quant(A, s));
  return W8A8_SUCCESS;
}

bool linear_can_fuse(const w8a8_linear *l, int T, int act_mode, FusedQuant *fq) {
  const int tg = std::min(T, 8);
  const int tt = tg <= 1 ? 1 : tg <= 2 ? 2 : tg <= 4 ? 4 : 8;
  if (act_mode != W8A8_ACT_STATIC || tt * l->k_pad > kFusedXMaxBytes) return false;
  *fq = FusedQuant{};
  fq->K = l->K;
  fq->inv_smooth = l->inv_smooth;
  fq->inv_step = l->inv_step;
  return true;
}

bool topk_on_tensor_cores(const w8a8_linear *l, int T) {
  return T >= W8A8_TC_MIN_TOKENS && l->path != W8A8_PATH_GEMV;
}

w8a8_status linear_topk_quantized(w8a8_linear *l, int T, int act_mode, int out_mode, int k,
                                  int row_offset, float *topk_val, int32_t *topk_idx,
                                  float *logits, int64_t ldl, const ShardSync &sync, bool pdl,
                                  cudaStream_t s, const FusedQuant *fq, const int8_t *x_rows,
                                  const TopkRoute *route) {
  if (((sync.seq && sync.n_ready == 0) || (fq && fq->pub_seq)) && T > 8)
    return fail(W8A8_ERR_INVALID_ARG, "a multi-device LM head takes at most 8 tokens a forward");
  const bool fused = fq && fq->x;
  if (topk_on_tensor_cores(l, T) && !fused && !route && !sync.seq && !sync.done &&
      !sync.done_peers) {
    // 16+ tokens: one tensor-core GEMM writes the logits (the weights stream once), then the
    // per-CTA row lists and the per-token selection
    float *lg = logits;
    int64_t ld = ldl;
    if (!lg) {
      w8a8_status st = grow_scratch(&l->logit_ws, &l->logit_ws_elems,
                                    static_cast<size_t>(T) * l->N);
      if (st != W8A8_SUCCESS) return st;
      lg = l->logit_ws;
      ld = l->N;
    }
    w8a8_status st = grow_scratch(&l->row_lists, &l->row_lists_keys,
                                  static_cast<size_t>(T) * topk_rows_grid(l->N) * (k + 1));
    if (st != W8A8_SUCCESS) return st;
    st = run_gemv(l, x_rows ? x_rows : l->xq, l->k_pad, T, act_mode, l->ratio, out_mode, lg, ld,
                  pdl, s);
    if (st != W8A8_SUCCESS) return st;
    TopK tk = {};
    tk.k = k;
    tk.row_offset = row_offset;
    tk.lists = l->row_lists;
    tk.counter = l->counter;
    tk.val = topk_val;
    tk.idx = topk_idx;
    W8A8_CUDA(launch_topk_rows(lg, ld, T, l->N, tk, true, s));
    return W8A8_SUCCESS;
  }
  for (int t0 = 0; t0 < T; t0 += 8) {
    const int tg = std::min(8, T - t0);
    GemvPlan plan;
    if (!plan_gemv(tg, l->N, l->k_pad, true, k, l->ctx->sm_count, &plan, fused))
      return fail(W8A8_ERR_NOT_SUPPORTED, "no top-k plan for T=%d N=%d K=%d k=%d", tg, l->N, l->K, k);
    if (static_cast<size_t>(tg) * plan.grid * (k + 1) > l->lists_keys)
      return fail(W8A8_ERR_NOT_SUPPORTED, "top-k scratch too small");
    GemvLaunch L = {};
    L.w = l->w;
    L.ldw = l->k_pad;
    L.x = (x_rows ? x_rows : l->xq) + static_cast<size_t>(t0) * l->k_pad;
    L.ldx = l->k_pad;
    L.T = tg;
    L.N = l->N;
    L.k_pad = l->k_pad;
    L.ep = make_epilogue(l, out_mode, act_mode, l->ratio + t0, nullptr, 0);
    L.topk = true;
    L.tk.k = k;
    L.tk.row_offset = row_offset;
    L.tk.lists = l->lists;
    L.tk.counter = l->counter;
    L.tk.val = topk_val + static_cast<size_t>(t0) * k;
    L.tk.idx = topk_idx + static_cast<size_t>(t0) * k;
    L.tk.logits = logits ? logits + static_cast<size_t>(t0) * ldl : nullptr;
    L.tk.ldl = ldl;
    L.err = l->ctx->d_err;
    L.sm_count = l->ctx->sm_count;
    L.pdl = pdl;
    L.trace = plan.grid <= 2 * l->ctx->sm_count ? l->tc_trace : nullptr;
    L.sync = sync;
    L.sync.hold = t0 + 8 < T ? 1 : 0;  // only the forward's last token group counts it
    if (route) {
      L.tk.val_dst = route->val_dst;
      L.tk.idx_dst = route->idx_dst;
      L.tk.dst_tokens = route->tokens;
      L.tk.tok0 = t0;
      L.tk.dst_row0 = route->row0;
      L.tk.dst_ld = route->ld;
    }
    if (fused) {
      L.fq = *fq;
      L.fq.x = fq->x + static_cast<size_t>(t0) * fq->ldx;
    }
    W8A8_CUDA(launch_gemv(L, plan, s));
  }
  return W8A8_SUCCESS;
}

int8_t *linear_staging(w8a8_linear *l) { return l->xq; }

int linear_staging_ld(const w8a8_linear *l) { return l->k_pad; }

w8a8_status linear_reserve_tokens(w8a8_linear *l, int T) {
  DeviceGuard g(l->ctx->device);
  return ensure_tokens(l, T);
}

int *linear_error_word(w8a8_linear *l) { return l->ctx->d_err; }

int *ctx_error_word(w8a8_ctx *ctx) { return ctx->d_err; }

}  // namespace w8a8


extern "C" {

const char *w8a8_status_to_string(w8a8_status s) {
  switch (s) {
    case W8A8_SUCCESS: return "success";
    case W8A8_ERR_INVALID_ARG: return "invalid argument";
    case W8A8_ERR_NO_MEMORY: return "out of device or host memory";
    case W8A8_ERR_DEVICE_BUSY: return "device busy";
    case W8A8_ERR_HARDWARE_FAULT: return "hardware fault";
    case W8A8_ERR_NOT_INITIALIZED: return "not initialized";
    case W8A8_ERR_NOT_SUPPORTED: return "not supported";
    case W8A8_ERR_IO: return "I/O error";
    case W8A8_ERR_CHECKSUM_MISMATCH: return "checksum mismatch";
    case W8A8_ERR_TIMEOUT: return "timeout";
    case W8A8_ERR_CUDA: return "CUDA error";
    case W8A8_ERR_PEER_TIMEOUT: return "peer timeout";
  }
  return "unknown status";
}

const char *w8a8_last_error(void) { return g_last_error.c_str(); }

const char *w8a8_version(void) { return "w8a8-b200 0.1.0 (sm_100a)"; }

w8a8_status w8a8_ctx_create(int device, w8a8_ctx **out_ctx) {
  if (!out_ctx) return fail(W8A8_ERR_INVALID_ARG, "out_ctx is NULL");
  *out_ctx = nullptr;
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess || ndev == 0)
    return fail(W8A8_ERR_NOT_INITIALIZED, "no CUDA device: %s", cudaGetErrorString(e));
  if (device < 0 || device >= ndev)
    return fail(W8A8_ERR_INVALID_ARG, "device %d out of range [0, %d)", device, ndev);
  // The caller's current device is restored on return: every call on this context's objects
  // selects the device itself.
  DeviceGuard guard(device);
  cudaDeviceProp prop;
  W8A8_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10 || prop.minor != 0)
    return fail(W8A8_ERR_NOT_SUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  w8a8_ctx *c = new (std::nothrow) w8a8_ctx();
  if (!c) return fail(W8A8_ERR_NO_MEMORY, "host allocation failed");
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  if (cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess) {
    delete c;
    return fail(W8A8_ERR_NO_MEMORY, "cudaMalloc of the error word failed");
  }
  cudaMemset(c->d_err, 0, sizeof(int));
  *out_ctx = c;
  return W8A8_SUCCESS;
}

void w8a8_ctx_destroy(w8a8_ctx *ctx) {
  if (!ctx) return;
  DeviceGuard g(ctx->device);
  cudaFree(ctx->d_err);
  delete ctx;
}

int w8a8_ctx_sm_count(const w8a8_ctx *ctx) { return ctx ? ctx->sm_count : 0; }

int w8a8_ctx_device(const w8a8_ctx *ctx) { return ctx ? ctx->device : -1; }

w8a8_status w8a8_ctx_check(w8a8_ctx *ctx) {
  if (!ctx) return fail(W8A8_ERR_INVALID_ARG, "ctx is NULL");
  DeviceGuard g(ctx->device);
  W8A8_CUDA(cudaDeviceSynchronize());
  int code = 0;
  W8A8_CUDA(cudaMemcpy(&code, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code == 0) return W8A8_SUCCESS;
  W8A8_CUDA(cudaMemset(ctx->d_err, 0, sizeof(int)));
  if (code == kDevPeerTimeout) return fail(W8A8_ERR_PEER_TIMEOUT, "a peer flag wait ran out");
  return fail(W8A8_ERR_TIMEOUT, "a bounded in-kernel wait ran out (code %d)", code);
}

w8a8_status w8a8_linear_create(w8a8_ctx *ctx, const w8a8_linear_desc *d, w8a8_linear **out) {
  if (!out) return fail(W8A8_ERR_INVALID_ARG, "out_linear is NULL");
  *out = nullptr;
  if (!ctx || !d) return fail(W8A8_ERR_INVALID_ARG, "ctx or desc is NULL");
  if (d->K < 1 || d->N < 1) return fail(W8A8_ERR_INVALID_ARG, "K=%d N=%d must be >= 1", d->K, d->N);
  if (!d->weights) return fail(W8A8_ERR_INVALID_ARG, "weights is NULL");
  if (d->weights_ld < d->K) return fail(W8A8_ERR_INVALID_ARG, "weights_ld %lld < K %d", (long long)d->weights_ld, d->K);
  if (d->quant_m && (d->trunc < 0 || d->trunc > 62))
    return fail(W8A8_ERR_INVALID_ARG, "trunc %d outside [0, 62]", d->trunc);
  if (d->quant_m && d->scale.out_dtype != W8A8_DTYPE_INT8 && d->scale.out_dtype != W8A8_DTYPE_INT16)
    return fail(W8A8_ERR_NOT_SUPPORTED, "requant out_dtype %d is not INT8 or INT16", d->scale.out_dtype);
  if (d->quant_m) {
    for (int n = 0; n < d->N; ++n)
      if (d->quant_m[n] < 1)
        return fail(W8A8_ERR_INVALID_ARG, "quant_m[%d] = %d is outside [1, 32767]", n, d->quant_m[n]);
  }
  DeviceGuard g(ctx->device);
  w8a8_linear *l = new (std::nothrow) w8a8_linear();
  if (!l) return fail(W8A8_ERR_NO_MEMORY, "host allocation failed");
  l->ctx = ctx;
  l->K = d->K;
  l->N = d->N;
  l->k_pad = static_cast<int>(round_up(d->K, 16));
  l->trunc = d->trunc;
  l->out_i16 = d->scale.out_dtype == W8A8_DTYPE_INT16 ? 1 : 0;
  l->qmax = l->out_i16 ? 32767 : 127;
  l->inv_step = (d->scale.in_step > 1e-12f) ? (1.0f / d->scale.in_step) : 0.0f;
  l->safe_thresh = std::max(d->scale.in_thresh, 1e-8f);
  w8a8_status st;
#define TRY(x)                 \
  do {                         \
    st = (x);                  \
    if (st != W8A8_SUCCESS) {  \
      linear_free(l);          \
      return st;               \
    }                          \
  } while (0)
  const size_t wbytes = static_cast<size_t>(l->N) * l->k_pad;
  TRY(dev_alloc(&l->w, wbytes, &l->device_bytes));
  {
    std::vector<int8_t> host(wbytes, 0);
    for (int n = 0; n < l->N; ++n)
      std::memcpy(host.data() + static_cast<size_t>(n) * l->k_pad,
                  d->weights + static_cast<int64_t>(n) * d->weights_ld, d->K);
    if (cudaMemcpy(l->w, host.data(), wbytes, cudaMemcpyHostToDevice) != cudaSuccess) {
      linear_free(l);
      return fail(W8A8_ERR_CUDA, "weight upload failed");
    }
  }
  TRY(dev_alloc(&l->quant_m, l->N, &l->device_bytes));
  TRY(dev_alloc(&l->quant_m32, l->N, &l->device_bytes));
  TRY(dev_alloc(&l->out_step, l->N, &l->device_bytes));
  TRY(dev_alloc(&l->acc_step, l->N, &l->device_bytes));
  {
    std::vector<int16_t> qm(l->N, 1);
    std::vector<float> os(l->N), as(l->N, 0.0f);
    if (d->quant_m) std::memcpy(qm.data(), d->quant_m, sizeof(int16_t) * l->N);
    std::vector<int32_t> qm32(qm.begin(), qm.end());
    for (int n = 0; n < l->N; ++n) os[n] = d->scale.out_step_chan ? d->scale.out_step_chan[n] : d->scale.out_step;
    if (d->acc_step) std::memcpy(as.data(), d->acc_step, sizeof(float) * l->N);
    l->has_quant_m = d->quant_m != nullptr;
    l->has_acc_step = d->acc_step != nullptr;
    if (cudaMemcpy(l->quant_m, qm.data(), sizeof(int16_t) * l->N, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->quant_m32, qm32.data(), sizeof(int32_t) * l->N, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->out_step, os.data(), sizeof(float) * l->N, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->acc_step, as.data(), sizeof(float) * l->N, cudaMemcpyHostToDevice) != cudaSuccess) {
      linear_free(l);
      return fail(W8A8_ERR_CUDA, "parameter upload failed");
    }
  }
  if (d->scale.in_inv_smooth) {
    TRY(dev_alloc(&l->inv_smooth, static_cast<size_t>(round_up(l->K, 4)), &l->device_bytes));
    if (cudaMemcpy(l->inv_smooth, d->scale.in_inv_smooth, sizeof(float) * l->K, cudaMemcpyHostToDevice) != cudaSuccess) {
      linear_free(l);
      return fail(W8A8_ERR_CUDA, "in_inv_smooth upload failed");
    }
  }
  TRY(ensure_tokens(l, kPreallocTokens));
  l->device_bytes += static_cast<size_t>(kPreallocTokens) * (l->k_pad + 4);
  // Top-k scratch sized for the largest plan over T <= 8, k <= 64.
  size_t max_keys = 0;
  for (int T = 1; T <= 8; ++T) {
    GemvPlan p;
    if (plan_gemv(T, l->N, l->k_pad, true, std::min(64, l->N), ctx->sm_count, &p))
      max_keys = std::max(max_keys, static_cast<size_t>(T) * p.grid * 65);
  }
  l->lists_keys = std::max<size_t>(max_keys, 64);
  TRY(dev_alloc(&l->lists, l->lists_keys, &l->device_bytes));
  TRY(dev_alloc(&l->counter, 1, &l->device_bytes));
  if (cudaMemset(l->counter, 0, sizeof(unsigned)) != cudaSuccess) {
    linear_free(l);
    return fail(W8A8_ERR_CUDA, "counter init failed");
  }
#undef TRY
  *out = l;
  return W8A8_SUCCESS;
}

void w8a8_linear_destroy(w8a8_linear *l) { linear_free(l); }

size_t w8a8_linear_device_bytes(const w8a8_linear *l) { return l ? l->device_bytes : 0; }

w8a8_status w8a8_linear_set_trace(w8a8_linear *l, unsigned long long *trace_dev) {
  if (!l) return fail(W8A8_ERR_INVALID_ARG, "linear is NULL");
  l->tc_trace = trace_dev;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_linear_set_input_norm(w8a8_linear *l, const float *emb_norm_scaled, float eps) {
  if (!l) return fail(W8A8_ERR_INVALID_ARG, "linear is NULL");
  if (emb_norm_scaled && l->K > 12288) return fail(W8A8_ERR_INVALID_ARG, "input norm needs K <= 12288");
  if (emb_norm_scaled && !(eps >= 0.0f)) return fail(W8A8_ERR_INVALID_ARG, "eps must be >= 0");
  l->emb_norm = emb_norm_scaled;
  l->norm_eps = eps;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_linear_set_path(w8a8_linear *l, int32_t path) {
  if (!l) return fail(W8A8_ERR_INVALID_ARG, "linear is NULL");
  if (path != W8A8_PATH_AUTO && path != W8A8_PATH_GEMV && path != W8A8_PATH_TENSOR &&
      path != W8A8_PATH_TENSOR_PAIR)
    return fail(W8A8_ERR_INVALID_ARG, "path %d is not a w8a8_path", path);
  l->path = path;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_linear_reserve(w8a8_linear *l, int32_t max_tokens, int32_t max_k, void *stream) {
  if (!l) return fail(W8A8_ERR_INVALID_ARG, "linear is NULL");
  if (max_tokens < 1) return fail(W8A8_ERR_INVALID_ARG, "max_tokens=%d must be >= 1", max_tokens);
  if (max_k < 0 || max_k > W8A8_TOPK_MAX)
    return fail(W8A8_ERR_INVALID_ARG, "max_k=%d outside [0, %d]", max_k, W8A8_TOPK_MAX);
  DeviceGuard g(l->ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  w8a8_status s = ensure_tokens(l, max_tokens);
  if (s != W8A8_SUCCESS) return s;
  const bool forced = l->path == W8A8_PATH_TENSOR || l->path == W8A8_PATH_TENSOR_PAIR;
  const bool any_tc = forced || (l->path == W8A8_PATH_AUTO && max_tokens >= W8A8_TC_MIN_TOKENS);
  if (!any_tc) return W8A8_SUCCESS;
  // the largest split-K accumulation plane and tile-counter arrays over every token count that
  // takes the tensor-core path
  size_t ws = 0, counters = 0;
  for (int T = forced ? 1 : W8A8_TC_MIN_TOKENS; T <= max_tokens; ++T) {
    TcPlan plan;
    if (!plan_tc(T, l->N, l->k_pad, l->ctx->sm_count, &plan, l->path == W8A8_PATH_TENSOR_PAIR))
      return fail(W8A8_ERR_NOT_SUPPORTED, "no tensor-core plan for T=%d N=%d K=%d", T, l->N, l->K);
    if (plan.splits > 1) {
      ws = std::max(ws, static_cast<size_t>(T) * l->N);
      counters = std::max(counters, static_cast<size_t>(plan.tiles_n) * plan.tiles_t);
    }
  }
  if (ws > 0 && (s = ensure_tc_scratch(l, ws, counters)) != W8A8_SUCCESS) return s;
  bool built = false;
  if ((s = ensure_tc_weights(l, st, &built)) != W8A8_SUCCESS) return s;
  if (max_k > 0 && max_tokens >= W8A8_TC_MIN_TOKENS && l->path != W8A8_PATH_GEMV) {
    if ((s = grow_scratch(&l->logit_ws, &l->logit_ws_elems,
                          static_cast<size_t>(max_tokens) * l->N)) != W8A8_SUCCESS)
      return s;
    if ((s = grow_scratch(&l->row_lists, &l->row_lists_keys,
                          static_cast<size_t>(max_tokens) * topk_rows_grid(l->N) * (max_k + 1))) !=
        W8A8_SUCCESS)
      return s;
  }
  return W8A8_SUCCESS;
}

w8a8_status w8a8_pack_input(w8a8_linear *l, const float *x, int64_t ldx, int32_t T, int32_t act_mode,
                            int8_t *q, int64_t ldq, float *ratio, void *stream) {
  if (!l || !x || !q) return fail(W8A8_ERR_INVALID_ARG, "linear, x or q is NULL");
  if (T < 1) return fail(W8A8_ERR_INVALID_ARG, "T=%d must be >= 1", T);
  if (ldx < l->K || ldq < l->K) return fail(W8A8_ERR_INVALID_ARG, "ldx/ldq below K");
  if (act_mode != W8A8_ACT_STATIC && act_mode != W8A8_ACT_DYNTOK)
    return fail(W8A8_ERR_INVALID_ARG, "act_mode %d", act_mode);
  if (act_mode == W8A8_ACT_DYNTOK && !ratio) return fail(W8A8_ERR_INVALID_ARG, "DYNTOK needs ratio");
  DeviceGuard g(l->ctx->device);
  ActQuantLaunch L = {};
  L.x = x;
  L.ldx = ldx;
  L.T = T;
  L.K = l->K;
  L.k_fill = l->K;
  L.inv_smooth = l->inv_smooth;
  L.act_mode = act_mode;
  L.inv_step = l->inv_step;
  L.safe_thresh = l->safe_thresh;
  L.q = q;
  L.ldq = ldq;
  L.ratio = ratio;
  L.pdl = false;
  W8A8_CUDA(launch_act_quant(L, static_cast<cudaStream_t>(stream)));
  return W8A8_SUCCESS;
}

w8a8_status w8a8_linear_forward_q(w8a8_linear *l, const int8_t *q, int64_t ldq, int32_t T,
                                  int32_t act_mode, const float *ratio, int32_t out_mode, void *y,
                                  int64_t ldy, void *stream) {
  if (!l || !q || !y) return fail(W8A8_ERR_INVALID_ARG, "linear, q or y is NULL");
  if (T < 1) return fail(W8A8_ERR_INVALID_ARG, "T=%d must be >= 1", T);
  if (ldq < l->K || ldy < l->N) return fail(W8A8_ERR_INVALID_ARG, "ldq < K or ldy < N");
  w8a8_status st = check_modes(l, act_mode, out_mode);
  if (st != W8A8_SUCCESS) return st;
  const bool needs_ratio = act_mode == W8A8_ACT_DYNTOK && (out_mode == W8A8_OUT_F32 || out_mode == W8A8_OUT_F32_ACC);
  if (needs_ratio && !ratio) return fail(W8A8_ERR_INVALID_ARG, "DYNTOK float output needs ratio");
  DeviceGuard g(l->ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int8_t *xin = q;
  int64_t ldx = ldq;
  if (!(aligned16(q) && ldq % 16 == 0 && l->K % 16 == 0)) {
    st = ensure_tokens(l, T);
    if (st != W8A8_SUCCESS) return st;
    W8A8_CUDA(launch_copy_pad_i8(q, ldq, T, l->K, l->xq, l->k_pad, l->k_pad, false, s));
    xin = l->xq;
    ldx = l->k_pad;
  }
  return run_gemv(l, xin, ldx, T, act_mode, ratio, out_mode, y, ldy, xin != q, s);
}

w8a8_status w8a8_unpack_output(w8a8_linear *l, const void *yq, int64_t ldyq, int32_t T, int32_t act_mode,
                               const float *ratio, float *y, int64_t ldy, void *stream) {
  if (!l || !yq || !y) return fail(W8A8_ERR_INVALID_ARG, "linear, yq or y is NULL");
  if (T < 1 || ldyq < l->N || ldy < l->N) return fail(W8A8_ERR_INVALID_ARG, "bad T or strides");
  if (act_mode == W8A8_ACT_DYNTOK && !ratio) return fail(W8A8_ERR_INVALID_ARG, "DYNTOK needs ratio");
  DeviceGuard g(l->ctx->device);
  UnpackLaunch L = {};
  L.yq = yq;
  L.ldyq = ldyq;
  L.in_i16 = l->out_i16;
  L.T = T;
  L.N = l->N;
  L.act_mode = act_mode;
  L.ratio = ratio;
  L.out_step = l->out_step;
  L.y = y;
  L.ldy = ldy;
  L.pdl = false;
  W8A8_CUDA(launch_unpack(L, static_cast<cudaStream_t>(stream)));
  return W8A8_SUCCESS;
}

w8a8_status w8a8_linear_forward(w8a8_linear *l, const float *x, int64_t ldx, int32_t T, int32_t act_mode,
                                int32_t out_mode, void *y, int64_t ldy, float *ratio_out, void *stream) {
  if (!l || !x || !y) return fail(W8A8_ERR_INVALID_ARG, "linear, x or y is NULL");
  if (T < 1) return fail(W8A8_ERR_INVALID_ARG, "T=%d must be >= 1", T);
  if (ldx < l->K || ldy < l->N) return fail(W8A8_ERR_INVALID_ARG, "ldx < K or ldy < N");
  w8a8_status st = check_modes(l, act_mode, out_mode);
  if (st != W8A8_SUCCESS) return st;
  DeviceGuard g(l->ctx->device);
  st = ensure_tokens(l, T);
  if (st != W8A8_SUCCESS) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float *ratio = ratio_out ? ratio_out : l->ratio;
  ActQuantLaunch A = {};
  A.x = x;
  A.ldx = ldx;
  A.T = T;
  A.K = l->K;
  A.k_fill = l->k_pad;
  A.inv_smooth = l->inv_smooth;
  A.act_mode = act_mode;
  A.inv_step = l->inv_step;
  A.safe_thresh = l->safe_thresh;
  A.q = l->xq;
  A.ldq = l->k_pad;
  A.ratio = ratio;
  A.pdl = true;
  W8A8_CUDA(launch_act_quant(A, s));
  return run_gemv(l, l->xq, l->k_pad, T, act_mode, ratio, out_mode, y, ldy, true, s);
}

w8a8_status w8a8_linear_forward_topk(w8a8_linear *l, const float *x, int64_t ldx, int32_t T,
                                     int32_t act_mode, int32_t out_mode, int32_t k, int32_t row_offset,
                                     float *topk_val, int32_t *topk_idx, float *logits, int64_t ldl,
                                     void *stream) {
  if (!l || !x || !topk_val || !topk_idx) return fail(W8A8_ERR_INVALID_ARG, "NULL argument");
  if (T < 1) return fail(W8A8_ERR_INVALID_ARG, "T=%d must be >= 1", T);
  if (ldx < l->K) return fail(W8A8_ERR_INVALID_ARG, "ldx < K");
  if (out_mode != W8A8_OUT_F32 && out_mode != W8A8_OUT_F32_ACC)
    return fail(W8A8_ERR_INVALID_ARG, "top-k needs a float out_mode (F32 or F32_ACC)");
  if (k < 1 || k > W8A8_TOPK_MAX || k > l->N)
    return fail(W8A8_ERR_INVALID_ARG, "k=%d outside [1, min(%d, N=%d)]", k, W8A8_TOPK_MAX, l->N);
  if (row_offset < 0 || static_cast<int64_t>(row_offset) + l->N > INT32_MAX)
    return fail(W8A8_ERR_INVALID_ARG, "row_offset %d out of range", row_offset);
  if (logits && ldl < l->N) return fail(W8A8_ERR_INVALID_ARG, "ldl < N");
  w8a8_status st = check_modes(l, act_mode, out_mode);
  if (st != W8A8_SUCCESS) return st;
  DeviceGuard g(l->ctx->device);
  st = ensure_tokens(l, T);
  if (st != W8A8_SUCCESS) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (l->emb_norm && act_mode == W8A8_ACT_STATIC) {
    st = w8a8::linear_quant_input(l, x, ldx, T, act_mode, nullptr, 0, nullptr, nullptr, s,
                                  nullptr, nullptr, 0, l->emb_norm, l->norm_eps);
    if (st != W8A8_SUCCESS) return st;
    return w8a8::linear_topk_quantized(l, T, act_mode, out_mode, k, row_offset, topk_val,
                                       topk_idx, logits, ldl, w8a8::ShardSync{}, true, s);
  }
  w8a8::FusedQuant fq;
  if (!w8a8::topk_on_tensor_cores(l, T) && w8a8::linear_can_fuse(l, T, act_mode, &fq)) {
    // static quantisation runs in the GEMV prologue: one launch per 8 tokens
    fq.x = x;
    fq.ldx = ldx;
    return w8a8::linear_topk_quantized(l, T, act_mode, out_mode, k, row_offset, topk_val,
                                       topk_idx, logits, ldl, w8a8::ShardSync{}, true, s, &fq);
  }
  st = w8a8::linear_quant_input(l, x, ldx, T, act_mode, nullptr, 0, nullptr, nullptr, s);
  if (st != W8A8_SUCCESS) return st;
  return w8a8::linear_topk_quantized(l, T, act_mode, out_mode, k, row_offset, topk_val, topk_idx,
                                     logits, ldl, w8a8::ShardSync{}, true, s);
}

w8a8_status w8a8_topk_merge(w8a8_ctx *ctx, const float *in_val, const int32_t *in_idx, int32_t T,
                            int32_t n_lists, int32_t k_in, int64_t list_stride, int64_t token_stride,
                            int32_t k_out, float *out_val, int32_t *out_idx, int32_t *argmax,
                            void *stream) {
  if (!ctx || !in_val || !in_idx || !out_val || !out_idx) return fail(W8A8_ERR_INVALID_ARG, "NULL argument");
  if (T < 1 || n_lists < 1 || n_lists > 64 || k_in < 1 || k_in > W8A8_TOPK_MAX || k_out < 1 ||
      k_out > W8A8_TOPK_MAX || k_out > n_lists * k_in)
    return fail(W8A8_ERR_INVALID_ARG, "bad merge shape T=%d n_lists=%d k_in=%d k_out=%d", T, n_lists, k_in, k_out);
  if (list_stride < k_in || token_stride < 0)
    return fail(W8A8_ERR_INVALID_ARG, "list_stride %lld < k_in %d or negative token_stride",
                (long long)list_stride, k_in);
  DeviceGuard g(ctx->device);
  MergeLaunch L = {};
  L.in_val = in_val;
  L.in_idx = in_idx;
  L.T = T;
  L.n_lists = n_lists;
  L.k_in = k_in;
  L.k_out = k_out;
  L.list_stride = list_stride;
  L.token_stride = token_stride;
  L.out_val = out_val;
  L.out_idx = out_idx;
  L.argmax = argmax;
  L.pdl = true;
  W8A8_CUDA(launch_topk_merge(L, static_cast<cudaStream_t>(stream)));
  return W8A8_SUCCESS;
}

}  // extern "C"

struct w8a8_chain {
  w8a8_ctx *ctx = nullptr;
  int n_ops = 0, T = 0, barriers = 0;
  size_t clear_bytes = 0;
  unsigned long long *trace = nullptr;
  ChainPlan plan = {};
  ChainOp *ops_dev = nullptr;
  unsigned *bar = nullptr;
  unsigned *tk_counter = nullptr;
  uint64_t *lists = nullptr;
};

namespace {

struct Range {
  uintptr_t lo, hi;
};

Range view_range(const void *p, int64_t ld, int rows, int cols, size_t elem) {
  const uintptr_t b = reinterpret_cast<uintptr_t>(p);
  return {b, b + (static_cast<uintptr_t>(rows - 1) * ld + cols) * elem};
}

bool overlap(const Range &a, const Range &b) { return a.lo < b.hi && b.lo < a.hi; }

void chain_free(w8a8_chain *c) {
  if (!c) return;
  DeviceGuard g(c->ctx ? c->ctx->device : 0);
  cudaFree(c->ops_dev);
  cudaFree(c->bar);
  cudaFree(c->tk_counter);
  cudaFree(c->lists);
  delete c;
}

size_t out_elem_bytes(const w8a8_linear *l, int out_mode) {
  return out_mode == W8A8_OUT_QUANT ? (l->out_i16 ? 2 : 1) : 4;
}

}  // namespace

extern "C" {

w8a8_status w8a8_chain_create(w8a8_ctx *ctx, const w8a8_chain_step *steps, int32_t n, int32_t T,
                              w8a8_chain **out) {
  if (!out) return fail(W8A8_ERR_INVALID_ARG, "out_chain is NULL");
  *out = nullptr;
  if (!ctx || !steps || n < 1) return fail(W8A8_ERR_INVALID_ARG, "ctx/steps NULL or n_steps < 1");
  if (T < 1 || T > 8) return fail(W8A8_ERR_INVALID_ARG, "T=%d outside [1, 8]", T);
  std::vector<ChainOp> ops(n);
  std::vector<Range> epoch_in, epoch_out;
  int barriers = 0;
  int topk_k = 0;
  for (int s = 0; s < n; ++s) {
    const w8a8_chain_step &st = steps[s];
    const w8a8_linear *l = st.linear;
    if (!l || l->ctx != ctx) return fail(W8A8_ERR_INVALID_ARG, "step %d: linear NULL or of another context", s);
    if (!st.x_dev || st.ldx < l->K) return fail(W8A8_ERR_INVALID_ARG, "step %d: x NULL or ldx < K", s);
    w8a8_status ms = check_modes(l, st.act_mode, st.out_mode);
    if (ms != W8A8_SUCCESS) return ms;
    const bool topk = st.topk_k != 0;
    if (topk) {
      if (s != n - 1) return fail(W8A8_ERR_INVALID_ARG, "step %d: the top-k step must be last", s);
      if (st.topk_k < 1 || st.topk_k > W8A8_TOPK_MAX || st.topk_k > l->N)
        return fail(W8A8_ERR_INVALID_ARG, "step %d: k=%d outside [1, min(64, N)]", s, st.topk_k);
      if (!st.topk_val_dev || !st.topk_idx_dev) return fail(W8A8_ERR_INVALID_ARG, "step %d: top-k outputs NULL", s);
      if (st.out_mode != W8A8_OUT_F32 && st.out_mode != W8A8_OUT_F32_ACC)
        return fail(W8A8_ERR_INVALID_ARG, "step %d: top-k needs F32 or F32_ACC", s);
      if (st.row_offset < 0) return fail(W8A8_ERR_INVALID_ARG, "step %d: negative row_offset", s);
      topk_k = st.topk_k;
    } else if (!st.y_dev || st.ldy < l->N) {
      return fail(W8A8_ERR_INVALID_ARG, "step %d: y NULL or ldy < N", s);
    }
    if (st.emb_norm_dev && st.act_mode != W8A8_ACT_STATIC)
      return fail(W8A8_ERR_INVALID_ARG, "step %d: emb_norm needs the STATIC act mode", s);
    if (st.emb_norm_dev && !(st.norm_eps >= 0.0f))
      return fail(W8A8_ERR_INVALID_ARG, "step %d: norm_eps must be >= 0", s);
    ChainOp &op = ops[s];
    op = ChainOp{};
    op.w = l->w;
    op.ldw = l->k_pad;
    op.N = l->N;
    op.K = l->K;
    op.k_pad = l->k_pad;
    op.x = st.x_dev;
    op.ldx = st.ldx;
    op.inv_smooth = l->inv_smooth;
    op.vec_x = (l->K % 4 == 0) && (st.ldx % 4 == 0) && aligned16(st.x_dev) ? 1 : 0;
    op.act_mode = st.act_mode;
    op.inv_step = l->inv_step;
    op.safe_thresh = l->safe_thresh;
    if (st.emb_norm_dev) {
      op.act_mode = kActEmbNorm;
      op.inv_smooth = st.emb_norm_dev;
      op.norm_eps = st.norm_eps;
    }
    op.ratio_out = st.ratio_dev;
    op.out_mode = st.out_mode;
    op.quant_m = l->quant_m;
    op.quant_m32 = l->quant_m32;
    op.trunc = l->trunc;
    op.qmax = l->qmax;
    op.out_i16 = l->out_i16;
    op.out_step = l->out_step;
    op.acc_step = l->acc_step;
    op.y = topk ? nullptr : st.y_dev;
    op.ldy = st.ldy;
    op.topk = topk ? 1 : 0;
    op.tk.k = st.topk_k;
    op.tk.row_offset = st.row_offset;
    op.tk.val = st.topk_val_dev;
    op.tk.idx = st.topk_idx_dev;
    // hazards against the steps since the last barrier: RAW (x vs y), WAR (y vs x), WAW
    const Range xin = view_range(st.x_dev, st.ldx, T, l->K, 4);
    Range yout = {0, 0};
    if (!topk) yout = view_range(st.y_dev, st.ldy, T, l->N, out_elem_bytes(l, st.out_mode));
    bool need = false;
    for (const Range &r : epoch_out) need = need || overlap(r, xin) || (!topk && overlap(r, yout));
    for (const Range &r : epoch_in) need = need || (!topk && overlap(r, yout));
    if (need && s > 0) {
      op.barrier_before = 1;
      ++barriers;
      epoch_in.clear();
      epoch_out.clear();
    }
    epoch_in.push_back(xin);
    if (!topk) epoch_out.push_back(yout);
  }
  ChainPlan plan;
  if (!plan_chain(ops.data(), n, T, ctx->sm_count, &plan))
    return fail(W8A8_ERR_NOT_SUPPORTED, "the chain does not fit the persistent kernel's shared memory plan");
  DeviceGuard g(ctx->device);
  w8a8_chain *c = new (std::nothrow) w8a8_chain();
  if (!c) return fail(W8A8_ERR_NO_MEMORY, "host allocation failed");
  c->ctx = ctx;
  c->n_ops = n;
  c->T = T;
  c->barriers = barriers;
  c->plan = plan;
  w8a8_status st;
  // zero-at-launch region: n arrival counters, then n amax slots of 8 floats
  c->clear_bytes = sizeof(unsigned) * n + sizeof(float) * 8 * n;
  if ((st = dev_alloc(&c->ops_dev, n, nullptr)) != W8A8_SUCCESS ||
      (st = dev_alloc(&c->bar, c->clear_bytes / sizeof(unsigned), nullptr)) != W8A8_SUCCESS ||
      (st = dev_alloc(&c->tk_counter, 1, nullptr)) != W8A8_SUCCESS ||
      (st = dev_alloc(&c->lists, static_cast<size_t>(T) * plan.grid * (std::max(topk_k, 1) + 1), nullptr)) !=
          W8A8_SUCCESS) {
    chain_free(c);
    return st;
  }
  // amax hand-off: a dyntok step whose input is a column block of exactly one earlier fp32
  // output (the latest step writing that memory) gets its per-token max |x * s| reduced by
  // that producer's epilogue, so it reads x once instead of twice.
  float *amax_dev = reinterpret_cast<float *>(c->bar + n);
  for (int s = 1; s < n; ++s) {
    const w8a8_chain_step &cs = steps[s];
    if (cs.act_mode != W8A8_ACT_DYNTOK) continue;
    const Range xin = view_range(cs.x_dev, cs.ldx, T, cs.linear->K, 4);
    int j = -1;
    for (int q = s - 1; q >= 0 && j < 0; --q) {
      if (steps[q].topk_k) continue;
      const Range yq = view_range(steps[q].y_dev, steps[q].ldy, T, steps[q].linear->N,
                                  out_elem_bytes(steps[q].linear, steps[q].out_mode));
      if (overlap(xin, yq)) j = q;
    }
    if (j < 0 || steps[j].out_mode != W8A8_OUT_F32 || steps[j].ldy != cs.ldx || ops[j].amax_dst)
      continue;
    const ptrdiff_t off = static_cast<const float *>(cs.x_dev) - static_cast<const float *>(steps[j].y_dev);
    if (off < 0 || off + cs.linear->K > steps[j].linear->N) continue;
    ops[j].amax_dst = amax_dev + 8 * s;
    ops[j].amax_c0 = static_cast<int>(off);
    ops[j].amax_cols = cs.linear->K;
    ops[j].amax_smooth = cs.linear->inv_smooth;
    ops[s].amax_src = amax_dev + 8 * s;
  }
  if (cudaMemcpy(c->ops_dev, ops.data(), sizeof(ChainOp) * n, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(c->tk_counter, 0, sizeof(unsigned)) != cudaSuccess) {
    chain_free(c);
    return fail(W8A8_ERR_CUDA, "chain upload failed");
  }
  const cudaError_t e = configure_chain(plan);
  if (e != cudaSuccess) {
    chain_free(c);
    return cuda_fail(e, "configure_chain");
  }
  *out = c;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_chain_forward(w8a8_chain *c, void *stream) {
  if (!c) return fail(W8A8_ERR_INVALID_ARG, "chain is NULL");
  DeviceGuard g(c->ctx->device);
  W8A8_CUDA(launch_chain(c->ops_dev, c->n_ops, c->T, c->plan, c->bar, c->clear_bytes,
                         c->tk_counter, c->lists, c->ctx->d_err, c->trace,
                         static_cast<cudaStream_t>(stream)));
  return W8A8_SUCCESS;
}

w8a8_status w8a8_chain_set_trace(w8a8_chain *c, unsigned long long *trace_dev) {
  if (!c) return fail(W8A8_ERR_INVALID_ARG, "chain is NULL");
  c->trace = trace_dev;
  return W8A8_SUCCESS;
}

int32_t w8a8_chain_grid(const w8a8_chain *c) { return c ? c->plan.grid : 0; }

void w8a8_chain_destroy(w8a8_chain *c) { chain_free(c); }

int32_t w8a8_chain_barriers(const w8a8_chain *c) { return c ? c->barriers : 0; }

}  // extern "C"
