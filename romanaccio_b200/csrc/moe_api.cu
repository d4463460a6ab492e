// C ABI w8a8_moe_*: the mixture-of-experts decode layer (router, W8A8 experts, combine) over
// device-resident expert tables.  Kernels in moe.cu; semantics in include/w8a8.h.
#include "../../include/w8a8.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "kernels.h"
#include "linear_internal.h"

using namespace w8a8;

struct w8a8_moe {
  w8a8_ctx *ctx = nullptr;
  int dev = 0;
  int H = 0, I = 0, E = 0, S = 0, k = 0, slots = 0, max_T = 0;
  int norm_topk = 0;
  float scaling = 1.0f;
  int gu_trunc = 0, dn_trunc = 0, dn_i16 = 0;
  int ldh = 0, ldi = 0;  // round_up(H, 16), round_up(I, 16)
  int own_rank = 0, own_world = 1;  // expert parallelism: experts e % own_world == own_rank
  // device tables
  float *gate_w = nullptr, *gate_b = nullptr;
  int8_t *gu_w = nullptr;          // [E+S, 2I, ldh]
  int16_t *gu_qm = nullptr;        // [E+S, 2I]
  float *gu_os = nullptr;          // [E+S, 2I]
  float *gu_s = nullptr;           // [E+S, H]
  float *gu_thr = nullptr;         // [E+S] max(in_thresh, 1e-8)
  int8_t *dn_w = nullptr;          // [E+S, H, ldi]
  int16_t *dn_qm = nullptr;        // [E+S, H]
  float *dn_os = nullptr;          // [E+S, H]
  float *dn_s = nullptr;           // [E+S, I]
  float *dn_inv = nullptr;         // [E+S] static 1/in_step
  // scratch (max_T tokens)
  int32_t *idx = nullptr;          // [T, k]
  float *w = nullptr;              // [T, k]
  int8_t *q1 = nullptr;            // [P, ldh]
  float *r1 = nullptr;             // [P]
  float *gu = nullptr;             // [P, 2I]
  float *h = nullptr;              // [P, I]
  int8_t *q2 = nullptr;            // [P, ldi]
  void *yq = nullptr;              // [P, H]
  int32_t *grp_off = nullptr;      // [E+S+1] pairs of each expert, then the grouped GEMV's work
                                   // items (T > 1)
  int32_t *grp_pairs = nullptr;    // [P]
  float *route_logits = nullptr;   // [max_T, E]
  int *route_cnt = nullptr;        // [max_T] arrival counters of the routing kernel
};

namespace {

class DeviceScope {
 public:
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

w8a8_status invalid(const char *msg) {
  set_last_error(msg);
  return W8A8_ERR_INVALID_ARG;
}

w8a8_status cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return W8A8_SUCCESS;
  char buf[256];
  std::snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  set_last_error(buf);
  return e == cudaErrorMemoryAllocation ? W8A8_ERR_NO_MEMORY : W8A8_ERR_CUDA;
}

int round16(int v) { return (v + 15) / 16 * 16; }

template <typename T>
cudaError_t upload(T **dst, const T *src, size_t count) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void **>(dst), count * sizeof(T) + 16);
  if (e != cudaSuccess) return e;
  if (src) return cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice);
  return cudaMemset(*dst, 0, count * sizeof(T));
}

// Rows of `cols` int8 values re-laid with a row stride of `ld` (zero padded).
cudaError_t upload_rows(int8_t **dst, const int8_t *src, size_t rows, int cols, int ld) {
  std::vector<int8_t> tmp(rows * ld, 0);
  for (size_t r = 0; r < rows; ++r) std::memcpy(&tmp[r * ld], src + r * cols, cols);
  return upload(dst, tmp.data(), tmp.size());
}

void moe_free(w8a8_moe *m) {
  if (!m) return;
  DeviceScope d(m->dev);
  void *ptrs[] = {m->gate_w, m->gate_b, m->gu_w, m->gu_qm, m->gu_os, m->gu_s, m->gu_thr,
                  m->dn_w,   m->dn_qm,  m->dn_os, m->dn_s, m->dn_inv, m->idx, m->w,
                  m->q1,     m->r1,     m->gu,   m->h,    m->q2,     m->yq,
                  m->grp_off, m->grp_pairs, m->route_logits, m->route_cnt};
  for (void *p : ptrs) cudaFree(p);
  delete m;
}

MoePairs pairs_of(const w8a8_moe *m, int T) {
  MoePairs P;
  P.T = T;
  P.k = m->k;
  P.slots = m->slots;
  P.n_routed = m->E;
  P.routed_idx = m->idx;
  P.routed_w = m->w;
  P.own_rank = m->own_rank;
  P.own_world = m->own_world;
  return P;
}

w8a8_status route(w8a8_moe *m, const float *hidden, int64_t ldh, int T, int32_t *idx, float *w,
                  cudaStream_t st) {
  MoeRouteLaunch L = {};
  L.hidden = hidden;
  L.ldh = ldh;
  L.gate_w = m->gate_w;
  L.bias = m->gate_b;
  L.T = T;
  L.H = m->H;
  L.E = m->E;
  L.k = m->k;
  L.norm_topk = m->norm_topk;
  L.scaling = m->scaling;
  L.logits = m->route_logits;
  L.cnt = m->route_cnt;
  L.pdl = false;
  for (int t0 = 0; t0 < T; t0 += m->max_T) {  // the scratch holds max_tokens rows
    L.hidden = hidden + static_cast<int64_t>(t0) * ldh;
    L.T = std::min(T - t0, m->max_T);
    L.idx = idx + static_cast<int64_t>(t0) * m->k;
    L.w = w + static_cast<int64_t>(t0) * m->k;
    const w8a8_status s = cuda_status(launch_moe_route(L, st), "moe route");
    if (s != W8A8_SUCCESS) return s;
  }
  return W8A8_SUCCESS;
}

}  // namespace

extern "C" {

w8a8_status w8a8_moe_create(w8a8_ctx *ctx, const w8a8_moe_desc *d, w8a8_moe **out) {
  if (!out) return invalid("out_moe is NULL");
  *out = nullptr;
  if (!ctx || !d) return invalid("ctx or desc is NULL");
  if (d->hidden < 1 || d->inter < 1 || d->n_routed < 1 || d->n_shared < 0 || d->top_k < 1 ||
      d->top_k > 16 || d->top_k > d->n_routed || d->max_tokens < 1)
    return invalid("bad MoE shape (hidden, inter, n_routed, n_shared, top_k, max_tokens)");
  if (round16(d->hidden) > 4096 || round16(d->inter) > 4096 || d->n_routed > 4096)
    return invalid("hidden, inter and n_routed must be at most 4096");
  if (!d->gate_w || !d->gu_weights || !d->gu_quant_m || !d->gu_out_step_chan ||
      !d->gu_inv_smooth || !d->gu_in_thresh || !d->dn_weights || !d->dn_quant_m ||
      !d->dn_out_step_chan || !d->dn_inv_smooth || !d->dn_in_step)
    return invalid("a MoE parameter array is NULL");
  if (d->gu_trunc < 0 || d->gu_trunc > 62 || d->dn_trunc < 0 || d->dn_trunc > 62)
    return invalid("trunc outside [0, 62]");
  if (d->dn_out_dtype != W8A8_DTYPE_INT8 && d->dn_out_dtype != W8A8_DTYPE_INT16)
    return invalid("dn_out_dtype must be INT8 or INT16");
  w8a8_moe *m = new (std::nothrow) w8a8_moe();
  if (!m) return W8A8_ERR_NO_MEMORY;
  m->ctx = ctx;
  m->dev = w8a8_ctx_device(ctx);
  m->H = d->hidden;
  m->I = d->inter;
  m->E = d->n_routed;
  m->S = d->n_shared;
  m->k = d->top_k;
  m->slots = d->top_k + d->n_shared;
  m->max_T = d->max_tokens;
  m->norm_topk = d->norm_topk_prob;
  m->scaling = d->routed_scaling;
  m->gu_trunc = d->gu_trunc;
  m->dn_trunc = d->dn_trunc;
  m->dn_i16 = d->dn_out_dtype == W8A8_DTYPE_INT16;
  m->ldh = round16(d->hidden);
  m->ldi = round16(d->inter);
  const size_t X = static_cast<size_t>(m->E + m->S);
  const size_t H = m->H, I = m->I;
  std::vector<float> thr(X), inv(X);
  for (size_t e = 0; e < X; ++e) {
    thr[e] = d->gu_in_thresh[e] > 1e-8f ? d->gu_in_thresh[e] : 1e-8f;
    inv[e] = d->dn_in_step[e] > 1e-12f ? 1.0f / d->dn_in_step[e] : 0.0f;
  }
  const size_t P = static_cast<size_t>(m->max_T) * m->slots;
  DeviceScope ds(m->dev);
  cudaError_t e = upload(&m->gate_w, d->gate_w, static_cast<size_t>(m->E) * H);
  if (e == cudaSuccess && d->gate_bias)
    e = upload(&m->gate_b, d->gate_bias, static_cast<size_t>(m->E));
  if (e == cudaSuccess) e = upload_rows(&m->gu_w, d->gu_weights, X * 2 * I, m->H, m->ldh);
  if (e == cudaSuccess) e = upload(&m->gu_qm, d->gu_quant_m, X * 2 * I);
  if (e == cudaSuccess) e = upload(&m->gu_os, d->gu_out_step_chan, X * 2 * I);
  if (e == cudaSuccess) e = upload(&m->gu_s, d->gu_inv_smooth, X * H);
  if (e == cudaSuccess) e = upload(&m->gu_thr, thr.data(), X);
  if (e == cudaSuccess) e = upload_rows(&m->dn_w, d->dn_weights, X * H, m->I, m->ldi);
  if (e == cudaSuccess) e = upload(&m->dn_qm, d->dn_quant_m, X * H);
  if (e == cudaSuccess) e = upload(&m->dn_os, d->dn_out_step_chan, X * H);
  if (e == cudaSuccess) e = upload(&m->dn_s, d->dn_inv_smooth, X * I);
  if (e == cudaSuccess) e = upload(&m->dn_inv, inv.data(), X);
  if (e == cudaSuccess)
    e = upload(&m->idx, static_cast<const int32_t *>(nullptr), static_cast<size_t>(m->max_T) * m->k);
  if (e == cudaSuccess)
    e = upload(&m->w, static_cast<const float *>(nullptr), static_cast<size_t>(m->max_T) * m->k);
  if (e == cudaSuccess) e = upload(&m->q1, static_cast<const int8_t *>(nullptr), P * m->ldh);
  if (e == cudaSuccess) e = upload(&m->r1, static_cast<const float *>(nullptr), P);
  if (e == cudaSuccess) e = upload(&m->gu, static_cast<const float *>(nullptr), P * 2 * I);
  if (e == cudaSuccess) e = upload(&m->h, static_cast<const float *>(nullptr), P * I);
  if (e == cudaSuccess) e = upload(&m->q2, static_cast<const int8_t *>(nullptr), P * m->ldi);
  if (e == cudaSuccess) e = cudaMalloc(&m->yq, P * H * (m->dn_i16 ? 2 : 1));
  if (e == cudaSuccess)
    e = upload(&m->grp_off, static_cast<const int32_t *>(nullptr),
               X + 2 + static_cast<size_t>(moe_max_group_items(static_cast<int>(X), static_cast<int>(P))));
  if (e == cudaSuccess) e = upload(&m->grp_pairs, static_cast<const int32_t *>(nullptr), P);
  if (e == cudaSuccess)
    e = upload(&m->route_logits, static_cast<const float *>(nullptr),
               static_cast<size_t>(m->max_T) * m->E);
  if (e == cudaSuccess)
    e = upload(&m->route_cnt, static_cast<const int *>(nullptr), static_cast<size_t>(m->max_T));
  if (e != cudaSuccess) {
    w8a8_status st = cuda_status(e, "MoE upload");
    moe_free(m);
    return st;
  }
  *out = m;
  return W8A8_SUCCESS;
}

void w8a8_moe_destroy(w8a8_moe *m) { moe_free(m); }

w8a8_status w8a8_moe_route(w8a8_moe *m, const float *hidden, int64_t ldh, int32_t T,
                           int32_t *idx, float *w, void *stream) {
  if (!m || !hidden || !idx || !w) return invalid("moe, hidden, idx or w is NULL");
  if (T < 1 || ldh < m->H) return invalid("T < 1 or ldh < hidden");
  DeviceScope d(m->dev);
  return route(m, hidden, ldh, T, idx, w, static_cast<cudaStream_t>(stream));
}

w8a8_status w8a8_moe_forward(w8a8_moe *m, const float *hidden, int64_t ldh, int32_t T,
                             float *out, int64_t ldo, void *stream) {
  if (!m || !hidden || !out) return invalid("moe, hidden or out is NULL");
  if (T < 1 || T > m->max_T) return invalid("T outside [1, max_tokens]");
  if (ldh < m->H || ldo < m->H) return invalid("ldh or ldo below hidden");
  DeviceScope d(m->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  w8a8_status s = route(m, hidden, ldh, T, m->idx, m->w, st);
  if (s != W8A8_SUCCESS) return s;
  const MoePairs P = pairs_of(m, T);
  // T > 1: the pairs are grouped by expert so that each expert's weight rows stream once for all
  // of its pairs; T = 1 keeps one CTA column per pair (every expert has at most one pair).
  const bool grouped = T > 1;
  const int n_experts = m->E + m->S;
  if (grouped) {
    s = cuda_status(launch_moe_group(P, n_experts, m->grp_off, m->grp_pairs, true, st),
                    "moe expert grouping");
    if (s != W8A8_SUCCESS) return s;
  }

  MoeActLaunch A = {};
  A.pairs = P;
  A.src = hidden;
  A.ld = ldh;
  A.per_pair_rows = 0;
  A.K = m->H;
  A.inv_smooth = m->gu_s;
  A.inv_step = nullptr;
  A.safe_thresh = m->gu_thr;
  A.q = m->q1;
  A.ldq = m->ldh;
  A.ratio = m->r1;
  A.pdl = true;
  s = cuda_status(launch_moe_act_quant(A, true, st), "moe gate_up act quant");
  if (s != W8A8_SUCCESS) return s;

  MoeGemvLaunch G = {};
  G.pairs = P;
  G.q = m->q1;
  G.ldq = m->ldh;
  G.w = m->gu_w;
  G.N = 2 * m->I;
  G.k_pad = m->ldh;
  G.quant_m = m->gu_qm;
  G.trunc = m->gu_trunc;
  G.qmax = 127;
  G.out_step = m->gu_os;
  G.ratio = m->r1;
  G.out_f32 = 1;
  G.y = m->gu;
  G.pdl = true;
  G.grp_off = m->grp_off;
  G.grp_pairs = m->grp_pairs;
  G.n_experts = n_experts;
  s = cuda_status(grouped ? launch_moe_gemv_grouped(G, st) : launch_moe_gemv(G, st),
                  "moe gate_up GEMV");
  if (s != W8A8_SUCCESS) return s;

  // SwiGLU (silu(gate) * up) fused into the down projection's static pack
  MoeActLaunch B = {};
  B.pairs = P;
  B.swiglu_gu = m->gu;
  B.src_out = m->h;
  B.src = m->h;
  B.ld = m->I;
  B.per_pair_rows = 1;
  B.K = m->I;
  B.inv_smooth = m->dn_s;
  B.inv_step = m->dn_inv;
  B.safe_thresh = nullptr;
  B.q = m->q2;
  B.ldq = m->ldi;
  B.ratio = nullptr;
  B.pdl = true;
  s = cuda_status(launch_moe_act_quant(B, false, st), "moe down act quant");
  if (s != W8A8_SUCCESS) return s;

  MoeGemvLaunch D = {};
  D.pairs = P;
  D.q = m->q2;
  D.ldq = m->ldi;
  D.w = m->dn_w;
  D.N = m->H;
  D.k_pad = m->ldi;
  D.quant_m = m->dn_qm;
  D.trunc = m->dn_trunc;
  D.qmax = m->dn_i16 ? 32767 : 127;
  D.out_step = m->dn_os;
  D.ratio = nullptr;
  D.out_f32 = 0;
  D.out_i16 = m->dn_i16;
  D.y = m->yq;
  D.pdl = true;
  D.grp_off = m->grp_off;
  D.grp_pairs = m->grp_pairs;
  D.n_experts = n_experts;
  s = cuda_status(grouped ? launch_moe_gemv_grouped(D, st) : launch_moe_gemv(D, st),
                  "moe down GEMV");
  if (s != W8A8_SUCCESS) return s;

  MoeCombineLaunch C = {};
  C.pairs = P;
  C.yq = m->yq;
  C.in_i16 = m->dn_i16;
  C.H = m->H;
  C.out_step = m->dn_os;
  C.out = out;
  C.ldo = ldo;
  C.pdl = true;
  return cuda_status(launch_moe_combine(C, st), "moe combine");
}

w8a8_status w8a8_moe_views(const w8a8_moe *m, const int32_t **idx, const float **w,
                           const float **gate_up, const float **act, const void **down_q) {
  if (!m) return invalid("moe is NULL");
  if (idx) *idx = m->idx;
  if (w) *w = m->w;
  if (gate_up) *gate_up = m->gu;
  if (act) *act = m->h;
  if (down_q) *down_q = m->yq;
  return W8A8_SUCCESS;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Expert parallelism over processes (w8a8_moe_ep_*): rank r computes the experts e with
// e % world == r for every token (the hidden states are the same on every rank), combines its
// own slots in slot order into a partial [T, H], and the library exchanges the partials (peer
// stores into CUDA-IPC-mapped memory, double-buffered by the forward's parity, device counters)
// and sums them in rank order on every rank.  With world = 2 that is the reference's even / odd
// split of the selected experts over its two dies and its die-by-die sum
// (src/LFM2.5-8B-A1B/lfm2_moe.cpp:2190-2432: mlp_out of die 0, mlp_out_d1 of die 1, added after).
// A rank publishes forward f + 1's partial only after its sum of forward f saw every rank's
// forward-f partial, so a rank is at most one forward ahead of any other: two buffers suffice.
struct w8a8_moe_ep {
  w8a8_moe *moe = nullptr;
  int rank = 0, world = 1, max_T = 0;
  unsigned char *arena = nullptr;  // [0] done[64], then gather [2][world][max_T][H] fp32
  size_t off_gather = 0, bytes = 0;
  std::vector<unsigned char *> base;
  std::vector<char> opened;
  bool connected = false;
  float *partial = nullptr;        // [max_T, H]
  unsigned *local = nullptr;       // [0] forwards published, [1] publication arrivals
  float **dst = nullptr;           // [world] gather base of every rank
  unsigned **done = nullptr;       // [world] done[rank] of every rank
};

namespace {

void ep_free(w8a8_moe_ep *x) {
  if (!x) return;
  DeviceScope d(x->moe ? x->moe->dev : 0);
  for (size_t p = 0; p < x->base.size(); ++p)
    if (x->opened[p] && x->base[p]) cudaIpcCloseMemHandle(x->base[p]);
  cudaFree(x->arena);
  cudaFree(x->partial);
  cudaFree(x->local);
  cudaFree(x->dst);
  cudaFree(x->done);
  if (x->moe) {
    x->moe->own_rank = 0;
    x->moe->own_world = 1;
  }
  delete x;
}

w8a8_status ep_tables(w8a8_moe_ep *x) {
  std::vector<float *> dst(x->world);
  std::vector<unsigned *> done(x->world);
  for (int p = 0; p < x->world; ++p) {
    dst[p] = reinterpret_cast<float *>(x->base[p] + x->off_gather);
    done[p] = reinterpret_cast<unsigned *>(x->base[p]) + x->rank;
  }
  cudaError_t e = cudaMemcpy(x->dst, dst.data(), x->world * sizeof(float *), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(x->done, done.data(), x->world * sizeof(unsigned *), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return cuda_status(e, "expert-parallel pointer tables");
}

}  // namespace

extern "C" {

w8a8_status w8a8_moe_ep_create(w8a8_moe *moe, int32_t rank, int32_t world, int32_t max_T,
                               w8a8_moe_ep **out) {
  if (!out) return invalid("out_ep is NULL");
  *out = nullptr;
  if (!moe) return invalid("moe is NULL");
  if (world < 1 || world > 64 || rank < 0 || rank >= world || max_T < 1 || max_T > moe->max_T)
    return invalid("bad expert-parallel shape (rank, world <= 64, max_tokens <= the layer's)");
  w8a8_moe_ep *x = new (std::nothrow) w8a8_moe_ep();
  if (!x) return W8A8_ERR_NO_MEMORY;
  x->moe = moe;
  x->rank = rank;
  x->world = world;
  x->max_T = max_T;
  DeviceScope d(moe->dev);
  x->off_gather = 256;
  x->bytes = x->off_gather + 2ull * world * max_T * moe->H * sizeof(float);
  cudaError_t e = cudaMalloc(&x->arena, x->bytes);
  if (e == cudaSuccess) e = cudaMemset(x->arena, 0, x->bytes);
  if (e == cudaSuccess) e = cudaMalloc(&x->partial, static_cast<size_t>(max_T) * moe->H * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&x->local, 2 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(x->local, 0, 2 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMalloc(&x->dst, world * sizeof(float *));
  if (e == cudaSuccess) e = cudaMalloc(&x->done, world * sizeof(unsigned *));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    ep_free(x);
    return cuda_status(e, "expert-parallel arena");
  }
  x->base.assign(world, nullptr);
  x->opened.assign(world, 0);
  x->base[rank] = x->arena;
  moe->own_rank = rank;
  moe->own_world = world;
  *out = x;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_moe_ep_export(const w8a8_moe_ep *x, void *handle_out) {
  if (!x || !handle_out) return invalid("ep or handle_out is NULL");
  DeviceScope d(x->moe->dev);
  cudaIpcMemHandle_t h;
  w8a8_status st = cuda_status(cudaIpcGetMemHandle(&h, x->arena), "cudaIpcGetMemHandle");
  if (st != W8A8_SUCCESS) return st;
  static_assert(sizeof(h) == W8A8_MOE_EP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return W8A8_SUCCESS;
}

w8a8_status w8a8_moe_ep_connect(w8a8_moe_ep *x, const void *handles) {
  if (!x || !handles) return invalid("ep or handles is NULL");
  if (x->connected) return invalid("ep is already connected");
  DeviceScope d(x->moe->dev);
  const unsigned char *hb = static_cast<const unsigned char *>(handles);
  for (int p = 0; p < x->world; ++p) {
    if (p == x->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + static_cast<size_t>(p) * W8A8_MOE_EP_HANDLE_BYTES, sizeof(h));
    void *ptr = nullptr;
    w8a8_status st = cuda_status(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess),
                                 "cudaIpcOpenMemHandle");
    if (st != W8A8_SUCCESS) return st;
    x->base[p] = static_cast<unsigned char *>(ptr);
    x->opened[p] = 1;
  }
  w8a8_status st = ep_tables(x);
  if (st == W8A8_SUCCESS) x->connected = true;
  return st;
}

w8a8_status w8a8_moe_ep_connect_local(w8a8_moe_ep *const *eps, int32_t world) {
  if (!eps || world < 1) return invalid("eps is NULL or world < 1");
  for (int p = 0; p < world; ++p)
    if (!eps[p] || eps[p]->world != world || eps[p]->rank != p || eps[p]->connected)
      return invalid("eps[p] must be rank p of the same world and not yet connected");
  for (int r = 0; r < world; ++r) {
    for (int p = 0; p < world; ++p) {
      const int dr = eps[r]->moe->dev, dp = eps[p]->moe->dev;
      if (dr != dp) {
        int can = 0;
        cudaDeviceCanAccessPeer(&can, dr, dp);
        if (!can) {
          set_last_error("no peer access between the ranks' devices");
          return W8A8_ERR_NOT_SUPPORTED;
        }
        DeviceScope d(dr);
        const cudaError_t e = cudaDeviceEnablePeerAccess(dp, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
        else if (e != cudaSuccess) return cuda_status(e, "cudaDeviceEnablePeerAccess");
      }
      eps[r]->base[p] = eps[p]->arena;
    }
  }
  for (int r = 0; r < world; ++r) {
    DeviceScope d(eps[r]->moe->dev);
    w8a8_status st = ep_tables(eps[r]);
    if (st != W8A8_SUCCESS) return st;
    eps[r]->connected = true;
  }
  return W8A8_SUCCESS;
}

w8a8_status w8a8_moe_ep_forward(w8a8_moe_ep *x, const float *hidden, int64_t ldh, int32_t T,
                                float *out, int64_t ldo, void *stream) {
  if (!x || !hidden || !out) return invalid("ep, hidden or out is NULL");
  if (!x->connected) return invalid("ep is not connected (w8a8_moe_ep_connect)");
  if (T < 1 || T > x->max_T) return invalid("T outside [1, max_tokens]");
  if (ldo < x->moe->H) return invalid("ldo below hidden");
  // this rank's experts and its partial combine
  w8a8_status s = w8a8_moe_forward(x->moe, hidden, ldh, T, x->partial, x->moe->H, stream);
  if (s != W8A8_SUCCESS) return s;
  DeviceScope d(x->moe->dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MoeEpLaunch L = {};
  L.partial = x->partial;
  L.dst = x->dst;
  L.done = x->done;
  L.rank = x->rank;
  L.world = x->world;
  L.T = T;
  L.H = x->moe->H;
  L.max_T = x->max_T;
  L.pub_seq = x->local;
  L.pub_arrive = x->local + 1;
  L.gather = reinterpret_cast<const float *>(x->arena + x->off_gather);
  L.done_here = reinterpret_cast<const unsigned *>(x->arena);
  L.out = out;
  L.ldo = ldo;
  L.err = w8a8::ctx_error_word(x->moe->ctx);
  L.pdl = true;
  s = cuda_status(launch_moe_ep_publish(L, st), "expert-parallel publication");
  if (s != W8A8_SUCCESS) return s;
  return cuda_status(launch_moe_ep_sum(L, st), "expert-parallel sum");
}

void w8a8_moe_ep_destroy(w8a8_moe_ep *x) { ep_free(x); }

}  // extern "C"

