// C ABI w8a8_moe_*: the mixture-of-experts decode layer (router, W8A8 experts, combine) over
// device-resident expert tables.  Kernels in moe.cu; semantics in include/w8a8.h.
#include "../../include/w8a8.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "kernels.h"

using namespace w8a8;

struct w8a8_moe {
  w8a8_ctx *ctx = nullptr;
  int dev = 0;
  int H = 0, I = 0, E = 0, S = 0, k = 0, slots = 0, max_T = 0;
  int norm_topk = 0;
  float scaling = 1.0f;
  int gu_trunc = 0, dn_trunc = 0, dn_i16 = 0;
  int ldh = 0, ldi = 0;  // round_up(H, 16), round_up(I, 16)
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
                  m->q1,     m->r1,     m->gu,   m->h,    m->q2,     m->yq};
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
  L.idx = idx;
  L.w = w;
  L.pdl = false;
  return cuda_status(launch_moe_route(L, st), "moe route");
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
  if (round16(d->hidden) > 4096 || round16(d->inter) > 4096)
    return invalid("hidden and inter must be at most 4096");
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
  const int n_pairs = T * m->slots;

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
  s = cuda_status(launch_moe_gemv(G, st), "moe gate_up GEMV");
  if (s != W8A8_SUCCESS) return s;

  s = cuda_status(launch_moe_swiglu(m->gu, m->I, n_pairs, m->h, true, st), "moe swiglu");
  if (s != W8A8_SUCCESS) return s;

  MoeActLaunch B = {};
  B.pairs = P;
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
  s = cuda_status(launch_moe_gemv(D, st), "moe down GEMV");
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
