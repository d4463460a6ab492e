// C ABI w8a8_lmhead_*: the vocab-sharded LM head over several devices of one process.
//
// Replaces the dual-die LM head of the reference (TransformerSession::forward_lm_head_dual_die,
// src/eswin_runtime/src/llm/transformer_session.cpp:538-614, and run_dual_die,
// src/LFM3/lfm3_v2.cpp:1311-1332, which runs one host thread per die and concatenates the two
// halves of the logits before Sampler::sample scans the full vocabulary).  Here every shard
// keeps only its top-k (logit, vocab id) pairs on chip and device 0 merges the n lists.
//
// Device 0 drives a forward; shards on other devices ("remote" shards) synchronise with it
// through counters in device memory instead of cross-device stream events:
//   * the remote shards' GEMVs are launched first, each on its own stream of its own device; a
//     remote GEMV streams its first weight stages at once (weights do not depend on h) and its
//     producer waits (bounded) until its x_ready counter reaches the forward's number;
//   * device 0 quantises h once (static in_step, the broadcast of fused_emb_norm_broadcast_t1,
//     lfm3_v2.cpp:810-831) and stores the int8 rows into every shard's staging buffer over
//     NVLink, then bumps every x_ready counter (system-scope release);
//   * each remote shard's last CTA stores its sorted top-k into device 0's gather buffer (peer
//     stores), then bumps its done counter on device 0;
//   * device 0 runs its own shard(s), then the merge kernel, which waits (bounded) for every
//     done counter before merging.
// A forward is therefore a handful of asynchronous launches with no host or cross-device
// stream dependency; the shards on device 0 follow the caller's stream.  Shards that share
// device 0 need no counters (stream order), and a head whose shards all live on device 0 can be
// captured in a CUDA graph; one with remote shards cannot (the remote launches are outside the
// captured stream), and forwards of one head must be issued on one stream, one at a time.
#include "../../include/w8a8.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "kernels.h"
#include "linear_internal.h"

struct w8a8_lmhead {
  int n = 0, K = 0, V = 0, max_T = 0, k_max = 0;
  float in_step = 0.0f;
  std::vector<w8a8_ctx *> ctxs;
  std::vector<int> dev;                 // device of each shard
  std::vector<int> lo;                  // first vocab id of each shard
  std::vector<w8a8_linear *> shards;
  std::vector<char> remote;             // shard on another device than shard 0
  std::vector<cudaStream_t> streams;    // per shard (remote shards only; else null)
  std::vector<unsigned *> counters;     // per shard s >= 1, on its device: [0] seq, [1] x_ready
  uint64_t remote_mask = 0;
  // device 0
  unsigned *ctr0 = nullptr;             // [0] forwards published, [1] arrival, [2 + s] done[s]
  w8a8::PublishPeer *peers = nullptr;   // [n - 1]: shards 1..n-1 staging buffers and x_ready
  float *cand_val = nullptr;            // [n][max_T * k_max]
  int32_t *cand_idx = nullptr;
  unsigned long long *trace = nullptr;  // optional diagnostics timeline (device 0)
  const float *emb_norm = nullptr;      // optional input RMSNorm (device 0), see set_input_norm
  float eps = 0.0f;
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

w8a8_status cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return W8A8_SUCCESS;
  char buf[256];
  std::snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  w8a8::set_last_error(buf);
  return W8A8_ERR_CUDA;
}

w8a8_status invalid(const char *msg) {
  w8a8::set_last_error(msg);
  return W8A8_ERR_INVALID_ARG;
}

void lmhead_free(w8a8_lmhead *lm) {
  if (!lm) return;
  for (w8a8_linear *l : lm->shards) w8a8_linear_destroy(l);
  for (size_t s = 0; s < lm->streams.size(); ++s) {
    if (!lm->streams[s]) continue;
    DeviceScope d(lm->dev[s]);
    cudaStreamDestroy(lm->streams[s]);
  }
  for (size_t s = 0; s < lm->counters.size(); ++s) {
    if (!lm->counters[s]) continue;
    DeviceScope d(lm->dev[s]);
    cudaFree(lm->counters[s]);
  }
  if (!lm->dev.empty()) {
    DeviceScope d(lm->dev[0]);
    cudaFree(lm->ctr0);
    cudaFree(lm->peers);
    cudaFree(lm->cand_val);
    cudaFree(lm->cand_idx);
  }
  delete lm;
}

// Peer access from device `from` to device `to` (idempotent).
w8a8_status enable_peer(int from, int to) {
  int can = 0;
  cudaDeviceCanAccessPeer(&can, from, to);
  if (!can) {
    w8a8::set_last_error("a shard device has no peer access to the first device");
    return W8A8_ERR_NOT_SUPPORTED;
  }
  DeviceScope d(from);
  const cudaError_t e = cudaDeviceEnablePeerAccess(to, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return W8A8_SUCCESS;
  }
  return cuda_status(e, "cudaDeviceEnablePeerAccess");
}

}  // namespace

extern "C" {

w8a8_status w8a8_lmhead_create(w8a8_ctx *const *ctxs, int32_t n, int32_t K, int32_t V,
                               const int8_t *weights, int64_t ld, const float *acc_step,
                               float in_step, int32_t max_T, int32_t k_max, w8a8_lmhead **out) {
  if (!out) return invalid("out_lmhead is NULL");
  *out = nullptr;
  if (!ctxs || !weights || !acc_step) return invalid("ctxs, weights or acc_step is NULL");
  if (n < 1 || n > 64 || K < 1 || V < n || ld < K || max_T < 1 || k_max < 1 ||
      k_max > W8A8_TOPK_MAX || k_max > V / n)
    return invalid("bad LM-head shape (n_shards, K, V, weights_ld, max_tokens or k_max)");
  for (int s = 0; s < n; ++s)
    if (!ctxs[s]) return invalid("ctxs[s] is NULL");
  w8a8_lmhead *lm = new (std::nothrow) w8a8_lmhead();
  if (!lm) return W8A8_ERR_NO_MEMORY;
  lm->n = n;
  lm->K = K;
  lm->V = V;
  lm->max_T = max_T;
  lm->k_max = k_max;
  lm->in_step = in_step;
  lm->ctxs.assign(ctxs, ctxs + n);
  for (int s = 0; s < n; ++s) lm->dev.push_back(w8a8_ctx_device(ctxs[s]));
  const int dev0 = lm->dev[0];
  for (int s = 0; s < n; ++s) {
    const bool r = lm->dev[s] != dev0;
    lm->remote.push_back(r ? 1 : 0);
    if (r) lm->remote_mask |= 1ull << s;
  }
  if (lm->remote_mask && max_T > 8) {
    lmhead_free(lm);
    return invalid("shards on other devices take at most 8 tokens a forward (max_tokens <= 8)");
  }

  // Shard linears: rows [lo, hi) with their acc_step slice; static input quantisation with
  // in_step (in_thresh = 127 * in_step keeps the descriptor consistent).
  for (int s = 0; s < n; ++s) {
    const int lo = static_cast<int>((static_cast<int64_t>(s) * V) / n);
    const int hi = static_cast<int>((static_cast<int64_t>(s + 1) * V) / n);
    lm->lo.push_back(lo);
    w8a8_linear_desc d;
    std::memset(&d, 0, sizeof(d));
    d.K = K;
    d.N = hi - lo;
    d.weights = weights + static_cast<int64_t>(lo) * ld;
    d.weights_ld = ld;
    d.quant_m = nullptr;
    d.trunc = 0;
    d.acc_step = acc_step + lo;
    d.scale.out_dtype = W8A8_DTYPE_INT8;
    d.scale.in_step = in_step;
    d.scale.in_thresh = in_step * 127.0f;
    d.scale.out_step = 1.0f;
    w8a8_linear *l = nullptr;
    w8a8_status st = w8a8_linear_create(ctxs[s], &d, &l);
    if (st == W8A8_SUCCESS) {
      lm->shards.push_back(l);
      // the staging buffers are written by device 0 and must not move afterwards
      st = w8a8::linear_reserve_tokens(l, max_T);
    }
    if (st != W8A8_SUCCESS) {
      lmhead_free(lm);
      return st;
    }
  }
  // Peer access both ways between device 0 and every remote shard's device: device 0 stores
  // activations and counters there, the shard stores candidates and its counter on device 0.
  for (int s = 1; s < n; ++s) {
    if (!lm->remote[s]) continue;
    w8a8_status st = enable_peer(lm->dev[s], dev0);
    if (st == W8A8_SUCCESS) st = enable_peer(dev0, lm->dev[s]);
    if (st != W8A8_SUCCESS) {
      lmhead_free(lm);
      return st;
    }
  }
  lm->streams.assign(n, nullptr);
  lm->counters.assign(n, nullptr);
  std::vector<w8a8::PublishPeer> table;
  for (int s = 1; s < n; ++s) {
    DeviceScope d(lm->dev[s]);
    cudaError_t e = cudaMalloc(&lm->counters[s], 2 * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(lm->counters[s], 0, 2 * sizeof(unsigned));
    if (e == cudaSuccess && lm->remote[s])
      e = cudaStreamCreateWithFlags(&lm->streams[s], cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      lmhead_free(lm);
      return cuda_status(e, "shard counters / stream");
    }
    table.push_back({w8a8::linear_staging(lm->shards[s]), lm->counters[s] + 1});
  }
  {
    DeviceScope d(dev0);
    const size_t cells = static_cast<size_t>(n) * max_T * k_max;
    cudaError_t e = cudaMalloc(&lm->cand_val, cells * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&lm->cand_idx, cells * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&lm->ctr0, (2 + n) * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(lm->ctr0, 0, (2 + n) * sizeof(unsigned));
    if (e == cudaSuccess && !table.empty()) {
      e = cudaMalloc(&lm->peers, table.size() * sizeof(w8a8::PublishPeer));
      if (e == cudaSuccess)
        e = cudaMemcpy(lm->peers, table.data(), table.size() * sizeof(w8a8::PublishPeer),
                       cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      lmhead_free(lm);
      return cuda_status(e, "LM-head gather buffers / counters");
    }
  }
  *out = lm;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_lmhead_forward(w8a8_lmhead *lm, const float *h, int32_t T, int32_t k,
                                float *val, int32_t *idx, int32_t *argmax, void *stream) {
  if (!lm || !h || !val || !idx) return invalid("lmhead, h, val or idx is NULL");
  if (T < 1 || T > lm->max_T || k < 1 || k > lm->k_max)
    return invalid("T or k outside [1, max_tokens] / [1, k_max]");
  cudaStream_t s0 = static_cast<cudaStream_t>(stream);
  const int n = lm->n;
  const int dev0 = lm->dev[0];
  if (lm->remote_mask) {
    DeviceScope d(dev0);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    w8a8_status st = cuda_status(cudaStreamIsCapturing(s0, &cs), "cudaStreamIsCapturing");
    if (st != W8A8_SUCCESS) return st;
    if (cs != cudaStreamCaptureStatusNone) {
      w8a8::set_last_error("an LM head with shards on other devices cannot be graph-captured");
      return W8A8_ERR_NOT_SUPPORTED;
    }
  }
  // Shard s writes its [T, k] block at cand + s * T * k: the merge reads candidate (t, s, j)
  // at t * k + s * (T * k) + j.
  const int64_t block = static_cast<int64_t>(T) * k;
  // 1. remote shards: launched first, they stream weights while waiting for the activations
  for (int s = 1; s < n; ++s) {
    if (!lm->remote[s]) continue;
    DeviceScope d(lm->dev[s]);
    w8a8::ShardSync sync = {};
    sync.seq = lm->counters[s];
    sync.x_ready = lm->counters[s] + 1;
    sync.done = lm->ctr0 + 2 + s;
    w8a8_status st = w8a8::linear_topk_quantized(
        lm->shards[s], T, W8A8_ACT_STATIC, W8A8_OUT_F32_ACC, k, lm->lo[s], lm->cand_val + s * block,
        lm->cand_idx + s * block, nullptr, 0, sync, false, lm->streams[s]);
    if (st != W8A8_SUCCESS) return st;
  }
  // 2. device 0: quantise h into every shard's staging buffer, then its own shards, then merge.
  // Shard 0's GEMV quantises h in its prologue and its last CTA publishes the rows (one launch);
  // when the rows do not fit that, a quantisation kernel publishes them first.
  DeviceScope d(dev0);
  w8a8::FusedQuant fq;
  const bool fused =
      !lm->emb_norm && w8a8::linear_can_fuse(lm->shards[0], T, W8A8_ACT_STATIC, &fq);
  w8a8_status st = W8A8_SUCCESS;
  if (fused) {
    fq.x = h;
    fq.ldx = lm->K;
    fq.peers = lm->peers;
    fq.n_peers = n - 1;
    fq.pub_seq = n > 1 ? lm->ctr0 : nullptr;
    fq.trace = lm->trace;
  } else {
    st = w8a8::linear_quant_input(lm->shards[0], h, lm->K, T, W8A8_ACT_STATIC, lm->peers, n - 1,
                                  lm->ctr0, lm->ctr0 + 1, s0, lm->trace, nullptr, 0,
                                  lm->emb_norm, lm->eps);
    if (st != W8A8_SUCCESS) return st;
  }
  for (int s = 0; s < n; ++s) {
    if (lm->remote[s]) continue;
    st = w8a8::linear_topk_quantized(lm->shards[s], T, W8A8_ACT_STATIC, W8A8_OUT_F32_ACC, k,
                                     lm->lo[s], lm->cand_val + s * block, lm->cand_idx + s * block,
                                     nullptr, 0, w8a8::ShardSync{}, true, s0,
                                     s == 0 && fused ? &fq : nullptr);
    if (st != W8A8_SUCCESS) return st;
  }
  w8a8::MergeLaunch L = {};
  L.in_val = lm->cand_val;
  L.in_idx = lm->cand_idx;
  L.T = T;
  L.n_lists = n;
  L.k_in = k;
  L.k_out = k;
  L.list_stride = block;
  L.token_stride = k;
  L.out_val = val;
  L.out_idx = idx;
  L.argmax = argmax;
  L.pdl = true;
  if (lm->remote_mask) {
    L.done = lm->ctr0 + 2;
    L.remote_mask = lm->remote_mask;
    L.pub_seq = lm->ctr0;
    L.err = w8a8::linear_error_word(lm->shards[0]);
  }
  L.trace = lm->trace;
  return cuda_status(w8a8::launch_topk_merge(L, s0), "LM-head merge launch");
}

w8a8_status w8a8_lmhead_set_input_norm(w8a8_lmhead *lm, const float *emb_norm_scaled, float eps) {
  if (!lm) return invalid("lmhead is NULL");
  if (emb_norm_scaled && lm->K > 12288) return invalid("input norm needs K <= 12288");
  lm->emb_norm = emb_norm_scaled;
  lm->eps = eps;
  return W8A8_SUCCESS;
}

void w8a8_lmhead_destroy(w8a8_lmhead *lm) { lmhead_free(lm); }

int32_t w8a8_lmhead_shards(const w8a8_lmhead *lm) { return lm ? lm->n : 0; }

w8a8_status w8a8_lmhead_set_trace(w8a8_lmhead *lm, unsigned long long *head_trace,
                                  unsigned long long *const *shard_traces) {
  if (!lm) return invalid("lmhead is NULL");
  lm->trace = head_trace;
  for (int s = 0; s < lm->n; ++s) {
    w8a8_status st = w8a8_linear_set_trace(lm->shards[s], shard_traces ? shard_traces[s] : nullptr);
    if (st != W8A8_SUCCESS) return st;
  }
  return W8A8_SUCCESS;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// One rank of a vocab-sharded LM head over processes (w8a8_lmhead_rank_*): one process per GPU,
// the exchange done by this library with peer stores into CUDA-IPC-mapped device memory and
// counters in device memory, so a rank's whole forward is three (with two or more tokens in all,
// four) stream-ordered launches that a CUDA graph can hold (no NCCL call, no host round trip, no
// cross-process stream event).
//
// Every rank exports one arena of its device memory:
//   x_ready[64]  counters: x_ready[p] = forwards whose int8 rows rank p stored here
//   done[64]     counters: done[s] = forwards whose candidates shard s stored here
//   staging      int8 [world * max_T][k_pad]: rank p's rows of a T-token forward at p * T
//   gather       fp32 / int32 [world lists][max_T][k_max]: list s = shard s's candidates for
//                this rank's tokens
// A forward of rank r (T tokens of its own, the same T on every rank):
//   1. the activation quantisation (static in_step, as the reference's broadcast of the final
//      hidden state to both dies, lfm3_v2.cpp:810-831) stores r's rows into every rank's staging
//      at rows [r * T, (r + 1) * T) and then bumps x_ready[r] on every rank (system-scope fence +
//      relaxed stores);
//   2. r's shard GEMV streams its weights at once, waits (bounded) until every x_ready has
//      reached the forward's number, runs the fused top-k over all world * T tokens, and its last
//      CTA stores token t's candidates into the gather buffer of t's owner (list r), then bumps
//      done[r] there;
//   3. the merge waits (bounded) for every other shard's done counter and merges the world lists
//      of r's own tokens (value desc, id asc).
// Hazards across forwards need no extra wait: a rank re-publishes rows only after its merge saw
// every shard finish (so every shard's GEMV has read the staging), and a shard stores candidates
// of the next forward only after every rank published that forward's rows (so every merge of
// the previous one has run).  Counters only grow; every rank must run the same forwards.
struct w8a8_lmhead_rank {
  w8a8_ctx *ctx = nullptr;
  int rank = 0, world = 1, K = 0, V = 0, max_T = 0, k_max = 0, k_pad = 0, lo = 0, hi = 0;
  float in_step = 0.0f;
  w8a8_linear *shard = nullptr;
  unsigned char *arena = nullptr;
  size_t off_staging = 0, off_val = 0, off_idx = 0, arena_bytes = 0;
  std::vector<unsigned char *> base;   // every rank's arena as seen from this process
  std::vector<char> opened;            // base[p] came from cudaIpcOpenMemHandle
  bool connected = false;
  unsigned *local = nullptr;           // [0] forwards published, [1] publication arrival, [2] shard seq
  w8a8::PublishPeer *peers = nullptr;  // [world] staging + x_ready[rank] of every rank
  float **val_dst = nullptr;           // [world] list `rank` of every rank's gather
  int32_t **idx_dst = nullptr;
  unsigned **done_dst = nullptr;       // [world] done[rank] of every rank
  const float *emb_norm = nullptr;     // optional input RMSNorm, see set_input_norm
  float eps = 0.0f;
};

namespace {

constexpr int kRankMax = 64;
constexpr size_t kCounterBytes = 2 * kRankMax * sizeof(unsigned);

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

void rank_free(w8a8_lmhead_rank *x) {
  if (!x) return;
  DeviceScope d(w8a8_ctx_device(x->ctx));
  for (size_t p = 0; p < x->base.size(); ++p)
    if (x->opened[p] && x->base[p]) cudaIpcCloseMemHandle(x->base[p]);
  w8a8_linear_destroy(x->shard);
  cudaFree(x->arena);
  cudaFree(x->local);
  cudaFree(x->peers);
  cudaFree(x->val_dst);
  cudaFree(x->idx_dst);
  cudaFree(x->done_dst);
  delete x;
}

// Device pointer tables of every rank's arena (base[p] for every p filled in).
w8a8_status rank_tables(w8a8_lmhead_rank *x) {
  const int W = x->world;
  std::vector<w8a8::PublishPeer> peers(W);
  std::vector<float *> val(W);
  std::vector<int32_t *> idx(W);
  std::vector<unsigned *> done(W);
  const size_t list = static_cast<size_t>(x->rank) * x->max_T * x->k_max;
  for (int p = 0; p < W; ++p) {
    unsigned char *b = x->base[p];
    unsigned *ctr = reinterpret_cast<unsigned *>(b);
    peers[p].q = reinterpret_cast<int8_t *>(b + x->off_staging);
    peers[p].flag = ctr + x->rank;                      // x_ready[rank] on rank p
    done[p] = ctr + kRankMax + x->rank;                 // done[rank] on rank p
    val[p] = reinterpret_cast<float *>(b + x->off_val) + list;
    idx[p] = reinterpret_cast<int32_t *>(b + x->off_idx) + list;
  }
  cudaError_t e = cudaMemcpy(x->peers, peers.data(), W * sizeof(peers[0]), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(x->val_dst, val.data(), W * sizeof(float *), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(x->idx_dst, idx.data(), W * sizeof(int32_t *), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(x->done_dst, done.data(), W * sizeof(unsigned *), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return cuda_status(e, "LM-head rank pointer tables");
}

}  // namespace

extern "C" {

w8a8_status w8a8_lmhead_rank_create(w8a8_ctx *ctx, int32_t rank, int32_t world, int32_t K,
                                    int32_t V, const int8_t *shard_weights, int64_t ld,
                                    const float *shard_acc_step, float in_step, int32_t max_T,
                                    int32_t k_max, w8a8_lmhead_rank **out) {
  if (!out) return invalid("out_rank is NULL");
  *out = nullptr;
  if (!ctx || !shard_weights || !shard_acc_step)
    return invalid("ctx, shard_weights or shard_acc_step is NULL");
  if (world < 1 || world > kRankMax || rank < 0 || rank >= world || K < 1 || V < world ||
      ld < K || max_T < 1 || world * max_T > 64 || k_max < 1 || k_max > W8A8_TOPK_MAX ||
      k_max > V / world)
    return invalid("bad LM-head rank shape (rank, world <= 64, K, V, ld, max_tokens with "
                   "world * max_tokens <= 64, or k_max)");
  w8a8_lmhead_rank *x = new (std::nothrow) w8a8_lmhead_rank();
  if (!x) return W8A8_ERR_NO_MEMORY;
  x->ctx = ctx;
  x->rank = rank;
  x->world = world;
  x->K = K;
  x->V = V;
  x->max_T = max_T;
  x->k_max = k_max;
  x->in_step = in_step;
  x->k_pad = (K + 15) / 16 * 16;
  x->lo = static_cast<int>((static_cast<int64_t>(rank) * V) / world);
  x->hi = static_cast<int>((static_cast<int64_t>(rank + 1) * V) / world);
  w8a8_linear_desc d;
  std::memset(&d, 0, sizeof(d));
  d.K = K;
  d.N = x->hi - x->lo;
  d.weights = shard_weights;
  d.weights_ld = ld;
  d.acc_step = shard_acc_step;
  d.scale.out_dtype = W8A8_DTYPE_INT8;
  d.scale.in_step = in_step;
  d.scale.in_thresh = in_step * 127.0f;
  d.scale.out_step = 1.0f;
  w8a8_status st = w8a8_linear_create(ctx, &d, &x->shard);
  if (st != W8A8_SUCCESS) {
    rank_free(x);
    return st;
  }
  DeviceScope ds(w8a8_ctx_device(ctx));
  x->off_staging = align256(kCounterBytes);
  x->off_val = x->off_staging + align256(static_cast<size_t>(world) * max_T * x->k_pad);
  const size_t cells = static_cast<size_t>(world) * max_T * k_max;
  x->off_idx = x->off_val + align256(cells * sizeof(float));
  x->arena_bytes = x->off_idx + align256(cells * sizeof(int32_t));
  cudaError_t e = cudaMalloc(&x->arena, x->arena_bytes);
  if (e == cudaSuccess) e = cudaMemset(x->arena, 0, x->arena_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&x->local, 4 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(x->local, 0, 4 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMalloc(&x->peers, world * sizeof(w8a8::PublishPeer));
  if (e == cudaSuccess) e = cudaMalloc(&x->val_dst, world * sizeof(float *));
  if (e == cudaSuccess) e = cudaMalloc(&x->idx_dst, world * sizeof(int32_t *));
  if (e == cudaSuccess) e = cudaMalloc(&x->done_dst, world * sizeof(unsigned *));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    rank_free(x);
    return cuda_status(e, "LM-head rank arena");
  }
  x->base.assign(world, nullptr);
  x->opened.assign(world, 0);
  x->base[rank] = x->arena;
  *out = x;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_lmhead_rank_export(const w8a8_lmhead_rank *x, void *handle_out) {
  if (!x || !handle_out) return invalid("rank or handle_out is NULL");
  DeviceScope d(w8a8_ctx_device(x->ctx));
  cudaIpcMemHandle_t h;
  w8a8_status st = cuda_status(cudaIpcGetMemHandle(&h, x->arena), "cudaIpcGetMemHandle");
  if (st != W8A8_SUCCESS) return st;
  static_assert(sizeof(h) == W8A8_LMHEAD_RANK_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return W8A8_SUCCESS;
}

w8a8_status w8a8_lmhead_rank_connect(w8a8_lmhead_rank *x, const void *handles) {
  if (!x || !handles) return invalid("rank or handles is NULL");
  if (x->connected) return invalid("rank is already connected");
  DeviceScope d(w8a8_ctx_device(x->ctx));
  const unsigned char *hb = static_cast<const unsigned char *>(handles);
  for (int p = 0; p < x->world; ++p) {
    if (p == x->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + static_cast<size_t>(p) * W8A8_LMHEAD_RANK_HANDLE_BYTES, sizeof(h));
    void *ptr = nullptr;
    w8a8_status st = cuda_status(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess),
                                 "cudaIpcOpenMemHandle");
    if (st != W8A8_SUCCESS) return st;
    x->base[p] = static_cast<unsigned char *>(ptr);
    x->opened[p] = 1;
  }
  w8a8_status st = rank_tables(x);
  if (st == W8A8_SUCCESS) x->connected = true;
  return st;
}

w8a8_status w8a8_lmhead_rank_connect_local(w8a8_lmhead_rank *const *ranks, int32_t world) {
  if (!ranks || world < 1) return invalid("ranks is NULL or world < 1");
  for (int p = 0; p < world; ++p)
    if (!ranks[p] || ranks[p]->world != world || ranks[p]->rank != p || ranks[p]->connected)
      return invalid("ranks[p] must be rank p of the same world and not yet connected");
  for (int r = 0; r < world; ++r) {
    for (int p = 0; p < world; ++p) {
      const int dr = w8a8_ctx_device(ranks[r]->ctx), dp = w8a8_ctx_device(ranks[p]->ctx);
      if (dr != dp) {
        w8a8_status st = enable_peer(dr, dp);
        if (st != W8A8_SUCCESS) return st;
      }
      ranks[r]->base[p] = ranks[p]->arena;
    }
  }
  for (int r = 0; r < world; ++r) {
    DeviceScope d(w8a8_ctx_device(ranks[r]->ctx));
    w8a8_status st = rank_tables(ranks[r]);
    if (st != W8A8_SUCCESS) return st;
    ranks[r]->connected = true;
  }
  return W8A8_SUCCESS;
}

w8a8_status w8a8_lmhead_rank_forward(w8a8_lmhead_rank *x, const float *h, int32_t T, int32_t k,
                                     float *val, int32_t *idx, int32_t *argmax, void *stream) {
  if (!x || !h || !val || !idx) return invalid("rank, h, val or idx is NULL");
  if (!x->connected) return invalid("rank is not connected (w8a8_lmhead_rank_connect)");
  if (T < 1 || T > x->max_T || k < 1 || k > x->k_max)
    return invalid("T or k outside [1, max_tokens] / [1, k_max]");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceScope d(w8a8_ctx_device(x->ctx));
  const int W = x->world;
  int8_t *staging = reinterpret_cast<int8_t *>(x->arena + x->off_staging);
  unsigned *ctr = reinterpret_cast<unsigned *>(x->arena);
  // 1. this rank's rows into every rank's staging, then x_ready[rank] everywhere
  w8a8_status st = w8a8::linear_quant_input(
      x->shard, h, x->K, T, W8A8_ACT_STATIC, x->peers, W, x->local, x->local + 1, s, nullptr,
      staging + static_cast<size_t>(x->rank) * T * x->k_pad, x->rank * T, x->emb_norm, x->eps);
  if (st != W8A8_SUCCESS) return st;
  // 2. the shard's top-k over every rank's tokens, each token's list to its owner
  w8a8::ShardSync sync = {};
  sync.seq = x->local + 2;
  sync.x_ready = ctr;
  sync.n_ready = W;
  sync.done_peers = x->done_dst;
  sync.n_done = W;
  w8a8::TopkRoute route = {x->val_dst, x->idx_dst, T, 0, x->k_max};
  float *own_val = reinterpret_cast<float *>(x->arena + x->off_val);
  int32_t *own_idx = reinterpret_cast<int32_t *>(x->arena + x->off_idx);
  st = w8a8::linear_topk_quantized(x->shard, W * T, W8A8_ACT_STATIC, W8A8_OUT_F32_ACC, k, x->lo,
                                   own_val, own_idx, nullptr, 0, sync, true, s, nullptr, staging,
                                   &route);
  if (st != W8A8_SUCCESS) return st;
  // 3. merge the world lists of this rank's tokens once every other shard has stored them
  w8a8::MergeLaunch L = {};
  L.in_val = own_val;
  L.in_idx = own_idx;
  L.T = T;
  L.n_lists = W;
  L.k_in = k;
  L.k_out = k;
  L.list_stride = static_cast<int64_t>(x->max_T) * x->k_max;
  L.token_stride = x->k_max;
  L.out_val = val;
  L.out_idx = idx;
  L.argmax = argmax;
  L.pdl = true;
  uint64_t mask = 0;
  for (int p = 0; p < W; ++p)
    if (p != x->rank) mask |= 1ull << p;
  if (mask) {
    L.done = ctr + kRankMax;
    L.remote_mask = mask;
    L.pub_seq = x->local;
    L.err = w8a8::linear_error_word(x->shard);
  }
  return cuda_status(w8a8::launch_topk_merge(L, s), "LM-head rank merge launch");
}

w8a8_status w8a8_lmhead_rank_set_input_norm(w8a8_lmhead_rank *x, const float *emb_norm_scaled,
                                            float eps) {
  if (!x) return invalid("rank is NULL");
  if (emb_norm_scaled && x->K > 12288) return invalid("input norm needs K <= 12288");
  x->emb_norm = emb_norm_scaled;
  x->eps = eps;
  return W8A8_SUCCESS;
}

void w8a8_lmhead_rank_destroy(w8a8_lmhead_rank *x) { rank_free(x); }

int32_t w8a8_lmhead_rank_shard_range(const w8a8_lmhead_rank *x, int32_t *lo, int32_t *hi) {
  if (!x) return 0;
  if (lo) *lo = x->lo;
  if (hi) *hi = x->hi;
  return x->hi - x->lo;
}

}  // extern "C"
