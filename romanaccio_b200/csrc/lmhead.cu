// C ABI w8a8_lmhead_*: the vocab-sharded LM head over several devices of one process.
//
// Replaces the dual-die LM head of the reference (TransformerSession::forward_lm_head_dual_die,
// src/eswin_runtime/src/llm/transformer_session.cpp:538-614, and run_dual_die,
// src/LFM3/lfm3_v2.cpp:1311-1332, which runs one host thread per die and concatenates the two
// halves of the logits before Sampler::sample scans the full vocabulary).  Here every shard
// keeps only its top-k (logit, vocab id) pairs on chip, stores them into a gather buffer on the
// first device with peer stores over NVLink, and one merge kernel on that device produces the
// global top-k and argmax.  The host issues everything asynchronously: the shards' streams are
// forked from and joined back to the caller's stream with events, so a whole forward is a DAG
// that a CUDA graph can capture.
#include "../../include/w8a8.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "kernels.h"

struct w8a8_lmhead {
  int n = 0, K = 0, V = 0, max_T = 0, k_max = 0;
  float in_step = 0.0f;
  std::vector<w8a8_ctx *> ctxs;
  std::vector<int> dev;                 // device of each shard
  std::vector<int> lo;                  // first vocab id of each shard
  std::vector<w8a8_linear *> shards;
  std::vector<cudaStream_t> streams;    // shards 1..n-1 (shard 0 runs on the caller's stream)
  std::vector<cudaEvent_t> done;        // shards 1..n-1
  cudaEvent_t h_ready = nullptr;        // on device 0
  float *cand_val = nullptr;            // device 0: [n][max_T * k_max]
  int32_t *cand_idx = nullptr;
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
  for (size_t i = 0; i < lm->streams.size(); ++i) {
    if (lm->streams[i]) {
      DeviceScope d(lm->dev[i + 1]);
      cudaStreamDestroy(lm->streams[i]);
      if (lm->done[i]) cudaEventDestroy(lm->done[i]);
    }
  }
  if (!lm->dev.empty()) {
    DeviceScope d(lm->dev[0]);
    if (lm->h_ready) cudaEventDestroy(lm->h_ready);
    cudaFree(lm->cand_val);
    cudaFree(lm->cand_idx);
  }
  delete lm;
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
    if (st != W8A8_SUCCESS) {
      lmhead_free(lm);
      return st;
    }
    lm->shards.push_back(l);
  }
  // Peer access from every other device to device 0 (activations read, candidates stored).
  for (int s = 1; s < n; ++s) {
    if (lm->dev[s] == dev0) continue;
    int can = 0;
    cudaDeviceCanAccessPeer(&can, lm->dev[s], dev0);
    if (!can) {
      lmhead_free(lm);
      w8a8::set_last_error("a shard device has no peer access to the first device");
      return W8A8_ERR_NOT_SUPPORTED;
    }
    DeviceScope d(lm->dev[s]);
    cudaError_t e = cudaDeviceEnablePeerAccess(dev0, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();
    } else if (e != cudaSuccess) {
      lmhead_free(lm);
      return cuda_status(e, "cudaDeviceEnablePeerAccess");
    }
  }
  for (int s = 1; s < n; ++s) {
    DeviceScope d(lm->dev[s]);
    cudaStream_t st = nullptr;
    cudaEvent_t ev = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    lm->streams.push_back(st);
    lm->done.push_back(ev);
    if (e != cudaSuccess) {
      lmhead_free(lm);
      return cuda_status(e, "shard stream / event");
    }
  }
  {
    DeviceScope d(dev0);
    cudaError_t e = cudaEventCreateWithFlags(&lm->h_ready, cudaEventDisableTiming);
    const size_t cells = static_cast<size_t>(n) * max_T * k_max;
    if (e == cudaSuccess) e = cudaMalloc(&lm->cand_val, cells * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&lm->cand_idx, cells * sizeof(int32_t));
    if (e != cudaSuccess) {
      lmhead_free(lm);
      return cuda_status(e, "LM-head gather buffers");
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
  // Shard s writes its [T, k] block at cand + s * T * k: the merge reads candidate (t, s, j)
  // at t * k + s * (T * k) + j.
  const int64_t block = static_cast<int64_t>(T) * k;
  if (n > 1) {
    DeviceScope d(lm->dev[0]);
    w8a8_status st = cuda_status(cudaEventRecord(lm->h_ready, s0), "cudaEventRecord");
    if (st != W8A8_SUCCESS) return st;
  }
  for (int s = 1; s < n; ++s) {
    DeviceScope d(lm->dev[s]);
    cudaStream_t ss = lm->streams[s - 1];
    w8a8_status st = cuda_status(cudaStreamWaitEvent(ss, lm->h_ready, 0), "cudaStreamWaitEvent");
    if (st != W8A8_SUCCESS) return st;
    st = w8a8_linear_forward_topk(lm->shards[s], h, lm->K, T, W8A8_ACT_STATIC, W8A8_OUT_F32_ACC,
                                  k, lm->lo[s], lm->cand_val + s * block,
                                  lm->cand_idx + s * block, nullptr, 0, ss);
    if (st != W8A8_SUCCESS) return st;
    st = cuda_status(cudaEventRecord(lm->done[s - 1], ss), "cudaEventRecord");
    if (st != W8A8_SUCCESS) return st;
  }
  // Shard 0 on the caller's stream, then the merge after every other shard's event (with one
  // shard the merge only copies its sorted list and writes the argmax).
  DeviceScope d(lm->dev[0]);
  w8a8_status st = w8a8_linear_forward_topk(lm->shards[0], h, lm->K, T, W8A8_ACT_STATIC,
                                            W8A8_OUT_F32_ACC, k, lm->lo[0], lm->cand_val,
                                            lm->cand_idx, nullptr, 0, s0);
  if (st != W8A8_SUCCESS) return st;
  for (int s = 1; s < n; ++s) {
    st = cuda_status(cudaStreamWaitEvent(s0, lm->done[s - 1], 0), "cudaStreamWaitEvent");
    if (st != W8A8_SUCCESS) return st;
  }
  return w8a8_topk_merge(lm->ctxs[0], lm->cand_val, lm->cand_idx, T, n, k, block, k, k, val, idx,
                         argmax, s0);
}

void w8a8_lmhead_destroy(w8a8_lmhead *lm) { lmhead_free(lm); }

int32_t w8a8_lmhead_shards(const w8a8_lmhead *lm) { return lm ? lm->n : 0; }

}  // extern "C"
