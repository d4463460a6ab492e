// Allocation-free LM-head shard top-k (w8a8_lmhead_topk_noalloc).
//
// Some callers cannot call cudaMalloc at all: code that runs inside a host-side allocator or
// memory-pool callback, plugins whose host process owns every device allocation and forbids
// others, and hot paths that must not take the driver's allocation locks.  Those callers
// already hold the weights, parameters, inputs and outputs in device memory; what the regular
// top-k entry point adds on top is scratch memory (int8 activation staging, per-token ratios,
// per-CTA candidate lists, an arrival counter), which w8a8_linear_create allocates.  This file
// keeps that scratch in one module-scope device array instead, so the entry point below
// allocates nothing.
//
// The array (kScratchBytes, about 1.4 MiB) is held by every GPU that loads the library until
// the process exits.  All calls on a device share it and it keeps the last call's contents, so
// calls whose executions overlap on the GPU (different streams, or different host threads
// without ordering) race and corrupt each other's results; the arrival counter, which must
// start at zero, is cleared on the call's stream before each launch.
//
// The first call on a device is a set-up call: it resolves the array's device address and,
// under CUDA's default lazy module loading, makes the driver load this library's kernels on that
// device, which allocates device memory inside the driver.  Make it (a warm-up call) before any
// stream capture and outside any context where allocating is not allowed; later calls allocate
// nothing.
#include "../../include/w8a8.h"
#include "kernels.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

namespace {

constexpr int kMaxTokens = 8;
constexpr size_t kXqBytes = 128 * 1024;     // int8 activations: T * round_up(K, 16) bytes
constexpr size_t kMiscBytes = 256;          // ratios [8] fp32, counter, error word
constexpr size_t kListKeys = 160 * 1024;    // per-CTA candidate keys (u64): 1.25 MiB
constexpr size_t kScratchBytes = kXqBytes + kMiscBytes + kListKeys * 8;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DeviceSlot {
  unsigned char *scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sm_count = 0;
  bool ok = false;
};

std::mutex g_mu;
DeviceSlot g_slots[kMaxDevices];

// Set-up, once per device, with that device current: resolves the device address of the
// scratch array (the host-side name g_noalloc_scratch is only a stand-in, not a device address).
w8a8_status device_slot(DeviceSlot *out, const char **why) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *why = "no current CUDA device";
    return W8A8_ERR_NOT_INITIALIZED;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceSlot &s = g_slots[dev];
  if (!s.ok) {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      *why = "device attribute query failed";
      return W8A8_ERR_CUDA;
    }
    if (major != 10 || minor != 0) {
      *why = "device is not sm_100";
      return W8A8_ERR_NOT_SUPPORTED;
    }
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *why = "cudaGetSymbolAddress of the scratch array failed";
      return W8A8_ERR_CUDA;
    }
    s.scratch = static_cast<unsigned char *>(p);
    s.sm_count = sms;
    s.ok = true;
  }
  *out = s;
  return W8A8_SUCCESS;
}

// Records the reason for w8a8_last_error() and returns the status.
w8a8_status reject(w8a8_status st, const char *fmt, long long a = 0, long long b = 0) {
  char msg[256];
  std::snprintf(msg, sizeof(msg), fmt, a, b);
  w8a8::set_last_error(msg);
  return st;
}

}  // namespace

extern "C" w8a8_status w8a8_lmhead_topk_noalloc(const int8_t *w_dev, int64_t ldw, int32_t K,
                                                int32_t N, const float *acc_step_dev,
                                                float in_step, const float *x_dev, int64_t ldx,
                                                int32_t T, int32_t k, int32_t row_offset,
                                                float *topk_val_dev, int32_t *topk_idx_dev,
                                                void *stream) {
  using namespace w8a8;
  if (!w_dev || !acc_step_dev || !x_dev || !topk_val_dev || !topk_idx_dev)
    return reject(W8A8_ERR_INVALID_ARG, "NULL pointer argument");
  if (T < 1 || T > kMaxTokens)
    return reject(W8A8_ERR_INVALID_ARG, "T=%lld outside [1, %lld]", T, kMaxTokens);
  if (K < 1 || N < 1) return reject(W8A8_ERR_INVALID_ARG, "K=%lld N=%lld must be >= 1", K, N);
  const int k_pad = (K + 15) / 16 * 16;
  if (ldw < k_pad || ldw % 16 != 0 || (reinterpret_cast<uintptr_t>(w_dev) & 15u) != 0)
    return reject(W8A8_ERR_INVALID_ARG,
                  "weights need a 16-byte aligned base and ldw (%lld) a multiple of 16 >= %lld",
                  ldw, k_pad);
  if (ldx < K) return reject(W8A8_ERR_INVALID_ARG, "ldx %lld < K %lld", ldx, K);
  if (k < 1 || k > W8A8_TOPK_MAX || k > N)
    return reject(W8A8_ERR_INVALID_ARG, "k=%lld outside [1, min(64, N=%lld)]", k, N);
  if (row_offset < 0 || static_cast<long long>(row_offset) + N > 0x7FFFFFFFLL)
    return reject(W8A8_ERR_INVALID_ARG, "row_offset %lld + N %lld out of range", row_offset, N);
  if (static_cast<size_t>(T) * k_pad > kXqBytes)
    return reject(W8A8_ERR_INVALID_ARG,
                  "T * round_up(K, 16) = %lld bytes exceeds the %lld-byte activation scratch",
                  static_cast<long long>(T) * k_pad, static_cast<long long>(kXqBytes));
  DeviceSlot slot;
  const char *why = "";
  w8a8_status st = device_slot(&slot, &why);
  if (st != W8A8_SUCCESS) return reject(st, why);
  GemvPlan plan;
  if (!plan_gemv(T, N, k_pad, true, k, slot.sm_count, &plan))
    return reject(W8A8_ERR_NOT_SUPPORTED, "no top-k plan for T=%lld N=%lld", T, N);
  if (static_cast<size_t>(T) * plan.grid * (k + 1) > kListKeys)
    return reject(W8A8_ERR_INVALID_ARG,
                  "T * grid * (k + 1) = %lld candidate keys exceed the scratch maximum of %lld",
                  static_cast<long long>(T) * plan.grid * (k + 1),
                  static_cast<long long>(kListKeys));

  int8_t *xq = reinterpret_cast<int8_t *>(slot.scratch);
  float *ratio = reinterpret_cast<float *>(slot.scratch + kXqBytes);
  unsigned *counter = reinterpret_cast<unsigned *>(slot.scratch + kXqBytes + 64);
  int *err = reinterpret_cast<int *>(slot.scratch + kXqBytes + 128);
  uint64_t *lists = reinterpret_cast<uint64_t *>(slot.scratch + kXqBytes + kMiscBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // the arrival counter must start at zero; the error word (which no call reads back) is
  // cleared with it so a bounded wait that ran out in an earlier call leaves nothing behind
  static_assert(128 + sizeof(int) <= kMiscBytes, "the error word lies inside the cleared range");
  if (cudaMemsetAsync(counter, 0, 64 + sizeof(int), s) != cudaSuccess)
    return reject(W8A8_ERR_CUDA, "clearing the arrival counter failed");

  ActQuantLaunch A = {};
  A.x = x_dev;
  A.ldx = ldx;
  A.T = T;
  A.K = K;
  A.k_fill = k_pad;
  A.inv_smooth = nullptr;
  A.act_mode = kActStatic;
  A.inv_step = (in_step > 1e-12f) ? (1.0f / in_step) : 0.0f;
  A.safe_thresh = 1.0f;
  A.q = xq;
  A.ldq = k_pad;
  A.ratio = ratio;
  A.pdl = false;
  if (launch_act_quant(A, s) != cudaSuccess)
    return reject(W8A8_ERR_CUDA, "activation quantisation launch failed");

  GemvLaunch L = {};
  L.w = w_dev;
  L.ldw = ldw;
  L.x = xq;
  L.ldx = k_pad;
  L.T = T;
  L.N = N;
  L.k_pad = k_pad;
  L.ep.out_mode = kOutF32Acc;
  L.ep.act_mode = kActStatic;
  L.ep.acc_step = acc_step_dev;
  L.ep.ratio = ratio;
  L.topk = true;
  L.tk.k = k;
  L.tk.row_offset = row_offset;
  L.tk.lists = lists;
  L.tk.counter = counter;
  L.tk.val = topk_val_dev;
  L.tk.idx = topk_idx_dev;
  L.tk.logits = nullptr;
  L.tk.ldl = 0;
  L.err = err;
  L.sm_count = slot.sm_count;
  L.pdl = true;
  if (launch_gemv(L, plan, s) != cudaSuccess)
    return reject(W8A8_ERR_CUDA, "top-k GEMV launch failed");
  return W8A8_SUCCESS;
}
