// int16 x int16 contraction with the SDP QuantM requant: the w2 stage of the reference's SwiGLU
// MLP subgraph, whose input is the int16 product silu(gate) * up and whose weights are int16
// per-output-row codes (C ABI w8a8_linear16_*).
//
// Reference: the weights are tile_int16_slice codes (src/LFM3/build_lfm3_int8_pkg.py:111-122,
// written for w2 at :290-306 with trunc 28 and per-channel out_step_chan); the arithmetic is the
// engine's MLP model in src/LFM3/attribute_int8_error.py:117-121:
//   out_q[t, n] = clip(round(sum_k x[t, k] * w[n, k] * (QuantM[n] / 2^trunc)), +-32767)
// computed there in float64.  The sum of int16 products is an integer below 2^53 for any K here
// (|x * w| < 2^30), so float64 holds it exactly in any order; this kernel accumulates it exactly
// in int64 and then performs the same float64 operations: one multiply by QuantM * 2^-trunc
// (exact), round-half-even, clip.  Optional unpack: y = float(out_q) * out_step_chan[n]
// (unpack_npu_output_int16, src/LFM3/lfm3_v2.cpp:1010-1046).
//
// One warp per output row at a time (four rows per warp, eight warps per CTA); each lane streams
// 16-byte chunks (8 codes) of the weight row and of every token's input row; two int16 products
// always fit int32 (|p| < 2^30), so each chunk adds four exact pair sums to int64 accumulators.
#include "../../include/w8a8.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <new>

#include "common.cuh"
#include "kernels.h"

namespace w8a8 {
namespace {

constexpr int kG16Threads = 256;
constexpr int kG16RowsPerWarp = 4;
constexpr int kG16RowsPerCta = kG16RowsPerWarp * (kG16Threads / 32);

struct Gemv16Args {
  const int16_t *w;      // [N, ldw] codes, zero past K up to k8 (a multiple of 8)
  int64_t ldw;
  const int16_t *x;      // [T, ldx] int16 activations, zero past K up to k8
  int64_t ldx;
  int T, N, k8;
  const int16_t *quant_m;
  int trunc;
  const float *out_step_chan;  // F32 output only
  int out_f32;
  void *y;
  int64_t ldy;
};

__device__ __forceinline__ int pair_dot(uint32_t a, uint32_t b) {
  const int a0 = static_cast<int16_t>(a & 0xFFFFu), a1 = static_cast<int16_t>(a >> 16);
  const int b0 = static_cast<int16_t>(b & 0xFFFFu), b1 = static_cast<int16_t>(b >> 16);
  return a0 * b0 + a1 * b1;  // |.| < 2^31: two products of magnitude < 2^30
}

__device__ __forceinline__ long long chunk_dot(const int4 &a, const int4 &b) {
  return static_cast<long long>(pair_dot(a.x, b.x)) + static_cast<long long>(pair_dot(a.y, b.y)) +
         static_cast<long long>(pair_dot(a.z, b.z)) + static_cast<long long>(pair_dot(a.w, b.w));
}

__device__ __forceinline__ long long warp_sum_ll(long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// The reference's float64 requant of an exact integer accumulator: round(acc * (qm / 2^trunc)),
// clipped to +-32767 (clipping before the round-half-even conversion gives the same integer).
__device__ __forceinline__ int requant_i16_f64(long long acc, int qm, int trunc) {
  double v = static_cast<double>(acc) *
             (static_cast<double>(qm) *
              __longlong_as_double(static_cast<long long>(1023 - trunc) << 52));
  v = v < -32767.0 ? -32767.0 : v;
  v = v > 32767.0 ? 32767.0 : v;
  return __double2int_rn(v);
}

template <int TT>
__global__ void __launch_bounds__(kG16Threads) gemv_i16_kernel(const Gemv16Args a) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kG16RowsPerCta + warp * kG16RowsPerWarp;
#pragma unroll 1
  for (int r = 0; r < kG16RowsPerWarp; ++r) {
    const int n = n0 + r;
    if (n >= a.N) break;
    long long acc[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[t] = 0;
    const int16_t *wr = a.w + static_cast<int64_t>(n) * a.ldw;
    for (int c = lane * 8; c < a.k8; c += 256) {
      const int4 wv = __ldg(reinterpret_cast<const int4 *>(wr + c));
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        if (t >= a.T) break;
        const int4 xv = __ldg(reinterpret_cast<const int4 *>(a.x + t * a.ldx + c));
        acc[t] += chunk_dot(wv, xv);
      }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (t >= a.T) break;
      const long long s = warp_sum_ll(acc[t]);
      if (lane == 0) {
        const int q = requant_i16_f64(s, a.quant_m[n], a.trunc);
        if (a.out_f32)
          static_cast<float *>(a.y)[t * a.ldy + n] = static_cast<float>(q) * a.out_step_chan[n];
        else
          static_cast<int16_t *>(a.y)[t * a.ldy + n] = static_cast<int16_t>(q);
      }
    }
  }
}

// Rows [N, K] of int16 codes copied into a zero-padded [N, k8] buffer (k8 = round_up(K, 8)).
__global__ void pad_rows_i16_kernel(const int16_t *src, int64_t lds, int N, int K, int16_t *dst,
                                    int k8) {
  const int64_t total = static_cast<int64_t>(N) * k8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / k8, k = i % k8;
    dst[i] = k < K ? src[n * lds + k] : static_cast<int16_t>(0);
  }
}

}  // namespace
}  // namespace w8a8

struct w8a8_linear16 {
  w8a8_ctx *ctx = nullptr;
  int dev = 0, K = 0, N = 0, k8 = 0, trunc = 0, max_T = 0;
  int16_t *w = nullptr;        // [N, k8]
  int16_t *quant_m = nullptr;  // [N]
  float *out_step = nullptr;   // [N] or null
  int16_t *xs = nullptr;       // [max_T, k8] staging of inputs whose rows are not 16-byte padded
};

namespace {

w8a8_status l16_fail(w8a8_status st, const char *msg) {
  w8a8::set_last_error(msg);
  return st;
}

w8a8_status l16_cuda(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return W8A8_SUCCESS;
  char buf[256];
  std::snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  w8a8::set_last_error(buf);
  return W8A8_ERR_CUDA;
}

class L16Device {
 public:
  explicit L16Device(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~L16Device() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

void l16_free(w8a8_linear16 *l) {
  if (!l) return;
  L16Device d(l->dev);
  cudaFree(l->w);
  cudaFree(l->quant_m);
  cudaFree(l->out_step);
  cudaFree(l->xs);
  delete l;
}

}  // namespace

extern "C" {

w8a8_status w8a8_linear16_create(w8a8_ctx *ctx, int32_t K, int32_t N, const int16_t *weights,
                                 int64_t ld, const int16_t *quant_m, int32_t trunc,
                                 const float *out_step_chan, int32_t max_T,
                                 w8a8_linear16 **out) {
  if (!out) return l16_fail(W8A8_ERR_INVALID_ARG, "out_linear16 is NULL");
  *out = nullptr;
  if (!ctx || !weights || !quant_m) return l16_fail(W8A8_ERR_INVALID_ARG, "ctx, weights or quant_m is NULL");
  if (K < 1 || N < 1 || ld < K || trunc < 0 || trunc > 62 || max_T < 1 || max_T > 4096)
    return l16_fail(W8A8_ERR_INVALID_ARG, "bad shape (K, N >= 1, ld >= K, trunc in [0, 62], 1 <= max_tokens <= 4096)");
  if (static_cast<int64_t>(K) * 32767 * 32767 >= (int64_t{1} << 53))
    return l16_fail(W8A8_ERR_INVALID_ARG, "K too large for an exact float64 accumulator");
  w8a8_linear16 *l = new (std::nothrow) w8a8_linear16();
  if (!l) return W8A8_ERR_NO_MEMORY;
  l->ctx = ctx;
  l->dev = w8a8_ctx_device(ctx);
  l->K = K;
  l->N = N;
  l->k8 = (K + 7) / 8 * 8;
  l->trunc = trunc;
  l->max_T = max_T;
  L16Device d(l->dev);
  const size_t row = static_cast<size_t>(l->k8) * sizeof(int16_t);
  cudaError_t e = cudaMalloc(&l->w, row * N);
  if (e == cudaSuccess) e = cudaMemset(l->w, 0, row * N);
  if (e == cudaSuccess)
    e = cudaMemcpy2D(l->w, row, weights, static_cast<size_t>(ld) * sizeof(int16_t),
                     static_cast<size_t>(K) * sizeof(int16_t), N, cudaMemcpyDefault);
  if (e == cudaSuccess) e = cudaMalloc(&l->quant_m, N * sizeof(int16_t));
  if (e == cudaSuccess) e = cudaMemcpy(l->quant_m, quant_m, N * sizeof(int16_t), cudaMemcpyDefault);
  if (e == cudaSuccess && out_step_chan) {
    e = cudaMalloc(&l->out_step, N * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(l->out_step, out_step_chan, N * sizeof(float), cudaMemcpyDefault);
  }
  if (e == cudaSuccess) e = cudaMalloc(&l->xs, row * max_T);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    l16_free(l);
    return l16_cuda(e, "linear16 upload");
  }
  *out = l;
  return W8A8_SUCCESS;
}

w8a8_status w8a8_linear16_forward(w8a8_linear16 *l, const int16_t *x_dev, int64_t ldx, int32_t T,
                                  int32_t out_mode, void *y_dev, int64_t ldy, void *stream) {
  using namespace w8a8;
  if (!l || !x_dev || !y_dev) return l16_fail(W8A8_ERR_INVALID_ARG, "linear16, x or y is NULL");
  if (T < 1 || T > l->max_T || ldx < l->K || ldy < l->N)
    return l16_fail(W8A8_ERR_INVALID_ARG, "T outside [1, max_tokens], ldx < K or ldy < N");
  if (out_mode != W8A8_OUT_QUANT && out_mode != W8A8_OUT_F32)
    return l16_fail(W8A8_ERR_NOT_SUPPORTED, "out_mode must be QUANT (int16) or F32");
  if (out_mode == W8A8_OUT_F32 && !l->out_step)
    return l16_fail(W8A8_ERR_INVALID_ARG, "F32 output needs out_step_chan at create");
  L16Device d(l->dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // inputs staged into 16-byte-padded rows (zero past K)
  const int64_t cells = static_cast<int64_t>(T) * l->k8;
  int blocks = static_cast<int>((cells + 255) / 256);
  blocks = blocks > 1024 ? 1024 : blocks;
  pad_rows_i16_kernel<<<blocks, 256, 0, s>>>(x_dev, ldx, T, l->K, l->xs, l->k8);
  w8a8_status st = l16_cuda(cudaGetLastError(), "linear16 input staging");
  if (st != W8A8_SUCCESS) return st;
  for (int t0 = 0; t0 < T; t0 += 8) {
    Gemv16Args a;
    a.w = l->w;
    a.ldw = l->k8;
    a.x = l->xs + static_cast<int64_t>(t0) * l->k8;
    a.ldx = l->k8;
    a.T = T - t0 < 8 ? T - t0 : 8;
    a.N = l->N;
    a.k8 = l->k8;
    a.quant_m = l->quant_m;
    a.trunc = l->trunc;
    a.out_step_chan = l->out_step;
    a.out_f32 = out_mode == W8A8_OUT_F32 ? 1 : 0;
    a.y = out_mode == W8A8_OUT_F32
              ? static_cast<void *>(static_cast<float *>(y_dev) + static_cast<int64_t>(t0) * ldy)
              : static_cast<void *>(static_cast<int16_t *>(y_dev) + static_cast<int64_t>(t0) * ldy);
    a.ldy = ldy;
    const dim3 grid((l->N + kG16RowsPerCta - 1) / kG16RowsPerCta);
    const cudaError_t e = a.T <= 1   ? launch_ex(gemv_i16_kernel<1>, grid, dim3(kG16Threads), 0, s, true, a)
                          : a.T <= 4 ? launch_ex(gemv_i16_kernel<4>, grid, dim3(kG16Threads), 0, s, true, a)
                                     : launch_ex(gemv_i16_kernel<8>, grid, dim3(kG16Threads), 0, s, true, a);
    st = l16_cuda(e, "linear16 GEMV launch");
    if (st != W8A8_SUCCESS) return st;
  }
  return W8A8_SUCCESS;
}

void w8a8_linear16_destroy(w8a8_linear16 *l) { l16_free(l); }

}  // extern "C"
