// The host-side steps on either side of each linear in the reference's decode loop, moved onto
// the GPU with the reference's float order (C ABI w8a8_rmsnorm_pack_dyntok / w8a8_post_op_ffn_pack):
//
//   rmsnorm_pack_kernel   fused_rms_norm_pack_dyntok_t1 (src/LFM3/lfm3_v2.cpp:652-700): RMSNorm,
//                         SmoothQuant and dynamic per-token int8 quantisation of a linear's input
//                         (+ the plain normalised row for the attention path);
//   post_op_pack_kernel   fused_post_op_residual_ffn_pack_mlp_t1 (:702-765): post-operator norm,
//                         residual add, FFN norm, SmoothQuant and static int8 quantisation.
//
// The sums of squares must round exactly as the reference's: four interleaved partial sums over
// the multiple-of-4 prefix, combined as (s0 + s1) + (s2 + s3), then the tail one by one (:659-667).
// Four threads of the CTA run those four chains in order over the row staged in shared memory
// (thread 0 then adds the tail); everything else (elementwise products in the reference's
// left-to-right order, IEEE sqrt and division, the max reduction, which is order-free) is spread
// over the CTA.  One CTA per token row.
#include "../../include/w8a8.h"

#include <cuda_runtime.h>

#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace w8a8 {
namespace {

constexpr int kNormThreads = 256;
constexpr int kNormMaxC = 12288;  // row staged in shared memory (48 KB + static, opted in)

// The reference's sum of squares of row[0..C) (see the file comment); valid in thread 0 after the
// call, which ends with a __syncthreads().
__device__ float sum_sq_ordered(const float *row, int C, float *s_part) {
  const int C4 = C & ~3;
  if (threadIdx.x < 4) {
    float s = 0.0f;
    for (int c = threadIdx.x; c < C4; c += 4) s += row[c] * row[c];
    s_part[threadIdx.x] = s;
  }
  __syncthreads();
  float sum = 0.0f;
  if (threadIdx.x == 0) {
    sum = (s_part[0] + s_part[1]) + (s_part[2] + s_part[3]);
    for (int c = C4; c < C; ++c) sum += row[c] * row[c];
  }
  __syncthreads();
  return sum;
}

// Max over the CTA of per-thread values (non-negative; the reduction order does not matter).
__device__ float block_amax(float v, float *s_red) {
  v = warp_amax(v);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) m = s_red[w] > m ? s_red[w] : m;
  __syncthreads();
  return m;
}

struct RmsPackArgs {
  const float *h;
  int64_t ldh;
  int C;
  const float *norm, *smooth;
  float in_thresh, eps;
  int8_t *q;
  int64_t ldq;
  float *ratio;
  float *u_out;
  int64_t ldu;
};

__global__ void __launch_bounds__(kNormThreads) rmsnorm_pack_kernel(const RmsPackArgs a) {
  extern __shared__ float row[];
  __shared__ float s_part[4], s_red[kNormThreads / 32], s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const float *h = a.h + t * a.ldh;
  for (int c = threadIdx.x; c < a.C; c += kNormThreads) row[c] = h[c];
  __syncthreads();
  const float sum = sum_sq_ordered(row, a.C, s_part);
  if (threadIdx.x == 0) s_inv = 1.0f / sqrtf(sum / static_cast<float>(a.C) + a.eps);
  __syncthreads();
  const float inv_rms = s_inv;
  float amax = 0.0f;
  for (int c = threadIdx.x; c < a.C; c += kNormThreads) {
    if (a.u_out) a.u_out[t * a.ldu + c] = row[c] * inv_rms * a.norm[c];
    const float v = fabsf(row[c] * inv_rms * a.smooth[c]);
    if (v > amax) amax = v;
  }
  amax = block_amax(amax, s_red);
  amax = amax < 1e-8f ? 1e-8f : amax;
  if (threadIdx.x == 0) a.ratio[t] = amax / (a.in_thresh < 1e-8f ? 1e-8f : a.in_thresh);
  const float inv_step = 127.0f / amax;
  for (int c = threadIdx.x; c < a.C; c += kNormThreads)
    a.q[t * a.ldq + c] =
        static_cast<int8_t>(round_clamp(row[c] * inv_rms * a.smooth[c] * inv_step, 127.0f));
}

struct PostOpArgs {
  const float *op_out;
  int64_t ldo;
  const float *post_norm;
  const float *h;
  int64_t ldh;
  int C;
  const float *ffn_scaled;
  float eps;
  float *h_mid;
  int64_t ldm;
  int8_t *q;
  int64_t ldq;
};

__global__ void __launch_bounds__(kNormThreads) post_op_pack_kernel(const PostOpArgs a) {
  extern __shared__ float row[];
  __shared__ float s_part[4], s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const float *o = a.op_out + t * a.ldo;
  for (int c = threadIdx.x; c < a.C; c += kNormThreads) row[c] = o[c];
  __syncthreads();
  float sum = sum_sq_ordered(row, a.C, s_part);
  if (threadIdx.x == 0) s_inv = 1.0f / sqrtf(sum / static_cast<float>(a.C) + a.eps);
  __syncthreads();
  const float inv_op = s_inv;
  // h_mid = h + op_out * inv_rms_op * post_norm, kept in place of op_out for the second norm
  const float *h = a.h + t * a.ldh;
  float *m = a.h_mid + t * a.ldm;
  for (int c = threadIdx.x; c < a.C; c += kNormThreads) {
    const float hm = h[c] + row[c] * inv_op * a.post_norm[c];
    row[c] = hm;
    m[c] = hm;
  }
  __syncthreads();
  sum = sum_sq_ordered(row, a.C, s_part);
  if (threadIdx.x == 0) s_inv = 1.0f / sqrtf(sum / static_cast<float>(a.C) + a.eps);
  __syncthreads();
  const float inv_ffn = s_inv;
  for (int c = threadIdx.x; c < a.C; c += kNormThreads)
    a.q[t * a.ldq + c] =
        static_cast<int8_t>(round_clamp(row[c] * inv_ffn * a.ffn_scaled[c], 127.0f));
}

class DeviceScope {
 public:
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() {
    if (prev_ >= 0) cudaSetDevice(prev_);
  }

 private:
  int prev_ = -1;
};

w8a8_status norm_error(w8a8_status st, const char *msg) {
  set_last_error(msg);
  return st;
}

w8a8_status norm_launch_status(cudaError_t e) {
  if (e == cudaSuccess) return W8A8_SUCCESS;
  char buf[200];
  std::snprintf(buf, sizeof(buf), "norm kernel launch: %s", cudaGetErrorString(e));
  set_last_error(buf);
  return W8A8_ERR_CUDA;
}

}  // namespace
}  // namespace w8a8

extern "C" {

w8a8_status w8a8_rmsnorm_pack_dyntok(w8a8_ctx *ctx, const float *h, int64_t ldh, int32_t T,
                                     int32_t C, const float *norm, const float *smooth,
                                     float in_thresh, float eps, int8_t *q, int64_t ldq,
                                     float *ratio, float *u_out, int64_t ldu, void *stream) {
  using namespace w8a8;
  if (!ctx || !h || !smooth || !q || !ratio)
    return norm_error(W8A8_ERR_INVALID_ARG, "ctx, h, smooth, q or ratio is NULL");
  if (u_out && !norm) return norm_error(W8A8_ERR_INVALID_ARG, "u_out needs norm");
  if (T < 1 || C < 1 || C > kNormMaxC || ldh < C || ldq < C || (u_out && ldu < C))
    return norm_error(W8A8_ERR_INVALID_ARG, "bad shape: 1 <= C <= 12288, strides >= C, T >= 1");
  DeviceScope d(w8a8_ctx_device(ctx));
  int limit = 0;
  w8a8_status st = norm_launch_status(opt_in_dyn_smem<rmsnorm_pack_kernel>(&limit));
  if (st != W8A8_SUCCESS) return st;
  RmsPackArgs a{h, ldh, C, norm, smooth, in_thresh, eps, q, ldq, ratio, u_out, ldu};
  return norm_launch_status(launch_ex(rmsnorm_pack_kernel, dim3(T), dim3(kNormThreads),
                                      static_cast<size_t>(C) * 4,
                                      static_cast<cudaStream_t>(stream), true, a));
}

w8a8_status w8a8_post_op_ffn_pack(w8a8_ctx *ctx, const float *op_out, int64_t ldo,
                                  const float *post_norm, const float *h, int64_t ldh, int32_t T,
                                  int32_t C, const float *ffn_scaled, float eps, float *h_mid,
                                  int64_t ldm, int8_t *q, int64_t ldq, void *stream) {
  using namespace w8a8;
  if (!ctx || !op_out || !post_norm || !h || !ffn_scaled || !h_mid || !q)
    return norm_error(W8A8_ERR_INVALID_ARG, "NULL argument");
  if (T < 1 || C < 1 || C > kNormMaxC || ldo < C || ldh < C || ldm < C || ldq < C)
    return norm_error(W8A8_ERR_INVALID_ARG, "bad shape: 1 <= C <= 12288, strides >= C, T >= 1");
  DeviceScope d(w8a8_ctx_device(ctx));
  int limit = 0;
  w8a8_status st = norm_launch_status(opt_in_dyn_smem<post_op_pack_kernel>(&limit));
  if (st != W8A8_SUCCESS) return st;
  PostOpArgs a{op_out, ldo, post_norm, h, ldh, C, ffn_scaled, eps, h_mid, ldm, q, ldq};
  return norm_launch_status(launch_ex(post_op_pack_kernel, dim3(T), dim3(kNormThreads),
                                      static_cast<size_t>(C) * 4,
                                      static_cast<cudaStream_t>(stream), true, a));
}

}  // extern "C"

extern "C" w8a8_status w8a8_emb_norm_pack(w8a8_ctx *ctx, const float *h_dev, int64_t ldh,
                                          int32_t T, int32_t C, const float *emb_norm_scaled_dev,
                                          float eps, int8_t *q_dev, int64_t ldq, void *stream) {
  if (!ctx || !h_dev || !emb_norm_scaled_dev || !q_dev) {
    w8a8::set_last_error("ctx, h, emb_norm_scaled or q is NULL");
    return W8A8_ERR_INVALID_ARG;
  }
  if (T < 1 || C < 1 || C > 12288 || ldh < C || ldq < C) {
    w8a8::set_last_error("T >= 1, 1 <= C <= 12288, ldh >= C and ldq >= C required");
    return W8A8_ERR_INVALID_ARG;
  }
  w8a8::ActQuantLaunch A = {};
  A.x = h_dev;
  A.ldx = ldh;
  A.T = T;
  A.K = C;
  A.k_fill = C;
  A.act_mode = w8a8::kActStatic;
  A.q = q_dev;
  A.ldq = ldq;
  A.emb_norm = emb_norm_scaled_dev;
  A.eps = eps;
  const cudaError_t e = w8a8::launch_act_quant(A, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "emb norm pack launch: %s", cudaGetErrorString(e));
    w8a8::set_last_error(buf);
    return W8A8_ERR_CUDA;
  }
  return W8A8_SUCCESS;
}

