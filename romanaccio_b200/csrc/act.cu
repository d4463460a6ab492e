// Boundary kernels around the contraction: activation quantisation (pack), int8 staging copy,
// output dequantisation (unpack) and the cross-shard top-k merge.
//
//   act_quant_kernel  pack_npu_input_int8 (src/LFM3/lfm3_v2.cpp:892-940) and
//                     pack_npu_input_int8_dyntok (src/LFM3/lfm3_v2.cpp:1050-1141), [T, K] layout
//   unpack_kernel     unpack_npu_output_int8 / _int16 / _int8_dyntok (src/LFM3/lfm3_v2.cpp:971-1046,
//                     1143-1183)
//   topk_merge_kernel merge of per-shard candidates; order (value desc, id asc) as the greedy
//                     rule of src/eswin_runtime/src/nlp/sampler.cpp:93-103
#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace w8a8 {

namespace {

constexpr int kActThreads = 256;

struct ActArgs {
  const float *x;
  int64_t ldx;
  int K, k_fill;
  const float *s;
  float inv_step, safe_thresh;
  int8_t *q;
  int64_t ldq;
  float *ratio;
  const PublishPeer *peers;
  int n_peers;
  unsigned *pub_seq, *pub_arrive;
  unsigned long long *trace;
  int pub_row0;
  const float *emb;
  float eps;
};

// Publication of the quantised rows to other devices: every CTA's stores are fenced at system
// scope before it arrives; the last CTA to arrive bumps the forward counter and stores it into
// each peer's flag with release semantics (the peer reads the rows after an acquire of it).
__device__ void publish_arrive(const ActArgs &a) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(a.pub_arrive, 1u) == gridDim.x - 1) {
    __threadfence_system();
    const unsigned e = *a.pub_seq + 1u;
    *a.pub_seq = e;
    *a.pub_arrive = 0u;
    // (the fence above makes these relaxed stores a release of every CTA's rows)
    for (int p = 0; p < a.n_peers; ++p) st_relaxed_sys(a.peers[p].flag, e);
    if (a.trace) a.trace[1] = global_timer_ns();
  }
}

// One CTA per token row.  DYN: amax_t = max_c |x*s| (NaN ignored as by `if (a > amax)`),
// amax_t = max(amax_t, 1e-8), ratio_t = amax_t / max(in_thresh, 1e-8), inv = 127 / amax_t.
// q = round_clamp(x * (s * inv), 127) with the reference's association of the products.
// fused_emb_norm_broadcast_t1 (src/LFM3/lfm3_v2.cpp:810-831) for one token row per CTA: the
// row is staged in shared memory, four threads run the reference's four interleaved
// sum-of-squares chains in order over the multiple-of-4 prefix, thread 0 combines them as
// (s0 + s1) + (s2 + s3) and adds the tail one by one, inv_rms = 1 / sqrt(sum / C + eps) (IEEE),
// and q[c] = round_clamp(x[c] * inv_rms * emb[c], 127) with the reference's left-to-right
// products; the rows go to q and, like act_quant_kernel, to every peer.
constexpr int kEmbNormMaxK = 12288;  // fp32 row in 48 KB of dynamic shared memory

__global__ void __launch_bounds__(kActThreads) emb_norm_pack_kernel(const ActArgs a) {
  extern __shared__ float row[];
  __shared__ float s_part[4], s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const float *x = a.x + t * a.ldx;
  for (int c = threadIdx.x; c < a.K; c += kActThreads) row[c] = x[c];
  __syncthreads();
  const int K4 = a.K & ~3;
  if (threadIdx.x < 4) {
    float sum = 0.0f;
    for (int c = threadIdx.x; c < K4; c += 4) sum += row[c] * row[c];
    s_part[threadIdx.x] = sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = (s_part[0] + s_part[1]) + (s_part[2] + s_part[3]);
    for (int c = K4; c < a.K; ++c) sum += row[c] * row[c];
    s_inv = 1.0f / sqrtf(sum / static_cast<float>(a.K) + a.eps);
  }
  __syncthreads();
  const float inv_rms = s_inv;
  int8_t *q = a.q + t * a.ldq;
  for (int c = threadIdx.x; c < a.k_fill; c += kActThreads) {
    const int8_t o = c < a.K ? static_cast<int8_t>(round_clamp(row[c] * inv_rms * a.emb[c], 127.0f))
                             : static_cast<int8_t>(0);
    q[c] = o;
    for (int p = 0; p < a.n_peers; ++p) a.peers[p].q[(a.pub_row0 + t) * a.ldq + c] = o;
  }
  if (a.ratio && threadIdx.x == 0) a.ratio[t] = 1.0f;
  if (a.pub_seq) publish_arrive(a);
}

template <bool DYN, bool SMOOTH, bool VEC>
__global__ void __launch_bounds__(kActThreads) act_quant_kernel(const ActArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) a.trace[0] = global_timer_ns();
  const int t = blockIdx.x;
  const float *x = a.x + t * a.ldx;
  int8_t *q = a.q + t * a.ldq;
  float inv = a.inv_step;
  if (DYN) {
    __shared__ float s_part[kActThreads / 32];
    float amax = 0.0f;
    if (VEC) {
      const float4 *x4 = reinterpret_cast<const float4 *>(x);
      const float4 *s4 = reinterpret_cast<const float4 *>(a.s);
      for (int c = threadIdx.x; c < a.K / 4; c += kActThreads) {
        const float4 v = x4[c];
        float4 m = v;
        if (SMOOTH) {
          const float4 sv = s4[c];
          m.x = v.x * sv.x; m.y = v.y * sv.y; m.z = v.z * sv.z; m.w = v.w * sv.w;
        }
        const float ax = fabsf(m.x), ay = fabsf(m.y), az = fabsf(m.z), aw = fabsf(m.w);
        if (ax > amax) amax = ax;
        if (ay > amax) amax = ay;
        if (az > amax) amax = az;
        if (aw > amax) amax = aw;
      }
    } else {
      for (int c = threadIdx.x; c < a.K; c += kActThreads) {
        const float v = SMOOTH ? fabsf(x[c] * a.s[c]) : fabsf(x[c]);
        if (v > amax) amax = v;
      }
    }
    amax = warp_amax(amax);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.0f;
#pragma unroll
    for (int w = 0; w < kActThreads / 32; ++w) amax = s_part[w] > amax ? s_part[w] : amax;
    amax = (amax < 1e-8f) ? 1e-8f : amax;
    if (threadIdx.x == 0) a.ratio[t] = amax / a.safe_thresh;
    inv = 127.0f / amax;
  }
  if (VEC) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    const float4 *s4 = reinterpret_cast<const float4 *>(a.s);
    char4 *q4 = reinterpret_cast<char4 *>(q);
    for (int c = threadIdx.x; c < a.K / 4; c += kActThreads) {
      const float4 v = x4[c];
      char4 o;
      if (SMOOTH) {
        const float4 sv = s4[c];
        o.x = static_cast<signed char>(round_clamp(v.x * (sv.x * inv), 127.0f));
        o.y = static_cast<signed char>(round_clamp(v.y * (sv.y * inv), 127.0f));
        o.z = static_cast<signed char>(round_clamp(v.z * (sv.z * inv), 127.0f));
        o.w = static_cast<signed char>(round_clamp(v.w * (sv.w * inv), 127.0f));
      } else {
        o.x = static_cast<signed char>(round_clamp(v.x * inv, 127.0f));
        o.y = static_cast<signed char>(round_clamp(v.y * inv, 127.0f));
        o.z = static_cast<signed char>(round_clamp(v.z * inv, 127.0f));
        o.w = static_cast<signed char>(round_clamp(v.w * inv, 127.0f));
      }
      q4[c] = o;
      for (int p = 0; p < a.n_peers; ++p)
        reinterpret_cast<char4 *>(a.peers[p].q + (a.pub_row0 + t) * a.ldq)[c] = o;
    }
  } else {
    for (int c = threadIdx.x; c < a.K; c += kActThreads) {
      const float v = SMOOTH ? x[c] * (a.s[c] * inv) : x[c] * inv;
      const int8_t o = static_cast<int8_t>(round_clamp(v, 127.0f));
      q[c] = o;
      for (int p = 0; p < a.n_peers; ++p) a.peers[p].q[(a.pub_row0 + t) * a.ldq + c] = o;
    }
  }
  for (int c = a.K + threadIdx.x; c < a.k_fill; c += kActThreads) {
    q[c] = 0;
    for (int p = 0; p < a.n_peers; ++p) a.peers[p].q[(a.pub_row0 + t) * a.ldq + c] = 0;
  }
  if (a.pub_seq) publish_arrive(a);
}

// Dyntok quantisation with the token row held in registers (NV float4 of x, and of the
// smoothing factors, per thread): every load of the row is issued at once and x is read once
// from memory (act_quant_kernel reads it twice).  The same arithmetic, association and NaN rule
// as act_quant_kernel<true, SMOOTH, true>; for rows of K <= 4 * kActThreads * NV, no publication.
template <bool SMOOTH, int NV>
__global__ void __launch_bounds__(kActThreads) act_quant_dyn_rows_kernel(const ActArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const float4 *x4 = reinterpret_cast<const float4 *>(a.x + t * a.ldx);
  const float4 *s4 = reinterpret_cast<const float4 *>(a.s);
  const int n4 = a.K / 4;
  float4 v[NV], sv[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int c = threadIdx.x + u * kActThreads;
    v[u] = c < n4 ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (SMOOTH) sv[u] = c < n4 ? s4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __shared__ float s_part[kActThreads / 32];
  float amax = 0.0f;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    float4 m = v[u];
    if (SMOOTH) {
      m.x = v[u].x * sv[u].x; m.y = v[u].y * sv[u].y; m.z = v[u].z * sv[u].z; m.w = v[u].w * sv[u].w;
    }
    const float ax = fabsf(m.x), ay = fabsf(m.y), az = fabsf(m.z), aw = fabsf(m.w);
    if (ax > amax) amax = ax;
    if (ay > amax) amax = ay;
    if (az > amax) amax = az;
    if (aw > amax) amax = aw;
  }
  amax = warp_amax(amax);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.0f;
#pragma unroll
  for (int w = 0; w < kActThreads / 32; ++w) amax = s_part[w] > amax ? s_part[w] : amax;
  amax = (amax < 1e-8f) ? 1e-8f : amax;
  if (threadIdx.x == 0) a.ratio[t] = amax / a.safe_thresh;
  const float inv = 127.0f / amax;
  char4 *q4 = reinterpret_cast<char4 *>(a.q + t * a.ldq);
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int c = threadIdx.x + u * kActThreads;
    if (c >= n4) break;
    char4 o;
    if (SMOOTH) {
      o.x = static_cast<signed char>(round_clamp(v[u].x * (sv[u].x * inv), 127.0f));
      o.y = static_cast<signed char>(round_clamp(v[u].y * (sv[u].y * inv), 127.0f));
      o.z = static_cast<signed char>(round_clamp(v[u].z * (sv[u].z * inv), 127.0f));
      o.w = static_cast<signed char>(round_clamp(v[u].w * (sv[u].w * inv), 127.0f));
    } else {
      o.x = static_cast<signed char>(round_clamp(v[u].x * inv, 127.0f));
      o.y = static_cast<signed char>(round_clamp(v[u].y * inv, 127.0f));
      o.z = static_cast<signed char>(round_clamp(v[u].z * inv, 127.0f));
      o.w = static_cast<signed char>(round_clamp(v[u].w * inv, 127.0f));
    }
    q4[c] = o;
  }
  int8_t *q = a.q + t * a.ldq;
  for (int c = a.K + threadIdx.x; c < a.k_fill; c += kActThreads) q[c] = 0;
}

template <bool SMOOTH>
cudaError_t act_dyn_rows(const ActArgs &a, int T, int n4, cudaStream_t st, bool pdl) {
  const dim3 g(T), b(kActThreads);
  if (n4 <= 1 * kActThreads) return launch_ex(act_quant_dyn_rows_kernel<SMOOTH, 1>, g, b, 0, st, pdl, a);
  if (n4 <= 2 * kActThreads) return launch_ex(act_quant_dyn_rows_kernel<SMOOTH, 2>, g, b, 0, st, pdl, a);
  if (n4 <= 4 * kActThreads) return launch_ex(act_quant_dyn_rows_kernel<SMOOTH, 4>, g, b, 0, st, pdl, a);
  return launch_ex(act_quant_dyn_rows_kernel<SMOOTH, 8>, g, b, 0, st, pdl, a);
}

template <bool DYN, bool SMOOTH>
cudaError_t act_dispatch_vec(const ActArgs &a, int T, bool vec, cudaStream_t st, bool pdl) {
  if (vec) return launch_ex(act_quant_kernel<DYN, SMOOTH, true>, dim3(T), dim3(kActThreads), 0, st, pdl, a);
  return launch_ex(act_quant_kernel<DYN, SMOOTH, false>, dim3(T), dim3(kActThreads), 0, st, pdl, a);
}

__global__ void copy_pad_kernel(const int8_t *src, int64_t lds, int K, int8_t *dst, int64_t ldd,
                                int k_pad) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.y;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < k_pad; c += gridDim.x * blockDim.x)
    dst[t * ldd + c] = c < K ? src[t * lds + c] : static_cast<int8_t>(0);
}

struct UnpackArgs {
  const void *yq;
  int64_t ldyq;
  int in_i16, N, dyn;
  const float *ratio, *out_step;
  float *y;
  int64_t ldy;
};

__global__ void unpack_kernel(const UnpackArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.y;
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < a.N; n += gridDim.x * blockDim.x) {
    const int v = a.in_i16 ? static_cast<const int16_t *>(a.yq)[t * a.ldyq + n]
                           : static_cast<const int8_t *>(a.yq)[t * a.ldyq + n];
    const float step = a.dyn ? a.ratio[t] * a.out_step[n] : a.out_step[n];
    a.y[t * a.ldy + n] = static_cast<float>(v) * step;
  }
}

struct MergeArgs {
  const float *in_val;
  const int32_t *in_idx;
  int n_lists, k_in, k_out, P;
  int64_t list_stride, token_stride;
  float *out_val;
  int32_t *out_idx;
  int32_t *argmax;
  const unsigned *done;
  uint64_t remote_mask;
  const unsigned *pub_seq;
  int *err;
  unsigned long long *trace;
};

constexpr int kMergeWarps = 8;

// One CTA per token: the candidates' order keys into shared memory, then the warp-list top-k
// (topk.cuh) of all of them.
__global__ void __launch_bounds__(kMergeWarps * 32) topk_merge_kernel(const MergeArgs a) {
  extern __shared__ __align__(16) uint64_t keys[];
  uint64_t *stage = keys + a.P;  // kMergeWarps * 64 keys
  pdl_launch_dependents();
  pdl_wait();
  const bool tr = a.trace && blockIdx.x == 0 && threadIdx.x == 0;
  if (tr) a.trace[2] = global_timer_ns();
  if (a.done) {
    // lists stored by other devices: wait until each has reached this forward's count
    const unsigned e = *a.pub_seq;
    for (int s = threadIdx.x; s < 64; s += blockDim.x)
      if ((a.remote_mask >> s) & 1ull) wait_flag_reached(a.done + s, e, kWaitLimitNs, a.err, kDevPeerTimeout);
    __syncthreads();
  }
  if (tr) a.trace[3] = global_timer_ns();
  const int t = blockIdx.x;
  const int n = a.n_lists * a.k_in;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t off = t * a.token_stride + (i / a.k_in) * a.list_stride + (i % a.k_in);
    keys[i] = topk_key(a.in_val[off], static_cast<uint32_t>(a.in_idx[off]));
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto sync = [] { __syncthreads(); };
  if (a.k_out > 32)
    cta_top_keys<2, kMergeWarps>(keys, n, false, stage, warp, lane, sync);
  else
    cta_top_keys<1, kMergeWarps>(keys, n, false, stage, warp, lane, sync);
  if (warp == 0) {
    for (int e = lane; e < a.k_out; e += 32) {
      a.out_val[t * a.k_out + e] = topk_key_value(stage[e]);
      a.out_idx[t * a.k_out + e] = topk_key_id(stage[e]);
    }
    if (a.argmax && lane == 0) a.argmax[t] = topk_key_id(stage[0]);
  }
  if (tr) a.trace[4] = global_timer_ns();
}

}  // namespace

cudaError_t launch_act_quant(const ActQuantLaunch &L, cudaStream_t st) {
  ActArgs a{L.x,     L.ldx,   L.K,       L.k_fill,  L.inv_smooth, L.inv_step,  L.safe_thresh,
            L.q,     L.ldq,   L.ratio,   L.peers,   L.n_peers,    L.pub_seq,   L.pub_arrive,
            L.trace, L.pub_row0, L.emb_norm, L.eps};
  const bool vec = (L.K % 4 == 0) && (L.ldx % 4 == 0) && (L.ldq % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(L.x) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(L.q) % 4 == 0) &&
                   (L.inv_smooth == nullptr || reinterpret_cast<uintptr_t>(L.inv_smooth) % 16 == 0);
  if (L.emb_norm) {
    if (L.K > kEmbNormMaxK || L.act_mode != kActStatic) return cudaErrorInvalidValue;
    return launch_ex(emb_norm_pack_kernel, dim3(L.T), dim3(kActThreads),
                     static_cast<size_t>(L.K) * sizeof(float), st, L.pdl, a);
  }
  const bool dyn = L.act_mode == kActDyntok;
  const bool sm = L.inv_smooth != nullptr;
  // register-resident rows: vector layout, K <= 8192, no publication to other devices
  if (dyn && vec && L.n_peers == 0 && !L.pub_seq && L.K / 4 <= 8 * kActThreads)
    return sm ? act_dyn_rows<true>(a, L.T, L.K / 4, st, L.pdl) : act_dyn_rows<false>(a, L.T, L.K / 4, st, L.pdl);
  if (dyn && sm) return act_dispatch_vec<true, true>(a, L.T, vec, st, L.pdl);
  if (dyn) return act_dispatch_vec<true, false>(a, L.T, vec, st, L.pdl);
  if (sm) return act_dispatch_vec<false, true>(a, L.T, vec, st, L.pdl);
  return act_dispatch_vec<false, false>(a, L.T, vec, st, L.pdl);
}

cudaError_t launch_copy_pad_i8(const int8_t *src, int64_t lds, int T, int K, int8_t *dst,
                               int64_t ldd, int k_pad, bool pdl, cudaStream_t st) {
  const int bx = (k_pad + 255) / 256;
  return launch_ex(copy_pad_kernel, dim3(bx < 64 ? bx : 64, T), dim3(256), 0, st, pdl, src, lds, K,
                   dst, ldd, k_pad);
}

cudaError_t launch_unpack(const UnpackLaunch &L, cudaStream_t st) {
  UnpackArgs a{L.yq, L.ldyq, L.in_i16, L.N, L.act_mode == kActDyntok ? 1 : 0, L.ratio, L.out_step,
               L.y, L.ldy};
  const int bx = (L.N + 255) / 256;
  return launch_ex(unpack_kernel, dim3(bx < 256 ? bx : 256, L.T), dim3(256), 0, st, L.pdl, a);
}

cudaError_t launch_topk_merge(const MergeLaunch &L, cudaStream_t st) {
  // keys, rounded up to an even count, then the warp lists' staging area
  const int P = (L.n_lists * L.k_in + 1) & ~1;
  MergeArgs a{L.in_val,  L.in_idx,  L.n_lists, L.k_in,        L.k_out,   P,
              L.list_stride, L.token_stride, L.out_val, L.out_idx, L.argmax,
              L.done,    L.remote_mask, L.pub_seq, L.err,     L.trace};
  const size_t smem = (static_cast<size_t>(P) + kMergeWarps * 64) * 8;
  return launch_ex(topk_merge_kernel, dim3(L.T), dim3(kMergeWarps * 32), smem, st, L.pdl, a);
}

}  // namespace w8a8
