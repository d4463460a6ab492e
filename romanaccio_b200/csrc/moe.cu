// Mixture-of-experts decode kernels: router, per-(token, expert) W8A8 expert GEMVs and the
// weighted combine of the experts' requantised outputs.
//
//   moe_route_kernel    MoERouter::route (src/eswin_runtime/src/llm/moe_router.cpp:211-260):
//                       logits = W_gate . h (+ bias), softmax with the max subtracted, exp in
//                       float and the sum in double (scores_from_logits, :108-130), top-k in the
//                       order (score desc, expert index asc), weights = raw probabilities unless
//                       norm_topk_prob (no renormalisation for DeepSeek-V2-Lite), times
//                       routed_scaling_factor.
//   moe_act_quant_kernel pack_npu_input_int8[_dyntok] (src/LFM3/lfm3_v2.cpp:892-940, 1050-1141)
//                       of each pair's token row with the pair's expert smoothing vector.
//   moe_gemv_kernel     the W8A8 contraction of each pair's token against its expert's weights
//                       with the SDP requant epilogue (QuantM, RNE shift, saturate), then either
//                       the unpack (F32) or the int16/int8 requantised value (QUANT).
//   moe_swiglu_kernel   silu(gate) * up between the two expert projections (float).
//   moe_combine_kernel  mlp_out[t, c] += float(y_q[pair, c]) * (w_pair * out_step_chan[e, c]),
//                       accumulated over the token's pairs in slot order
//                       (src/LFM2.5-8B-A1B/lfm2_moe.cpp:2300-2318).
//
// A pair is one (token, slot): slots 0..k-1 are the routed experts of the token, the following
// ones the shared experts (weight 1).  Everything stays on the device; no host round trip
// between the router and the experts.
#include "common.cuh"
#include "kernels.h"

#include <cmath>

namespace w8a8 {

namespace {

constexpr int kMoeThreads = 256;
constexpr int kRowsPerWarp = 8;
constexpr int kRowsPerCta = kRowsPerWarp * (kMoeThreads / 32);

// One CTA per token.  Warp w computes the logits of experts w, w + 8, ... (lane-strided partial
// sums reduced across the warp); thread 0 then runs the reference's softmax and top-k serially
// (at most a few hundred experts).
__global__ void __launch_bounds__(kMoeThreads) moe_route_kernel(const MoeRouteLaunch L) {
  extern __shared__ float s_route[];
  float *h = s_route;                 // [H]
  float *logit = s_route + L.H;       // [E]
  float *score = logit + L.E;         // [E]
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  for (int i = tid; i < L.H; i += kMoeThreads) h[i] = L.hidden[static_cast<int64_t>(t) * L.ldh + i];
  __syncthreads();
  for (int e = warp; e < L.E; e += kMoeThreads / 32) {
    const float *w = L.gate_w + static_cast<int64_t>(e) * L.H;
    float acc = 0.0f;
    for (int i = lane; i < L.H; i += 32) acc += w[i] * h[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) logit[e] = L.bias ? acc + L.bias[e] : acc;
  }
  __syncthreads();
  if (tid == 0) {
    const int E = L.E;
    float mx = logit[0];
    for (int e = 1; e < E; ++e)
      if (logit[e] > mx) mx = logit[e];
    double sum = 0.0;
    for (int e = 0; e < E; ++e) {
      score[e] = expf(logit[e] - mx);
      sum += score[e];
    }
    if (sum > 0.0) {
      const float inv = static_cast<float>(1.0 / sum);
      for (int e = 0; e < E; ++e) score[e] *= inv;
    }
    // top-k by (score desc, index asc): k passes of a max scan over the untaken experts
    float wsum = 0.0f;
    for (int j = 0; j < L.k; ++j) {
      int best = -1;
      for (int e = 0; e < E; ++e) {
        if (score[e] < 0.0f) continue;  // taken (probabilities are >= 0)
        if (best < 0 || score[e] > score[best]) best = e;
      }
      L.idx[t * L.k + j] = best;
      L.w[t * L.k + j] = score[best];
      wsum += score[best];
      score[best] = -1.0f;
    }
    if (L.norm_topk && wsum > 0.0f) {
      const float inv = 1.0f / wsum;
      for (int j = 0; j < L.k; ++j) L.w[t * L.k + j] *= inv;
    }
    if (L.scaling != 1.0f)
      for (int j = 0; j < L.k; ++j) L.w[t * L.k + j] *= L.scaling;
  }
}

__device__ __forceinline__ int pair_expert(const MoePairs &P, int p) {
  const int t = p / P.slots, j = p % P.slots;
  return j < P.k ? P.routed_idx[t * P.k + j] : P.n_routed + (j - P.k);
}

// Whether this rank computes expert e (expert parallelism: e % world == rank).
__device__ __forceinline__ bool expert_owned(const MoePairs &P, int e) {
  return P.own_world <= 1 || e % P.own_world == P.own_rank;
}

// One CTA per pair: x = src[token or pair row], smoothed by the pair's expert vector.
template <bool DYN>
__global__ void __launch_bounds__(kMoeThreads) moe_act_quant_kernel(const MoeActLaunch L) {
  pdl_launch_dependents();
  pdl_wait();
  const int p = blockIdx.x;
  const int e = pair_expert(L.pairs, p);
  if (!expert_owned(L.pairs, e)) return;  // another rank's expert
  const int row = L.per_pair_rows ? p : p / L.pairs.slots;
  const float *x = L.src + static_cast<int64_t>(row) * L.ld;
  const float *s = L.inv_smooth + static_cast<int64_t>(e) * L.K;
  int8_t *q = L.q + static_cast<int64_t>(p) * L.ldq;
  float inv = L.inv_step ? L.inv_step[e] : 0.0f;
  if (DYN) {
    __shared__ float s_part[kMoeThreads / 32];
    float amax = 0.0f;
    for (int c = threadIdx.x; c < L.K; c += kMoeThreads) {
      const float v = fabsf(x[c] * s[c]);
      if (v > amax) amax = v;
    }
    amax = warp_amax(amax);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.0f;
#pragma unroll
    for (int w = 0; w < kMoeThreads / 32; ++w) amax = s_part[w] > amax ? s_part[w] : amax;
    amax = (amax < 1e-8f) ? 1e-8f : amax;
    if (threadIdx.x == 0) L.ratio[p] = amax / L.safe_thresh[e];
    inv = 127.0f / amax;
  }
  for (int c = threadIdx.x; c < L.K; c += kMoeThreads)
    q[c] = static_cast<int8_t>(round_clamp(x[c] * (s[c] * inv), 127.0f));
  for (int c = L.K + threadIdx.x; c < L.ldq; c += kMoeThreads) q[c] = 0;
}

// grid (ceil(N / 64), pairs).  Warp w of the CTA owns 8 consecutive rows of the pair's expert;
// each lane holds its 16-byte chunks of the pair's int8 row in registers and streams the
// matching chunks of every weight row (two rows at a time for independent loads).
template <int MAXC>
__global__ void __launch_bounds__(kMoeThreads) moe_gemv_kernel(const MoeGemvLaunch L) {
  pdl_launch_dependents();
  pdl_wait();
  const int p = blockIdx.y;
  const int e = pair_expert(L.pairs, p);
  if (!expert_owned(L.pairs, e)) return;  // another rank's expert
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunks = L.k_pad >> 4;  // 16-byte chunks per row
  const int8_t *xq = L.q + static_cast<int64_t>(p) * L.ldq;
  int4 xv[MAXC];
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int ci = lane + 32 * c;
    xv[c] = ci < chunks ? *reinterpret_cast<const int4 *>(xq + ci * 16) : make_int4(0, 0, 0, 0);
  }
  const int8_t *W = L.w + static_cast<int64_t>(e) * L.N * L.k_pad;
  const int n0 = blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
#pragma unroll 1
  for (int r = 0; r < kRowsPerWarp; r += 2) {
    int acc[2] = {0, 0};
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int n = n0 + r + u;
      if (n >= L.N) continue;
      const int8_t *wr = W + static_cast<int64_t>(n) * L.k_pad;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int ci = lane + 32 * c;
        if (ci < chunks) {
          const int4 wv = __ldg(reinterpret_cast<const int4 *>(wr + ci * 16));
          int s = acc[u];
          s = __dp4a(wv.x, xv[c].x, s);
          s = __dp4a(wv.y, xv[c].y, s);
          s = __dp4a(wv.z, xv[c].z, s);
          s = __dp4a(wv.w, xv[c].w, s);
          acc[u] = s;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int n = n0 + r + u;
      const int s = warp_sum(acc[u]);
      if (lane == 0 && n < L.N) {
        const int64_t pe = static_cast<int64_t>(e) * L.N + n;
        const int yq = requant_quantm(s, L.quant_m[pe], L.trunc, L.qmax);
        const int64_t o = static_cast<int64_t>(p) * L.N + n;
        if (L.out_f32) {
          const float step = L.ratio ? L.ratio[p] * L.out_step[pe] : L.out_step[pe];
          static_cast<float *>(L.y)[o] = static_cast<float>(yq) * step;
        } else if (L.out_i16) {
          static_cast<int16_t *>(L.y)[o] = static_cast<int16_t>(yq);
        } else {
          static_cast<int8_t *>(L.y)[o] = static_cast<int8_t>(yq);
        }
      }
    }
  }
}

// h[p, i] = silu(gu[p, i]) * gu[p, I + i], silu(g) = g / (1 + exp(-g)).
__global__ void __launch_bounds__(kMoeThreads) moe_swiglu_kernel(const float *gu, int I, int pairs,
                                                                 float *h, const MoePairs P) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = static_cast<int64_t>(pairs) * I;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kMoeThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kMoeThreads) {
    const int64_t p = i / I, c = i % I;
    if (!expert_owned(P, pair_expert(P, static_cast<int>(p)))) continue;
    const float g = gu[p * 2 * I + c];
    const float u = gu[p * 2 * I + I + c];
    h[i] = (g / (1.0f + expf(-g))) * u;
  }
}

// out[t, c] = sum over the token's slots j (in order, from 0.0f) of
// float(yq[p, c]) * (w_j * out_step_chan[e_j, c]).
__global__ void __launch_bounds__(kMoeThreads) moe_combine_kernel(const MoeCombineLaunch L) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.y;
  for (int c = blockIdx.x * kMoeThreads + threadIdx.x; c < L.H; c += gridDim.x * kMoeThreads) {
    float acc = 0.0f;
    for (int j = 0; j < L.pairs.slots; ++j) {
      const int p = t * L.pairs.slots + j;
      const int e = pair_expert(L.pairs, p);
      if (!expert_owned(L.pairs, e)) continue;  // summed by its owner
      const float w = j < L.pairs.k ? L.pairs.routed_w[t * L.pairs.k + j] : 1.0f;
      const int64_t o = static_cast<int64_t>(p) * L.H + c;
      const float v = L.in_i16 ? static_cast<float>(static_cast<const int16_t *>(L.yq)[o])
                               : static_cast<float>(static_cast<const int8_t *>(L.yq)[o]);
      acc += v * (w * L.out_step[static_cast<int64_t>(e) * L.H + c]);
    }
    L.out[static_cast<int64_t>(t) * L.ldo + c] = acc;
  }
}

// Expert-parallel exchange, step 1: this rank's partial [T, H] into buffer (e & 1), list `rank`,
// of every rank's gather (peer stores; e = this forward's number), then the last CTA to arrive
// counts the forward and stores it into done[rank] on every rank (system-scope fence + relaxed
// stores: a release of the rows).
__global__ void __launch_bounds__(kMoeThreads) moe_ep_publish_kernel(const MoeEpLaunch L) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ unsigned s_e;
  __shared__ int s_last;
  if (threadIdx.x == 0) s_e = *L.pub_seq + 1u;
  __syncthreads();
  const unsigned e = s_e;
  const int t = blockIdx.y;
  const int c = blockIdx.x * kMoeThreads + threadIdx.x;
  if (c < L.H) {
    const float v = L.partial[static_cast<int64_t>(t) * L.H + c];
    const int64_t off =
        ((static_cast<int64_t>(e & 1u) * L.world + L.rank) * L.max_T + t) * L.H + c;
    for (int p = 0; p < L.world; ++p) L.dst[p][off] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(L.pub_arrive, 1u) == gridDim.x * gridDim.y - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence_system();
    *L.pub_seq = e;
    *L.pub_arrive = 0u;
    for (int p = 0; p < L.world; ++p) st_relaxed_sys(L.done[p], e);
  }
}

// Step 2: once every other rank's partial of this forward has arrived (bounded waits), the
// layer output out[t, c] = sum over ranks in rank order (from 0.0f) of the partials -- the
// reference's per-die partial sums added die after die (lfm2_moe.cpp:2432).
__global__ void __launch_bounds__(kMoeThreads) moe_ep_sum_kernel(const MoeEpLaunch L) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned e = *L.pub_seq;  // bumped by this rank's publication (stream order)
  if (threadIdx.x < 32) {
    for (int p = threadIdx.x; p < L.world; p += 32)
      if (p != L.rank) wait_flag_reached(L.done_here + p, e, kWaitLimitNs, L.err, kDevPeerTimeout);
  }
  __syncthreads();
  const int t = blockIdx.y;
  const int c = blockIdx.x * kMoeThreads + threadIdx.x;
  if (c >= L.H) return;
  const float *g = L.gather + static_cast<int64_t>(e & 1u) * L.world * L.max_T * L.H;
  float acc = 0.0f;
  for (int p = 0; p < L.world; ++p) acc += g[(static_cast<int64_t>(p) * L.max_T + t) * L.H + c];
  L.out[static_cast<int64_t>(t) * L.ldo + c] = acc;
}

}  // namespace

cudaError_t launch_moe_ep_publish(const MoeEpLaunch &L, cudaStream_t st) {
  const int bx = (L.H + kMoeThreads - 1) / kMoeThreads;
  return launch_ex(moe_ep_publish_kernel, dim3(bx, L.T), dim3(kMoeThreads), 0, st, L.pdl, L);
}

cudaError_t launch_moe_ep_sum(const MoeEpLaunch &L, cudaStream_t st) {
  const int bx = (L.H + kMoeThreads - 1) / kMoeThreads;
  return launch_ex(moe_ep_sum_kernel, dim3(bx, L.T), dim3(kMoeThreads), 0, st, L.pdl, L);
}

cudaError_t launch_moe_route(const MoeRouteLaunch &L, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(L.H + 2 * L.E) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(moe_route_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  return launch_ex(moe_route_kernel, dim3(L.T), dim3(kMoeThreads), smem, st, L.pdl, L);
}

cudaError_t launch_moe_act_quant(const MoeActLaunch &L, bool dyn, cudaStream_t st) {
  const int P = L.pairs.T * L.pairs.slots;
  if (dyn) return launch_ex(moe_act_quant_kernel<true>, dim3(P), dim3(kMoeThreads), 0, st, L.pdl, L);
  return launch_ex(moe_act_quant_kernel<false>, dim3(P), dim3(kMoeThreads), 0, st, L.pdl, L);
}

cudaError_t launch_moe_gemv(const MoeGemvLaunch &L, cudaStream_t st) {
  const int P = L.pairs.T * L.pairs.slots;
  const dim3 grid((L.N + kRowsPerCta - 1) / kRowsPerCta, P);
  const int chunks = L.k_pad / 16;
  if (chunks <= 32 * 4)
    return launch_ex(moe_gemv_kernel<4>, grid, dim3(kMoeThreads), 0, st, L.pdl, L);
  if (chunks <= 32 * 8)
    return launch_ex(moe_gemv_kernel<8>, grid, dim3(kMoeThreads), 0, st, L.pdl, L);
  return cudaErrorInvalidValue;  // K above 4096 is not an expert shape here
}

cudaError_t launch_moe_swiglu(const float *gu, int I, int pairs, float *h, bool pdl,
                              cudaStream_t st, const MoePairs &P) {
  const int64_t total = static_cast<int64_t>(pairs) * I;
  int blocks = static_cast<int>((total + kMoeThreads - 1) / kMoeThreads);
  if (blocks > 4096) blocks = 4096;
  return launch_ex(moe_swiglu_kernel, dim3(blocks), dim3(kMoeThreads), 0, st, pdl, gu, I, pairs,
                   h, P);
}

cudaError_t launch_moe_combine(const MoeCombineLaunch &L, cudaStream_t st) {
  const int bx = (L.H + kMoeThreads - 1) / kMoeThreads;
  return launch_ex(moe_combine_kernel, dim3(bx, L.pairs.T), dim3(kMoeThreads), 0, st, L.pdl, L);
}

}  // namespace w8a8
