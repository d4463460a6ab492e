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
//   moe_swiglu_kernel   silu(gate) * up between the two expert projections (float); the layer
//                       runs it fused into the down projection's moe_act_quant_kernel.
//   moe_combine_kernel  mlp_out[t, c] += float(y_q[pair, c]) * (w_pair * out_step_chan[e, c]),
//                       accumulated over the token's pairs in slot order
//                       (src/LFM2.5-8B-A1B/lfm2_moe.cpp:2300-2318).
//
// A pair is one (token, slot): slots 0..k-1 are the routed experts of the token, the following
// ones the shared experts (weight 1).  Everything stays on the device; no host round trip
// between the router and the experts.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cmath>

namespace w8a8 {

namespace {

constexpr int kMoeThreads = 256;
constexpr int kRowsPerWarp = 8;
constexpr int kRowsPerCta = kRowsPerWarp * (kMoeThreads / 32);

// grid (ceil(E / 8), T).  Warp w of CTA (x, t) computes the logit of expert 8x + w for token t
// (16-byte loads, four partial sums per lane, warp-shuffle total) into logits[t, E]; the last CTA
// of token t to arrive (counter cnt[t], reset by that CTA) runs the reference's softmax and top-k
// with its first warp: max, exp and a double-precision sum across the lanes, then k rounds of a
// warp arg-max by (score desc, index asc) over the untaken experts.
template <bool VEC>
__global__ void __launch_bounds__(kMoeThreads) moe_route_kernel(const MoeRouteLaunch L) {
  extern __shared__ float s_route[];  // [E] logits, [E] scores (last CTA)
  __shared__ int s_last;
  const int t = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_launch_dependents();
  pdl_wait();
  const int e = blockIdx.x * (kMoeThreads / 32) + warp;
  if (e < L.E) {
    const float *hr = L.hidden + static_cast<int64_t>(t) * L.ldh;
    const float *wr = L.gate_w + static_cast<int64_t>(e) * L.H;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (VEC) {
      const float4 *h4 = reinterpret_cast<const float4 *>(hr);
      const float4 *w4 = reinterpret_cast<const float4 *>(wr);
      const int n4 = L.H >> 2;
#pragma unroll 4
      for (int i = lane; i < n4; i += 32) {
        const float4 x = __ldg(h4 + i), w = __ldg(w4 + i);
        acc[0] += w.x * x.x;
        acc[1] += w.y * x.y;
        acc[2] += w.z * x.z;
        acc[3] += w.w * x.w;
      }
    } else {
      for (int i = lane; i < L.H; i += 32) acc[i & 3] += __ldg(wr + i) * __ldg(hr + i);
    }
    float v = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if (lane == 0) L.logits[static_cast<int64_t>(t) * L.E + e] = L.bias ? v + L.bias[e] : v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(&L.cnt[t], 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!s_last || warp != 0) return;
  if (lane == 0) L.cnt[t] = 0;  // every CTA of token t has arrived
  __threadfence();
  const int E = L.E;
  float *logit = s_route, *score = s_route + E;
  for (int i = lane; i < E; i += 32) logit[i] = __ldcg(L.logits + static_cast<int64_t>(t) * E + i);
  __syncwarp();
  float mx = logit[0];
  for (int i = lane; i < E; i += 32) mx = logit[i] > mx ? logit[i] : mx;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float other = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
    mx = other > mx ? other : mx;
  }
  double sum = 0.0;
  for (int i = lane; i < E; i += 32) {
    score[i] = expf(logit[i] - mx);
    sum += score[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
  const float inv = sum > 0.0 ? static_cast<float>(1.0 / sum) : 1.0f;
  for (int i = lane; i < E; i += 32) {
    const float sc = sum > 0.0 ? score[i] * inv : score[i];
    score[i] = sc >= 0.0f ? sc : 0.0f;  // a NaN score ranks as 0, so every round finds an expert
  }
  __syncwarp();
  float wsum = 0.0f;
  for (int j = 0; j < L.k; ++j) {
    int best = -1;
    float bs = 0.0f;
    for (int i = lane; i < E; i += 32) {  // ascending i: strict > keeps the lower index on ties
      const float sc = score[i];
      if (sc >= 0.0f && (best < 0 || sc > bs)) {
        best = i;
        bs = sc;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const float os = __shfl_xor_sync(0xFFFFFFFFu, bs, o);
      if (ob >= 0 && (best < 0 || os > bs || (os == bs && ob < best))) {
        best = ob;
        bs = os;
      }
    }
    if (lane == 0) {
      L.idx[t * L.k + j] = best;
      L.w[t * L.k + j] = bs;
      score[best] = -1.0f;  // taken (probabilities are >= 0)
    }
    wsum += bs;
    __syncwarp();
  }
  if (lane == 0) {
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
  if (!DYN && L.swiglu_gu) {
    // SwiGLU fused: the same float steps as moe_swiglu_kernel, h kept for the stage views
    const float *g = L.swiglu_gu + static_cast<int64_t>(p) * 2 * L.K;
    float *h = L.src_out + static_cast<int64_t>(p) * L.K;
    for (int c = threadIdx.x; c < L.K; c += kMoeThreads) {
      const float gv = g[c];
      const float xv = (gv / (1.0f + expf(-gv))) * g[L.K + c];
      h[c] = xv;
      q[c] = static_cast<int8_t>(round_clamp(xv * (s[c] * inv), 127.0f));
    }
  } else {
    for (int c = threadIdx.x; c < L.K; c += kMoeThreads)
      q[c] = static_cast<int8_t>(round_clamp(x[c] * (s[c] * inv), 127.0f));
  }
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

constexpr int kGroupTokens = 8;   // pairs of one expert per CTA of the grouped GEMV

// One CTA: the pairs of every expert this rank owns, as lists (counting sort; the order inside an
// expert's list does not matter: every pair's outputs are computed independently), then the
// grouped GEMV's work items after the offsets: off[n_experts + 1] = their count, then one item
// e << 16 | z per block of up to 8 pairs of expert e, so that no CTA of that GEMV is launched
// for an empty block.
__global__ void __launch_bounds__(kMoeThreads) moe_group_kernel(const MoePairs P, int n_experts,
                                                               int32_t *off, int32_t *list) {
  // [n_experts] counts (then scatter cursors), [n_experts] list starts, [n_experts] first items
  extern __shared__ int s_cnt[];
  int *s_start = s_cnt + n_experts, *s_item = s_start + n_experts;
  pdl_launch_dependents();
  pdl_wait();
  for (int e = threadIdx.x; e < n_experts; e += kMoeThreads) s_cnt[e] = 0;
  __syncthreads();
  const int n = P.T * P.slots;
  for (int p = threadIdx.x; p < n; p += kMoeThreads) {
    const int e = pair_expert(P, p);
    if (expert_owned(P, e)) atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // prefix sums in shared memory
    int acc = 0, ni = 0;
    for (int e = 0; e < n_experts; ++e) {
      s_start[e] = acc;
      s_item[e] = ni;
      acc += s_cnt[e];
      ni += (s_cnt[e] + kGroupTokens - 1) / kGroupTokens;
    }
    off[n_experts] = acc;
    off[n_experts + 1] = ni;
  }
  __syncthreads();
  int32_t *items = off + n_experts + 2;
  for (int e = threadIdx.x; e < n_experts; e += kMoeThreads) {
    off[e] = s_start[e];
    const int nz = (s_cnt[e] + kGroupTokens - 1) / kGroupTokens;
    for (int z = 0; z < nz; ++z) items[s_item[e] + z] = (e << 16) | z;
    s_cnt[e] = s_start[e];  // this expert's scatter cursor (each expert has one thread here)
  }
  __syncthreads();
  for (int p = threadIdx.x; p < n; p += kMoeThreads) {
    const int e = pair_expert(P, p);
    if (expert_owned(P, e)) list[atomicAdd(&s_cnt[e], 1)] = p;
  }
}

constexpr int kGroupRows = 4;     // weight rows a warp streams together
constexpr int kGroupMaxK = 6144;  // widest staged row (kGroupTokens rows = 48 KB)

// Sums v[0..31] over the warp: afterwards lane l holds the total of value l.  Each halving step
// sends the half that the partner lane keeps (31 shuffles for 32 values).
__device__ __forceinline__ int warp_sum32(int (&v)[32], int lane) {
#pragma unroll
  for (int off = 16, c = 32; off >= 1; off >>= 1, c >>= 1) {
    const bool hi = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < c / 2; ++i) {
      const int send = hi ? v[i] : v[i + c / 2];
      const int keep = hi ? v[i + c / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// grid (ceil(N / 64), most work items).  CTA (rb, i) takes work item i (if there is one): pairs
// 8z .. 8z + 7 of expert e's list, stages their int8 rows in shared memory and streams its 64 weight rows once for all
// of them: each warp owns 8 rows, 4 at a time, each lane its 16-byte chunks of the 4 rows, dp4a
// against the 8 staged rows; the 32 sums of a pass are reduced together and lane l writes
// (row l / 8, pair l % 8) through the epilogue of moe_gemv_kernel.
__global__ void __launch_bounds__(kMoeThreads, 2) moe_gemv_grouped_kernel(const MoeGemvLaunch L) {
  extern __shared__ __align__(16) int4 s_x[];  // [kGroupTokens][chunks]
  pdl_launch_dependents();
  pdl_wait();
  const int32_t *items = L.grp_off + L.n_experts + 1;  // [0] count, then the items
  if (static_cast<int>(blockIdx.y) >= items[0]) return;
  const int item = items[1 + blockIdx.y];
  const int e = item >> 16;
  const int beg = L.grp_off[e] + (item & 0xffff) * kGroupTokens, end = L.grp_off[e + 1];
  if (beg >= end) return;
  const int ng = min(kGroupTokens, end - beg);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunks = L.k_pad >> 4;
  for (int i = threadIdx.x; i < kGroupTokens * chunks; i += kMoeThreads) {
    const int t = i / chunks, c = i % chunks;
    s_x[i] = t < ng ? *reinterpret_cast<const int4 *>(
                          L.q + static_cast<int64_t>(L.grp_pairs[beg + t]) * L.ldq + c * 16)
                    : make_int4(0, 0, 0, 0);
  }
  __syncthreads();
  const int8_t *W = L.w + static_cast<int64_t>(e) * L.N * L.k_pad;
  const int n0 = blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
  // this lane's (row, pair) of the reduced sums
  const int my_u = lane >> 3, my_t = lane & 7;
  const int my_p = my_t < ng ? L.grp_pairs[beg + my_t] : 0;
#pragma unroll 1
  for (int r = 0; r < kRowsPerWarp; r += kGroupRows) {
    if (n0 + r >= L.N) break;
    const int8_t *wr[kGroupRows];
#pragma unroll
    for (int u = 0; u < kGroupRows; ++u)  // rows past N re-read row N - 1; their sums are dropped
      wr[u] = W + static_cast<int64_t>(min(n0 + r + u, L.N - 1)) * L.k_pad;
    int acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0;
    // the next chunk's weight loads are issued before this chunk's products (two chunks of
    // loads in flight per lane)
    int4 wv[kGroupRows];
#pragma unroll
    for (int u = 0; u < kGroupRows; ++u)
      wv[u] = lane < chunks ? __ldg(reinterpret_cast<const int4 *>(wr[u] + lane * 16))
                            : make_int4(0, 0, 0, 0);
    for (int ci = lane; ci < chunks; ci += 32) {
      const int cn = ci + 32;
      int4 wn[kGroupRows];
#pragma unroll
      for (int u = 0; u < kGroupRows; ++u)
        wn[u] = cn < chunks ? __ldg(reinterpret_cast<const int4 *>(wr[u] + cn * 16))
                            : make_int4(0, 0, 0, 0);
#pragma unroll
      for (int t = 0; t < kGroupTokens; ++t) {
        const int4 xv = s_x[t * chunks + ci];
#pragma unroll
        for (int u = 0; u < kGroupRows; ++u) {
          int s = acc[u * kGroupTokens + t];
          s = __dp4a(wv[u].x, xv.x, s);
          s = __dp4a(wv[u].y, xv.y, s);
          s = __dp4a(wv[u].z, xv.z, s);
          s = __dp4a(wv[u].w, xv.w, s);
          acc[u * kGroupTokens + t] = s;
        }
      }
#pragma unroll
      for (int u = 0; u < kGroupRows; ++u) wv[u] = wn[u];
    }
    const int sum = warp_sum32(acc, lane);
    const int n = n0 + r + my_u;
    if (my_t < ng && n < L.N) {
      const int64_t pe = static_cast<int64_t>(e) * L.N + n;
      const int yq = requant_quantm(sum, L.quant_m[pe], L.trunc, L.qmax);
      const int64_t o = static_cast<int64_t>(my_p) * L.N + n;
      if (L.out_f32) {
        const float step = L.ratio ? L.ratio[my_p] * L.out_step[pe] : L.out_step[pe];
        static_cast<float *>(L.y)[o] = static_cast<float>(yq) * step;
      } else if (L.out_i16) {
        static_cast<int16_t *>(L.y)[o] = static_cast<int16_t>(yq);
      } else {
        static_cast<int8_t *>(L.y)[o] = static_cast<int8_t>(yq);
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
  if (L.E < 1 || L.H < 1 || L.T < 1 || L.k < 1 || L.k > L.E || !L.logits || !L.cnt)
    return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(2 * L.E) * sizeof(float);
  if (smem > 48 * 1024) return cudaErrorInvalidValue;  // more than 6144 experts
  const bool vec = L.H % 4 == 0 && L.ldh % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(L.hidden) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(L.gate_w) % 16 == 0;
  const dim3 grid((L.E + kMoeThreads / 32 - 1) / (kMoeThreads / 32), L.T);
  if (vec) return launch_ex(moe_route_kernel<true>, grid, dim3(kMoeThreads), smem, st, L.pdl, L);
  return launch_ex(moe_route_kernel<false>, grid, dim3(kMoeThreads), smem, st, L.pdl, L);
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

cudaError_t launch_moe_group(const MoePairs &P, int n_experts, int32_t *off, int32_t *pairs,
                             bool pdl, cudaStream_t st) {
  return launch_ex(moe_group_kernel, dim3(1), dim3(kMoeThreads),
                   3 * static_cast<size_t>(n_experts) * sizeof(int), st, pdl, P, n_experts, off,
                   pairs);
}

cudaError_t launch_moe_gemv_grouped(const MoeGemvLaunch &L, cudaStream_t st) {
  if (L.k_pad <= 0 || L.k_pad % 16 != 0 || L.n_experts <= 0) return cudaErrorInvalidValue;
  if (L.k_pad > kGroupMaxK) return launch_moe_gemv(L, st);  // rows too wide to stage: per pair
  // one CTA row per work item that launch_moe_group can have written
  const dim3 grid((L.N + kRowsPerCta - 1) / kRowsPerCta,
                  moe_max_group_items(L.n_experts, L.pairs.T * L.pairs.slots));
  if (grid.y > 65535u) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(kGroupTokens) * L.k_pad;
  return launch_ex(moe_gemv_grouped_kernel, grid, dim3(kMoeThreads), smem, st, L.pdl, L);
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
