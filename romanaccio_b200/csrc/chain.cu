// Persistent decode-chain kernel: a whole sequence of W8A8 linears (and optionally the LM-head
// shard with its top-k) in ONE cooperative launch.
//
// It replaces the per-token sequence of NPU submits of the reference's decode loop
// (Lfm3Engine::forward_chunk, src/LFM3/lfm3_v2.cpp:1743-1990; TransformerSession::step,
// src/eswin_runtime/src/llm/transformer_session.cpp:650-844), where every linear is a separate
// pack -> submit_task -> unpack round trip with ~0.41 ms of fixed overhead (FINDINGS.md:1883).
//
// One CTA per SM, 8 consumer warps + 1 producer warp.  The producer warp streams the int8
// weight slabs of every step this CTA owns, step after step, through an NS-deep shared-memory
// ring with 1-D bulk copies (TMA engine, no tensor map, one CTA per copy) completing on mbarriers.
// Weights do not depend on activations, so the producer runs ahead into the next linears while
// the consumers are still busy or waiting: HBM never idles at a linear boundary.  Consumers,
// per step: wait at a grid barrier when the step reads an earlier step's output, quantise the
// step's fp32 input into shared memory (dyntok amax / static step, the reference's
// pack_npu_input_int8[_dyntok] arithmetic), run dp4a over the landed slabs, and apply the
// requant / unpack epilogue (or keep LM-head logits on chip for the grid top-k of topk.cuh).
// The grid barrier is a per-step arrival counter (release: fence + atomic add; acquire:
// ld.acquire spin, bounded by 2 s of %globaltimer).
#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

#include <algorithm>

namespace w8a8 {

namespace {

constexpr int kCW = 8;              // consumer warps
constexpr int kCT = kCW * 32;       // consumer threads
constexpr int kThreads = kCT + 32;  // + producer warp
constexpr int kMaxStages = 8;
// Weight stages in flight per CTA.  When a CTA streams little per dependent step (latency-bound
// chains), two stages of ~24 KB beat a deeper ring: bytes queued in the memory system lengthen
// every L2 round trip on the step-to-step critical path (the arrival fence, the counter poll, the
// activation read) more than they add overlap (28-layer Qwen2.5-1.5B-shaped step, ~47 KB per CTA
// per step: 688 us at two stages against 723 us at four).  Chains streaming more per step keep
// every stage that fits (48-layer Gemma-12B-shaped step, ~200 KB: 2716 us at four against 2990 us
// at two).
constexpr int kLatencyRingStages = 2;
constexpr size_t kDeepRingBytesPerStep = 96 * 1024;  // weight bytes per CTA per step
// activation float4 loads in flight per thread in quantise_input (more registers at TT = 1,
// fewer at TT = 8, whose accumulators and activation vectors leave less room)
template <int TT>
__host__ __device__ constexpr int quant_batch() { return TT == 1 ? 5 : TT == 8 ? 3 : 4; }

struct ChainArgs {
  const ChainOp *ops;
  int n_ops;
  int T;
  unsigned *bar;      // [n_ops] arrival counters, zero at launch
  unsigned *tk_counter;  // top-k arrival counter (zero between launches)
  uint64_t *lists;       // [T][grid * (k + 1)] top-k lists, then heads
  int *err;
  int ns;
  uint32_t stage_bytes;
  int kpad_max;
  int cand_cap;
  int max_rows;       // most rows one CTA owns in any step (epilogue parameter staging)
  uint32_t ring_bytes;
  int norm_floats;    // fp32 staging row of a kActEmbNorm step (0: none)
  uint32_t xq_off, cand_off, bars_off, ep_off, norm_off;  // ChainPlan's shared-memory layout
  unsigned long long *trace;  // optional [grid][n_ops][8] %globaltimer stamps
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void split_range(int total, int parts, int idx, int &b, int &e) {
  b = static_cast<int>((static_cast<long long>(total) * idx) / parts);
  e = static_cast<int>((static_cast<long long>(total) * (idx + 1)) / parts);
}

// Quantises the step's fp32 input [T, K] into xq [TT][kpad_max] (zero past K) and the per-token
// ratio / inverse step, exactly as pack_npu_input_int8[_dyntok].
// When the step that produced x already reduced max_c |x*s| per token (amax_src), x is read
// once; otherwise (the chain's external input) once for the amax and once to quantise.
__device__ __forceinline__ char4 quant4(const float4 v, const float4 sv, bool smooth, float inv,
                                        bool emb = false) {
  char4 o;
  if (smooth) {
    // smoothing: x * (s * inv) == (s * inv) * x; RMSNorm pack (emb): (x * inv_rms) * emb[c]
    const float4 p = emb ? v : sv, r = emb ? sv : v;
    o.x = static_cast<signed char>(round_clamp(p.x * inv * r.x, 127.0f));
    o.y = static_cast<signed char>(round_clamp(p.y * inv * r.y, 127.0f));
    o.z = static_cast<signed char>(round_clamp(p.z * inv * r.z, 127.0f));
    o.w = static_cast<signed char>(round_clamp(p.w * inv * r.w, 127.0f));
  } else {
    o.x = static_cast<signed char>(round_clamp(v.x * inv, 127.0f));
    o.y = static_cast<signed char>(round_clamp(v.y * inv, 127.0f));
    o.z = static_cast<signed char>(round_clamp(v.z * inv, 127.0f));
    o.w = static_cast<signed char>(round_clamp(v.w * inv, 127.0f));
  }
  return o;
}

// Smoothing factors of this thread's first 4 float4 columns, loaded before the grid barrier
// (they do not depend on the previous step).
__device__ __forceinline__ void preload_smooth(const ChainOp &op, int tid, float4 (&s_pre)[4]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) s_pre[u] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (!op.vec_x || !op.inv_smooth) return;
  const int n4 = op.K / 4;
  const float4 *s4 = reinterpret_cast<const float4 *>(op.inv_smooth);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int c = tid + u * kCT;
    if (c < n4) s_pre[u] = s4[c];
  }
}

// kActEmbNorm (the LM head's input, fused_emb_norm_broadcast_t1, src/LFM3/lfm3_v2.cpp:810-831):
// inv_rms per token into s_inv.  The row is staged in shared memory (xs); four threads form the
// reference's interleaved sums of squares s0..s3 (column c into s_{c mod 4}, in column order) and
// one thread adds (s0 + s1) + (s2 + s3) and the K mod 4 tail: inv_rms = 1 / sqrt(sum / K + eps).
// The pack itself is the static one with the product taken as (x * inv_rms) * emb_norm_scaled[c].
__device__ void emb_norm_inv(const ChainOp &op, int T, float *xs, float *s_inv, int tid) {
  __shared__ float s_sq[4];
  const int K = op.K, K4 = K & ~3;
  for (int t = 0; t < T; ++t) {
    const float *xr = op.x + t * op.ldx;
    if (op.vec_x) {
      const float4 *x4 = reinterpret_cast<const float4 *>(xr);
      for (int c = tid; c < K / 4; c += kCT) reinterpret_cast<float4 *>(xs)[c] = __ldcg(x4 + c);
    } else {
      for (int c = tid; c < K; c += kCT) xs[c] = __ldcg(xr + c);
    }
    consumer_sync();
    if (tid < 4) {
      float sum = 0.0f;
#pragma unroll 8
      for (int c = tid; c < K4; c += 4) sum += xs[c] * xs[c];
      s_sq[tid] = sum;
    }
    __syncwarp();
    if (tid == 0) {
      float sum = (s_sq[0] + s_sq[1]) + (s_sq[2] + s_sq[3]);
      for (int c = K4; c < K; ++c) sum += xs[c] * xs[c];
      s_inv[t] = 1.0f / sqrtf(sum / static_cast<float>(K) + op.norm_eps);
    }
    consumer_sync();  // s_inv[t] visible; xs is restaged for the next token
  }
}

template <int TT>
__device__ void quantise_input(const ChainOp &op, int T, int8_t *xq, int kpad_max, float *s_ratio,
                               float *s_inv, float (*s_part)[TT], int tid,
                               const float4 (&s_pre)[4], float *xs) {
  const int warp = tid >> 5, lane = tid & 31;
  const bool vec = op.vec_x;
  const bool emb = op.act_mode == kActEmbNorm;
  float inv_r[TT];
  // amax already reduced by the producing step: every thread derives the inverse steps itself
  // (no barrier before the x pass).  The loads are issued here; the divisions wait until the
  // first activation loads of the token are in flight (see `lazy` below), so the two L2 round
  // trips overlap.
  const bool lazy = op.act_mode == kActDyntok && op.amax_src != nullptr;
  if (lazy) {
#pragma unroll
    for (int t = 0; t < TT; ++t) inv_r[t] = t < T ? __ldcg(op.amax_src + t) : 1.0f;
  } else if (op.act_mode == kActDyntok) {
    float amax[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) amax[t] = 0.0f;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (t >= T) break;
      const float *xr = op.x + t * op.ldx;
      if (vec) {
        const int n4 = op.K / 4;
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        const float4 *s4 = reinterpret_cast<const float4 *>(op.inv_smooth);
        for (int c0 = tid; c0 < n4; c0 += 4 * kCT) {
          float4 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = c0 + u * kCT;
            v[u] = c < n4 ? __ldcg(x4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = c0 + u * kCT;
            if (c >= n4) continue;
            float4 m = v[u];
            if (op.inv_smooth) {
              const float4 sv = s4[c];
              m.x = m.x * sv.x; m.y = m.y * sv.y; m.z = m.z * sv.z; m.w = m.w * sv.w;
            }
            const float a0 = fabsf(m.x), a1 = fabsf(m.y), a2 = fabsf(m.z), a3 = fabsf(m.w);
            if (a0 > amax[t]) amax[t] = a0;
            if (a1 > amax[t]) amax[t] = a1;
            if (a2 > amax[t]) amax[t] = a2;
            if (a3 > amax[t]) amax[t] = a3;
          }
        }
      } else {
        for (int c = tid; c < op.K; c += kCT) {
          const float v = __ldcg(xr + c);
          const float a = op.inv_smooth ? fabsf(v * op.inv_smooth[c]) : fabsf(v);
          if (a > amax[t]) amax[t] = a;
        }
      }
      const float m = warp_amax(amax[t]);
      if (lane == 0) s_part[warp][t] = m;
    }
    consumer_sync();
    if (tid < T) {
      float m = 0.0f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) m = s_part[w][tid] > m ? s_part[w][tid] : m;
      m = (m < 1e-8f) ? 1e-8f : m;
      s_ratio[tid] = m / op.safe_thresh;
      s_inv[tid] = 127.0f / m;
    }
    consumer_sync();
#pragma unroll
    for (int t = 0; t < TT; ++t) inv_r[t] = t < T ? s_inv[t] : 0.0f;
  } else {
    if (tid < T) s_ratio[tid] = 1.0f;
    if (emb) emb_norm_inv(op, T, xs, s_inv, tid);
#pragma unroll
    for (int t = 0; t < TT; ++t) inv_r[t] = emb ? (t < T ? s_inv[t] : 0.0f) : op.inv_step;
  }
  // the reference's amax floor, ratio and inverse step from a reduced amax
  auto derive = [&](int t, float m) {
    m = (m < 1e-8f) ? 1e-8f : m;
    if (tid == t) s_ratio[t] = m / op.safe_thresh;
    return 127.0f / m;
  };
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    if (t >= T) break;
    float inv = inv_r[t];
    bool pending = lazy;
    const float *xr = op.x + t * op.ldx;
    int8_t *q = xq + t * kpad_max;
    if (vec) {
      // QB independent 16-byte loads (and their smoothing factors) in flight per thread before
      // any use: K = 8960 takes two batches of L2 round trips instead of three
      const int n4 = op.K / 4;
      const bool smooth = op.inv_smooth != nullptr;
      const float4 *x4 = reinterpret_cast<const float4 *>(xr);
      const float4 *s4 = reinterpret_cast<const float4 *>(op.inv_smooth);
      constexpr int QB = quant_batch<TT>();
      for (int c0 = tid; c0 < n4; c0 += QB * kCT) {
        float4 v[QB], sv[QB];
#pragma unroll
        for (int u = 0; u < QB; ++u) {
          const int c = c0 + u * kCT;
          v[u] = c < n4 ? __ldcg(x4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
          sv[u] = (c0 == tid && u < 4)
                      ? s_pre[u & 3]
                      : ((smooth && c < n4) ? s4[c] : make_float4(0.f, 0.f, 0.f, 0.f));
        }
        if (pending) {
          inv = derive(t, inv_r[t]);
          pending = false;
        }
#pragma unroll
        for (int u = 0; u < QB; ++u) {
          const int c = c0 + u * kCT;
          if (c < n4) reinterpret_cast<char4 *>(q)[c] = quant4(v[u], sv[u], smooth, inv, emb);
        }
      }
      if (pending) inv = derive(t, inv_r[t]);  // (this thread had no column)
      for (int c = (op.K & ~3) + tid; c < op.k_pad; c += kCT) q[c] = 0;
    } else {
      if (pending) inv = derive(t, inv_r[t]);
      for (int c = tid; c < op.k_pad; c += kCT) {
        int8_t v = 0;
        if (c < op.K) {
          const float xv = __ldcg(xr + c);
          const float y = emb ? xv * inv * op.inv_smooth[c]
                              : (op.inv_smooth ? xv * (op.inv_smooth[c] * inv) : xv * inv);
          v = static_cast<int8_t>(round_clamp(y, 127.0f));
        }
        q[c] = v;
      }
    }
  }
  consumer_sync();
}

// Per-row epilogue parameters of the CTA's rows of the current step, in shared memory.
__host__ __device__ constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v >> 1); }

// Sums of NV (a power of two <= 32) per-lane values over the warp.  Each halving step sends the
// half of the values that the partner lane keeps (offsets 16, 8, ...), then the remaining
// offsets add whole: lane l ends with the total of value l >> (5 - log2 NV), in
// NV - 1 + 5 - log2 NV shuffles instead of 5 NV.
template <int NV>
__device__ __forceinline__ int warp_sum_multi(int (&v)[NV], int lane) {
  constexpr int kSteps = ilog2(NV);
#pragma unroll
  for (int step = 0; step < kSteps; ++step) {
    const int off = 16 >> step;
    const int c = NV >> step;
    const bool hi = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < c / 2; ++i) {
      const int send = hi ? v[i] : v[i + c / 2];
      const int keep = hi ? v[i + c / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, off);
    }
  }
#pragma unroll
  for (int off = 16 >> kSteps; off > 0; off >>= 1) v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], off);
  return v[0];
}

// Position in the weight ring: slot = it % ns and phase = (it / ns) & 1 of the ring iteration
// it, advanced incrementally (no integer division on the per-stage path).
struct RingPos {
  int slot = 0;
  uint32_t phase = 0;
  bool lapped = false;  // it >= ns: the slot has been filled before
  __device__ __forceinline__ void advance(int ns) {
    if (++slot == ns) {
      slot = 0;
      phase ^= 1u;
      lapped = true;
    }
  }
};

struct EpiSmem {
  int *qm;        // QuantM
  float *step;    // out_step_chan / out_step / acc_step
  float *smooth;  // the consuming dyntok step's smoothing factor, or -1 outside its columns
};

__device__ __forceinline__ void cp_async4(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all_but_newest() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// Stages the epilogue parameters of rows [tb*rb, min(te*rb, N)) with asynchronous copies
// (cp.async): the issuing threads do not wait for the loads, so staging the next step's
// parameters costs the current step nothing.  The caller commits the copy group.
__device__ void stage_epilogue_params(const ChainOp &op, int tb, int te, const EpiSmem &ep,
                                      int tid) {
  if (op.topk) return;  // the LM-head step reads its per-row parameters from global memory
  const int r0 = tb * op.rb;
  const int rows = te > tb ? min((te - tb) * op.rb, op.N - r0) : 0;
  const float *step = op.out_mode == kOutF32Acc ? op.acc_step : op.out_step;
  for (int i = tid; i < rows; i += kCT) {
    const int n = r0 + i;
    cp_async4(ep.qm + i, op.quant_m32 + n);
    cp_async4(ep.step + i, step + n);
    const int c = n - op.amax_c0;
    if (op.amax_dst && c >= 0 && c < op.amax_cols) {
      if (op.amax_smooth)
        cp_async4(ep.smooth + i, op.amax_smooth + c);
      else
        ep.smooth[i] = 1.0f;
    } else {
      ep.smooth[i] = -1.0f;
    }
  }
}

// Step descriptors live in a window of kWindow shared-memory slots, refilled kWindow - 1
// steps ahead with asynchronous copies, so the consumers never wait on a descriptor load.
constexpr int kWindow = 8;
constexpr int kOpChunks = static_cast<int>(sizeof(ChainOp) / 16);

__device__ __forceinline__ void fetch_descriptor(ChainOp *window, const ChainOp *ops, int s,
                                                 int lane) {
  const uint4 *src = reinterpret_cast<const uint4 *>(ops + s);
  uint4 *dst = reinterpret_cast<uint4 *>(window + (s % kWindow));
  for (int c = lane; c < kOpChunks; c += 32) cp_async16(dst + c, src + c);
}

// Consumes this CTA's tiles [tb, te) of one step.  `it` is the ring iteration counter shared
// with the producer's issue order.
template <int TT, int RPW, bool TOPK>
__device__ void consume_tiles(const ChainOp &op, const ChainArgs &a, int tb, int te, RingPos &rp,
                              const uint8_t *ring, const int8_t *xq, uint64_t *bars,
                              const float *s_ratio, uint64_t *cand, int *s_amax,
                              const EpiSmem &ep, int tid, bool &ok, unsigned long long *tr) {
  const int warp = tid >> 5, lane = tid & 31;
  bool first = true;
  constexpr int RB = kCW * RPW;
  const bool dyn = op.act_mode == kActDyntok;
  for (int tile = tb; tile < te; ++tile) {
    int acc[RPW * TT];  // value r * TT + t: row r, token t
#pragma unroll
    for (int i = 0; i < RPW * TT; ++i) acc[i] = 0;
    for (int kci = 0; kci < op.nk; ++kci, rp.advance(a.ns)) {
      const int slot = rp.slot;
      if (ok) ok = mbar_wait_bounded(smem_addr(&bars[slot]), rp.phase, a.err, kDevTimeoutFull);
      if (tr && first && tid == 0) tr[6] = global_timer_ns();
      first = false;
      const int k0 = kci * op.kc;
      const int bytes = min(op.kc, op.k_pad - k0);
      const uint8_t *sw = ring + static_cast<size_t>(slot) * a.stage_bytes;
      if (ok) {
        for (int kk = lane * 16; kk < bytes; kk += 512) {
          int4 xv[TT];
#pragma unroll
          for (int t = 0; t < TT; ++t)
            xv[t] = *reinterpret_cast<const int4 *>(xq + t * a.kpad_max + k0 + kk);
#pragma unroll
          for (int r = 0; r < RPW; ++r) {
            const int4 wv = *reinterpret_cast<const int4 *>(sw + (warp * RPW + r) * op.kc + kk);
#pragma unroll
            for (int t = 0; t < TT; ++t) {
              int s = acc[r * TT + t];
              s = __dp4a(wv.x, xv[t].x, s);
              s = __dp4a(wv.y, xv[t].y, s);
              s = __dp4a(wv.z, xv[t].z, s);
              s = __dp4a(wv.w, xv[t].w, s);
              acc[r * TT + t] = s;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&bars[kMaxStages + slot]));
    }
    // the RPW x TT sums reduced together: lane l ends with value l >> kShift
    constexpr int kNV = RPW * TT;
    constexpr int kShift = 5 - ilog2(kNV);
    int mine = 0;
    if constexpr (kNV <= 4) {
      mine = warp_sum_multi<kNV>(acc, lane);
    } else {  // (the halving form's extra live values spill at 96 registers)
#pragma unroll
      for (int i = 0; i < kNV; ++i) {
        const int s2 = warp_sum(acc[i]);
        if (lane == (i << kShift)) mine = s2;
      }
    }
    if ((lane & ((1 << kShift) - 1)) == 0) {
      const int vi = lane >> kShift;
      const int r = vi / TT, t = vi % TT;
      const int row = warp * RPW + r;
      const int n = tile * RB + row;
      if (t < a.T && n < op.N && ok) {
        // per-row parameters: staged in shared memory before the step's grid barrier, or for
        // the LM-head step (hundreds of rows a CTA, streaming-bound) read from global memory
        const int lr = (tile - tb) * RB + row;
        int e_qm;
        float e_step, e_smooth;
        if (TOPK) {
          e_qm = op.out_mode == kOutF32 ? __ldg(op.quant_m32 + n) : 0;
          e_step = __ldg((op.out_mode == kOutF32Acc ? op.acc_step : op.out_step) + n);
          e_smooth = -1.0f;
        } else {
          e_qm = ep.qm[lr];
          e_step = ep.step[lr];
          e_smooth = ep.smooth[lr];
        }
        const bool e_amax = e_smooth >= 0.0f;
        const float step = dyn ? s_ratio[t] * e_step : e_step;
        if (op.out_mode == kOutAccI32) {
          static_cast<int32_t *>(op.y)[t * op.ldy + n] = mine;
        } else if (op.out_mode == kOutQuant) {
          const int yq = requant_quantm(mine, e_qm, op.trunc, op.qmax);
          if (op.out_i16)
            static_cast<int16_t *>(op.y)[t * op.ldy + n] = static_cast<int16_t>(yq);
          else
            static_cast<int8_t *>(op.y)[t * op.ldy + n] = static_cast<int8_t>(yq);
        } else {
          const float v = op.out_mode == kOutF32
                              ? static_cast<float>(requant_quantm(mine, e_qm, op.trunc, op.qmax)) * step
                              : __int2float_rn(mine) * step;
          if (TOPK) {
            if (op.tk.logits) op.tk.logits[t * op.tk.ldl + n] = v;
            cand[t * a.cand_cap + (tile - tb) * RB + row] =
                topk_key(v, static_cast<uint32_t>(op.tk.row_offset + n));
          } else {
            static_cast<float *>(op.y)[t * op.ldy + n] = v;
            if (e_amax) {
              // fp32 output consumed by a dyntok step: reduce its amax |y * s_next| per token
              // (e_smooth is 1 when that step has no smoothing: v * 1 == v exactly)
              const float av = fabsf(v * e_smooth);
              if (av > 0.0f) atomicMax(s_amax + t, __float_as_int(av));
            }
          }
        }
      }
    }
  }
}

template <int TT, bool TOPK>
__device__ void consume_dispatch(const ChainOp &op, const ChainArgs &a, int tb, int te, RingPos &it,
                                 const uint8_t *ring, const int8_t *xq, uint64_t *bars,
                                 const float *s_ratio, uint64_t *cand, int *s_amax,
                                 const EpiSmem &ep, int tid, bool &ok, unsigned long long *tr) {
  // (the planner never gives TT = 8 more than 2 rows per warp: 4 x 8 accumulators spill)
  constexpr int kRpwMax = TT >= 8 ? 2 : 4;
  switch (op.rpw) {
    case 1: consume_tiles<TT, 1, TOPK>(op, a, tb, te, it, ring, xq, bars, s_ratio, cand, s_amax, ep, tid, ok, tr); break;
    case 2: consume_tiles<TT, 2, TOPK>(op, a, tb, te, it, ring, xq, bars, s_ratio, cand, s_amax, ep, tid, ok, tr); break;
    default: consume_tiles<TT, kRpwMax, TOPK>(op, a, tb, te, it, ring, xq, bars, s_ratio, cand, s_amax, ep, tid, ok, tr); break;
  }
}

// The LM-head step's grid top-k (topk.cuh): every CTA writes its sorted top-k list per token,
// and the last CTA to arrive selects the shard's top-k.  Consumer warps only; the drained weight
// ring holds the warps' staged lists and the gathered candidates.
template <int R>
__device__ void topk_finish(const ChainOp &op, const ChainArgs &a, int tb, int te, const uint64_t *cand,
                            uint64_t *ring, int tid) {
  __shared__ int s_last;
  __shared__ int s_n;
  const int k = op.tk.k;
  const int rows_here = te > tb ? min((te - tb) * op.rb, op.N - tb * op.rb) : 0;
  const int warp = tid >> 5, lane = tid & 31;
  const GridTopkState st{a.tk_counter, a.lists};
  uint64_t *stage = ring;
  uint64_t *gather = ring + kCW * 64;
  auto sync = [] { consumer_sync(); };
  for (int t = 0; t < a.T; ++t)
    grid_topk_offer<R, kCW>(cand + t * a.cand_cap, rows_here, k, t, st, stage, warp, lane, sync);
  if (!grid_topk_arrive(st, tid, &s_last, sync)) return;
  // CTA g owns the tiles split_range(num_tiles, G, g): tile i belongs to
  // g = ceil((i + 1) * G / num_tiles) - 1
  // (32-bit arithmetic: tile < num_tiles and (tile + 1) * G < 2^32 for any chain shape, and a
  // 32-bit division is a short inline sequence where a 64-bit one is a slow-path call)
  const int row_offset = op.tk.row_offset;
  const unsigned rb = static_cast<unsigned>(op.rb), num_tiles = static_cast<unsigned>(op.num_tiles);
  const unsigned G = gridDim.x;
  auto list_of = [row_offset, rb, num_tiles, G](uint64_t key) {
    const unsigned tile = static_cast<unsigned>(topk_key_id(key) - row_offset) / rb;
    return static_cast<int>(((tile + 1u) * G + num_tiles - 1u) / num_tiles - 1u);
  };
  for (int t = 0; t < a.T; ++t)
    grid_topk_select<R, kCW>(static_cast<int>(gridDim.x), k, t, st, op.tk.val + t * k, op.tk.idx + t * k, stage, gather, &s_n, warp, lane,
                             sync, list_of);
  if (tid == 0) *st.arrive = 0u;
}

template <int TT>
__global__ void __launch_bounds__(kThreads, 2) chain_kernel(const ChainArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  ChainOp *window = reinterpret_cast<ChainOp *>(smem);
  uint8_t *ring = smem + kWindow * sizeof(ChainOp);
  int8_t *xq = reinterpret_cast<int8_t *>(smem + a.xq_off);
  uint64_t *cand = reinterpret_cast<uint64_t *>(smem + a.cand_off);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.bars_off);
  EpiSmem ep_buf[2];
  {
    int *p = reinterpret_cast<int *>(smem + a.ep_off);
    for (int b = 0; b < 2; ++b) {
      ep_buf[b].qm = p;
      ep_buf[b].step = reinterpret_cast<float *>(p + a.max_rows);
      ep_buf[b].smooth = ep_buf[b].step + a.max_rows;
      p += 3 * a.max_rows;
    }
  }
  float *xs = a.norm_floats ? reinterpret_cast<float *>(smem + a.norm_off) : nullptr;
  __shared__ float s_part[kCW][TT];
  __shared__ float s_ratio[TT];
  __shared__ float s_inv[TT];
  __shared__ int s_amax[TT];  // float bits of a non-negative max (int order == float order)
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int t = 0; t < TT; ++t) s_amax[t] = 0;
    for (int s = 0; s < a.ns; ++s) {
      mbar_init(smem_addr(&bars[s]), 1);
      mbar_init(smem_addr(&bars[kMaxStages + s]), kCW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kCW) {
    // ------------------------------- producer warp -------------------------------
    const uint64_t pol = policy_evict_first();
    RingPos rp;
    bool ok = true;
    for (int s = 0; s < a.n_ops && ok; ++s) {
      // The producer runs ahead of the consumers: fetch the next descriptor into L1 now, and
      // keep this one's fields in registers (the barrier asm would otherwise force reloads).
      if (lane < 3 && s + 1 < a.n_ops)
        asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const char *>(a.ops + s + 1) + lane * 128));
      const ChainOp &op = a.ops[s];
      const int8_t *w = op.w;
      const int64_t ldw = op.ldw;
      const int N = op.N, rb = op.rb, kc = op.kc, nk = op.nk, k_pad = op.k_pad;
      const bool whole_rows = nk == 1 && kc == ldw;
      int tb, te;
      split_range(op.num_tiles, G, blockIdx.x, tb, te);
      unsigned long long *ptr =
          a.trace ? a.trace + (static_cast<size_t>(blockIdx.x) * a.n_ops + s) * 8 : nullptr;
      if (ptr && lane == 0) ptr[4] = global_timer_ns();
      for (int tile = tb; tile < te && ok; ++tile) {
        const int rows = min(rb, N - tile * rb);
        for (int kci = 0; kci < nk; ++kci, rp.advance(a.ns)) {
          const int slot = rp.slot;
          if (rp.lapped) {
            // the consumers' release of this slot's previous fill (phase of the lap before)
            ok = mbar_wait_bounded(smem_addr(&bars[kMaxStages + slot]), rp.phase ^ 1u, a.err,
                                   kDevTimeoutEmpty);
            if (!ok) break;
          }
          const int k0 = kci * kc;
          const int bytes = min(kc, k_pad - k0);
          const uint32_t full = smem_addr(&bars[slot]);
          const uint32_t dst = smem_addr(ring + static_cast<size_t>(slot) * a.stage_bytes);
          const int8_t *src = w + static_cast<int64_t>(tile * rb) * ldw + k0;
          if (whole_rows) {
            // whole rows: the tile is one contiguous block of rows * k_pad bytes, one copy
            if (lane == 0) {
              mbar_arrive_expect_tx(full, static_cast<uint32_t>(rows * bytes));
              bulk_g2s(dst, src, static_cast<uint32_t>(rows * bytes), full, pol);
            }
          } else {
            if (lane == 0) mbar_arrive_expect_tx(full, static_cast<uint32_t>(rows * bytes));
            __syncwarp();
            for (int r = lane; r < rows; r += 32)
              bulk_g2s(dst + r * kc, src + static_cast<int64_t>(r) * ldw, bytes, full, pol);
          }
          __syncwarp();
        }
      }
      if (ptr && lane == 0) ptr[5] = global_timer_ns();
    }
    return;
  }

  // ------------------------------- consumer warps -------------------------------
  const int tid = threadIdx.x;
  RingPos it;
  bool ok = true;
  // descriptors 0 .. kWindow-2 into the window, then step 0's per-row epilogue parameters;
  // every later descriptor is fetched kWindow-1 steps ahead and every later step's
  // parameters one step ahead
  if (tid < 32)
    for (int s = 0; s < kWindow - 1 && s < a.n_ops; ++s) fetch_descriptor(window, a.ops, s, tid);
  cp_async_commit();
  cp_async_wait_all();
  consumer_sync();
  {
    int tb0, te0;
    split_range(window[0].num_tiles, G, blockIdx.x, tb0, te0);
    stage_epilogue_params(window[0], tb0, te0, ep_buf[0], tid);
    cp_async_commit();
  }
  for (int s = 0; s < a.n_ops; ++s) {
    const ChainOp &op = window[s % kWindow];
    const EpiSmem &ep = ep_buf[s & 1];
    int tb, te;
    split_range(op.num_tiles, G, blockIdx.x, tb, te);
    // Work that does not depend on the previous step goes before its grid barrier: the
    // descriptor kWindow-1 steps ahead, the next step's per-row epilogue parameters into the
    // other shared-memory buffer, this thread's first smoothing factors into registers, the
    // candidate slots of a top-k step.  Exactly one copy group is committed per step, so
    // "all but the newest group" is this step's parameters (and older descriptors).
    if (tid < 32 && s + kWindow - 1 < a.n_ops) fetch_descriptor(window, a.ops, s + kWindow - 1, tid);
    if (s + 1 < a.n_ops) {
      const ChainOp &op1 = window[(s + 1) % kWindow];
      int tb1, te1;
      split_range(op1.num_tiles, G, blockIdx.x, tb1, te1);
      stage_epilogue_params(op1, tb1, te1, ep_buf[(s + 1) & 1], tid);
    }
    cp_async_commit();
    cp_async_wait_all_but_newest();
    float4 s_pre[4];
    preload_smooth(op, tid, s_pre);
    if (op.barrier_before && s > 0) {
      // Once one grid wait has run out, later ones are skipped so the kernel still ends.
      if (tid == 0 && !s_abort) {
        const unsigned *cnt = a.bar + (s - 1);
        if (ld_acquire_gpu(cnt) < static_cast<unsigned>(G)) {
          const unsigned long long t0 = global_timer_ns();
          for (uint32_t i = 1; ld_acquire_gpu(cnt) < static_cast<unsigned>(G); ++i) {
            if ((i & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
              atomicExch(a.err, kDevPeerTimeout);
              s_abort = 1;
              break;
            }
          }
        }
      }
      consumer_sync();
    }
    unsigned long long *tr =
        a.trace ? a.trace + (static_cast<size_t>(blockIdx.x) * a.n_ops + s) * 8 : nullptr;
    if (tr && tid == 0) tr[0] = global_timer_ns();
    if (te > tb || op.topk) {
      // (quantise_input ends with a consumer barrier: the staged parameters are visible)
      if (te > tb) quantise_input<TT>(op, a.T, xq, a.kpad_max, s_ratio, s_inv, s_part, tid, s_pre, xs);
      else consumer_sync();
      if (op.topk) {
        // candidate slots (they may share bytes with the activation rows' tail and the norm
        // staging row, both dead once the input is quantised)
        for (int i = tid; i < TT * a.cand_cap; i += kCT) cand[i] = 0ull;
        consumer_sync();
      }
      if (tr && tid == 0) tr[1] = global_timer_ns();
      // the CTA owning tile 0 publishes the per-token ratios
      if (tb == 0 && te > 0 && op.ratio_out && tid < a.T && op.act_mode == kActDyntok)
        op.ratio_out[tid] = s_ratio[tid];
      if (op.topk) {
        consume_dispatch<TT, true>(op, a, tb, te, it, ring, xq, bars, s_ratio, cand, s_amax, ep, tid, ok, tr);
        consumer_sync();
        uint64_t *ring64 = reinterpret_cast<uint64_t *>(ring);
        if (op.tk.k > 32)
          topk_finish<2>(op, a, tb, te, cand, ring64, tid);
        else
          topk_finish<1>(op, a, tb, te, cand, ring64, tid);
      } else {
        consume_dispatch<TT, false>(op, a, tb, te, it, ring, xq, bars, s_ratio, cand, s_amax, ep, tid, ok, tr);
      }
    }
    // arrival: every output of this CTA for step s is written (and its amax share reduced).
    // (read from the descriptor before the barrier: its window slot is refilled right after)
    float *const amax_dst = op.amax_dst;
    consumer_sync();
    if (tid == 0) {
      if (tr) tr[2] = global_timer_ns();
      if (amax_dst)
        for (int t = 0; t < a.T; ++t)
          if (s_amax[t] > 0) atomicMax(reinterpret_cast<int *>(amax_dst) + t, s_amax[t]);
      // only this thread touches s_amax between the consume phases: reset for the next step
      for (int t = 0; t < TT; ++t) s_amax[t] = 0;
      // release: the CTA's writes (ordered before this by the consumer barrier, and this
      // thread's amax reductions) become visible to any CTA that acquires the counter
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.bar + s), "r"(1u) : "memory");
      if (tr) tr[3] = global_timer_ns();
    }
  }
}

}  // namespace

cudaError_t configure_chain(const ChainPlan &plan) {
  // Opt the instantiation in (once per device) to the largest dynamic shared memory allowed.
  int limit = 0;
  cudaError_t e;
  switch (plan.tt) {
    case 1: e = opt_in_dyn_smem<chain_kernel<1>>(&limit); break;
    case 2: e = opt_in_dyn_smem<chain_kernel<2>>(&limit); break;
    case 4: e = opt_in_dyn_smem<chain_kernel<4>>(&limit); break;
    default: e = opt_in_dyn_smem<chain_kernel<8>>(&limit); break;
  }
  if (e != cudaSuccess) return e;
  if (plan.smem > static_cast<size_t>(limit)) return cudaErrorInvalidValue;
  return cudaSuccess;
}

namespace {

// Plans the chain for `cps` co-resident CTAs per SM; false when it does not fit.
bool plan_chain_cps(ChainOp *ops, int n_ops, int T, int sm_count, int cps, ChainPlan *plan) {
  ChainPlan p = {};
  p.tt = T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8;
  p.grid = cps * sm_count;
  int kpad_max = 16;
  size_t stage = 0;
  size_t cand_cap = 0;
  int max_rows = 8;
  int norm_floats = 0;
  int kpad_topk = 0;
  // Stage size target: every stage carries ~24 KB (whole-row tiles of up to 32 rows, or 8-row
  // K chunks of 3 KB per row for long rows), so the fixed-size ring slots stay full.
  constexpr int kMaxStage = 24576;
  for (int s = 0; s < n_ops; ++s) {
    ChainOp &op = ops[s];
    if (op.topk && s != n_ops - 1) return false;  // the LM-head step must be last
    auto tiles = [&](int rb) { return (op.N + rb - 1) / rb; };
    const int min_tiles = op.topk ? p.grid : 2 * p.grid;
    if (op.k_pad * 8 <= kMaxStage) {
      // whole-row tiles: a tile is one contiguous rb x k_pad block (one bulk copy per stage)
      op.rpw = 1;
      for (int r : {4, 2})
        if ((r < 4 || p.tt < 8) && 8 * r * op.k_pad <= kMaxStage && tiles(8 * r) >= min_tiles) {
          op.rpw = r;
          break;
        }
      op.kc = op.k_pad;
    } else {
      // long rows: 8-row tiles streamed in K chunks
      op.rpw = 1;
      op.kc = kMaxStage / 8;
    }
    op.rb = 8 * op.rpw;
    op.nk = (op.k_pad + op.kc - 1) / op.kc;
    op.num_tiles = tiles(op.rb);
    stage = std::max(stage, static_cast<size_t>(op.rb) * op.kc);
    kpad_max = std::max(kpad_max, op.k_pad);
    if (op.act_mode == kActEmbNorm) norm_floats = std::max(norm_floats, (op.K + 3) / 4 * 4);
    const int max_tiles = (op.num_tiles + p.grid - 1) / p.grid;
    if (op.topk) {
      // candidate slots of the LM-head step (its epilogue parameters are not staged)
      cand_cap = (static_cast<size_t>(max_tiles) * op.rb + 7) / 8 * 8;
      kpad_topk = op.k_pad;
    } else {
      max_rows = std::max(max_rows, max_tiles * op.rb);
    }
  }
  auto up16 = [](size_t v) { return (v + 15) / 16 * 16; };
  p.kpad_max = static_cast<int>(up16(kpad_max));
  p.cand_cap = static_cast<int>(cand_cap);
  p.max_rows = (max_rows + 3) / 4 * 4;
  p.stage_bytes = static_cast<uint32_t>(stage);
  p.norm_floats = norm_floats;
  // Layout after the ring, relative to the activation rows: xq [tt][kpad_max]; the LM-head
  // step's candidates in the rows' tail when one token leaves room after its row (the
  // candidates are written only once that step's input is quantised), else after xq; the
  // mbarriers; the two epilogue parameter buffers; the norm staging row, inside xq when it fits
  // (it is dead before the step writes its quantised rows).
  const size_t xq_bytes = static_cast<size_t>(p.tt) * p.kpad_max;
  const size_t cand_bytes = static_cast<size_t>(p.tt) * cand_cap * 8;
  const bool cand_in_xq = p.tt == 1 && cand_bytes > 0 && up16(kpad_topk) + cand_bytes <= xq_bytes;
  const bool norm_in_xq = static_cast<size_t>(norm_floats) * 4 <= xq_bytes;
  const size_t cand_rel = cand_in_xq ? up16(kpad_topk) : xq_bytes;
  const size_t bars_rel = up16(cand_in_xq ? xq_bytes : xq_bytes + cand_bytes);
  const size_t ep_rel = bars_rel + 2 * kMaxStages * 8;
  const size_t norm_rel = norm_in_xq ? 0 : up16(ep_rel + 2 * static_cast<size_t>(p.max_rows) * 12);
  const size_t tail = norm_in_xq ? ep_rel + 2 * static_cast<size_t>(p.max_rows) * 12
                                 : norm_rel + static_cast<size_t>(norm_floats) * 4;
  const size_t window = kWindow * sizeof(ChainOp);
  const size_t fixed = window + up16(tail);
  // the SM's 228 KB split between the co-resident CTAs, less the per-CTA reservation and
  // static shared memory (a few hundred bytes)
  const size_t budget = 233472 / cps - 1024 - 1024;
  if (fixed + 2 * stage > budget) return false;
  size_t weight_bytes = 0;
  for (int s = 0; s < n_ops; ++s) weight_bytes += static_cast<size_t>(ops[s].N) * ops[s].k_pad;
  const bool deep = weight_bytes / (static_cast<size_t>(n_ops) * p.grid) >= kDeepRingBytesPerStep;
  p.ns = static_cast<int>(std::min<size_t>(deep ? kMaxStages : kLatencyRingStages, (budget - fixed) / stage));
  p.ring_bytes = static_cast<uint32_t>(p.ns * stage);
  const size_t xq_off = window + p.ring_bytes;
  p.xq_off = static_cast<uint32_t>(xq_off);
  p.cand_off = static_cast<uint32_t>(xq_off + cand_rel);
  p.bars_off = static_cast<uint32_t>(xq_off + bars_rel);
  p.ep_off = static_cast<uint32_t>(xq_off + ep_rel);
  p.norm_off = static_cast<uint32_t>(xq_off + norm_rel);
  // the top-k step reuses the drained ring for its staged lists and gathered candidates
  bool any_topk = false;
  for (int s = 0; s < n_ops; ++s) any_topk = any_topk || ops[s].topk;
  if (any_topk && p.ring_bytes < (kCW * 64 + kTopkGatherKeys) * 8) return false;
  p.smem = p.ring_bytes + fixed;  // (fixed includes the window)
  *plan = p;
  return true;
}

}  // namespace

bool plan_chain(ChainOp *ops, int n_ops, int T, int sm_count, ChainPlan *plan) {
  if (n_ops < 1 || T < 1 || T > 8 || sm_count < 1) return false;
  // Two co-resident CTAs per SM give two independent weight pipelines per SM (more bytes in
  // flight than one CTA whose 8 warps release each stage together); large T x K inputs fall
  // back to one CTA per SM with the whole shared memory.
  return plan_chain_cps(ops, n_ops, T, sm_count, 2, plan) ||
         plan_chain_cps(ops, n_ops, T, sm_count, 1, plan);
}

cudaError_t launch_chain(const ChainOp *ops_dev, int n_ops, int T, const ChainPlan &plan,
                         unsigned *bar, size_t clear_bytes, unsigned *tk_counter,
                         uint64_t *lists, int *err, unsigned long long *trace,
                         cudaStream_t stream) {
  ChainArgs a;
  a.ops = ops_dev;
  a.n_ops = n_ops;
  a.T = T;
  a.bar = bar;
  a.tk_counter = tk_counter;
  a.lists = lists;
  a.err = err;
  a.ns = plan.ns;
  a.stage_bytes = plan.stage_bytes;
  a.kpad_max = plan.kpad_max;
  a.cand_cap = plan.cand_cap;
  a.max_rows = plan.max_rows;
  a.ring_bytes = plan.ring_bytes;
  a.norm_floats = plan.norm_floats;
  a.xq_off = plan.xq_off;
  a.cand_off = plan.cand_off;
  a.bars_off = plan.bars_off;
  a.ep_off = plan.ep_off;
  a.norm_off = plan.norm_off;
  a.trace = trace;
  void (*kern)(ChainArgs) = nullptr;
  switch (plan.tt) {
    case 1: kern = chain_kernel<1>; break;
    case 2: kern = chain_kernel<2>; break;
    case 4: kern = chain_kernel<4>; break;
    default: kern = chain_kernel<8>; break;
  }
  cudaError_t e = configure_chain(plan);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(bar, 0, clear_bytes, stream);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace w8a8
