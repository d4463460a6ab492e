// Decode-shaped W8A8 contraction (T <= 8 tokens) for sm_100a.
//
// One CTA = 8 consumer warps + 1 producer warp.  The CTA owns a contiguous range of row
// tiles (RB = 8 * RPW output channels each) and streams their int8 weights through an
// NS-deep ring of shared-memory stages filled by 1-D bulk copies (cp.async.bulk, TMA engine,
// no tensor map, one CTA per copy) that complete on mbarriers.  Each stage holds an [RB, KC] weight
// slab plus the matching [T, KC] slab of the int8 activations.  Consumers read 16-byte
// vectors, accumulate with dp4a into int32 registers, and reduce across the warp with
// shuffles.  The epilogue applies the reference's SDP requant (QuantM, RNE shift, saturate)
// and the unpack step (per-channel / per-token dequant), or keeps the logits on chip: each CTA
// writes its sorted top-k (warp bitonic networks, topk.cuh) and the last CTA to finish selects
// the shard's top-k from the few list prefixes that can hold it.
//
// The weight copies of the first NS stages are issued before griddepcontrol.wait, so under
// programmatic dependent launch the weight stream of this linear overlaps the tail of the
// kernel that produces its activations.
//
// Reference semantics: CMAC int8 GEMM -> CACC int32 (src/eswin_simulator/eswin_simulator/
// engines/cmac.py:300-383), SDP CvtPrecision_QuantM (src/LFM3/attribute_int8_error.py:104-122),
// unpack_npu_output_int8[_dyntok] (src/LFM3/lfm3_v2.cpp:971-1008, 1143-1183), LM-head merge
// (src/LFM3/lfm3_v2.cpp:2360-2405) + greedy / top-k (src/eswin_runtime/src/nlp/sampler.cpp:93-121).
#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

#include <algorithm>

namespace w8a8 {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxStages = 8;
// 227 KB opt-in per block on sm_100, less a margin for the kernels' static shared memory.
constexpr size_t kMaxDynSmem = 232448 - 1024;

struct GemvArgs {
  const int8_t *w;
  int64_t ldw;
  const int8_t *x;
  int64_t ldx;
  int T, N, k_pad, kc, nk, ns, num_tiles, tiles_per_cta, cand_cap;
  uint32_t stage_bytes;
  uint32_t ring_bytes;  // stage ring (top-k: at least kTopkStageBytes); barriers follow it
  Epilogue ep;
  TopK tk;
  int *err;
  unsigned long long *trace;
  ShardSync sync;
  FusedQuant fq;
  uint32_t xres_off;  // fused quantisation: resident [TT][k_pad] int8 slab
  int split_select;   // top-k of several tokens: the selection runs in topk_select_kernel
};

// A shard on another device than GPU 0 waits at most this long for GPU 0 to store its
// activations (less than the consumers' 2 s stage wait, so the producer gives up first).
constexpr unsigned long long kXReadyLimitNs = 1000000000ull;

// Diagnostic timeline of a CTA (only when a trace buffer is attached): 0 entry, 1 setup done,
// 2 first stage landed (consumer warp 0), 3 streaming done, 4 top-k lists written, 5 arrived,
// 6 top-k selected (last CTA only), 7 exit.
__device__ __forceinline__ void stamp(const GemvArgs &a, int i) {
  if (a.trace && (threadIdx.x & 31) == 0) a.trace[blockIdx.x * 8 + i] = global_timer_ns();
}

__device__ __forceinline__ void store_output(const Epilogue &ep, int acc, int t, int n) {
  switch (ep.out_mode) {
    case kOutAccI32:
      static_cast<int32_t *>(ep.y)[t * ep.ldy + n] = acc;
      break;
    case kOutQuant: {
      const int yq = requant_quantm(acc, ep.quant_m[n], ep.trunc, ep.qmax);
      if (ep.out_i16)
        static_cast<int16_t *>(ep.y)[t * ep.ldy + n] = static_cast<int16_t>(yq);
      else
        static_cast<int8_t *>(ep.y)[t * ep.ldy + n] = static_cast<int8_t>(yq);
      break;
    }
    case kOutF32: {
      const int yq = requant_quantm(acc, ep.quant_m[n], ep.trunc, ep.qmax);
      const float step = ep.act_mode == kActDyntok ? ep.ratio[t] * ep.out_step[n] : ep.out_step[n];
      static_cast<float *>(ep.y)[t * ep.ldy + n] = static_cast<float>(yq) * step;
      break;
    }
    default: {
      const float step = ep.act_mode == kActDyntok ? ep.ratio[t] * ep.acc_step[n] : ep.acc_step[n];
      static_cast<float *>(ep.y)[t * ep.ldy + n] = __int2float_rn(acc) * step;
      break;
    }
  }
}

// Float logit of one (token, row) for the top-k path (F32 or F32_ACC).
__device__ __forceinline__ float logit_value(const Epilogue &ep, int acc, int t, int n) {
  if (ep.out_mode == kOutF32) {
    const int yq = requant_quantm(acc, ep.quant_m[n], ep.trunc, ep.qmax);
    const float step = ep.act_mode == kActDyntok ? ep.ratio[t] * ep.out_step[n] : ep.out_step[n];
    return static_cast<float>(yq) * step;
  }
  const float step = ep.act_mode == kActDyntok ? ep.ratio[t] * ep.acc_step[n] : ep.acc_step[n];
  return __int2float_rn(acc) * step;
}

struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

// Barrier over the consumer warps only (the producer warp keeps streaming).
__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// True in the CTA that publishes the activations to other devices (quantise_resident).
__device__ __forceinline__ bool is_publisher(const GemvArgs &a) {
  return a.fq.x != nullptr && a.fq.pub_seq != nullptr && blockIdx.x == gridDim.x - 1;
}

// Producer side of the publisher CTA: no weight copy of this CTA is in flight while its
// consumers fence the peer stores at system scope (the fence would wait for them too), so the
// producer waits here until the publication is done.  The publisher owns the grid's last,
// shortest tile range.
__device__ __forceinline__ void publish_gate() {
  asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory");
}

// Fused prologue: the T fp32 rows quantised into the resident slab xres ([TT][k_pad]; rows >= T
// and columns >= K zero) by the consumer threads, with the arithmetic of act_quant_kernel's
// static path: q = round_clamp(x * (s * inv_step), 127), or x * inv_step without smoothing.
// The last CTA of a multi-device LM head's shard-0 grid (it owns the fewest tiles, so the time
// it spends here is least likely to delay the grid) then stores rows [0, T) into every peer's
// staging buffer and bumps the peers' x_ready counters (one system-scope fence, then relaxed
// stores: a release).
template <int TT>
__device__ void quantise_resident(const GemvArgs &a, int8_t *xres, int tid) {
  const FusedQuant &f = a.fq;
  // The publishing CTA fetches its metadata (peer buffers, forward counter) first, so those
  // reads overlap the activations' instead of following them.
  __shared__ int8_t *s_peer_q[64];
  __shared__ unsigned *s_peer_flag[64];
  __shared__ unsigned s_seq;
  const bool publisher = is_publisher(a);
  if (publisher) {
    if (tid < f.n_peers) {
      s_peer_q[tid] = f.peers[tid].q;
      s_peer_flag[tid] = f.peers[tid].flag;
    }
    if (tid == 0) s_seq = *f.pub_seq;
  }
  const float inv = f.inv_step;
  const bool vec = (f.K % 4 == 0) && (f.ldx % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(f.x) % 16 == 0) &&
                   (f.inv_smooth == nullptr || reinterpret_cast<uintptr_t>(f.inv_smooth) % 16 == 0);
  constexpr int NT = kConsumerWarps * 32;
  for (int t = 0; t < TT; ++t) {
    int8_t *q = xres + t * a.k_pad;
    if (t >= a.T) {
      for (int c = tid * 16; c < a.k_pad; c += NT * 16)
        *reinterpret_cast<int4 *>(q + c) = make_int4(0, 0, 0, 0);
      continue;
    }
    const float *x = f.x + t * f.ldx;
    if (vec) {
      const float4 *x4 = reinterpret_cast<const float4 *>(x);
      const float4 *s4 = reinterpret_cast<const float4 *>(f.inv_smooth);
      for (int c = tid; c < f.K / 4; c += NT) {
        const float4 v = x4[c];
        char4 o;
        if (s4) {
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
        reinterpret_cast<char4 *>(q)[c] = o;
      }
    } else {
      for (int c = tid; c < f.K; c += NT) {
        const float v = f.inv_smooth ? x[c] * (f.inv_smooth[c] * inv) : x[c] * inv;
        q[c] = static_cast<int8_t>(round_clamp(v, 127.0f));
      }
    }
    for (int c = f.K + tid; c < a.k_pad; c += NT) q[c] = 0;
  }
  consumer_bar();
  if (!publisher) return;
  if (tid == 0 && f.trace) f.trace[0] = global_timer_ns();
  const int vecs = a.k_pad / 16;
  for (int p = 0; p < f.n_peers; ++p) {
    int8_t *dst = s_peer_q[p];
    for (int i = tid; i < a.T * vecs; i += NT) {
      const int t = i / vecs, c = (i - t * vecs) * 16;
      *reinterpret_cast<int4 *>(dst + t * a.k_pad + c) =
          *reinterpret_cast<const int4 *>(xres + t * a.k_pad + c);
    }
  }
  __threadfence_system();
  consumer_bar();
  if (tid == 0) {
    __threadfence_system();
    const unsigned e = s_seq + 1u;
    *f.pub_seq = e;
    for (int p = 0; p < f.n_peers; ++p) st_relaxed_sys(s_peer_flag[p], e);
    if (f.trace) f.trace[1] = global_timer_ns();
  }
  // releases the producer warp, which held this CTA's weight copies back (publish_gate)
  asm volatile("bar.arrive 2, %0;" ::"n"(kThreads) : "memory");
}

// Shared memory of the top-k epilogue (in the drained stage ring): the warps' staged lists (64
// keys each), then the last CTA's gathered candidates.
constexpr uint32_t kTopkStageBytes = ((kConsumerWarps + 1) * 64 + kTopkGatherKeys) * 8;

// Every token's share of the grid top-k from this CTA's candidate keys, then, in the CTA that
// arrives last, the selection of the shard's top-k (R = 1 for k <= 32, else 2).
template <int R>
__device__ void topk_epilogue(const GemvArgs &a, const GridTopkState &st, const uint64_t *cand,
                              int rows_here, int rows_per_cta, uint64_t *stage, int *s_last) {
  constexpr int NW = kConsumerWarps + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (a.T > 1) {
    // one warp per token: the warps fold different tokens' candidates at once (sort each chunk
    // of 32R keys, merge it into the running list), where grid_topk_offer would run the tokens
    // one after another with most warps idle on a CTA's few chunks
    for (int t = warp; t < a.T; t += NW) {
      uint64_t v[R];
      for (int c = 0; c < rows_here; c += 32 * R) {
        uint64_t b[R];
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const int i = c + lane + 32 * j;
          b[j] = i < rows_here ? cand[t * a.cand_cap + i] : 0ull;
        }
        warp_sort_desc<R>(b, lane);
        if (c == 0) {
#pragma unroll
          for (int j = 0; j < R; ++j) v[j] = b[j];
        } else {
          warp_merge_desc<R>(v, b, lane);
        }
      }
      uint64_t *base = st.keys + t * grid_topk_stride(gridDim.x, a.tk.k);
      uint64_t *list = base + static_cast<size_t>(blockIdx.x) * a.tk.k;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (lane + 32 * j < a.tk.k) list[lane + 32 * j] = v[j];
      if (lane == 0) base[static_cast<size_t>(gridDim.x) * a.tk.k + blockIdx.x] = v[0];
    }
    __syncthreads();
  } else {
    for (int t = 0; t < a.T; ++t)
      grid_topk_offer<R, NW>(cand + t * a.cand_cap, rows_here, a.tk.k, t, st, stage, warp, lane,
                             BlockSync{});
  }
  if (threadIdx.x == 0) stamp(a, 4);
  const bool last = grid_topk_arrive(st, threadIdx.x, s_last, BlockSync{});
  if (threadIdx.x == 0) stamp(a, 5);
  if (!last) {
    if (threadIdx.x == 0) stamp(a, 7);
    return;
  }
  if (a.split_select) {
    // every token's lists are written: the selection kernel (one CTA per token) takes over
    if (threadIdx.x == 0) {
      *st.arrive = 0u;
      stamp(a, 7);
    }
    return;
  }
  __shared__ int s_n;
  uint64_t *gather = stage + NW * 64;
  // CTA b owns rows [b * rows_per_cta, (b + 1) * rows_per_cta) of the shard
  const int row_offset = a.tk.row_offset;
  auto list_of = [row_offset, rows_per_cta](uint64_t key) {
    return (topk_key_id(key) - row_offset) / rows_per_cta;
  };
  for (int t = 0; t < a.T; ++t) {
    float *vr = a.tk.val + t * a.tk.k;
    int32_t *ir = a.tk.idx + t * a.tk.k;
    if (a.tk.val_dst) {
      // the token's owner gathers it: row (g % dst_tokens) of owner g / dst_tokens
      const int g = a.tk.tok0 + t;
      const int64_t off = a.tk.dst_row0 + static_cast<int64_t>(g % a.tk.dst_tokens) * a.tk.dst_ld;
      vr = a.tk.val_dst[g / a.tk.dst_tokens] + off;
      ir = a.tk.idx_dst[g / a.tk.dst_tokens] + off;
    }
    grid_topk_select<R, NW>(static_cast<int>(gridDim.x), a.tk.k, t, st, vr, ir, stage, gather, &s_n, warp, lane, BlockSync{},
                            list_of);
  }
  if ((a.sync.done || a.sync.done_peers) && !a.sync.hold) {
    // LM-head shard storing into other devices: publish the rows, then count the forward
    // (system-scope fence, then relaxed counter stores = a release of the rows).
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned e = *a.sync.seq + 1u;
      *a.sync.seq = e;
      if (a.sync.done) st_relaxed_sys(a.sync.done, e);
      for (int p = 0; p < a.sync.n_done; ++p) st_relaxed_sys(a.sync.done_peers[p], e);
    }
  }
  if (threadIdx.x == 0) {
    *st.arrive = 0u;
    stamp(a, 6);
    stamp(a, 7);
  }
}

template <int TT, int RPW, bool TOPK>
__global__ void __launch_bounds__(kThreads, 2) gemv_w8a8_kernel(const GemvArgs a) {
  constexpr int RB = kConsumerWarps * RPW;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *stages = smem;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.ring_bytes);
  uint64_t *cand = bars + 2 * kMaxStages;  // TOPK: [TT][cand_cap]
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile0 = blockIdx.x * a.tiles_per_cta;
  const int tile_end = min(tile0 + a.tiles_per_cta, a.num_tiles);
  const int ntiles = tile_end - tile0;
  const int total = ntiles * a.nk;
  if (threadIdx.x == 0) stamp(a, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.ns; ++s) {
      mbar_init(smem_addr(&bars[s]), 1);
      mbar_init(smem_addr(&bars[kMaxStages + s]), kConsumerWarps);
    }
    fence_barrier_init();
  }
  if (TOPK) {
    for (int i = threadIdx.x; i < TT * a.cand_cap; i += blockDim.x) cand[i] = 0ull;
  }
  __syncthreads();
  if (threadIdx.x == 0) stamp(a, 1);

  if (warp == kConsumerWarps) {
    // ------------------------------- producer warp -------------------------------
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const int pre = min(a.ns, total);
    // fused quantisation: the stages carry weights only
    const int x_rows = a.fq.x ? 0 : a.T;
    auto stage_geom = [&](int it, int &tile, int &k0, int &bytes, int &rows) {
      tile = tile0 + it / a.nk;
      k0 = (it % a.nk) * a.kc;
      bytes = min(a.kc, a.k_pad - k0);
      rows = min(RB, a.N - tile * RB);
    };
    // Whole-row tiles are one contiguous rows x k_pad block: one copy; else one per row.
    const bool whole_rows = a.nk == 1 && a.kc == a.ldw;
    auto copy_w = [&](uint32_t dst, int tile, int k0, int bytes, int rows, uint32_t full) {
      const int8_t *src = a.w + static_cast<int64_t>(tile * RB) * a.ldw + k0;
      if (whole_rows) {
        if (lane == 0) bulk_g2s(dst, src, static_cast<uint32_t>(rows * bytes), full, pol_w);
      } else {
        for (int r = lane; r < rows; r += 32)
          bulk_g2s(dst + r * a.kc, src + static_cast<int64_t>(r) * a.ldw, bytes, full, pol_w);
      }
    };
    auto issue_w = [&](int it) {
      int tile, k0, bytes, rows;
      stage_geom(it, tile, k0, bytes, rows);
      const uint32_t full = smem_addr(&bars[it]);
      if (lane == 0) mbar_arrive_expect_tx(full, static_cast<uint32_t>((rows + x_rows) * bytes));
      __syncwarp();
      copy_w(smem_addr(stages + static_cast<size_t>(it) * a.stage_bytes), tile, k0, bytes, rows, full);
    };
    // With fused quantisation the consumers read the fp32 activations right after the
    // dependency wait: only one stage goes ahead of them, so that read does not queue behind
    // the whole grid's prefetch.
    const bool publisher = is_publisher(a);
    const int early = publisher ? 0 : a.fq.x ? min(1, pre) : pre;
    for (int it = 0; it < early; ++it) issue_w(it);
    // Activations (and everything written by the previous kernel) are read only after this.
    pdl_wait();
    if (publisher) publish_gate();
    for (int it = early; it < pre; ++it) issue_w(it);
    if (a.sync.x_ready) {
      // Remote LM-head shard: GPU 0 stores this forward's activations into our staging buffer
      // and then bumps x_ready.  On a timeout the (stale) rows are still copied so the kernel
      // ends promptly; the error word records the failure.
      if (lane == 0) {
        const unsigned target = *a.sync.seq + 1u;
        const int nr = a.sync.n_ready > 0 ? a.sync.n_ready : 1;
        for (int p = 0; p < nr; ++p)
          if (!wait_flag_reached(a.sync.x_ready + p, target, kXReadyLimitNs, a.err,
                                 kDevPeerTimeout))
            break;  // (one wait that ran out is enough: the rest would only add their limits)
        fence_proxy_async_global();
      }
      __syncwarp();
    }
    for (int it = 0; it < pre; ++it) {
      int tile, k0, bytes, rows;
      stage_geom(it, tile, k0, bytes, rows);
      const uint32_t full = smem_addr(&bars[it]);
      const uint32_t dst = smem_addr(stages + static_cast<size_t>(it) * a.stage_bytes) + RB * a.kc;
      for (int t = lane; t < x_rows; t += 32)
        bulk_g2s(dst + t * a.kc, a.x + t * a.ldx + k0, bytes, full, pol_x);
    }
    bool ok = true;
    for (int it = pre; it < total; ++it) {
      const int slot = it % a.ns;
      const int use = it / a.ns;
      if (ok)
        ok = mbar_wait_bounded(smem_addr(&bars[kMaxStages + slot]), (use - 1) & 1, a.err,
                               kDevTimeoutEmpty);
      if (!ok) break;
      int tile, k0, bytes, rows;
      stage_geom(it, tile, k0, bytes, rows);
      const uint32_t full = smem_addr(&bars[slot]);
      if (lane == 0) mbar_arrive_expect_tx(full, static_cast<uint32_t>((rows + x_rows) * bytes));
      __syncwarp();
      const uint32_t dst = smem_addr(stages + static_cast<size_t>(slot) * a.stage_bytes);
      copy_w(dst, tile, k0, bytes, rows, full);
      for (int t = lane; t < x_rows; t += 32)
        bulk_g2s(dst + RB * a.kc + t * a.kc, a.x + t * a.ldx + k0, bytes, full, pol_x);
    }
  } else {
    // ------------------------------- consumer warps -------------------------------
    pdl_wait();
    int8_t *xres = reinterpret_cast<int8_t *>(smem + a.xres_off);
    const bool fused = a.fq.x != nullptr;
    if (fused) quantise_resident<TT>(a, xres, threadIdx.x);
    int acc[RPW][TT];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int t = 0; t < TT; ++t) acc[r][t] = 0;
    bool ok = true;
    for (int it = 0; it < total; ++it) {
      const int slot = it % a.ns;
      const int use = it / a.ns;
      if (ok) ok = mbar_wait_bounded(smem_addr(&bars[slot]), use & 1, a.err, kDevTimeoutFull);
      if (it == 0 && warp == 0) stamp(a, 2);
      const int kci = it % a.nk;
      const int bytes = min(a.kc, a.k_pad - kci * a.kc);
      const uint8_t *sw = stages + static_cast<size_t>(slot) * a.stage_bytes;
      // activations: the stage's slab (row stride kc) or the resident slab (row stride k_pad)
      const uint8_t *sx =
          fused ? reinterpret_cast<const uint8_t *>(xres) + kci * a.kc : sw + RB * a.kc;
      const int ldsx = fused ? a.k_pad : a.kc;
      if (ok) {
        for (int kk = lane * 16; kk < bytes; kk += 512) {
          int4 xv[TT];
#pragma unroll
          for (int t = 0; t < TT; ++t) xv[t] = *reinterpret_cast<const int4 *>(sx + t * ldsx + kk);
#pragma unroll
          for (int r = 0; r < RPW; ++r) {
            const int4 wv =
                *reinterpret_cast<const int4 *>(sw + (warp * RPW + r) * a.kc + kk);
#pragma unroll
            for (int t = 0; t < TT; ++t) {
              int s = acc[r][t];
              s = __dp4a(wv.x, xv[t].x, s);
              s = __dp4a(wv.y, xv[t].y, s);
              s = __dp4a(wv.z, xv[t].z, s);
              s = __dp4a(wv.w, xv[t].w, s);
              acc[r][t] = s;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&bars[kMaxStages + slot]));
      if (kci == a.nk - 1) {
        // Tile finished: butterfly-reduce every (row, token) sum; lane r*TT+t keeps it.
        const int tile = tile0 + it / a.nk;
        int mine = 0;
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            const int s = warp_sum(acc[r][t]);
            if (lane == r * TT + t) mine = s;
            acc[r][t] = 0;
          }
        if (lane < RPW * TT) {
          const int r = lane / TT;
          const int t = lane % TT;
          const int row = warp * RPW + r;
          const int n = tile * RB + row;
          if (t < a.T && n < a.N && ok) {
            if (TOPK) {
              const float v = logit_value(a.ep, mine, t, n);
              if (a.tk.logits) a.tk.logits[t * a.tk.ldl + n] = v;
              cand[t * a.cand_cap + (tile - tile0) * RB + row] =
                  topk_key(v, static_cast<uint32_t>(a.tk.row_offset + n));
            } else {
              store_output(a.ep, mine, t, n);
            }
          }
        }
      }
    }
  }
  pdl_launch_dependents();
  if (!TOPK) {
    if (a.trace) {
      __syncthreads();
      if (threadIdx.x == 0) {
        stamp(a, 3);
        stamp(a, 7);
      }
    }
    return;
  }

  // ------------------------------- top-k epilogue -------------------------------
  // The drained stage ring (at least kTopkStageBytes) stages the warps' sorted lists.
  __syncthreads();
  if (threadIdx.x == 0) stamp(a, 3);
  const int rows_here = min(ntiles * RB, a.N - tile0 * RB);
  const GridTopkState st{a.tk.counter, a.tk.lists};
  uint64_t *stage = reinterpret_cast<uint64_t *>(smem);
  if (a.tk.k > 32)
    topk_epilogue<2>(a, st, cand, rows_here, a.tiles_per_cta * RB, stage, &s_last);
  else
    topk_epilogue<1>(a, st, cand, rows_here, a.tiles_per_cta * RB, stage, &s_last);
}

template <int TT, int RPW, bool TOPK>
cudaError_t launch_one(const GemvArgs &args, const GemvPlan &plan, cudaStream_t stream, bool pdl) {
  auto kern = gemv_w8a8_kernel<TT, RPW, TOPK>;
  int max_dyn = 0;
  cudaError_t e = opt_in_dyn_smem<gemv_w8a8_kernel<TT, RPW, TOPK>>(&max_dyn);
  if (e != cudaSuccess) return e;
  if (plan.smem > static_cast<size_t>(max_dyn)) return cudaErrorInvalidValue;
  return launch_ex(kern, dim3(plan.grid), dim3(kThreads), plan.smem, stream, pdl, args);
}

template <int TT>
cudaError_t dispatch_rpw(const GemvArgs &args, const GemvPlan &plan, cudaStream_t stream, bool pdl,
                         bool topk) {
  if (topk) {
    switch (plan.rpw) {
      case 1: return launch_one<TT, 1, true>(args, plan, stream, pdl);
      case 2: return launch_one<TT, 2, true>(args, plan, stream, pdl);
      default: return launch_one<TT, 4, true>(args, plan, stream, pdl);
    }
  }
  switch (plan.rpw) {
    case 1: return launch_one<TT, 1, false>(args, plan, stream, pdl);
    case 2: return launch_one<TT, 2, false>(args, plan, stream, pdl);
    default: return launch_one<TT, 4, false>(args, plan, stream, pdl);
  }
}

size_t pow2_ceil(size_t v) {
  size_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

}  // namespace

bool plan_gemv(int T, int N, int k_pad, bool topk, int k, int sm_count, GemvPlan *plan,
               bool fused_x) {
  if (T < 1 || T > 8 || N < 1 || k_pad < 16 || (k_pad % 16) != 0 || sm_count < 1) return false;
  GemvPlan p = {};
  p.tt = T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8;
  if (fused_x && p.tt * k_pad > kFusedXMaxBytes) return false;
  p.fused_x = fused_x;
  const size_t xres = fused_x ? static_cast<size_t>(p.tt) * k_pad : 0;
  auto tiles = [&](int rb) { return (N + rb - 1) / rb; };
  const int min_tiles = 2 * sm_count;
  constexpr int kMaxStage = 32768;
  p.rpw = 1;
  if (k_pad * 8 <= kMaxStage) {
    // whole-row tiles (one contiguous block per stage), as many rows as balance allows
    for (int r : {4, 2})
      if (8 * r * k_pad <= kMaxStage && tiles(8 * r) >= min_tiles) {
        p.rpw = r;
        break;
      }
    p.kc = k_pad;
  } else {
    p.kc = kMaxStage / 8;
  }
  p.rb = 8 * p.rpw;
  p.nk = (k_pad + p.kc - 1) / p.kc;
  const size_t stage = static_cast<size_t>(p.rb + (fused_x ? 0 : p.tt)) * p.kc;
  p.num_tiles = tiles(p.rb);
  const size_t bars = 2 * kMaxStages * 8;
  if (!topk) {
    const size_t budget = 110 * 1024 - xres;
    p.ns = static_cast<int>(std::min<size_t>(kMaxStages, std::max<size_t>(2, budget / stage)));
    p.grid = std::min(p.num_tiles, 2 * sm_count);
    p.tiles_per_cta = (p.num_tiles + p.grid - 1) / p.grid;
    p.grid = (p.num_tiles + p.tiles_per_cta - 1) / p.tiles_per_cta;
    p.cand_cap = 0;
    p.xres_off = static_cast<uint32_t>(p.ns * stage + bars);
    p.smem = p.ns * stage + bars + xres;
  } else {
    if (k < 1 || k > 64 || k > N) return false;
    int grid = std::min(p.num_tiles, 2 * sm_count);
    size_t cap = 0;
    while (true) {
      const int tpc = (p.num_tiles + grid - 1) / grid;
      cap = pow2_ceil(static_cast<size_t>(tpc) * p.rb);
      if (static_cast<size_t>(p.tt) * cap * 8 <= 96 * 1024) break;
      if (grid >= p.num_tiles) return false;
      grid = std::min(p.num_tiles, grid * 2);
    }
    p.tiles_per_cta = (p.num_tiles + grid - 1) / grid;
    p.grid = (p.num_tiles + p.tiles_per_cta - 1) / p.tiles_per_cta;
    p.cand_cap = static_cast<int>(cap);
    const size_t cand_bytes = static_cast<size_t>(p.tt) * cap * 8;
    const size_t used = cand_bytes + xres;
    const size_t budget = 110 * 1024 > used + 2 * stage ? 110 * 1024 - used : 2 * stage;
    p.ns = static_cast<int>(std::min<size_t>(kMaxStages, std::max<size_t>(2, budget / stage)));
    const size_t ring = std::max<size_t>(p.ns * stage, kTopkStageBytes);
    p.xres_off = static_cast<uint32_t>(ring + bars + cand_bytes);
    p.smem = ring + bars + cand_bytes + xres;
  }
  if (p.smem > kMaxDynSmem) return false;
  *plan = p;
  return true;
}

namespace {

// The grid top-k selection of a multi-token GEMV, one CTA per token (tokens in parallel instead
// of one after another in the GEMV's last CTA): token blockIdx.x's top-k over the G per-CTA lists
// the GEMV wrote, into its output rows (or its owner's gather rows); then, in the last selection
// CTA to finish, the same publication as the GEMV's last CTA (system-scope fence, forward count,
// done counters).  The GEMV left st.arrive at zero; it counts the selection CTAs here and the
// last one re-zeroes it.
struct SelectArgs {
  GridTopkState st;
  int G, k, T, rows_per_cta;
  TopK tk;
  ShardSync sync;
};

constexpr int kSelectWarps = 8;
constexpr uint32_t kSelectSmemBytes = (kSelectWarps * 64 + kTopkGatherKeys) * 8;

template <int R>
__global__ void __launch_bounds__(kSelectWarps * 32) topk_select_kernel(const SelectArgs a) {
  extern __shared__ __align__(16) uint64_t sel_smem[];
  __shared__ int s_n, s_last;
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  uint64_t *stage = sel_smem;
  uint64_t *gather = sel_smem + kSelectWarps * 64;
  const int row_offset = a.tk.row_offset, rows_per_cta = a.rows_per_cta;
  auto list_of = [row_offset, rows_per_cta](uint64_t key) {
    return (topk_key_id(key) - row_offset) / rows_per_cta;
  };
  float *vr = a.tk.val + t * a.tk.k;
  int32_t *ir = a.tk.idx + t * a.tk.k;
  if (a.tk.val_dst) {
    const int g = a.tk.tok0 + t;
    const int64_t off = a.tk.dst_row0 + static_cast<int64_t>(g % a.tk.dst_tokens) * a.tk.dst_ld;
    vr = a.tk.val_dst[g / a.tk.dst_tokens] + off;
    ir = a.tk.idx_dst[g / a.tk.dst_tokens] + off;
  }
  grid_topk_select<R, kSelectWarps>(a.G, a.k, t, a.st, vr, ir, stage, gather, &s_n, warp, lane,
                                    BlockSync{}, list_of);
  const bool publish = (a.sync.done || a.sync.done_peers) && !a.sync.hold;
  if (publish) __threadfence_system();
  else __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    s_last = atomicAdd(a.st.arrive, 1u) == gridDim.x - 1;
    if (s_last) {
      *a.st.arrive = 0u;
      if (publish) {
        // every token's rows are stored: count the forward (a release of the rows)
        __threadfence_system();
        const unsigned e = *a.sync.seq + 1u;
        *a.sync.seq = e;
        if (a.sync.done) st_relaxed_sys(a.sync.done, e);
        for (int p = 0; p < a.sync.n_done; ++p) st_relaxed_sys(a.sync.done_peers[p], e);
      }
    }
  }
}

// One CTA's share of a token's grid top-k over kTopkRowsPerCta rows of fp32 logits (16 per
// thread, coalesced loads).  A key can be among the CTA's k largest only if it reaches T0, the
// k-th largest of the 256 threads' maxima (k distinct threads each hold a key >= T0), so only the
// keys >= T0 are gathered and sorted: on random logits about k + a few of the 4096.  Ties cannot
// defeat the bound (keys are unique: the vocab id is part of the key); adversarial logits only
// gather more keys, up to all of them.
constexpr int kRowsPerThread = kTopkRowsPerCta / (kSelectWarps * 32);
constexpr uint32_t kRowsOfferSmemBytes = (kSelectWarps * 64 + kTopkRowsPerCta) * 8;

struct RowsOfferArgs {
  const float *logits;
  int64_t ldl;
  int N, k, row_offset;
  GridTopkState st;
};

template <int R>
__global__ void __launch_bounds__(kSelectWarps * 32) topk_rows_offer_kernel(const RowsOfferArgs a) {
  extern __shared__ __align__(16) uint64_t offer_smem[];
  __shared__ int s_n;
  uint64_t *stage = offer_smem;                     // kSelectWarps * 32R keys
  uint64_t *pool = offer_smem + kSelectWarps * 64;  // the threads' maxima, then the survivors
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x, b = blockIdx.x, t = blockIdx.y;
  const int n0 = b * kTopkRowsPerCta;
  const int rows = min(kTopkRowsPerCta, a.N - n0);
  const float *row = a.logits + static_cast<size_t>(t) * a.ldl + n0;
  uint64_t key[kRowsPerThread];
  uint64_t m = 0ull;
#pragma unroll
  for (int j = 0; j < kRowsPerThread; ++j) {
    const int i = tid + j * kSelectWarps * 32;
    key[j] = i < rows ? topk_key(row[i], static_cast<uint32_t>(a.row_offset + n0 + i)) : 0ull;
    m = max_u64(m, key[j]);
  }
  pool[tid] = m;
  if (tid == 0) s_n = 0;
  __syncthreads();
  cta_top_keys<R, kSelectWarps>(pool, kSelectWarps * 32, false, stage, warp, lane, BlockSync{});
  // 0 when fewer than k threads hold a row: every key survives
  const uint64_t t0 = stage[a.k - 1];
  // append the survivors to the pool (warp-aggregated slots)
#pragma unroll
  for (int j = 0; j < kRowsPerThread; ++j) {
    const bool keep = key[j] != 0ull && key[j] >= t0;
    const unsigned mask = __ballot_sync(0xFFFFFFFFu, keep);
    if (mask) {
      int slot = 0;
      if (lane == 0) slot = atomicAdd(&s_n, __popc(mask));
      slot = __shfl_sync(0xFFFFFFFFu, slot, 0);
      if (keep) pool[slot + __popc(mask & ((1u << lane) - 1u))] = key[j];
    }
  }
  __syncthreads();
  cta_top_keys<R, kSelectWarps>(pool, s_n, false, stage, warp, lane, BlockSync{});
  if (warp == 0) {
    uint64_t *base = a.st.keys + t * grid_topk_stride(G, a.k);
    uint64_t *list = base + static_cast<size_t>(b) * a.k;
    for (int e = lane; e < a.k; e += 32) list[e] = stage[e];
    if (lane == 0) base[static_cast<size_t>(G) * a.k + b] = stage[0];
  }
}

}  // namespace

cudaError_t launch_topk_rows(const float *logits, int64_t ldl, int T, int N, const TopK &tk,
                             bool pdl, cudaStream_t stream) {
  const int G = topk_rows_grid(N);
  const GridTopkState st{tk.counter, tk.lists};
  const RowsOfferArgs oa{logits, ldl, N, tk.k, tk.row_offset, st};
  static_assert(kRowsOfferSmemBytes <= 48 * 1024, "within the default dynamic shared memory");
  cudaError_t e =
      tk.k > 32 ? launch_ex(topk_rows_offer_kernel<2>, dim3(G, T), dim3(kSelectWarps * 32),
                            kRowsOfferSmemBytes, stream, pdl, oa)
                : launch_ex(topk_rows_offer_kernel<1>, dim3(G, T), dim3(kSelectWarps * 32),
                            kRowsOfferSmemBytes, stream, pdl, oa);
  if (e != cudaSuccess) return e;
  SelectArgs sa = {};
  sa.st = st;
  sa.G = G;
  sa.k = tk.k;
  sa.T = T;
  sa.rows_per_cta = kTopkRowsPerCta;
  sa.tk = tk;
  if (tk.k > 32)
    return launch_ex(topk_select_kernel<2>, dim3(T), dim3(kSelectWarps * 32), kSelectSmemBytes,
                     stream, true, sa);
  return launch_ex(topk_select_kernel<1>, dim3(T), dim3(kSelectWarps * 32), kSelectSmemBytes,
                   stream, true, sa);
}

cudaError_t launch_gemv(const GemvLaunch &L, const GemvPlan &plan, cudaStream_t stream) {
  GemvArgs a;
  a.w = L.w;
  a.ldw = L.ldw;
  a.x = L.x;
  a.ldx = L.ldx;
  a.T = L.T;
  a.N = L.N;
  a.k_pad = L.k_pad;
  a.kc = plan.kc;
  a.nk = plan.nk;
  a.ns = plan.ns;
  a.num_tiles = plan.num_tiles;
  a.tiles_per_cta = plan.tiles_per_cta;
  a.cand_cap = plan.cand_cap;
  a.stage_bytes = static_cast<uint32_t>((plan.rb + (plan.fused_x ? 0 : plan.tt)) * plan.kc);
  a.ring_bytes = static_cast<uint32_t>(plan.ns) * a.stage_bytes;
  if (L.topk) a.ring_bytes = std::max(a.ring_bytes, kTopkStageBytes);
  a.ep = L.ep;
  a.tk = L.tk;
  a.err = L.err;
  a.trace = L.trace;
  a.sync = L.sync;
  a.fq = L.fq;
  a.xres_off = plan.xres_off;
  if ((L.fq.x != nullptr) != plan.fused_x) return cudaErrorInvalidValue;
  // several tokens: their selections run in parallel in a kernel of their own
  a.split_select = (L.topk && L.T >= 2) ? 1 : 0;
  cudaError_t e;
  switch (plan.tt) {
    case 1: e = dispatch_rpw<1>(a, plan, stream, L.pdl, L.topk); break;
    case 2: e = dispatch_rpw<2>(a, plan, stream, L.pdl, L.topk); break;
    case 4: e = dispatch_rpw<4>(a, plan, stream, L.pdl, L.topk); break;
    default: e = dispatch_rpw<8>(a, plan, stream, L.pdl, L.topk); break;
  }
  if (e != cudaSuccess || !a.split_select) return e;
  SelectArgs sa;
  sa.st = GridTopkState{L.tk.counter, L.tk.lists};
  sa.G = plan.grid;
  sa.k = L.tk.k;
  sa.T = L.T;
  sa.rows_per_cta = plan.tiles_per_cta * plan.rb;
  sa.tk = L.tk;
  sa.sync = L.sync;
  static_assert(kSelectSmemBytes <= 48 * 1024, "within the default dynamic shared memory");
  if (L.tk.k > 32)
    return launch_ex(topk_select_kernel<2>, dim3(L.T), dim3(kSelectWarps * 32), kSelectSmemBytes,
                     stream, true, sa);
  return launch_ex(topk_select_kernel<1>, dim3(L.T), dim3(kSelectWarps * 32), kSelectSmemBytes,
                   stream, true, sa);
}

}  // namespace w8a8
