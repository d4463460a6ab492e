// Grid-wide top-k (k <= 64) of the LM-head logits, fused into the epilogue of a GEMV grid.
//
// Keys are the 64-bit order keys of topk_key (value descending, then vocab id ascending; key 0
// marks an empty slot and sorts last), so "the k largest keys" is the reference's greedy /
// top-k order (src/eswin_runtime/src/nlp/sampler.cpp:93-121, ties to the lower id).
//
// Three pieces:
//   * warp lists: a warp holds 32*R keys (R = 1 or 2), lane l owning elements l and l + 32, and
//     sorts them (bitonic network over shuffles) or merges a second sorted list into them,
//     keeping the larger half (max of a[e] and b[last - e] is bitonic, then one bitonic merge);
//   * cta_top_keys: every warp folds chunks of 32R keys into its own list, then the warps'
//     lists are merged pairwise in a tree through shared memory;
//   * the grid protocol: each CTA writes its sorted top-k list and, separately, the list's head
//     (its largest key).  The last CTA to arrive takes T0 = the k-th largest head: k distinct
//     keys are >= T0, so every key of the grid's top-k is >= T0, and only the k lists whose
//     head reaches T0 can hold such keys.  One thread per such list walks its prefix >= T0 (on
//     random logits about k + a few keys in all; never more than k * k) and the top-k of the
//     gathered keys is the grid's.
#pragma once

#include "common.cuh"

namespace w8a8 {

// Buffers of one grid-wide top-k.  Per token t, keys + t * stride(k) holds gridDim.x sorted
// lists of k keys, then gridDim.x heads.
struct GridTopkState {
  unsigned *arrive;  // CTA arrival counter (zero between launches; the last CTA re-zeroes it)
  uint64_t *keys;
};

__host__ __device__ inline size_t grid_topk_stride(int grid, int k) {
  return static_cast<size_t>(grid) * (k + 1);
}

// Shared memory the last CTA gathers the candidate prefixes in.
constexpr int kTopkGatherKeys = 64 * 64;

__device__ __forceinline__ uint64_t max_u64(uint64_t a, uint64_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint64_t min_u64(uint64_t a, uint64_t b) { return a < b ? a : b; }

// One compare-exchange stage of a bitonic network on a warp list: elements e and e ^ d, the
// lower one keeping the larger key where (e & size) == 0 (descending runs of `size`).
template <int R>
__device__ __forceinline__ void warp_bitonic_stage(uint64_t (&v)[R], int lane, int size, int d) {
  if (R == 2 && d == 32) {
    // partner in the same lane; only reached with size 64, a single descending run
    const uint64_t hi = max_u64(v[0], v[R - 1]);
    const uint64_t lo = min_u64(v[0], v[R - 1]);
    v[0] = hi;
    v[R - 1] = lo;
    return;
  }
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v[j], d);
    const int e = lane + 32 * j;
    const bool keep_max = ((lane & d) == 0) == ((e & size) == 0);
    v[j] = keep_max ? max_u64(v[j], w) : min_u64(v[j], w);
  }
}

// Sorts a warp list descending.
template <int R>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&v)[R], int lane) {
#pragma unroll
  for (int size = 2; size <= 32 * R; size <<= 1)
#pragma unroll
    for (int d = size >> 1; d > 0; d >>= 1) warp_bitonic_stage<R>(v, lane, size, d);
}

// a := the 32R largest of a and b (both sorted descending), sorted descending.
template <int R>
__device__ __forceinline__ void warp_merge_desc(uint64_t (&a)[R], const uint64_t (&b)[R], int lane) {
#pragma unroll
  for (int j = 0; j < R; ++j) {
    // element 32R-1-e of b, e = lane + 32 j, sits in lane 31 - lane, register R-1-j
    const uint64_t w = __shfl_sync(0xFFFFFFFFu, b[R - 1 - j], 31 - lane);
    a[j] = max_u64(a[j], w);
  }
#pragma unroll
  for (int d = 16 * R; d > 0; d >>= 1) warp_bitonic_stage<R>(a, lane, 64 * R, d);
}

// The 32R largest of keys[0..n) (0 past n), sorted descending, into stage[0..32R), visible to
// every warp when the call returns.  Warps 0..NW-1 take part and sync() is a barrier over
// exactly them; `stage` holds NW * 32R keys of shared memory.  Only the first ceil(n / 32R)
// warps (at most NW) hold a chunk and take part in the tree.  cg: the keys were written by
// other CTAs of the grid (read through L2).  Not inlined: the per-CTA lists and the last CTA's
// selection run the same code, so the selection finds it in the SM's instruction cache.
template <int R, int NW, typename Sync>
__device__ __noinline__ void cta_top_keys(const uint64_t *keys, int n, bool cg, uint64_t *stage,
                                          int warp, int lane, Sync sync) {
  constexpr int L = 32 * R;
  const int chunks = (n + L - 1) / L;
  const int act = chunks < 1 ? 1 : (chunks < NW ? chunks : NW);
  uint64_t a[R];
  bool first = true;
#pragma unroll
  for (int j = 0; j < R; ++j) a[j] = 0ull;
  for (int c = warp * L; c < n; c += NW * L) {
    uint64_t b[R];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int i = c + lane + 32 * j;
      b[j] = i >= n ? 0ull
             : cg   ? __ldcg(reinterpret_cast<const unsigned long long *>(keys) + i)
                    : keys[i];
    }
    warp_sort_desc<R>(b, lane);
    if (first) {
#pragma unroll
      for (int j = 0; j < R; ++j) a[j] = b[j];
      first = false;
    } else {
      warp_merge_desc<R>(a, b, lane);
    }
  }
  if (warp < act) {
#pragma unroll
    for (int j = 0; j < R; ++j) stage[warp * L + lane + 32 * j] = a[j];
  }
  sync();
  for (int s = 1; s < act; s <<= 1) {
    if ((warp & (2 * s - 1)) == 0 && warp + s < act) {
      uint64_t b[R];
#pragma unroll
      for (int j = 0; j < R; ++j) b[j] = stage[(warp + s) * L + lane + 32 * j];
      warp_merge_desc<R>(a, b, lane);
#pragma unroll
      for (int j = 0; j < R; ++j) stage[warp * L + lane + 32 * j] = a[j];
    }
    sync();
  }
}

// This CTA's share of token t's grid top-k: its sorted top k of cand[0..n) (0 past n) and the
// list's head.  Returns after a sync() over the NW warps.
template <int R, int NW, typename Sync>
__device__ void grid_topk_offer(const uint64_t *cand, int n, int k, int t, const GridTopkState &st,
                                uint64_t *stage, int warp, int lane, Sync sync) {
  cta_top_keys<R, NW>(cand, n, false, stage, warp, lane, sync);
  if (warp == 0) {
    uint64_t *base = st.keys + t * grid_topk_stride(gridDim.x, k);
    uint64_t *list = base + static_cast<size_t>(blockIdx.x) * k;
    for (int e = lane; e < k; e += 32) list[e] = stage[e];
    if (lane == 0) base[static_cast<size_t>(gridDim.x) * k + blockIdx.x] = stage[0];
  }
  sync();
}

// Arrival after every token's offer: true in the one CTA that arrives last (which then runs
// grid_topk_select).  Publishes this CTA's lists first.
template <typename Sync>
__device__ bool grid_topk_arrive(const GridTopkState &st, int tid, int *s_flag, Sync sync) {
  __threadfence();
  sync();
  if (tid == 0) *s_flag = atomicAdd(st.arrive, 1u) == gridDim.x - 1;
  sync();
  const bool last = *s_flag != 0;
  if (last) __threadfence();
  return last;
}

// Last CTA (or a selection CTA of its own): token t's top-k over the G lists of the grid into
// val_row[0 .. k) / idx_row[0 .. k) (the token's output rows).  NW * 32 threads (tid < NW * 32)
// take part;
// `stage` holds NW * 32R keys and `gather` kTopkGatherKeys keys of shared memory; s_int is one
// shared int.  list_of(key) gives the index of the CTA (list) that owns a key's vocab row.
// Returns after a sync() over the NW warps.
template <int R, int NW, typename Sync, typename ListOf>
__device__ void grid_topk_select(int G, int k, int t, const GridTopkState &st, float *val_row,
                                 int32_t *idx_row, uint64_t *stage, uint64_t *gather, int *s_int,
                                 int warp, int lane, Sync sync, ListOf list_of) {
  const uint64_t *base = st.keys + t * grid_topk_stride(G, k);
  const uint64_t *heads = base + static_cast<size_t>(G) * k;
  // the k largest heads; T0 = the k-th (0 when fewer than k lists are non-empty)
  cta_top_keys<R, NW>(heads, G, true, stage, warp, lane, sync);
  const uint64_t t0 = stage[k - 1];
  const int tid = warp * 32 + lane;
  if (tid == 0) *s_int = 0;
  sync();
  // Thread j < k walks the list headed by the j-th largest head: the head itself, then the
  // entries after it while they reach T0 (four loads in flight per step).
  if (tid < k) {
    const uint64_t head = stage[tid];
    if (head != 0ull) {
      gather[atomicAdd(s_int, 1)] = head;
      const unsigned long long *list =
          reinterpret_cast<const unsigned long long *>(base) + static_cast<size_t>(list_of(head)) * k;
      for (int j = 1; j < k; j += 4) {
        uint64_t e[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) e[u] = j + u < k ? __ldcg(list + j + u) : 0ull;
        bool more = true;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          more = more && e[u] != 0ull && e[u] >= t0;
          if (more) gather[atomicAdd(s_int, 1)] = e[u];
        }
        if (!more) break;
      }
    }
  }
  sync();
  // the usual case is about k + a few candidates: one chunk, no tree
  cta_top_keys<R, NW>(gather, *s_int, false, stage, warp, lane, sync);
  if (warp == 0) {
    for (int e = lane; e < k; e += 32) {
      val_row[e] = topk_key_value(stage[e]);
      idx_row[e] = topk_key_id(stage[e]);
    }
  }
  sync();
}

}  // namespace w8a8
