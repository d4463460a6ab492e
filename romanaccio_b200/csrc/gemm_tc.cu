// Tensor-core W8A8 contraction for token counts above the GEMV range (prefill, batched decode):
// tcgen05.mma kind::i8 with int32 accumulators in TMEM.  Weights live in HBM as contiguous 16 KB
// tiles already in the 128-byte-swizzled shared-memory image (launch_tile_weights), so one 1-D bulk
// copy per stage streams them at full DRAM efficiency; activations arrive by 2-D TMA tiles with the
// 128-byte swizzle.  Every copy is a plain per-CTA load.
//
// Math: acc[t, n] = sum_k q[t, k] * Wq[n, k] in exact int32 (the CMAC step, cmac.py:300-383 of
// the reference's NPU model), then the per-output-channel epilogue shared with the GEMV kernels:
// CvtPrecision_QuantM requant (attribute_int8_error.py:104-122) and the out_step / acc_step
// dequant with the dyntok ratio (src/LFM3/lfm3_v2.cpp:971-1008, 1143-1183).
//
// Orientation: the weight tile is the MMA's A operand (M = 128 output channels = the 128 TMEM
// lanes) and the token tile is B (N = BT tokens = TMEM columns).  Each epilogue thread owns one
// output channel, so QuantM / out_step are per-thread constants and one warp's stores for one
// token are 32 consecutive channels.
//
// Work split: units of (channel block, token block, K split), walked persistently by the CTAs
// (unit = blockIdx.x + i * gridDim.x).  The accumulator is double-buffered in TMEM, so the
// epilogue of one unit overlaps the main loop of the next.  When the channel x token tiles do not
// fill the SMs, K is split: each split adds its int32 partial tile into one accumulation plane
// (L2 reductions), and the last split of a tile to arrive (an arrival counter per tile) reads the
// totals, resets them to zero and runs the epilogue.  Integer sums are exact in any order.
//
// Warp roles (576 threads): warp 0 issues the TMA copies, warp 1 owns TMEM and issues the MMAs
// (one thread), warps 2..17 run the epilogue; warp w reads TMEM lanes 32*(w%4)..+31 (the lane
// quarter a warp may access is fixed by its id modulo 4) and every 4th column chunk from (w-2)/4.
#include <cuda.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace w8a8 {
namespace {

constexpr int kEpiWarps = 16;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer warp, MMA warp, epilogue warps
constexpr int kColGroups = kEpiWarps / 4;    // epilogue warps sharing one TMEM lane quarter
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kBM = 128;                       // output channels per tile (MMA M)
constexpr int kBK = 128;                       // K bytes per stage = one 128-byte swizzle row
constexpr int kMmaK = 32;                      // K of one tcgen05.mma kind::i8
constexpr uint32_t kTileWBytes = kBM * kBK;    // weight bytes per stage
constexpr int kMaxStages = 16;
constexpr int kMaxBT = 256;
constexpr int kMaxDynSmem = 232448;            // sm_100 opt-in limit per block

struct TcArgs {
  int N, T, BT;
  int tiles_t, splits, k_iters, ips, units, ns;
  uint32_t stage_bytes, buf_stride, tmem_cols, idesc;
  Epilogue ep;
  const int8_t *w_tiles;  // [tiles_n][k_iters] contiguous 16 KB swizzled weight tiles
  int32_t *ws;            // split-K accumulation plane [T, N] (all zero between launches)
  unsigned *tile_count;   // split-K arrival counters [tiles] (all zero between launches)
  int *err;
  int w_stream;           // weights read once (one token block): evict-first L2 policy
  unsigned long long *trace;  // optional [grid, 8] %globaltimer stamps (see stamp())
};

// Diagnostic timeline of a CTA (only when a trace buffer is attached): 0 entry, 1 setup done,
// 2 first stage issued, 3 first stage landed (MMA issuer), 4 first unit's MMAs committed,
// 5 epilogue saw the first accumulator, 6 epilogue released it, 7 exit.
__device__ __forceinline__ void stamp(const TcArgs &a, int i) {
  if (a.trace) a.trace[blockIdx.x * 8 + i] = global_timer_ns();
}

// ------------------------------------------------------------------------------------------
// tcgen05 / TMA wrappers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; the wait is inside the same statement so no use of
// the registers can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  __syncwarp();  // .sync.aligned: the whole warp executes it together
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- CTA pair (cluster of two) helpers ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrives on an mbarrier of the other CTA of the pair (address from map_to_rank).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Bounded wait on a local mbarrier phase completed by arrivals from the other CTA (acquire at
// cluster scope).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, int *err, int code) {
  auto try_wait = [&]() {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
  };
  if (try_wait()) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (try_wait()) return true;
    if ((i & 511u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, code);
      return false;
    }
  }
}

// 2-D tensor copy into this CTA's shared memory whose completion (complete_tx) is signalled on
// the mbarrier at cluster address `bar`, which may be the other CTA's of the pair (.cta_group::2).
// A plain per-CTA load: no multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair_hint(uint32_t dst, const CUtensorMap *map, int c0,
                                                      int c1, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// The pair's MMA (issued by the even CTA): A = both CTAs' 128-row weight halves (M = 256),
// B = both CTAs' token halves (N = BT), D = each CTA's own TMEM (its 128 channels).
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on the mbarrier at offset `bar` in both CTAs of the pair once the MMAs issued so far
// have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar), "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte swizzle:
// rows of 128 bytes, 8-row swizzle atoms 1024 bytes apart (stride byte offset), leading byte
// offset unused (encoded 1), descriptor version 1, layout type 2 = SWIZZLE_128B.  The tile base
// is 1024-byte aligned, so the base-offset field is 0.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
}

// ------------------------------------------------------------------------------------------
// Epilogue: one thread = one output channel n; TMEM columns = tokens.  Specialised per output
// mode so that the per-element code is a short straight line.  MODE = w8a8_out_mode, plus
// kRqInt when the requant runs in 32-bit funnel-shift arithmetic (15 <= trunc <= 31) rather than
// in float64; both give the exact integer of requant_quantm.
// ------------------------------------------------------------------------------------------
constexpr int kRqInt = 4;

struct ChanParams {
  int32_t qm;
  long long bias;  // 2^(trunc-1) - 1
  double scale;    // QuantM[n] * 2^-trunc
  double qmax;
  float step;      // out_step[n] (F32) or acc_step[n] (F32_ACC)
};

template <int MODE>
__device__ __forceinline__ ChanParams chan_params(const Epilogue &ep, int n, bool n_ok) {
  constexpr int base = MODE & 3;
  ChanParams cp{0, (1LL << (ep.trunc > 0 ? ep.trunc - 1 : 0)) - 1, 0.0,
                static_cast<double>(ep.qmax), 0.0f};
  if (!n_ok) return cp;
  if (base == kOutQuant || base == kOutF32) {
    cp.qm = ep.quant_m[n];
    cp.scale = quantm_scale(cp.qm, ep.trunc);
  }
  if (base == kOutF32) cp.step = ep.out_step[n];
  if (base == kOutF32Acc) cp.step = ep.acc_step[n];
  return cp;
}

template <int MODE>
__device__ __forceinline__ int out_size(const Epilogue &ep) {
  return (MODE & 3) == kOutQuant ? (ep.out_i16 ? 2 : 1) : 4;
}

template <int MODE>
__device__ __forceinline__ int32_t requant(const Epilogue &ep, const ChanParams &cp, int32_t acc) {
  if (MODE & kRqInt) return requant_quantm_t15(acc, cp.qm, ep.trunc, cp.bias, ep.qmax);
  return requant_f64(acc, cp.scale, cp.qmax);
}

// Output value of (channel, token t) written at p.
template <int MODE>
__device__ __forceinline__ void emit(const Epilogue &ep, const ChanParams &cp, int32_t acc, int t,
                                     char *p) {
  constexpr int base = MODE & 3;
  if (base == kOutAccI32) {
    *reinterpret_cast<int32_t *>(p) = acc;
  } else if (base == kOutQuant) {
    const int yq = requant<MODE>(ep, cp, acc);
    if (ep.out_i16)
      *reinterpret_cast<int16_t *>(p) = static_cast<int16_t>(yq);
    else
      *reinterpret_cast<int8_t *>(p) = static_cast<int8_t>(yq);
  } else if (base == kOutF32) {
    const int yq = requant<MODE>(ep, cp, acc);
    const float step = ep.act_mode == kActDyntok ? ep.ratio[t] * cp.step : cp.step;
    *reinterpret_cast<float *>(p) = static_cast<float>(yq) * step;
  } else {
    const float step = ep.act_mode == kActDyntok ? ep.ratio[t] * cp.step : cp.step;
    *reinterpret_cast<float *>(p) = __int2float_rn(acc) * step;
  }
}

// Epilogue column chunk: 16 TMEM columns per tcgen05.ld (keeps the 16 epilogue warps within
// their register budget).
constexpr int kCW = 16;

template <int CW>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[CW]) {
  static_assert(CW == 16, "16-column TMEM loads");
  tmem_ld16(taddr, v);
}

// Split-K: this split's partial tile added into the workspace's accumulation plane (reductions
// in L2, no result awaited; int32 sums wrap, so their order does not change the total).
template <int CW>
__device__ __forceinline__ void add_partials(int32_t *plane_n, int N, uint32_t trow, int c_first,
                                             int t_base, int t_lim, bool n_ok) {
  for (int c = c_first; c < t_lim; c += kColGroups * CW) {
    uint32_t v[CW];
    tmem_ld<CW>(trow + c, v);
    if (!n_ok) continue;
    int32_t *p = plane_n + static_cast<size_t>(t_base + c) * N;
#pragma unroll
    for (int i = 0; i < CW; ++i)
      if (c + i < t_lim) atomicAdd(p + static_cast<size_t>(i) * N, static_cast<int32_t>(v[i]));
  }
}

// Final values of this thread's channel for its columns through the output mode: the
// accumulator, or with split-K the accumulation plane's totals (every split's partial tile, this
// one's included), which are read once and reset to zero for the next launch.
template <int MODE, int CW>
__device__ __forceinline__ void finish_columns(const Epilogue &ep, const ChanParams &cp,
                                               uint32_t trow, int c_first, int t_base, int t_lim,
                                               int n, bool n_ok, int32_t *ws, int N, int splits) {
  const int esize = out_size<MODE>(ep);
  char *col = static_cast<char *>(ep.y) + static_cast<size_t>(n) * esize;
  const size_t ldb = static_cast<size_t>(ep.ldy) * esize;
  for (int c = c_first; c < t_lim; c += kColGroups * CW) {
    uint32_t v[CW];
    tmem_ld<CW>(trow + c, v);
    if (!n_ok) continue;
    if (splits > 1) {
      int32_t *p = ws + static_cast<size_t>(t_base + c) * N + n;
#pragma unroll
      for (int i = 0; i < CW; ++i)
        if (c + i < t_lim) v[i] = static_cast<uint32_t>(__ldcg(p + static_cast<size_t>(i) * N));
#pragma unroll
      for (int i = 0; i < CW; ++i)
        if (c + i < t_lim) __stcg(p + static_cast<size_t>(i) * N, 0);
    }
#pragma unroll
    for (int i = 0; i < CW; ++i) {
      if (c + i < t_lim) {
        const int t = t_base + c + i;
        emit<MODE>(ep, cp, static_cast<int32_t>(v[i]), t, col + static_cast<size_t>(t) * ldb);
      }
    }
  }
}

struct Unit {
  int nb, tb, split, tile, k_begin, k_end;
};

__device__ __forceinline__ Unit decode_unit(const TcArgs &a, int u) {
  Unit r;
  r.split = u % a.splits;
  r.tile = u / a.splits;
  r.tb = r.tile % a.tiles_t;
  r.nb = r.tile / a.tiles_t;
  r.k_begin = r.split * a.ips;
  r.k_end = min(r.k_begin + a.ips, a.k_iters);
  return r;
}

// A CTA pair's unit u: 256 channels (this CTA's 128: channel block 2 * (u / tiles_t) + rank)
// by BT tokens, the whole K.
__device__ __forceinline__ Unit decode_pair_unit(const TcArgs &a, int u, uint32_t rank) {
  Unit r;
  r.split = 0;
  r.tile = u;
  r.tb = u % a.tiles_t;
  r.nb = 2 * (u / a.tiles_t) + static_cast<int>(rank);
  r.k_begin = 0;
  r.k_end = a.k_iters;
  return r;
}

// The epilogue warps' loop over this CTA's units (PAIR: over its pair's units, handing the
// accumulator buffer back to the even CTA, which issues the pair's MMAs).
template <int MODE, bool PAIR>
__device__ __forceinline__ void epilogue_role(const TcArgs &a, uint32_t tmem, uint32_t tfull0,
                                              uint32_t tempty0, int warp, int lane, int *s_last) {
  const Epilogue &ep = a.ep;
  const int q = warp & 3;
  const int group = (warp - 2) >> 2;  // column group of this warp
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  bool ok = true;
  int j = 0;
  const int u0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int du = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  for (int u = u0; u < a.units; u += du, ++j) {
    const Unit un = PAIR ? decode_pair_unit(a, u, rank) : decode_unit(a, u);
    const int buf = j & 1, use = j >> 1;
    if (ok) ok = mbar_wait_bounded(tfull0 + 8 * buf, use & 1, a.err, kDevTimeoutFull);
    // tcgen05.ld is warp-collective: the whole warp takes the same branch.
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (j == 0 && threadIdx.x == 64) stamp(a, 5);
    const int n = un.nb * kBM + q * 32 + lane;
    const bool n_ok = n < a.N;
    const int t_base = un.tb * a.BT;
    const int t_lim = min(a.BT, a.T - t_base);
    const uint32_t trow = tmem + buf * a.buf_stride + (static_cast<uint32_t>(q * 32) << 16);
    bool finish = true;
    if (a.splits > 1) {
      // Split-K: every split adds its partial tile into the accumulation plane (coalesced L2
      // reductions); the last split of the tile to arrive reads the totals in one pass, resets
      // them to zero and runs the epilogue.
      if (ok) add_partials<kCW>(a.ws + n, a.N, trow, group * kCW, t_base, t_lim, n_ok);
      __threadfence();
      epi_bar_sync();
      if (threadIdx.x == 64) {
        const unsigned prev = atomicAdd(a.tile_count + un.tile, 1u);
        *s_last = (prev == static_cast<unsigned>(a.splits - 1)) ? 1 : 0;
        if (*s_last) a.tile_count[un.tile] = 0u;
      }
      epi_bar_sync();
      finish = *s_last != 0;
      if (finish) __threadfence();
    }
    if (ok && finish) {
      const ChanParams cp = chan_params<MODE>(ep, n, n_ok);
      finish_columns<MODE, kCW>(ep, cp, trow, group * kCW, t_base, t_lim, n, n_ok, a.ws, a.N,
                                a.splits);
    }
    // TMEM buffer free for the next unit's MMAs.
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (PAIR && rank != 0)
        mbar_arrive_remote(map_to_rank(tempty0 + 8 * buf, 0));
      else
        mbar_arrive(tempty0 + 8 * buf);
    }
    if (j == 0 && threadIdx.x == 64) stamp(a, 6);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8a8_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 5];
  __shared__ uint32_t s_tmem;
  __shared__ int s_last;

  // Tiles start on a 1024-byte boundary (the 128-byte swizzle pattern repeats every 1024 bytes).
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t tiles = (raw + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full0 = smem_addr(&bars[0]);
  const uint32_t empty0 = smem_addr(&bars[kMaxStages]);
  const uint32_t tfull0 = smem_addr(&bars[2 * kMaxStages]);
  const uint32_t tempty0 = smem_addr(&bars[2 * kMaxStages + 2]);
  const uint32_t epi_done = smem_addr(&bars[2 * kMaxStages + 4]);

  if (threadIdx.x == 0) {
    stamp(a, 0);
    for (int s = 0; s < a.ns; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, kEpiWarps);
    }
    mbar_init(epi_done, kEpiWarps);
    fence_barrier_init();
  }
  __syncwarp();
  if (warp == 1) tmem_alloc(smem_addr(&s_tmem), a.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  if (threadIdx.x == 0) stamp(a, 1);

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      const uint64_t pol_w = a.w_stream ? policy_evict_first() : policy_evict_last();
      bool ok = true, dep_done = false;
      uint32_t g = 0;
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        const Unit un = decode_unit(a, u);
        for (int kit = un.k_begin; kit < un.k_end; ++kit, ++g) {
          const uint32_t s = g % a.ns, use = g / a.ns;
          if (use > 0) ok = mbar_wait_bounded(empty0 + 8 * s, (use - 1) & 1, a.err, kDevTimeoutEmpty);
          if (!ok) break;
          const uint32_t full = full0 + 8 * s;
          const uint32_t dst = tiles + s * a.stage_bytes;
          mbar_arrive_expect_tx(full, a.stage_bytes);
          // One contiguous 16 KB weight tile, already in the swizzled shared-memory image.
          bulk_g2s(dst, a.w_tiles + (static_cast<size_t>(un.nb) * a.k_iters + kit) * kTileWBytes,
                   kTileWBytes, full, pol_w);
          // Activations are written by the previous kernel in the stream: wait for it only now,
          // after the first weight copy is in flight.
          if (!dep_done) {
            pdl_wait();
            dep_done = true;
          }
          tma_load_2d(dst + kTileWBytes, &tm_x, kit * kBK, un.tb * a.BT, full);
          if (g == 0) stamp(a, 2);
        }
      }
      // Copies still in flight target this CTA's shared memory: let the last ones land before
      // the CTA may exit (the earlier ones were waited for by the MMA issuer).
      const uint32_t first = g > static_cast<uint32_t>(a.ns) ? g - a.ns : 0u;
      for (uint32_t i = first; i < g; ++i)
        if (!mbar_wait_bounded(full0 + 8 * (i % a.ns), (i / a.ns) & 1, a.err, kDevTimeoutFull)) break;
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      bool ok = true;
      uint32_t g = 0;
      int j = 0;
      for (int u = blockIdx.x; u < a.units; u += gridDim.x, ++j) {
        const Unit un = decode_unit(a, u);
        const int buf = j & 1, use = j >> 1;
        if (ok && use > 0)
          ok = mbar_wait_bounded(tempty0 + 8 * buf, (use - 1) & 1, a.err, kDevTimeoutEmpty);
        tc_fence_after();
        const uint32_t d = tmem + buf * a.buf_stride;
        for (int kit = un.k_begin; kit < un.k_end && ok; ++kit, ++g) {
          const uint32_t s = g % a.ns, su = g / a.ns;
          ok = mbar_wait_bounded(full0 + 8 * s, su & 1, a.err, kDevTimeoutFull);
          if (!ok) break;
          if (g == 0) stamp(a, 3);
          tc_fence_after();
          const uint32_t base = tiles + s * a.stage_bytes;
          const uint64_t adesc = smem_desc_sw128(base);
          const uint64_t bdesc = smem_desc_sw128(base + kTileWBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk) {
            // +32 bytes along K inside the swizzled row = +2 in the descriptor's address field.
            mma_i8(d, adesc + 2 * kk, bdesc + 2 * kk, a.idesc,
                   (kit > un.k_begin || kk > 0) ? 1u : 0u);
          }
          mma_commit(empty0 + 8 * s);
        }
        // Always released (also after a timeout) so that the epilogue warps do not wait twice.
        mma_commit(tfull0 + 8 * buf);
        if (j == 0) stamp(a, 4);
        if (!ok) break;
      }
    }
  } else {
    // ------------------------------- epilogue -------------------------------
    pdl_wait();
    const int rq_int = (a.ep.trunc >= 15 && a.ep.trunc <= 31) ? kRqInt : 0;
    switch (a.ep.out_mode | rq_int) {
      case kOutAccI32:
      case kOutAccI32 | kRqInt:
        epilogue_role<kOutAccI32, false>(a, tmem, tfull0, tempty0, warp, lane, &s_last);
        break;
      case kOutQuant: epilogue_role<kOutQuant, false>(a, tmem, tfull0, tempty0, warp, lane, &s_last); break;
      case kOutQuant | kRqInt:
        epilogue_role<kOutQuant | kRqInt, false>(a, tmem, tfull0, tempty0, warp, lane, &s_last);
        break;
      case kOutF32: epilogue_role<kOutF32, false>(a, tmem, tfull0, tempty0, warp, lane, &s_last); break;
      case kOutF32 | kRqInt:
        epilogue_role<kOutF32 | kRqInt, false>(a, tmem, tfull0, tempty0, warp, lane, &s_last);
        break;
      default: epilogue_role<kOutF32Acc, false>(a, tmem, tfull0, tempty0, warp, lane, &s_last); break;
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(epi_done);
  }

  // TMEM is released only after every epilogue warp has signalled, through an mbarrier, that its
  // last TMEM read completed (the block barrier alone was seen to let the producer and MMA warps
  // through while the epilogue was still draining).
  __syncwarp();
  if (warp == 1) {
    mbar_wait_bounded(epi_done, 0, a.err, kDevTimeoutFull);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
  __syncthreads();
  if (threadIdx.x == 0) stamp(a, 7);
}

// The CTA-pair kernel (clusters of two, launched with a cluster dimension of 2).  Each CTA loads
// its own operand halves into the same shared-memory offsets as its peer, by 2-D tensor copies
// (weights: the pre-swizzled 16 KB tiles viewed as a [tiles * 128, 128] byte matrix, copied
// unswizzled) whose completion both CTAs signal on the even CTA's full barrier (.cta_group::2; the
// even CTA announces both halves' bytes).  The even CTA ("leader") issues the pair's cta_group::2
// MMAs once a stage's barrier completes; the MMA commits arrive on both CTAs' empty / tfull
// barriers (tcgen05.commit multicast); both CTAs' epilogue warps hand an accumulator buffer back
// to the leader's tempty barrier.  Before either CTA deallocates TMEM and exits, the two exchange
// a final arrival (bye), so no arrival targets a CTA that has exited.  Every wait is bounded.
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8a8_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                             const __grid_constant__ CUtensorMap tm_w, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 6];
  __shared__ uint32_t s_tmem;
  __shared__ int s_last;

  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t tiles = (raw + 1023u) & ~1023u;  // (the same offset in both CTAs)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t full0 = smem_addr(&bars[0]);
  const uint32_t empty0 = smem_addr(&bars[kMaxStages]);
  const uint32_t tfull0 = smem_addr(&bars[2 * kMaxStages]);
  const uint32_t tempty0 = smem_addr(&bars[2 * kMaxStages + 2]);
  const uint32_t epi_done = smem_addr(&bars[2 * kMaxStages + 4]);
  const uint32_t bye = smem_addr(&bars[2 * kMaxStages + 5]);
  const int u0 = static_cast<int>(blockIdx.x >> 1), du = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    stamp(a, 0);
    for (int s = 0; s < a.ns; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 2 * kEpiWarps);
    }
    mbar_init(epi_done, kEpiWarps);
    mbar_init(bye, 1);
    fence_barrier_init();
  }
  // both CTAs' barriers are initialised before either CTA arrives on the other's
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (warp == 1) tmem_alloc_pair(smem_addr(&s_tmem), a.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  if (threadIdx.x == 0) stamp(a, 1);

  if (warp == 0) {
    // ------------------------------- TMA producer (both CTAs) -------------------------------
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      prefetch_tensormap(&tm_w);
      const uint64_t pol_w = a.w_stream ? policy_evict_first() : policy_evict_last();
      const uint32_t full_leader = map_to_rank(full0, 0);  // (the even CTA's own address for it)
      const int tiles_n = (a.N + kBM - 1) / kBM;
      bool ok = true, dep_done = false;
      uint32_t g = 0;
      for (int u = u0; u < a.units && ok; u += du) {
        const Unit un = decode_pair_unit(a, u, rank);
        const int nb = un.nb < tiles_n ? un.nb : tiles_n - 1;  // (a missing half: outputs masked)
        for (int kit = 0; kit < a.k_iters; ++kit, ++g) {
          const uint32_t s = g % a.ns, use = g / a.ns;
          if (use > 0) ok = mbar_wait_bounded(empty0 + 8 * s, (use - 1) & 1, a.err, kDevTimeoutEmpty);
          if (!ok) break;
          const uint32_t full = full_leader + 8 * s;
          const uint32_t dst = tiles + s * a.stage_bytes;
          // the leader announces both CTAs' bytes of the stage; either CTA's copies may complete
          // first (the transaction count may go below zero until the announcement)
          if (rank == 0) mbar_arrive_expect_tx(full0 + 8 * s, 2 * a.stage_bytes);
          tma_load_2d_pair_hint(dst, &tm_w, 0, (nb * a.k_iters + kit) * kBM, full, pol_w);
          if (!dep_done) {
            pdl_wait();
            dep_done = true;
          }
          tma_load_2d_pair(dst + kTileWBytes, &tm_x, kit * kBK,
                           un.tb * a.BT + static_cast<int>(rank) * (a.BT / 2), full);
          if (g == 0) stamp(a, 2);
        }
      }
      // Every MMA reading this CTA's stages has completed (the leader's commits on the empty
      // barriers) before the CTA may exit.
      const uint32_t first = g > static_cast<uint32_t>(a.ns) ? g - a.ns : 0u;
      for (uint32_t i = first; i < g && ok; ++i)
        ok = mbar_wait_bounded(empty0 + 8 * (i % a.ns), (i / a.ns) & 1, a.err, kDevTimeoutEmpty);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------- MMA issuer (even CTA) -------------------------------
      bool ok = true;
      uint32_t g = 0;
      int j = 0;
      for (int u = u0; u < a.units; u += du, ++j) {
        const int buf = j & 1, use = j >> 1;
        if (ok && use > 0)
          ok = mbar_wait_cluster(tempty0 + 8 * buf, (use - 1) & 1, a.err, kDevTimeoutEmpty);
        tc_fence_after();
        const uint32_t d = tmem + buf * a.buf_stride;
        for (int kit = 0; kit < a.k_iters && ok; ++kit, ++g) {
          const uint32_t s = g % a.ns, su = g / a.ns;
          ok = mbar_wait_cluster(full0 + 8 * s, su & 1, a.err, kDevTimeoutFull);
          if (!ok) break;
          if (g == 0) stamp(a, 3);
          tc_fence_after();
          const uint32_t base = tiles + s * a.stage_bytes;
          const uint64_t adesc = smem_desc_sw128(base);
          const uint64_t bdesc = smem_desc_sw128(base + kTileWBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk)
            mma_i8_pair(d, adesc + 2 * kk, bdesc + 2 * kk, a.idesc, (kit > 0 || kk > 0) ? 1u : 0u);
          mma_commit_pair(empty0 + 8 * s);
        }
        // always released (also after a timeout) so that the epilogue warps do not wait twice
        mma_commit_pair(tfull0 + 8 * buf);
        if (j == 0) stamp(a, 4);
        if (!ok) break;
      }
    }
  } else {
    // ------------------------------- epilogue (both CTAs) -------------------------------
    pdl_wait();
    const int rq_int = (a.ep.trunc >= 15 && a.ep.trunc <= 31) ? kRqInt : 0;
    switch (a.ep.out_mode | rq_int) {
      case kOutAccI32:
      case kOutAccI32 | kRqInt:
        epilogue_role<kOutAccI32, true>(a, tmem, tfull0, tempty0, warp, lane, &s_last);
        break;
      case kOutQuant: epilogue_role<kOutQuant, true>(a, tmem, tfull0, tempty0, warp, lane, &s_last); break;
      case kOutQuant | kRqInt:
        epilogue_role<kOutQuant | kRqInt, true>(a, tmem, tfull0, tempty0, warp, lane, &s_last);
        break;
      case kOutF32: epilogue_role<kOutF32, true>(a, tmem, tfull0, tempty0, warp, lane, &s_last); break;
      case kOutF32 | kRqInt:
        epilogue_role<kOutF32 | kRqInt, true>(a, tmem, tfull0, tempty0, warp, lane, &s_last);
        break;
      default: epilogue_role<kOutF32Acc, true>(a, tmem, tfull0, tempty0, warp, lane, &s_last); break;
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(epi_done);
  }

  __syncwarp();
  if (warp == 1) {
    bool ok = mbar_wait_bounded(epi_done, 0, a.err, kDevTimeoutFull);
    if (lane == 0) {
      mbar_arrive_remote(map_to_rank(bye, rank ^ 1u));
      if (ok) mbar_wait_cluster(bye, 0, a.err, kDevPeerTimeout);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, a.tmem_cols);
  }
  __syncthreads();
  if (threadIdx.x == 0) stamp(a, 7);
}

// ------------------------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no link-time libcuda dependency).
// ------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Row-major int8 matrix [rows, cols] (row stride ld bytes) read in boxes of box_rows x 128.
bool encode_i8_rows(CUtensorMap *map, const int8_t *base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tile-ordered weights as a [rows, 128] byte matrix read in 128 x 128 boxes without swizzle
// (each box is one 16 KB tile, already in its shared-memory image).
bool encode_w_tiles(CUtensorMap *map, const int8_t *tiles, int64_t rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kBK), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kBK)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(kBM)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(tiles), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One CTA per 128 x 128-byte tile: 16-byte chunk c of row r goes to chunk c ^ (r % 8) of the
// row, the pattern TMA writes for CU_TENSOR_MAP_SWIZZLE_128B into a 1024-byte aligned tile.
__global__ void tile_weights_kernel(const int8_t *__restrict__ w, int64_t ldw, int N, int k_pad,
                                    int k_iters, int8_t *__restrict__ tiles) {
  const int tile = blockIdx.x;
  const int nb = tile / k_iters, kb = tile % k_iters;
  int8_t *dst = tiles + static_cast<size_t>(tile) * kTileWBytes;
  for (int i = threadIdx.x; i < kBM * (kBK / 16); i += blockDim.x) {
    const int r = i >> 3, c = i & 7;
    const int row = nb * kBM + r, col = kb * kBK + c * 16;
    int4 v = make_int4(0, 0, 0, 0);
    if (row < N && col < k_pad)
      v = *reinterpret_cast<const int4 *>(w + static_cast<size_t>(row) * ldw + col);
    *reinterpret_cast<int4 *>(dst + r * kBK + ((c ^ (r & 7)) << 4)) = v;
  }
}

}  // namespace

bool plan_tc(int T, int N, int k_pad, int sm_count, TcPlan *p, bool force_pair) {
  if (T < 1 || N < 1 || k_pad < 16 || sm_count < 1) return false;
  TcPlan r = {};
  r.tiles_t = (T + kMaxBT - 1) / kMaxBT;
  const int per = (T + r.tiles_t - 1) / r.tiles_t;
  r.BT = (per + 15) / 16 * 16;
  r.tiles_n = (N + kBM - 1) / kBM;
  r.k_iters = (k_pad + kBK - 1) / kBK;
  const size_t budget = kMaxDynSmem - 1024 - 1024;  // alignment slack + static barriers
  // CTA pairs only on request: half the tokens per CTA, token tiles a multiple of 32.  Measured
  // on B200 they stream 1.5x fewer L2 -> SM bytes but run slower than single CTAs on the prefill
  // shapes (2048 x 8192 x 8192: 2127 against 2271 TOPS, GEMM alone), so AUTO / TENSOR keep one
  // CTA per 128-channel tile.
  const int pair_units = ((r.tiles_n + 1) / 2) * r.tiles_t;
  if (force_pair) {
    r.pair = 1;
    r.BT = (per + 31) / 32 * 32;
    r.splits = 1;
    r.ips = r.k_iters;
    r.units = pair_units;
    r.grid = 2 * (pair_units < sm_count / 2 ? pair_units : sm_count / 2);
    r.stage_bytes = kTileWBytes + static_cast<uint32_t>(r.BT / 2) * kBK;
    int ns = static_cast<int>(budget / r.stage_bytes);
    if (ns > kMaxStages) ns = kMaxStages;
    r.ns = ns;
    r.smem = static_cast<size_t>(ns) * r.stage_bytes + 1024;
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(2 * r.BT)) cols <<= 1;
    r.tmem_cols = cols;
    *p = r;
    return true;
  }
  const int tiles = r.tiles_n * r.tiles_t;
  r.splits = 1;
  if (tiles < sm_count) {
    // Fill the SMs, but keep each split's operand bytes ((128 + BT) * K / splits) well above the
    // partial tile it writes and the last split reads back (4 * BT * 128 bytes per split).
    int s = sm_count / tiles;
    if (s > r.k_iters / 4) s = r.k_iters / 4;  // at least 4 K stages per split
    const int by_bytes = k_pad / (2 * r.BT);
    if (s > by_bytes) s = by_bytes;
    if (s < 1) s = 1;
    r.splits = s;
  }
  r.ips = (r.k_iters + r.splits - 1) / r.splits;
  r.splits = (r.k_iters + r.ips - 1) / r.ips;  // no empty split
  r.units = tiles * r.splits;
  r.grid = r.units < sm_count ? r.units : sm_count;
  r.stage_bytes = kTileWBytes + static_cast<uint32_t>(r.BT) * kBK;
  int ns = static_cast<int>(budget / r.stage_bytes);
  if (ns > kMaxStages) ns = kMaxStages;
  const int total_iters = r.ips * ((r.units + r.grid - 1) / r.grid);
  if (ns > total_iters && total_iters >= 2) ns = total_iters;
  if (ns < 2) return false;
  r.ns = ns;
  r.smem = static_cast<size_t>(ns) * r.stage_bytes + 1024;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(2 * r.BT)) cols <<= 1;
  r.tmem_cols = cols;
  *p = r;
  return true;
}

// Co-resident clusters of two of the pair kernel at `smem` bytes (per device and size, queried
// once): the persistent grid is no larger, so no cluster waits for another to finish.
int pair_clusters(size_t smem, int sm_count) {
  static std::mutex mu;
  static int cached_dev[16] = {}, cached_n[16] = {};
  static size_t cached_smem[16] = {};
  static int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  for (int i = 0; i < used; ++i)
    if (cached_dev[i] == dev && cached_smem[i] == smem) return cached_n[i];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sm_count / 2 * 2));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_w8a8_tc_pair_kernel, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 0;
  }
  if (used < 16) {
    cached_dev[used] = dev;
    cached_smem[used] = smem;
    cached_n[used] = n;
    ++used;
  }
  return n;
}

cudaError_t launch_tc(const TcLaunch &L, const TcPlan &p, cudaStream_t stream) {
  CUtensorMap tm_x;
  if (!encode_i8_rows(&tm_x, L.x, L.T, L.k_extent_x, L.ldx, p.pair ? p.BT / 2 : p.BT)) {
    set_last_error("cuTensorMapEncodeTiled failed (driver entry point missing or bad operand)");
    return cudaErrorInvalidValue;
  }
  int limit = 0;
  cudaError_t attr_err = p.pair ? opt_in_dyn_smem<gemm_w8a8_tc_pair_kernel>(&limit)
                                : opt_in_dyn_smem<gemm_w8a8_tc_kernel>(&limit);
  if (attr_err != cudaSuccess) return attr_err;
  if (p.smem > static_cast<size_t>(limit)) return cudaErrorInvalidValue;
  TcArgs a = {};
  a.N = L.N;
  a.T = L.T;
  a.BT = p.BT;
  a.tiles_t = p.tiles_t;
  a.splits = p.splits;
  a.k_iters = p.k_iters;
  a.ips = p.ips;
  a.units = p.units;
  a.ns = p.ns;
  a.stage_bytes = p.stage_bytes;
  a.buf_stride = static_cast<uint32_t>(p.BT);
  a.tmem_cols = p.tmem_cols;
  // Instruction descriptor: D int32 (bits 4-5 = 2), A and B signed int8 (bits 7-9, 10-12 = 1),
  // both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
  a.idesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(p.BT >> 3) << 17) |
            (static_cast<uint32_t>((p.pair ? 2 * kBM : kBM) >> 4) << 24);
  a.ep = L.ep;
  a.ws = L.ws;
  a.tile_count = L.tile_count;
  a.err = L.err;
  a.w_tiles = L.w_tiles;
  a.trace = L.trace;
  a.w_stream = p.tiles_t == 1 ? 1 : 0;
  if (!p.pair)
    return launch_ex(gemm_w8a8_tc_kernel, dim3(p.grid), dim3(kThreads), p.smem, stream, L.pdl, tm_x,
                     a);
  int sm_count = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
  const int clusters = pair_clusters(p.smem, sm_count);
  if (clusters < 1) {
    set_last_error("no cluster of two CTAs of the pair GEMM fits on this device");
    return cudaErrorInvalidConfiguration;
  }
  const int grid = 2 * std::min(p.grid / 2, clusters);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 2 : 1;
  CUtensorMap tm_w;
  if (!encode_w_tiles(&tm_w, L.w_tiles, static_cast<int64_t>(p.tiles_n) * p.k_iters * kBM)) {
    set_last_error("cuTensorMapEncodeTiled failed for the weight tiles");
    return cudaErrorInvalidValue;
  }
  return cudaLaunchKernelEx(&cfg, gemm_w8a8_tc_pair_kernel, tm_x, tm_w, a);
}

size_t tc_tile_bytes(int N, int k_pad) {
  return static_cast<size_t>((N + kBM - 1) / kBM) * ((k_pad + kBK - 1) / kBK) * kTileWBytes;
}

cudaError_t launch_tile_weights(const int8_t *w, int64_t ldw, int N, int k_pad, int8_t *tiles,
                                cudaStream_t stream) {
  const int k_iters = (k_pad + kBK - 1) / kBK;
  const int n_tiles = ((N + kBM - 1) / kBM) * k_iters;
  tile_weights_kernel<<<n_tiles, 256, 0, stream>>>(w, ldw, N, k_pad, k_iters, tiles);
  return cudaGetLastError();
}

}  // namespace w8a8
