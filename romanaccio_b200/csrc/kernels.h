// Internal launch interface between the C-ABI layer (api.cu) and the kernel files.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <mutex>
#include <utility>

namespace w8a8 {

// Device error codes written into the context's error word.
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,   // a consumer waited too long for a bulk copy to land
  kDevTimeoutEmpty = 2,  // the producer waited too long for a stage to be released
  kDevPeerTimeout = 3,   // a peer flag never arrived
};

// Output modes (values of w8a8_out_mode).
enum OutMode : int { kOutAccI32 = 0, kOutQuant = 1, kOutF32 = 2, kOutF32Acc = 3 };
// Activation modes (values of w8a8_act_mode).
enum ActMode : int { kActStatic = 0, kActDyntok = 1,
                     // chain only: RMSNorm folded into a static pack (fused_emb_norm_broadcast_t1)
                     kActEmbNorm = 2 };

// Epilogue parameters shared by every contraction kernel.
struct Epilogue {
  int out_mode;
  int act_mode;
  const int16_t *quant_m;   // [N]
  int trunc;
  int qmax;                 // 127 or 32767
  int out_i16;              // QUANT output element type: 0 = int8, 1 = int16
  const float *out_step;    // [N] out_step_chan[n] or the scalar out_step repeated
  const float *acc_step;    // [N] F32_ACC step
  const float *ratio;       // [T] dyntok ratios (read in DYNTOK mode)
  void *y;                  // [T, ldy]
  int64_t ldy;
};

// Top-k epilogue (LM head shard).
struct TopK {
  int k;                    // 1..64
  int row_offset;           // vocab id of row 0
  uint64_t *lists;          // scratch [T][grid * (k + 1)]: per-CTA sorted lists, then heads
  unsigned *counter;        // scratch arrival counter (0 between launches)
  float *val;               // [T, k]
  int32_t *idx;             // [T, k]
  float *logits;            // optional [T, ldl]
  int64_t ldl;
  // Optional per-token destinations of the selected (val, idx) rows (an LM-head rank storing
  // each token's candidates into the token owner's gather buffer): token t of the launch (global
  // token tok0 + t) goes to val_dst[g / dst_tokens] + dst_row0 + (g % dst_tokens) * dst_ld.
  float *const *val_dst;    // device array [n owners] (null: val / idx above)
  int32_t *const *idx_dst;
  int dst_tokens;
  int tok0;
  int64_t dst_row0, dst_ld;
};

// A destination of the int8 activation rows on another device (multi-device LM head).
struct PublishPeer {
  int8_t *q;       // peer's int8 staging buffer
  unsigned *flag;  // peer's x_ready counter
};

// Cross-device handshake of an LM-head shard on another device than the merging one (GPU 0).
// All three are counters of forwards that only grow.
struct ShardSync {
  unsigned *seq;            // shard device: forwards this shard completed (last CTA bumps it)
  const unsigned *x_ready;  // shard device: forwards whose int8 activations GPU 0 stored here
  unsigned *done;           // GPU 0 (peer pointer): forwards whose candidates this shard stored
  // Multi-process head: x_ready holds n_ready counters (one per source rank, all must reach the
  // forward's number) and the candidates' completion is stored into every done_peers[p].  With
  // publish == 0 (a token group before the last of a forward) neither seq nor done is bumped.
  int n_ready;              // 0 or 1: the single counter above
  unsigned *const *done_peers;  // device array [n_done] (peer pointers) or null
  int n_done;
  int hold;                 // 1: do not bump seq / done (not the forward's last token group)
};

// Activation quantisation fused into a GEMV's prologue: every CTA quantises the fp32 rows into
// a resident shared-memory slab itself (the arithmetic of launch_act_quant), so no separate
// quantisation kernel precedes the GEMV.  Optionally one CTA also stores the int8 rows into other
// devices' staging buffers and bumps their x_ready counters (the multi-device LM head; the
// grid's last CTA does it).
// Static (per-tensor in_step) quantisation only: a per-token dyntok ratio would have to be
// agreed on by every CTA before its epilogue.
struct FusedQuant {
  const float *x;              // [T, ldx] fp32; null: the GEMV reads int8 rows (GemvLaunch::x)
  int64_t ldx;
  int K;
  const float *inv_smooth;     // [K] or null
  float inv_step;
  const PublishPeer *peers;    // device array [n_peers]
  int n_peers;
  unsigned *pub_seq;           // null: no publication
  unsigned long long *trace;   // optional: [0] publishing CTA quantised, [1] counters stored
};

struct GemvLaunch {
  const int8_t *w;          // [N, ldw] zero-padded up to k_pad
  int64_t ldw;
  const int8_t *x;          // [T, ldx] int8 activations, 16-byte aligned rows, k_pad readable
  int64_t ldx;
  int T, N, k_pad;
  Epilogue ep;
  bool topk;
  TopK tk;
  int *err;
  int sm_count;
  bool pdl;
  unsigned long long *trace;  // optional [grid, 8] %globaltimer stamps (diagnostics)
  ShardSync sync;             // all null: activations are local and ordered by the stream
  FusedQuant fq;              // fq.x null: int8 activations from x
};

// Shape plan of one GEMV launch (filled by plan_gemv; the scratch sizes of the top-k path
// depend on it).
struct GemvPlan {
  int tt;          // token template (1, 2, 4, 8)
  int rpw;         // rows per consumer warp (1, 2, 4)
  int rb;          // rows per tile = 8 * rpw
  int kc;          // bytes of K per stage
  int nk;          // stages per tile
  int ns;          // pipeline depth
  int num_tiles;
  int tiles_per_cta;
  int grid;
  int cand_cap;    // top-k: power-of-two candidate slots per token per CTA
  size_t smem;     // dynamic shared memory bytes
  bool fused_x;    // activations quantised in the prologue into a resident slab
  uint32_t xres_off;  // offset of that slab ([tt][k_pad] int8) in dynamic shared memory
};

// Largest resident activation slab (tt * k_pad bytes) of a fused-quantisation plan.
constexpr int kFusedXMaxBytes = 16 * 1024;

bool plan_gemv(int T, int N, int k_pad, bool topk, int k, int sm_count, GemvPlan *plan,
               bool fused_x = false);
cudaError_t launch_gemv(const GemvLaunch &L, const GemvPlan &plan, cudaStream_t stream);

// Top-k of fp32 logits already in memory ([T, ldl], N rows, vocab id tk.row_offset + n): the LM
// head of 16+ tokens, whose logits come from one tensor-core GEMM that reads the weights once
// (a GEMV top-k streams them again for every 8 tokens).  One CTA per (kTopkRowsPerCta rows,
// token) writes its sorted k-list and head in the grid top-k layout (tk.lists, G =
// topk_rows_grid(N) lists per token), then one selection CTA per token merges them into
// tk.val / tk.idx.  Two launches; tk.counter must be zero and is left zero.
constexpr int kTopkRowsPerCta = 4096;
inline int topk_rows_grid(int N) { return (N + kTopkRowsPerCta - 1) / kTopkRowsPerCta; }
cudaError_t launch_topk_rows(const float *logits, int64_t ldl, int T, int N, const TopK &tk,
                             bool pdl, cudaStream_t stream);

// Tensor-core (tcgen05 kind::i8) contraction for larger token counts.
struct TcPlan {
  int BT;          // tokens per tile (multiple of 16, <= 256) = MMA N
  int tiles_n;     // 128-channel blocks
  int tiles_t;     // token blocks
  int splits;      // K splits per tile
  int k_iters;     // 128-byte K stages per tile
  int ips;         // K stages per split
  int units;       // tiles * splits
  int grid;        // persistent CTAs
  int ns;          // pipeline depth
  uint32_t stage_bytes, tmem_cols;
  size_t smem;
  // CTA pairs (clusters of two, tcgen05 cta_group::2): a unit is a 256-channel x BT-token tile;
  // each CTA of the pair loads its 128 channels and BT / 2 tokens, and the pair's MMAs (M = 256)
  // read both CTAs' halves, so each SM streams 1.5x fewer operand bytes per MAC.  No split-K.
  int pair;
};

struct TcLaunch {
  const int8_t *w_tiles;    // weights in tensor-core tile order (launch_tile_weights)
  const int8_t *x;          // [T, ldx] int8 activations (16-byte aligned base, ldx % 16 == 0)
  int64_t ldx;
  int k_extent_x;           // readable columns of x; columns beyond read as zero
  int T, N;
  Epilogue ep;
  int32_t *ws;              // split-K accumulation plane [T, N], zero between launches (splits > 1)
  unsigned *tile_count;     // split-K counters [tiles_n * tiles_t], zero between launches
  int *err;
  unsigned long long *trace;  // optional per-CTA timeline [grid, 8]
  bool pdl;
};

// force_pair: CTA pairs whatever the size (otherwise only when they fill the SMs).
bool plan_tc(int T, int N, int k_pad, int sm_count, TcPlan *plan, bool force_pair = false);
cudaError_t launch_tc(const TcLaunch &L, const TcPlan &plan, cudaStream_t stream);
// Weights [N, ldw] (k_pad readable columns) re-laid as contiguous 128 x 128-byte tiles
// [ceil(N/128)][ceil(k_pad/128)], each stored exactly as the 128-byte-swizzled shared-memory
// image the MMA reads, zero-filled past N and k_pad.
size_t tc_tile_bytes(int N, int k_pad);
cudaError_t launch_tile_weights(const int8_t *w, int64_t ldw, int N, int k_pad, int8_t *tiles,
                                cudaStream_t stream);

// ---- mixture of experts (decode) ----
// Pair p = t * slots + j: slot j < k is the token's j-th routed expert, the rest are the shared
// experts (stored after the n_routed routed ones).
struct MoePairs {
  int T, k, slots, n_routed;
  const int32_t *routed_idx;  // [T, k]
  const float *routed_w;      // [T, k]
  // Expert parallelism: only experts e with e % own_world == own_rank are computed and combined
  // here (own_world <= 1: every expert).
  int own_rank, own_world;
};

struct MoeRouteLaunch {
  const float *hidden;  // [T, ldh]
  int64_t ldh;
  const float *gate_w;  // [E, H]
  const float *bias;    // [E] or null
  int T, H, E, k, norm_topk;
  float scaling;
  int32_t *idx;         // [T, k]
  float *w;             // [T, k]
  float *logits;        // [T, E] scratch
  int *cnt;             // [T] arrival counters, zero between launches
  bool pdl;
};

struct MoeActLaunch {
  MoePairs pairs;
  const float *src;          // rows: token t (per_pair_rows = 0) or pair p (1)
  int64_t ld;
  int per_pair_rows;
  int K;
  const float *inv_smooth;   // [E_total, K]
  const float *inv_step;     // [E_total] static 1/in_step, or null in dyntok mode
  const float *safe_thresh;  // [E_total] max(in_thresh, 1e-8) (dyntok)
  int8_t *q;                 // [pairs, ldq], ldq = round_up(K, 16)
  int64_t ldq;
  float *ratio;              // [pairs] (dyntok)
  bool pdl;
  // static mode with per-pair rows: when set, row p of the input is computed here as
  // silu(gu[p, c]) * gu[p, K + c] from the gate|up outputs gu [pairs, 2K] and also stored into
  // src_out [pairs, K] (the SwiGLU step between the two expert projections, fused)
  const float *swiglu_gu;
  float *src_out;
};

// Most (expert, 8-pair block) work items a grouped GEMV can have: sum over experts of
// ceil(count / 8) <= pairs / 8 + experts.
inline int moe_max_group_items(int n_experts, int pairs) { return n_experts + (pairs + 7) / 8; }

struct MoeGemvLaunch {
  MoePairs pairs;
  const int8_t *q;          // [pairs, ldq]
  int64_t ldq;
  const int8_t *w;          // [E_total, N, k_pad]
  int N, k_pad;
  const int16_t *quant_m;   // [E_total, N]
  int trunc, qmax;
  const float *out_step;    // [E_total, N]
  const float *ratio;       // [pairs] (dyntok unpack) or null
  int out_f32, out_i16;     // F32 (unpack) or QUANT int16 / int8
  void *y;                  // [pairs, N]
  bool pdl;
  // Expert-grouped form (launch_moe_gemv_grouped): the pairs of expert e are
  // grp_pairs[grp_off[e] .. grp_off[e + 1]) (from launch_moe_group), followed in the same array
  // by the count of work items and the items (e << 16 | z: pairs 8z .. 8z + 7 of expert e).
  const int32_t *grp_off;   // [n_experts + 2 + moe_max_group_items(n_experts, pairs)]
  const int32_t *grp_pairs; // [pairs]
  int n_experts;
};

struct MoeCombineLaunch {
  MoePairs pairs;
  const void *yq;           // [pairs, H] int16 or int8
  int in_i16;
  int H;
  const float *out_step;    // [E_total, H]
  float *out;               // [T, ldo]
  int64_t ldo;
  bool pdl;
};

cudaError_t launch_moe_route(const MoeRouteLaunch &L, cudaStream_t stream);
cudaError_t launch_moe_act_quant(const MoeActLaunch &L, bool dyn, cudaStream_t stream);
cudaError_t launch_moe_gemv(const MoeGemvLaunch &L, cudaStream_t stream);
// Pair lists per expert (this rank's experts only): off [n_experts + 1], pairs [T * slots].
cudaError_t launch_moe_group(const MoePairs &P, int n_experts, int32_t *off, int32_t *pairs,
                             bool pdl, cudaStream_t stream);
// The expert GEMV with each expert's weight rows streamed once per group of its pairs.
cudaError_t launch_moe_gemv_grouped(const MoeGemvLaunch &L, cudaStream_t stream);
cudaError_t launch_moe_swiglu(const float *gu, int I, int pairs, float *h, bool pdl,
                              cudaStream_t stream, const MoePairs &P);
cudaError_t launch_moe_combine(const MoeCombineLaunch &L, cudaStream_t stream);

// Expert-parallel exchange of the per-rank partial combines [T, H] (w8a8_moe_ep_*).
struct MoeEpLaunch {
  const float *partial;       // this rank's [T, H] partial
  float *const *dst;          // device array [world]: every rank's gather base
  unsigned *const *done;      // device array [world]: done[rank] on every rank
  int rank, world, T, H, max_T;
  unsigned *pub_seq;          // this rank: partials published (the last CTA bumps it)
  unsigned *pub_arrive;       // this rank: CTA arrivals (zero between launches)
  const float *gather;        // this rank's gather base [2][world][max_T][H]
  const unsigned *done_here;  // this rank's done[world]
  float *out;                 // [T, ldo]
  int64_t ldo;
  int *err;
  bool pdl;
};
cudaError_t launch_moe_ep_publish(const MoeEpLaunch &L, cudaStream_t stream);
cudaError_t launch_moe_ep_sum(const MoeEpLaunch &L, cudaStream_t stream);

// Activation quantisation (pack) of x [T, K] fp32 into q [T, ldq] int8 (+ ratio [T]).
struct ActQuantLaunch {
  const float *x;
  int64_t ldx;
  int T, K;
  int k_fill;               // columns [K, k_fill) of q are zero-filled
  const float *inv_smooth;  // [K] or null
  int act_mode;
  float inv_step;           // static: (in_step > 1e-12f) ? 1/in_step : 0
  float safe_thresh;        // dyntok: max(in_thresh, 1e-8f)
  int8_t *q;
  int64_t ldq;
  float *ratio;             // [T] (dyntok)
  bool pdl;
  // Optional publication to LM-head shards on other devices: every quantised row is also
  // stored into each peer's staging buffer (same ldq), then the last CTA bumps *pub_seq and
  // stores it into every peer's flag.
  const PublishPeer *peers;  // device array [n_peers]
  int n_peers;
  unsigned *pub_seq;         // this device; null: no publication
  unsigned *pub_arrive;      // this device, zero between launches
  unsigned long long *trace; // optional: [0] entry of CTA 0, [1] peers' flags stored
  int pub_row0;              // row t is stored at row pub_row0 + t of every peer's buffer
  // Optional RMSNorm in front of a static quantisation (the LM head's input step,
  // fused_emb_norm_broadcast_t1): q = round_clamp(x * inv_rms * emb_norm[c], 127) with inv_rms
  // from the reference's ordered sum of squares; emb_norm = norm weight / in_step (K <= 12288).
  const float *emb_norm;
  float eps;
};
cudaError_t launch_act_quant(const ActQuantLaunch &L, cudaStream_t stream);

// int8 row copy with zero fill of [K, k_pad) (used when a caller's int8 activations are not
// 16-byte aligned / padded).
cudaError_t launch_copy_pad_i8(const int8_t *src, int64_t lds, int T, int K, int8_t *dst,
                               int64_t ldd, int k_pad, bool pdl, cudaStream_t stream);

// Unpack (dequant) of requantised outputs.
struct UnpackLaunch {
  const void *yq;
  int64_t ldyq;
  int in_i16;
  int T, N;
  int act_mode;
  const float *ratio;
  const float *out_step;    // [N]
  float *y;
  int64_t ldy;
  bool pdl;
};
cudaError_t launch_unpack(const UnpackLaunch &L, cudaStream_t stream);

// Merge of n_lists candidate lists per token into the top k_out.
struct MergeLaunch {
  const float *in_val;
  const int32_t *in_idx;
  int T, n_lists, k_in, k_out;
  int64_t list_stride, token_stride;
  float *out_val;
  int32_t *out_idx;
  int32_t *argmax;
  bool pdl;
  // Optional: lists s with bit s of remote_mask are stored by other devices; the merge first
  // waits (bounded) until done[s] reaches *pub_seq, recording kDevPeerTimeout in *err if not.
  const unsigned *done;
  uint64_t remote_mask;
  const unsigned *pub_seq;
  int *err;
  unsigned long long *trace;  // optional: [2] CTA 0 past its stream wait, [3] flags seen, [4] end
};
cudaError_t launch_topk_merge(const MergeLaunch &L, cudaStream_t stream);

// One step of the persistent decode-chain kernel (device-resident op table).  128-byte aligned:
// an op is exactly three cache lines, which the kernel prefetches ahead of use.
struct alignas(128) ChainOp {
  // weights and tiling
  const int8_t *w;
  int64_t ldw;
  int N, K, k_pad;
  int rpw, rb, kc, nk, num_tiles;  // filled by plan_chain
  // input view and activation quantisation
  const float *x;
  int64_t ldx;
  int vec_x;                 // x rows 16-byte aligned, K % 4 == 0
  const float *inv_smooth;   // [K] or null (16-byte aligned); kActEmbNorm: emb_norm_scaled [K]
  int act_mode;
  float inv_step, safe_thresh;
  float norm_eps;            // kActEmbNorm: the RMSNorm epsilon
  float *ratio_out;          // optional [T]
  // epilogue
  int out_mode;
  const int16_t *quant_m;
  const int32_t *quant_m32;  // the same values widened (4-byte asynchronous staging)
  int trunc, qmax, out_i16;
  const float *out_step;
  const float *acc_step;
  void *y;
  int64_t ldy;
  // per-token amax hand-off between a producing step and the dyntok step that reads its output
  const float *amax_src;     // this step's amax [T] was reduced by its producer (or null)
  float *amax_dst;           // reduce max |y[:, c0 + c] * amax_smooth[c]| into [T] (or null)
  int amax_c0, amax_cols;
  const float *amax_smooth;  // the consuming step's in_inv_smooth (or null)
  // scheduling
  int barrier_before;        // wait for every CTA to finish the previous steps first
  int topk;                  // LM-head step (must be the last step)
  TopK tk;                   // k, row_offset, val, idx, logits, ldl (lists / counter unused)
};

struct ChainPlan {
  int tt, grid, kpad_max, cand_cap, max_rows, ns;
  int norm_floats;  // fp32 staging of one token's input row for kActEmbNorm steps (0: none)
  uint32_t stage_bytes, ring_bytes;
  // byte offsets in dynamic shared memory (the descriptor window sits at 0, the ring after it):
  // activation rows, top-k candidate keys, mbarriers, epilogue parameters, norm staging row.
  // The candidates and the staging row may lie inside the activation rows' unused bytes.
  uint32_t xq_off, cand_off, bars_off, ep_off, norm_off;
  size_t smem;
};

bool plan_chain(ChainOp *ops, int n_ops, int T, int sm_count, ChainPlan *plan);
cudaError_t configure_chain(const ChainPlan &plan);
// `bar` starts a zero-at-launch region of clear_bytes (arrival counters, then amax slots).
cudaError_t launch_chain(const ChainOp *ops_dev, int n_ops, int T, const ChainPlan &plan,
                         unsigned *bar, size_t clear_bytes, unsigned *tk_counter,
                         uint64_t *lists, int *err, unsigned long long *trace,
                         cudaStream_t stream);

// Records `msg` as the calling thread's w8a8_last_error() text (defined in api.cu).
void set_last_error(const char *msg);

// Opts kernel Kern in, once per device (function attributes belong to a device's context), to
// the largest dynamic shared memory the device allows next to the kernel's static shared
// memory; *limit receives that size for the current device.
template <auto Kern>
cudaError_t opt_in_dyn_smem(int *limit) {
  constexpr int kDevices = 64;
  static int cached[kDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int optin = 0;
    cudaFuncAttributes fa;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, Kern);
    if (e != cudaSuccess) return e;
    const int lim = optin - static_cast<int>(fa.sharedSizeBytes);
    e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    if (e != cudaSuccess) return e;
    cached[dev] = lim;
  }
  *limit = cached[dev];
  return cudaSuccess;
}

// Launch helper: cudaLaunchKernelEx with the programmatic-stream-serialisation attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, bool pdl, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace w8a8
