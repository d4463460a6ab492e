/*
 * w8a8.h - C ABI of the B200 (sm_100a) SmoothQuant W8A8 linear and vocab-sharded LM head.
 *
 * This library replaces the NPU side of romanaccio's quantised-linear boundary:
 *
 *   pack_npu_input(...)          src/LFM3/lfm3_v2.cpp:1186-1204   (fp32 -> int8, static or dyntok)
 *   WorkerPool::submit_task(...) src/eswin_runtime/src/backend/worker_pool.hpp:232-254
 *                                (NPU CMAC int8 GEMM -> CACC int32 -> SDP CvtPrecision_QuantM)
 *   unpack_npu_output(...)       src/LFM3/lfm3_v2.cpp:1207-1225   (int8/int16 -> fp32)
 *
 * and the host-side LM-head merge that follows the dual-die vocab split:
 *
 *   compute_logits_from_ptr(...)                src/LFM3/lfm3_v2.cpp:2320-2416
 *   TransformerSession::forward_lm_head_dual_die src/eswin_runtime/src/llm/transformer_session.cpp:538-614
 *   Sampler::sample greedy / top-k              src/eswin_runtime/src/nlp/sampler.cpp:93-121
 *
 * Conventions follow es_runtime.h (src/eswin_runtime/include/es_runtime.h:24-35): every call
 * returns a status code, no C++ exception crosses this boundary, destroy functions accept NULL,
 * and the caller owns every buffer it passes in.  Device pointers are plain CUDA device
 * addresses on the device the context was created for; `stream` is a cudaStream_t passed as
 * void* (NULL = legacy default stream).  Every forward call is asynchronous on `stream`.
 *
 * Thread safety: a w8a8_linear may be used by several host threads only on one stream at a
 * time (its scratch buffer is per object).  Different objects are independent.
 */
#ifndef W8A8_H
#define W8A8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------------------------
 * Status codes: values 0..-9 mirror es_status_t (es_runtime.h:24-35).
 * ------------------------------------------------------------------------------------- */
typedef enum {
    W8A8_SUCCESS               =  0,
    W8A8_ERR_INVALID_ARG       = -1,
    W8A8_ERR_NO_MEMORY         = -2,
    W8A8_ERR_DEVICE_BUSY       = -3,
    W8A8_ERR_HARDWARE_FAULT    = -4,
    W8A8_ERR_NOT_INITIALIZED   = -5,
    W8A8_ERR_NOT_SUPPORTED     = -6,
    W8A8_ERR_IO                = -7,
    W8A8_ERR_CHECKSUM_MISMATCH = -8,
    W8A8_ERR_TIMEOUT           = -9,
    W8A8_ERR_CUDA              = -10, /* a CUDA runtime call failed; see w8a8_last_error() */
    W8A8_ERR_PEER_TIMEOUT      = -11  /* a bounded wait on another GPU's flag ran out */
} w8a8_status;

/* Mirrors es_status_to_string (es_runtime.h:37). */
const char *w8a8_status_to_string(w8a8_status status);
/* Detail text of the last failure on the calling host thread ("" if none). */
const char *w8a8_last_error(void);
/* Library version string. */
const char *w8a8_version(void);

/* ---------------------------------------------------------------------------------------
 * Enumerations
 * ------------------------------------------------------------------------------------- */
/* Mirrors BoundaryDtype (lfm3_v2.cpp:550-554).  Only INT8 and INT16 are requant targets. */
typedef enum {
    W8A8_DTYPE_FP16  = 0,
    W8A8_DTYPE_INT8  = 1,
    W8A8_DTYPE_INT16 = 2
} w8a8_boundary_dtype;

/* Activation quantisation: pack_npu_input_int8 (static, lfm3_v2.cpp:892-940) or
 * pack_npu_input_int8_dyntok (per-token amax, lfm3_v2.cpp:1050-1141). */
typedef enum {
    W8A8_ACT_STATIC = 0,
    W8A8_ACT_DYNTOK = 1
} w8a8_act_mode;

/* What a forward call writes into y:
 *   ACC_I32  int32 accumulators acc[t,n] = sum_k q[t,k] * Wq[n,k]  (CMAC/CACC, cmac.py:300-383)
 *   QUANT    int8 (or int16) y_q = clip(RNE(acc * QuantM[n] / 2^trunc), +-Qmax)
 *            (SDP CvtPrecision_QuantM; attribute_int8_error.py:104-122, FINDINGS.md:2447)
 *   F32      QUANT followed by the reference unpack: y = float(y_q) * step
 *            (unpack_npu_output_int8[_dyntok], lfm3_v2.cpp:971-1008, 1143-1183)
 *   F32_ACC  float(acc) * (ratio[t] * acc_step[n]) without the requant stage (logit mode of the
 *            LM head: logit = acc * in_step * w_step[n]) */
typedef enum {
    W8A8_OUT_ACC_I32 = 0,
    W8A8_OUT_QUANT   = 1,
    W8A8_OUT_F32     = 2,
    W8A8_OUT_F32_ACC = 3
} w8a8_out_mode;

/* ---------------------------------------------------------------------------------------
 * Context: one per device.
 * ------------------------------------------------------------------------------------- */
typedef struct w8a8_ctx w8a8_ctx;

/* Creates a context on CUDA device `device`; the calling thread's current device is left as it was. */
w8a8_status w8a8_ctx_create(int device, w8a8_ctx **out_ctx);
void        w8a8_ctx_destroy(w8a8_ctx *ctx);
/* Number of SMs of the context's device. */
int         w8a8_ctx_sm_count(const w8a8_ctx *ctx);
/* CUDA device ordinal of the context (-1 for NULL). */
int         w8a8_ctx_device(const w8a8_ctx *ctx);
/* Synchronises the context's device and reports a device-side failure recorded by a kernel
 * (a bounded wait that ran out: W8A8_ERR_TIMEOUT / W8A8_ERR_PEER_TIMEOUT), then clears it.
 * Plays the role of the worker liveness checks of worker_pool.cpp:180-193.  After a timeout,
 * destroy and recreate the linears whose forwards were in flight: a tensor-core forward cut short
 * may leave its split-K accumulation plane non-zero. */
w8a8_status w8a8_ctx_check(w8a8_ctx *ctx);

/* ---------------------------------------------------------------------------------------
 * Per-linear scale parameters: mirrors SubgraphScaleInfo (lfm3_v2.cpp:556-565) and the
 * quant_scales.json entry (build_lfm3_int8_pkg.py:452-463).  Host pointers; copied at create.
 * ------------------------------------------------------------------------------------- */
typedef struct {
    int32_t      out_dtype;      /* w8a8_boundary_dtype: INT8 (Qmax 127) or INT16 (Qmax 32767) */
    float        in_thresh;      /* dyntok: ratio[t] = amax_t / max(in_thresh, 1e-8) */
    float        in_step;        /* static: q = RNE(clamp(x * (inv_smooth * (1/in_step)), +-127)) */
    float        out_thresh;     /* informational (output_threshold) */
    float        out_step;       /* scalar output step used when out_step_chan == NULL */
    const float *in_inv_smooth;  /* [K] or NULL: SmoothQuant 1/s_in[c] */
    const float *out_step_chan;  /* [N] or NULL: per-channel step in_s*w_step*2^trunc/QuantM */
} w8a8_scale_info;

/* A W8A8 linear: int8 weights [N, K] (row n = output channel, K contiguous), per-channel
 * QuantM, trunc and the scale info.  Mirrors one INT8 Class-B subgraph of the LFM3 package
 * (build_single_conv_region, build_lfm3_int8_pkg.py:171-224) with the NVDLA weight tiling
 * replaced by a row-major device layout. */
typedef struct {
    int32_t         K;           /* in-features  (>= 1) */
    int32_t         N;           /* out-features (>= 1) */
    const int8_t   *weights;     /* host [N, weights_ld] int8, values in [-127, 127] */
    int64_t         weights_ld;  /* elements between consecutive rows (>= K) */
    const int16_t  *quant_m;     /* host [N] QuantM in [1, 32767], or NULL (QUANT/F32 then unsupported) */
    int32_t         trunc;       /* SDP right shift, 0..62 */
    const float    *acc_step;    /* host [N] or NULL: step for W8A8_OUT_F32_ACC */
    w8a8_scale_info scale;
} w8a8_linear_desc;

typedef struct w8a8_linear w8a8_linear;

/* Uploads the weights and parameters to the context's device.  Replaces the package load of
 * one subgraph (load_quant_scales / parse_entry, lfm3_v2.cpp:3743, 3807-3826). */
w8a8_status w8a8_linear_create(w8a8_ctx *ctx, const w8a8_linear_desc *desc, w8a8_linear **out_linear);
void        w8a8_linear_destroy(w8a8_linear *linear);
/* Device bytes held by the linear (weights + parameters + scratch). */
size_t      w8a8_linear_device_bytes(const w8a8_linear *linear);

/* Boundary stage 1 -- replaces pack_npu_input (lfm3_v2.cpp:1186-1204) for INT8 inputs.
 * x_dev: fp32 [T, K] with row stride ldx (elements).  q_dev: int8 [T, K] with row stride ldq.
 * ratio_dev: fp32 [T]; written in DYNTOK mode (amax_t / max(in_thresh,1e-8)), ignored (may be
 * NULL) in STATIC mode.  Layout is [T, K] row-major for every T (the NVDLA [C/32, T, 32]
 * surface of the reference is not reproduced). */
w8a8_status w8a8_pack_input(w8a8_linear *linear, const float *x_dev, int64_t ldx, int32_t T,
                            int32_t act_mode, int8_t *q_dev, int64_t ldq, float *ratio_dev,
                            void *stream);

/* Boundary stage 2 -- replaces submit_task of the INT8 loadable (CMAC + CACC + SDP).
 * q_dev: int8 [T, K] (stride ldq).  Writes y_dev [T, N] (stride ldy elements) as int32 (ACC_I32),
 * int8/int16 per scale.out_dtype (QUANT), or fp32 (F32 / F32_ACC, which need ratio_dev in
 * DYNTOK mode). */
w8a8_status w8a8_linear_forward_q(w8a8_linear *linear, const int8_t *q_dev, int64_t ldq, int32_t T,
                                  int32_t act_mode, const float *ratio_dev, int32_t out_mode,
                                  void *y_dev, int64_t ldy, void *stream);

/* Boundary stage 3 -- replaces unpack_npu_output (lfm3_v2.cpp:1207-1225) for INT8/INT16
 * outputs.  yq_dev: [T, N] int8 or int16 per scale.out_dtype (stride ldyq); y_dev fp32 [T, N]
 * (stride ldy).  ratio_dev is read in DYNTOK mode. */
w8a8_status w8a8_unpack_output(w8a8_linear *linear, const void *yq_dev, int64_t ldyq, int32_t T,
                               int32_t act_mode, const float *ratio_dev, float *y_dev, int64_t ldy,
                               void *stream);

/* The three stages fused: pack -> int8 contraction -> requant -> unpack, one call.
 * x_dev fp32 [T, K] (stride ldx); y_dev per out_mode (stride ldy); ratio_dev [T] optional
 * output of the per-token ratios (DYNTOK), may be NULL. */
w8a8_status w8a8_linear_forward(w8a8_linear *linear, const float *x_dev, int64_t ldx, int32_t T,
                                int32_t act_mode, int32_t out_mode, void *y_dev, int64_t ldy,
                                float *ratio_dev, void *stream);

/* Contraction engine used by forward / forward_q (no reference counterpart: the reference has
 * one NPU engine).  AUTO streams the weights through the GEMV kernels for small token counts and
 * switches to the tcgen05 tensor-core GEMM above W8A8_TC_MIN_TOKENS; GEMV and TENSOR force one.
 * TENSOR runs one CTA per 128-channel tile; TENSOR_PAIR runs CTA pairs (clusters of two SMs
 * sharing each 256-channel tile, tcgen05 cta_group::2 MMAs: 1.5x fewer operand bytes per SM, but
 * slower on B200 for the prefill shapes measured, so AUTO does not choose it).  All give
 * bit-identical results. */
typedef enum {
    W8A8_PATH_AUTO        = 0,
    W8A8_PATH_GEMV        = 1,
    W8A8_PATH_TENSOR      = 2,
    W8A8_PATH_TENSOR_PAIR = 3
} w8a8_path;
#define W8A8_TC_MIN_TOKENS 16
w8a8_status w8a8_linear_set_path(w8a8_linear *linear, int32_t path);
/* Set-up call (no reference counterpart: the reference's NPU loadables own fixed buffers).
 * Allocates, once, every piece of device scratch that forward calls of up to max_tokens tokens
 * on the linear's current path would otherwise allocate on first use: the activation staging
 * rows, the tensor-core copy of the weights (built on `stream`), the split-K accumulation plane
 * and tile counters, and with max_k > 0 the logits and row lists of a 16+ token top-k forward with k <=
 * max_k.  Afterwards forward, forward_q and forward_topk calls within those limits allocate and
 * synchronise nothing, so a caller can capture them in a CUDA graph.  Call it outside any
 * capture; set the path first. */
w8a8_status w8a8_linear_reserve(w8a8_linear *linear, int32_t max_tokens, int32_t max_k,
                                void *stream);
/* The LM-head shard's input RMSNorm (fused_emb_norm_broadcast_t1, lfm3_v2.cpp:810-831): when
 * emb_norm_scaled_dev ([K] fp32 = norm weight / in_step, lfm3_v2.cpp:3906-3912) is non-NULL,
 * w8a8_linear_forward_topk with the STATIC act mode packs each row as
 * round_clamp(x * inv_rms * emb_norm_scaled[c], 127) with the reference's four interleaved sums
 * of squares.  K <= 12288.  NULL turns it off.  The pointer must stay valid while set. */
w8a8_status w8a8_linear_set_input_norm(w8a8_linear *linear, const float *emb_norm_scaled_dev,
                                       float eps);
/* Diagnostics (no reference counterpart): attaches a device buffer of 2 x sm_count x 8 uint64
 * that each launch of this linear fills with per-CTA %globaltimer stamps.  Tensor-core launches
 * (grid <= sm_count): entry, setup done, first stage issued, first stage landed, first MMAs
 * committed, first accumulator seen by the epilogue, released, exit.  GEMV launches (when their
 * grid is at most 2 x sm_count): entry, setup done, first stage landed, streaming done, top-k
 * lists written, arrived, top-k selected (last CTA), exit.  NULL detaches. */
w8a8_status w8a8_linear_set_trace(w8a8_linear *linear, unsigned long long *trace_dev);

/* ---------------------------------------------------------------------------------------
 * LM head shard: a linear over a contiguous block of vocab rows [row_offset, row_offset + N)
 * (the contiguous vocab split of dual_die_splitter.py:63-147 and
 * transformer_session.cpp:575-596) whose logits never leave the SM: the kernel keeps, per
 * token, the k largest (logit, vocab id) pairs in the total order (logit desc, id asc).
 * Greedy argmax (sampler.cpp:93-103, strict '>' keeps the lowest id) is element 0.
 * ------------------------------------------------------------------------------------- */
#define W8A8_TOPK_MAX 64

/* x_dev fp32 [T, K] (stride ldx).  out_mode F32 (requant + unpack, the LFM3 INT8 LM head) or
 * F32_ACC (logit = float(acc) * ratio * acc_step[n]).  k in [1, min(W8A8_TOPK_MAX, N)].
 * Writes topk_val_dev fp32 [T, k] and topk_idx_dev int32 [T, k] (vocab ids = row_offset + n),
 * sorted.  logits_dev: optional fp32 [T, N] (stride ldl) copy of the shard's logits, may be
 * NULL.  Scratch: per-CTA candidate lists held inside the linear. */
w8a8_status w8a8_linear_forward_topk(w8a8_linear *linear, const float *x_dev, int64_t ldx,
                                     int32_t T, int32_t act_mode, int32_t out_mode, int32_t k,
                                     int32_t row_offset, float *topk_val_dev,
                                     int32_t *topk_idx_dev, float *logits_dev, int64_t ldl,
                                     void *stream);

/* Merges n_lists candidate lists per token into the global top-k_out (the cross-shard merge
 * that replaces the logit concatenation + Sampler pass over the full vocab, i.e.
 * transformer_session.cpp:575-596 followed by sampler.cpp:93-121).  Candidate (t, l, j) is read
 * at in_val_dev[t * token_stride + l * list_stride + j] (same for in_idx_dev); lists need not
 * be sorted.  out: [T, k_out] sorted (value desc, id asc); argmax_dev: optional int32 [T]
 * (= out_idx[t, 0]).  k_out <= n_lists * k_in, k_out <= W8A8_TOPK_MAX, n_lists <= 64. */
w8a8_status w8a8_topk_merge(w8a8_ctx *ctx, const float *in_val_dev, const int32_t *in_idx_dev,
                            int32_t T, int32_t n_lists, int32_t k_in, int64_t list_stride,
                            int64_t token_stride, int32_t k_out, float *out_val_dev,
                            int32_t *out_idx_dev, int32_t *argmax_dev, void *stream);

/* ---------------------------------------------------------------------------------------
 * Vocab-sharded LM head over several devices driven by one process: the single-process form of
 * the dual-die LM head (TransformerSession::forward_lm_head_dual_die,
 * transformer_session.cpp:538-614; run_dual_die, lfm3_v2.cpp:1311-1332) for n = 1..8 shards.
 * Shard s holds the contiguous vocab rows [s*V/n, (s+1)*V/n) (floor split; n = 2 gives the
 * reference's halves, dual_die_splitter.py:95-141) on the device of ctxs[s].
 *
 * forward: h_dev lives on the device of ctxs[0] ("device 0").  Device 0 quantises h once
 * (static in_step, the broadcast of fused_emb_norm_broadcast_t1, lfm3_v2.cpp:810-831) and
 * stores the int8 rows into every shard's staging buffer over NVLink; each shard runs its top-k
 * GEMV and stores its k (logit, vocab id) pairs into a gather buffer on device 0; device 0
 * merges them (value desc, id asc).  Shards on other devices synchronise with device 0 through
 * counters in device memory (no host or cross-device stream dependency): they are launched on
 * their own streams first, stream their first weight stages at once, and wait (at most 1 s) for
 * device 0's activations, so device 0's `stream` must reach the forward within 1 s of the call;
 * a wait that runs out records W8A8_ERR_PEER_TIMEOUT (w8a8_ctx_check) and the head must then be
 * destroyed.  Forwards of one head are issued on one stream, one at a time.  A head with every
 * shard on device 0 is ordered on `stream` alone and can be captured in a CUDA graph; one with
 * shards elsewhere cannot (W8A8_ERR_NOT_SUPPORTED while `stream` is capturing) and takes at most
 * 8 tokens a forward (max_tokens <= 8).  Logits: float(acc) * in_step * w_step[v]
 * (acc_step = in_step * w_step).  Shard devices need peer access to and from device 0.
 * ------------------------------------------------------------------------------------- */
typedef struct w8a8_lmhead w8a8_lmhead;

w8a8_status w8a8_lmhead_create(w8a8_ctx *const *ctxs, int32_t n_shards, int32_t K, int32_t V,
                               const int8_t *weights_host, int64_t weights_ld,
                               const float *acc_step_host, float in_step, int32_t max_tokens,
                               int32_t k_max, w8a8_lmhead **out_lmhead);
/* topk_val_dev fp32 [T, k], topk_idx_dev int32 [T, k] (sorted), argmax_dev int32 [T] or NULL,
 * all on the device of ctxs[0].  1 <= T <= max_tokens, 1 <= k <= k_max. */
w8a8_status w8a8_lmhead_forward(w8a8_lmhead *lmhead, const float *h_dev, int32_t T, int32_t k,
                                float *topk_val_dev, int32_t *topk_idx_dev, int32_t *argmax_dev,
                                void *stream);
/* Fuses the LM head's input RMSNorm (fused_emb_norm_broadcast_t1, lfm3_v2.cpp:810-831; the
 * arithmetic of w8a8_emb_norm_pack, emb_norm_scaled_dev on the device of ctxs[0]) into the
 * forward's quantisation: h is then the un-normalised final hidden state.  NULL turns it off. */
w8a8_status w8a8_lmhead_set_input_norm(w8a8_lmhead *lmhead, const float *emb_norm_scaled_dev,
                                       float eps);
void        w8a8_lmhead_destroy(w8a8_lmhead *lmhead);
int32_t     w8a8_lmhead_shards(const w8a8_lmhead *lmhead);
/* Diagnostics (no reference counterpart): head_trace_dev (device 0, 8 uint64, or NULL) receives
 * %globaltimer stamps of a forward with several shards: [0] activations quantised (by the
 * publishing CTA, or entry of the quantisation kernel when shard 0 cannot fuse it), [1] every
 * shard's activations stored, [2] merge past its stream wait, [3] every remote shard's candidates seen, [4] merge
 * end; shard_traces[s] (device of shard s, 2 x sm_count x 8 uint64, or NULL; the array itself
 * may be NULL) is attached to shard s's linear as by w8a8_linear_set_trace. */
w8a8_status w8a8_lmhead_set_trace(w8a8_lmhead *lmhead, unsigned long long *head_trace_dev,
                                  unsigned long long *const *shard_traces);

/* ---------------------------------------------------------------------------------------
 * Mixture-of-experts layer (decode): router + W8A8 experts + weighted combine, all on the
 * device (no host round trip between routing and the experts).
 *
 *   route:   MoERouter::route (src/eswin_runtime/src/llm/moe_router.cpp:211-260): fp32 logits
 *            W_gate . h (+ bias), softmax (max subtracted, float exp, double sum,
 *            scores_from_logits :108-130), top-k by (score desc, expert index asc), weights =
 *            the probabilities (renormalised only when norm_topk_prob), times routed_scaling.
 *   experts: every (token, slot) pair, slots = top_k routed experts then n_shared shared ones
 *            (weight 1): gate|up W8A8 linear (dyntok input, F32 output) -> silu(gate) * up ->
 *            down W8A8 linear (static input, QUANT int8/int16 output y_q).
 *   combine: out[t, c] = sum over the token's slots in order of
 *            float(y_q[c]) * (w_slot * down_out_step_chan[e, c])
 *            (src/LFM2.5-8B-A1B/lfm2_moe.cpp:2300-2318).
 * Expert e (0 <= e < n_routed + n_shared) parameters are expert-major host arrays, copied at
 * create.  The router's logits are a warp-parallel fp32 sum (not the reference's serial
 * order), so routing weights agree within float rounding; the expert stages and the combine
 * are exact given the routing.
 * ------------------------------------------------------------------------------------- */
typedef struct {
    int32_t        hidden;            /* H <= 4096 */
    int32_t        inter;             /* I <= 4096, expert intermediate size */
    int32_t        n_routed;          /* E <= 4096 */
    int32_t        n_shared;          /* S */
    int32_t        top_k;             /* k <= 16 */
    int32_t        norm_topk_prob;    /* 0: raw softmax probabilities (DeepSeek-V2-Lite) */
    float          routed_scaling;    /* routed_scaling_factor (1.0 for none) */
    int32_t        max_tokens;        /* largest T of a forward */
    const float   *gate_w;            /* [E, H] router weights */
    const float   *gate_bias;         /* [E] or NULL */
    const int8_t  *gu_weights;        /* [E+S, 2I, H]: gate rows then up rows */
    const int16_t *gu_quant_m;        /* [E+S, 2I] */
    const float   *gu_out_step_chan;  /* [E+S, 2I] */
    const float   *gu_inv_smooth;     /* [E+S, H] */
    const float   *gu_in_thresh;      /* [E+S] dyntok input threshold */
    int32_t        gu_trunc;
    const int8_t  *dn_weights;        /* [E+S, H, I] */
    const int16_t *dn_quant_m;        /* [E+S, H] */
    const float   *dn_out_step_chan;  /* [E+S, H] */
    const float   *dn_inv_smooth;     /* [E+S, I] */
    const float   *dn_in_step;        /* [E+S] static input step */
    int32_t        dn_trunc;
    int32_t        dn_out_dtype;      /* W8A8_DTYPE_INT8 or W8A8_DTYPE_INT16 */
} w8a8_moe_desc;

typedef struct w8a8_moe w8a8_moe;

w8a8_status w8a8_moe_create(w8a8_ctx *ctx, const w8a8_moe_desc *desc, w8a8_moe **out_moe);
void        w8a8_moe_destroy(w8a8_moe *moe);
/* Router only: idx_dev int32 [T, k], w_dev fp32 [T, k]. */
w8a8_status w8a8_moe_route(w8a8_moe *moe, const float *hidden_dev, int64_t ldh, int32_t T,
                           int32_t *idx_dev, float *w_dev, void *stream);
/* Whole layer: hidden_dev fp32 [T, ldh] -> out_dev fp32 [T, ldo] (T <= max_tokens). */
w8a8_status w8a8_moe_forward(w8a8_moe *moe, const float *hidden_dev, int64_t ldh, int32_t T,
                             float *out_dev, int64_t ldo, void *stream);
/* Device views of the last forward's intermediates (for tests and tracing): routed ids
 * [T, k], weights [T, k], gate|up outputs fp32 [T*slots, 2I], silu(gate)*up fp32
 * [T*slots, I], down requantised outputs [T*slots, H] (int16 or int8 per dn_out_dtype). */
w8a8_status w8a8_moe_views(const w8a8_moe *moe, const int32_t **idx_dev, const float **w_dev,
                           const float **gate_up_dev, const float **act_dev,
                           const void **down_q_dev);

/* ---------------------------------------------------------------------------------------
 * One rank of a vocab-sharded LM head over processes: one process per GPU, each holding the
 * contiguous vocab rows [rank * V / world, (rank + 1) * V / world) (the reference's contiguous
 * die split, dual_die_splitter.py:95-141, transformer_session.cpp:588-596, for any world <= 64).
 * Replaces the dual-die LM-head merge of TransformerSession::forward_lm_head_dual_die
 * (transformer_session.cpp:538-614) and run_dual_die (lfm3_v2.cpp:1311-1332), where each die's
 * worker computes its half of the logits and the host concatenates them before Sampler::sample:
 * here every rank's GEMV keeps only the top-k (logit, vocab id) pairs of every rank's tokens,
 * stores each token's pairs into the token owner's device memory, and each rank merges its own
 * tokens' lists.  The exchange is done by this library: peer stores into CUDA-IPC-mapped device
 * memory with counters that only grow, each device-side wait bounded (1 to 2 s, then
 * W8A8_ERR_PEER_TIMEOUT through w8a8_ctx_check) -- no NCCL call and no host round trip, so a
 * forward (three launches on `stream`, four when world * T >= 2) can be captured in a CUDA graph.
 *
 * Set-up: every rank calls w8a8_lmhead_rank_create, then w8a8_lmhead_rank_export (64 bytes),
 * the caller exchanges the handles between the processes by any means (they are plain bytes),
 * and every rank calls w8a8_lmhead_rank_connect with all world handles in rank order.  Ranks
 * driven by one process (one per device) connect with w8a8_lmhead_rank_connect_local instead.
 * Forward: every rank calls w8a8_lmhead_rank_forward for the same sequence of forwards, with the
 * same T on every rank (world * max_tokens <= 64), on one stream per rank; the calls of
 * different ranks may be issued in any order and need not overlap in time beyond the bounded
 * waits.  h_dev: this rank's T hidden states fp32 [T, K]; outputs this rank's tokens' merged
 * top-k (value desc, id asc) [T, k] and argmax [T] (may be NULL).
 * ------------------------------------------------------------------------------------- */
#define W8A8_LMHEAD_RANK_HANDLE_BYTES 64
typedef struct w8a8_lmhead_rank w8a8_lmhead_rank;

/* shard_weights: int8 rows of THIS rank's shard [hi - lo, ld] (host or device memory),
 * shard_acc_step fp32 [hi - lo] (logit = float(acc) * acc_step); static input step in_step. */
w8a8_status w8a8_lmhead_rank_create(w8a8_ctx *ctx, int32_t rank, int32_t world, int32_t K,
                                    int32_t V, const int8_t *shard_weights, int64_t ld,
                                    const float *shard_acc_step, float in_step, int32_t max_tokens,
                                    int32_t k_max, w8a8_lmhead_rank **out_rank);
/* Writes W8A8_LMHEAD_RANK_HANDLE_BYTES bytes naming this rank's exchange memory. */
w8a8_status w8a8_lmhead_rank_export(const w8a8_lmhead_rank *rank, void *handle_out);
/* handles: world * W8A8_LMHEAD_RANK_HANDLE_BYTES bytes, rank p's at offset p * 64. */
w8a8_status w8a8_lmhead_rank_connect(w8a8_lmhead_rank *rank, const void *handles);
/* All world ranks of one process (ranks[p] = rank p), connected to each other directly. */
w8a8_status w8a8_lmhead_rank_connect_local(w8a8_lmhead_rank *const *ranks, int32_t world);
w8a8_status w8a8_lmhead_rank_forward(w8a8_lmhead_rank *rank, const float *h_dev, int32_t T,
                                     int32_t k, float *topk_val_dev, int32_t *topk_idx_dev,
                                     int32_t *argmax_dev, void *stream);
void        w8a8_lmhead_rank_destroy(w8a8_lmhead_rank *rank);
/* Fuses the LM head's input RMSNorm (w8a8_emb_norm_pack's arithmetic) into the forward's
 * quantisation step: h is then the un-normalised final hidden state.  NULL turns it off. */
w8a8_status w8a8_lmhead_rank_set_input_norm(w8a8_lmhead_rank *rank,
                                            const float *emb_norm_scaled_dev, float eps);
/* Number of vocab rows of this rank's shard; *lo / *hi (may be NULL) its first / end vocab id. */
int32_t     w8a8_lmhead_rank_shard_range(const w8a8_lmhead_rank *rank, int32_t *lo, int32_t *hi);

/* ---------------------------------------------------------------------------------------
 * Expert parallelism of a MoE layer over processes (one process per GPU, every rank holding the
 * same hidden states): rank r computes the experts e with e % world == r (shared expert s counts
 * as e = n_routed + s) for every token, combines its own slots in slot order into a partial
 * [T, H], and the library exchanges the partials -- peer stores into CUDA-IPC-mapped device
 * memory, device counters with bounded waits, no NCCL call -- and sums them in rank order, so
 * every rank gets the same [T, H] output.  With world = 2 this is the reference's even / odd
 * split of the selected experts over its two dies and its die-by-die sum
 * (src/LFM2.5-8B-A1B/lfm2_moe.cpp:2190-2432; MoERouter's per-die grouping, moe_router.hpp:100-130).
 * Set-up as for w8a8_lmhead_rank_*: create, export (64 bytes), exchange, connect (or
 * connect_local for ranks of one process).  While the ep object lives, w8a8_moe_forward of
 * its layer computes only this rank's partial.  Forwards of every rank: the same sequence, the
 * same T, on one stream per rank; graph-capturable.
 * ------------------------------------------------------------------------------------- */
#define W8A8_MOE_EP_HANDLE_BYTES 64
typedef struct w8a8_moe_ep w8a8_moe_ep;

w8a8_status w8a8_moe_ep_create(w8a8_moe *moe, int32_t rank, int32_t world, int32_t max_tokens,
                               w8a8_moe_ep **out_ep);
w8a8_status w8a8_moe_ep_export(const w8a8_moe_ep *ep, void *handle_out);
w8a8_status w8a8_moe_ep_connect(w8a8_moe_ep *ep, const void *handles);
w8a8_status w8a8_moe_ep_connect_local(w8a8_moe_ep *const *eps, int32_t world);
/* hidden_dev fp32 [T, ldh] (the same on every rank) -> out_dev fp32 [T, ldo]. */
w8a8_status w8a8_moe_ep_forward(w8a8_moe_ep *ep, const float *hidden_dev, int64_t ldh, int32_t T,
                                float *out_dev, int64_t ldo, void *stream);
void        w8a8_moe_ep_destroy(w8a8_moe_ep *ep);

/* ---------------------------------------------------------------------------------------
 * int16 x int16 linear: the w2 stage of the reference's SwiGLU MLP subgraph, whose input is the
 * int16 product silu(gate) * up and whose weights are int16 per-row codes (tile_int16_slice,
 * build_lfm3_int8_pkg.py:111-122, written for w2 at :290-306 with trunc 28).  It replaces the
 * NPU's int16 CMAC + SDP step modelled by attribute_int8_error.py:117-121:
 *   y_q[t, n] = clip(round(sum_k x[t, k] * w[n, k] * (QuantM[n] / 2^trunc)), +-32767)
 * (float64 in the reference; the sum is accumulated exactly here, so the result is the same
 * integer), and optionally the unpack y = float(y_q) * out_step_chan[n]
 * (unpack_npu_output_int16, lfm3_v2.cpp:1010-1046).  weights int16 [N, ld] (host or device),
 * quant_m int16 [N], out_step_chan fp32 [N] or NULL.  K * 32767^2 < 2^53.
 * ------------------------------------------------------------------------------------- */
typedef struct w8a8_linear16 w8a8_linear16;

w8a8_status w8a8_linear16_create(w8a8_ctx *ctx, int32_t K, int32_t N, const int16_t *weights,
                                 int64_t ld, const int16_t *quant_m, int32_t trunc,
                                 const float *out_step_chan, int32_t max_tokens,
                                 w8a8_linear16 **out_linear16);
/* x_dev int16 [T, ldx] -> y_dev int16 [T, ldy] (W8A8_OUT_QUANT) or fp32 [T, ldy] (W8A8_OUT_F32). */
w8a8_status w8a8_linear16_forward(w8a8_linear16 *linear16, const int16_t *x_dev, int64_t ldx,
                                  int32_t T, int32_t out_mode, void *y_dev, int64_t ldy,
                                  void *stream);
void        w8a8_linear16_destroy(w8a8_linear16 *linear16);

/* ---------------------------------------------------------------------------------------
 * Decode chain: a fixed sequence of linears, optionally ending with an LM-head top-k step, run
 * by ONE persistent cooperative kernel launch per forward.  Replaces the per-linear
 * pack -> submit_task -> unpack round trips of the reference's decode loop
 * (Lfm3Engine::forward_chunk, lfm3_v2.cpp:1743-1990; TransformerSession::step,
 * transformer_session.cpp:650-844).  All pointers are fixed at create time (like a recorded
 * graph); a step whose input or output overlaps an earlier step's buffers since the last grid
 * barrier gets a barrier in front of it.  The linears must outlive the chain.
 * ------------------------------------------------------------------------------------- */
typedef struct {
    w8a8_linear *linear;       /* weights + parameters of this step */
    const float *x_dev;        /* fp32 [T, ldx] input view (chain input or a slice of an earlier y) */
    int64_t      ldx;
    int32_t      act_mode;     /* w8a8_act_mode */
    int32_t      out_mode;     /* w8a8_out_mode (F32 or F32_ACC for a top-k step) */
    void        *y_dev;        /* [T, ldy] output per out_mode (unused by a top-k step) */
    int64_t      ldy;
    float       *ratio_dev;    /* optional [T] per-token ratios (DYNTOK), may be NULL */
    int32_t      topk_k;       /* 0, or k (1..64) for an LM-head step; must be the last step */
    int32_t      row_offset;   /* top-k: vocab id of the linear's row 0 */
    float       *topk_val_dev; /* top-k: [T, k] */
    int32_t     *topk_idx_dev; /* top-k: [T, k] */
    /* Optional RMSNorm folded into a STATIC pack (the LM head's fused_emb_norm_broadcast_t1,
     * lfm3_v2.cpp:810-831): when non-NULL, x rows are packed as
     * round_clamp(x * inv_rms * emb_norm_dev[c], 127), inv_rms = 1 / sqrt(sum / K + norm_eps)
     * with the reference's four interleaved sums of squares; emb_norm_dev = norm weight / in_step
     * ([K] fp32, lfm3_v2.cpp:3906-3912).  act_mode must be STATIC. */
    const float *emb_norm_dev;
    float        norm_eps;
} w8a8_chain_step;

typedef struct w8a8_chain w8a8_chain;

/* T in [1, 8].  Returns W8A8_ERR_NOT_SUPPORTED when the steps do not fit the kernel's shared
 * memory plan. */
w8a8_status w8a8_chain_create(w8a8_ctx *ctx, const w8a8_chain_step *steps, int32_t n_steps,
                              int32_t T, w8a8_chain **out_chain);
/* Runs every step once, asynchronously on `stream` (one memset + one kernel launch). */
w8a8_status w8a8_chain_forward(w8a8_chain *chain, void *stream);
void        w8a8_chain_destroy(w8a8_chain *chain);
/* Number of grid barriers the chain executes per forward. */
int32_t     w8a8_chain_barriers(const w8a8_chain *chain);
/* Number of CTAs of the chain kernel (one per SM). */
int32_t     w8a8_chain_grid(const w8a8_chain *chain);
/* Per-step stage timers, the counterpart of the reference's StageTimers (lfm3_v2.cpp:431-530):
 * when trace_dev is non-NULL, every forward writes uint64 %globaltimer stamps (ns) into
 * trace_dev[(cta * n_steps + step) * 8 + i]: i = 0 step entered (after its grid barrier),
 * 1 input quantised, 2 outputs written, 3 arrival published, 4 / 5 first / last weight copy of
 * the step issued, 6 first weight stage of the step landed.  NULL turns tracing off. */
w8a8_status w8a8_chain_set_trace(w8a8_chain *chain, unsigned long long *trace_dev);

/* Allocation-free LM-head shard top-k.  This entry point has no counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: code running inside an allocator or memory-pool
 * callback, plugins whose host process owns every device allocation, and hot paths that must
 * not take the driver's allocation locks.  It computes what w8a8_linear_forward_topk computes
 * for a static-input shard in F32_ACC mode (logit = float(acc) * acc_step[n]), but takes the
 * weights and parameters as device pointers (no w8a8_linear, no w8a8_ctx) and keeps its scratch
 * (int8 activations, per-CTA candidate lists, arrival counter) in one module-scope device array
 * of about 1.4 MiB that every GPU loading the library holds until the process exits.  It calls
 * no cudaMalloc, cudaFree or allocating library routine.
 *
 * w_dev: int8 [N, ldw] on the current device, 16-byte aligned, ldw a multiple of 16 and
 * >= round_up(K, 16) (bytes past K in a row may hold anything).  acc_step_dev: fp32 [N].
 * x_dev: fp32 [T, ldx].  in_step: static input step (q = RNE(clamp(x * (1 / in_step), +-127))).
 * Outputs topk_val_dev fp32 [T, k], topk_idx_dev int32 [T, k] (ids = row_offset + n), sorted
 * (value desc, id asc).  Limits: T <= 8, T * round_up(K, 16) <= 128 KiB, and
 * T * (CTAs of the launch, at most two per SM) * (k + 1) <= 163840 candidate keys; larger requests
 * return W8A8_ERR_INVALID_ARG with the reason in w8a8_last_error().
 *
 * The first call on a device is a set-up call: it resolves the scratch array's device address
 * (with that device current) and, under CUDA's default lazy module loading, makes the driver
 * load the library's kernels on that device, which allocates device memory inside the driver.
 * Make that first call (a warm-up call) before any stream capture and outside any context where
 * allocating is not allowed; later calls allocate nothing.  Every call on a device shares the
 * array and it keeps the last call's contents: calls whose executions overlap on the GPU race
 * and corrupt each other's results, so order them on one stream.  A bounded in-kernel wait that
 * runs out is not reported by this entry point (it has no context). */
w8a8_status w8a8_lmhead_topk_noalloc(const int8_t *w_dev, int64_t ldw, int32_t K, int32_t N,
                                     const float *acc_step_dev, float in_step, const float *x_dev,
                                     int64_t ldx, int32_t T, int32_t k, int32_t row_offset,
                                     float *topk_val_dev, int32_t *topk_idx_dev, void *stream);

/* ---------------------------------------------------------------------------------------
 * The steps on either side of each linear of the reference's decode loop, on the GPU with the
 * reference's float order (sums of squares in its four interleaved chains, then its tail; IEEE
 * sqrt and division; products left to right), bit-identical to it.  One token row per CTA;
 * every pointer is device memory; C <= 12288.
 *
 * w8a8_rmsnorm_pack_dyntok replaces fused_rms_norm_pack_dyntok_t1 (lfm3_v2.cpp:652-700) for T
 * rows: inv_rms = 1 / sqrt(sum_sq / C + eps); u = h * inv_rms * smooth[c];
 * ratio[t] = max(max|u|, 1e-8) / max(in_thresh, 1e-8); q = round_clamp(u * (127 / amax), 127),
 * and (u_out non-NULL) u_out = h * inv_rms * norm[c].  q / ratio feed w8a8_linear_forward_q in
 * W8A8_ACT_DYNTOK mode.
 *
 * w8a8_post_op_ffn_pack replaces fused_post_op_residual_ffn_pack_mlp_t1 (lfm3_v2.cpp:702-765):
 * h_mid = h + op_out * inv_rms(op_out) * post_norm[c]; q = round_clamp(h_mid * inv_rms(h_mid)
 * * ffn_scaled[c], 127) (ffn_scaled folds the FFN norm weight, the smoothing and 1 / in_step:
 * a static-mode input for the MLP's first linear).  h_mid may alias h.
 * ------------------------------------------------------------------------------------- */
w8a8_status w8a8_rmsnorm_pack_dyntok(w8a8_ctx *ctx, const float *h_dev, int64_t ldh, int32_t T,
                                     int32_t C, const float *norm_dev, const float *smooth_dev,
                                     float in_thresh, float eps, int8_t *q_dev, int64_t ldq,
                                     float *ratio_dev, float *u_out_dev, int64_t ldu,
                                     void *stream);
/* w8a8_emb_norm_pack replaces fused_emb_norm_broadcast_t1 (lfm3_v2.cpp:810-831), the LM head's
 * input step: q[t, c] = round_clamp(h * inv_rms * emb_norm_scaled[c], 127) with inv_rms from the
 * reference's ordered sum of squares and emb_norm_scaled[c] = norm_weight[c] * (1 / in_step)
 * (lfm3_v2.cpp:3906-3912): a static-mode int8 input of the LM head.  C <= 12288. */
w8a8_status w8a8_emb_norm_pack(w8a8_ctx *ctx, const float *h_dev, int64_t ldh, int32_t T,
                               int32_t C, const float *emb_norm_scaled_dev, float eps,
                               int8_t *q_dev, int64_t ldq, void *stream);
w8a8_status w8a8_post_op_ffn_pack(w8a8_ctx *ctx, const float *op_out_dev, int64_t ldo,
                                  const float *post_norm_dev, const float *h_dev, int64_t ldh,
                                  int32_t T, int32_t C, const float *ffn_scaled_dev, float eps,
                                  float *h_mid_dev, int64_t ldm, int8_t *q_dev, int64_t ldq,
                                  void *stream);

/* ---------------------------------------------------------------------------------------
 * Token sampler over the merged LM-head candidates: Sampler::sample (sampler.cpp:83-179) with
 * its SamplerParams (sampler.hpp:10-19) and history (Sampler::accept / reset), run on the host
 * over the k (logit, vocab id) pairs that w8a8_lmhead_forward / w8a8_topk_merge leave, instead
 * of over the full vocabulary: repetition penalty over the history window, loop breaking,
 * greedy argmax or temperature, top-k, softmax, min-p, top-p and the draw from std::mt19937
 * (seed 0 = a random seed, as the reference).  The float steps use the host's libm and the
 * same order of operations, so a sampler given the same seed returns the reference's token.
 *
 * cand_val / cand_id: host arrays of n_cand pairs that are the n_cand largest raw logits of the
 * vocabulary in (logit desc, id asc) order (the merge's output).  The result is the reference's
 * whenever the candidates decide it; when they cannot (top_k = 0 or >= vocab with
 * n_cand < vocab, too few candidates left above the smallest one after the penalties, or a
 * repeat_penalty below 1 with history tokens outside the candidates) the call returns
 * W8A8_ERR_NOT_SUPPORTED and consumes no random number, so the caller can retry with more
 * candidates.  Ties among the top_k kept logits are ordered by id here, while the reference's
 * std::partial_sort leaves their order unspecified: the drawn token can differ only then.
 * Host only: no device memory, no CUDA call.
 * ------------------------------------------------------------------------------------- */
typedef struct {
    float    temperature;                 /* <= 0: greedy */
    int32_t  top_k;                       /* 0 disables */
    float    top_p;                       /* 1 disables */
    float    min_p;                       /* 0 disables */
    float    repeat_penalty;              /* 1 disables */
    int32_t  repeat_window;
    int32_t  max_consecutive_duplicates;  /* <= 0 disables */
    uint32_t seed;                        /* 0: random seed */
} w8a8_sampler_params;

typedef struct w8a8_sampler w8a8_sampler;

/* NULL params: the reference defaults (0.7, 40, 0.9, 0.05, 1.15, 64, 2, seed 0). */
w8a8_status w8a8_sampler_create(const w8a8_sampler_params *params, w8a8_sampler **out_sampler);
void        w8a8_sampler_destroy(w8a8_sampler *sampler);
w8a8_status w8a8_sampler_accept(w8a8_sampler *sampler, int32_t token_id);
w8a8_status w8a8_sampler_reset(w8a8_sampler *sampler);
w8a8_status w8a8_sampler_sample(w8a8_sampler *sampler, const float *cand_val,
                                const int32_t *cand_id, int32_t n_cand, int32_t vocab_size,
                                int32_t *token_out);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* W8A8_H */
